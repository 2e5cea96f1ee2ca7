#!/usr/bin/env python
"""Decode benchmark for the hymt2 B200 backend.

Workload (config 0 of the baseline): the reference's own bench GGUF
(Hy-MT2-1.8B shape, 32 layers, STQ1_0 layers + Q6_K tied LM head, written
byte-identically by hymt2_b200/synth), greedy decode at batch 1 after a
48-token prompt of ids uniform in [0, 120818) (numpy PCG64 seed 1).  One
benchmark step = one decoded token; steps cycle through positions 48..111
(the 64 generated tokens of the config).  Weights (613 MB) exceed L2, so no
flush is needed between steps.

  value        device-timed decode tok/s (CUDA events on the backend stream,
               max over ranks; whole job = ranks * steps / max time)
  e2e          the same decode through the public C ABI with every step's
               token copied in from / out to pinned host memory, wall-clock
  roofline     the dominant kernel: the persistent decode kernel (one launch
               runs up to 64 decode steps), each launch timed with CUDA
               events; algorithmic bytes = every weight byte of a step plus
               the K/V rows attention reads, per step times steps per launch
  cpu_baseline the reference's CPU library on this host (rank 0, N = 1)

`--impl reference` times the reference's own CPU implementation of the path
(oracle/_ref/libhymt2_ref.so, built from its sources) on the same config.
Multi-GPU: one process per GPU, independent replicas (no collective on the
data path); the process group only carries the barrier and the max-time.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Hy-MT2-1.8B STQ1_0 decode tok/s (bs1; bs256/GPU at 1/2/4/8); quant-GEMV HBM GB/s"
UNIT = "tok/s"
PROMPT_LEN, GEN_LEN, VOCAB = 48, 64, 120818
# algorithmic bytes per launch (weights as streamed: panel 64 B codes + 4 B scale per 256 weights;
# Q6_K 210 B per 256)
H, FFN, QD, KVD, L = 2048, 6144, 2048, 512, 32
PANEL = 68 / 256
OPS = {
    0: ("lm_head_q6k_argmax", 1, VOCAB * H * 210 // 256),
    1: ("qkv_gemv_panel", L, int((QD + 2 * KVD) * H * PANEL)),
    2: ("gate_up_gemv_panel", L, int(2 * FFN * H * PANEL)),
    3: ("down_gemv_panel", L, int(H * FFN * PANEL)),
    4: ("o_proj_gemv_panel", L, int(H * QD * PANEL)),
    5: ("attention_decode", L, 2 * (PROMPT_LEN + GEN_LEN // 2) * KVD * 2),  # K+V bf16 rows at mid window
}
STEP_WEIGHT_BYTES = sum(b * n for op, (_, n, b) in OPS.items() if op != 5)
# K/V rows read per step at the window's mean position (positions 48..111)
STEP_KV_BYTES = L * 2 * (PROMPT_LEN + (GEN_LEN - 1) / 2) * KVD * 2
STEP_BYTES = STEP_WEIGHT_BYTES + int(STEP_KV_BYTES)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=16)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--model-dir", default=os.environ.get("HYMT2_MODEL_DIR",
                                                         os.path.join(tempfile.gettempdir(), "hymt2_models")))
    p.add_argument("--cpu-tokens", type=int, default=24, help="decode tokens in the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--graph-breakdown", action="store_true",
                   help="also time each kernel of the per-layer graph path alone")
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampler during the timed region."""

    def __init__(self, dev: int):
        self.samples = []
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(dev), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.p = None

    def _read(self):
        for line in self.p.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def stop(self):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        sms = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def ensure_model(rank, local, world, model_dir, dist):
    from hymt2_b200 import synth
    if world > 1 and local != 0:
        dist.barrier()
        return synth.ensure("c0_stq", model_dir)
    path = synth.ensure("c0_stq", model_dir)
    if world > 1:
        dist.barrier()
    return path


def prompt_ids():
    return np.random.default_rng(1).integers(0, VOCAB, PROMPT_LEN).astype(np.int32)


def cpu_baseline(path: str, ntok: int) -> dict:
    """The reference's own CPU path on this host (all physical cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    os.environ["HYMT2_DEVICE"] = "cpu"
    ref = O.Reference()
    cores = int(ref.lib.refh_physical_cores())
    m = ref.load(path, threads=cores, ctx=1024)
    try:
        ids = prompt_ids().tolist()
        _, _, pre_ms, dec_ms, _ = m.greedy(ids, ntok + 1)
        threads = m.threads()
    finally:
        m.close()
    import platform
    cpu = platform.processor() or ""
    try:
        with open("/proc/cpuinfo") as f:
            cpu = next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), cpu)
    except OSError:
        pass
    return {"value": round(ntok / (dec_ms / 1000.0), 3), "unit": UNIT, "cores": threads, "kind": "reference",
            "isa": ref.isa(), "cpu": cpu,
            "sample": f"reference hymt2 CPU path (oracle/_ref, {ref.isa()}, {threads} threads): 48-token prompt "
                      f"prefill ({pre_ms:.0f} ms) then {ntok} greedy decode tokens at positions 48..{47 + ntok}"}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    from hymt2_b200 import synth
    path = synth.ensure("c0_stq", args.model_dir)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    os.environ["HYMT2_DEVICE"] = "cpu"
    try:
        ref = O.Reference()
    except (FileNotFoundError, OSError) as e:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU library not built: {e}"}))
        return
    cores = int(ref.lib.refh_physical_cores())
    m = ref.load(path, threads=cores, ctx=1024)
    ids = prompt_ids().tolist()
    steps = max(1, min(args.steps, GEN_LEN))
    m.greedy(ids, max(1, min(args.warmup, GEN_LEN)) + 1)           # warm-up (full prefill)
    _, _, pre_ms, dec_ms, cached = m.greedy(ids, steps + 1)         # prefix reuse, `steps` decode forwards
    threads = m.threads()
    m.close()
    v = steps / (dec_ms / 1000.0)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(dec_ms / steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8+fp32", "data": "synthetic",
        "config": {"workload": "c0_stq bs1 greedy decode, 48-token prompt, positions 48..111", "parallelism": "none"},
        "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"reference CPU ({ref.isa()}, {threads} threads), {steps} decode steps after a "
                                   f"cached 48-token prompt"},
        "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    args = parse()
    rank, local, world = dist_env()
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from hymt2_b200.device import Backend, DeviceModel
    path = ensure_model(rank, local, world, args.model_dir, dist)
    be = Backend(local)
    dm = DeviceModel(path, be, ctx=1024)
    lib, impl = be.lib, be.impl
    stream = torch.cuda.ExternalStream(be.stream())
    ids = prompt_ids()

    def check(rc, what):
        if rc != 0:
            raise RuntimeError(f"{what}: {be.error()}")

    check(lib.hyc_decode_begin(impl, ids.ctypes.data, PROMPT_LEN, 0, GEN_LEN, None, 0, dm.vocab_out), "begin")
    import ctypes
    why = ctypes.create_string_buffer(128)
    persistent = lib.hyc_decode_path(impl, why, 128) == 1
    path_name = why.value.decode()
    first = np.zeros(1, dtype=np.int32)
    lib.hyc_decode_read(impl, first.ctypes.data, 1)
    tok0 = int(first[0])

    def run_steps(n, host_io=None):
        s = 0
        while s < n:
            check(lib.hyc_decode_rewind(impl, PROMPT_LEN, tok0), "rewind")
            m = min(GEN_LEN, n - s)
            if host_io is None:
                check(lib.hyc_decode_steps(impl, m), "steps")
            else:
                check(lib.hyc_decode_steps_host(impl, m, host_io), "steps_host")
            s += m

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        be.sync()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident decode
    w0 = time.perf_counter()
    run_steps(max(3, args.warmup))
    barrier()
    per_step = (time.perf_counter() - w0) / max(3, args.warmup)
    # keep the GPU busy ~0.6 s on both sides of the timed region so the clock
    # sampler (200 ms period) sees the load that the timed steps run under
    pad = max(1, int(0.6 / max(per_step, 1e-5)))
    clocks = Clocks(local)
    run_steps(pad)
    l0 = be.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run_steps(args.steps)
    e1.record(stream)
    launches = be.launches() - l0
    run_steps(pad)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))

    # ---- end to end: every step's token through pinned host memory, wall clock
    host = lib.hyc_host_alloc(4 * (GEN_LEN + 1))
    run_steps(max(3, args.warmup), host)
    barrier()
    t0 = time.perf_counter()
    run_steps(args.steps, host)
    be.sync()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    lib.hyc_host_free(host)

    # ---- roofline of the dominant kernel
    peak, peak_kind = peaks()
    kernels = {}
    dom_entry = None
    if persistent:
        # one launch of the persistent kernel = GEN_LEN decode steps (the
        # rewind before it is a 8-byte copy); CUDA events around each launch
        n_launch = max(2, min(8, args.steps // GEN_LEN or 2))
        evs = []
        for _ in range(n_launch):
            check(lib.hyc_decode_rewind(impl, PROMPT_LEN, tok0), "rewind")
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            check(lib.hyc_decode_steps(impl, GEN_LEN), "steps")
            b.record(stream)
            evs.append((a, b))
        be.sync()
        t = statistics.mean(x.elapsed_time(y) for x, y in evs)
        nbytes = STEP_BYTES * GEN_LEN
        dom_entry = ("decode_mega", {"ms_per_launch": round(t, 4), "launches_per_step": 1.0 / GEN_LEN,
                                     "steps_per_launch": GEN_LEN, "bytes_per_launch": nbytes,
                                     "gbs": round(nbytes / (t / 1e3) / 1e9, 1)})
    for op, (name, per_step, nbytes) in (OPS.items() if (args.graph_breakdown or not persistent) else []):
        iters = 20 if op == 0 else 64
        check(lib.hyc_bench_op(impl, op, 4), "bench_op warm")
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        check(lib.hyc_bench_op(impl, op, iters), "bench_op")
        b.record(stream)
        be.sync()
        t = a.elapsed_time(b) / iters
        kernels[name] = {"ms_per_launch": round(t, 5), "launches_per_step": per_step, "bytes_per_launch": nbytes,
                         "gbs": round(nbytes / (t / 1e3) / 1e9, 1), "share_of_step_ms": round(t * per_step, 4)}
    if dom_entry:
        dom, dk = dom_entry
    else:
        dom = max(kernels, key=lambda k: kernels[k]["share_of_step_ms"])
        dk = kernels[dom]
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "dram_traffic_c0_stq.json")
    if os.path.exists(tfile):
        with open(tfile) as f:
            tj = json.load(f).get(dom)
        if tj:  # per-step DRAM bytes of one ncu capture, scaled to a launch
            traffic = int(tj["dram_bytes_per_step"] * dk.get("steps_per_launch", 1))

    if rank == 0:
        step_ms = ms / args.steps
        value = world * args.steps / (ms / 1e3)
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8+fp32", "data": "synthetic",
            "config": {"workload": "c0_stq: Hy-MT2-1.8B shape, 32 layers STQ1_0 (panel) + Q6_K tied head, reference "
                                   "bench GGUF; bs1 greedy decode after a 48-token prompt, positions 48..111",
                       "global_batch": world, "seq_len": PROMPT_LEN + GEN_LEN, "parallelism": f"dp{world} replicas",
                       "l2": "weights 613 MB per step > 126 MB L2 (no flush needed)"},
            "e2e": {"value": round(world * args.steps / e2e_s, 2), "unit": UNIT, "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4,
                    "path": f"hyc_decode_steps_host: token in from pinned host, one decode step ({path_name}), "
                            f"token out to pinned host"},
            "decode_path": path_name,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": dk["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": round(dk["gbs"] / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "bytes_per_launch": dk["bytes_per_launch"], "ms_per_launch": dk["ms_per_launch"]},
            "roofline_step": {"bytes_per_step": STEP_BYTES, "achieved_gbs": round(STEP_BYTES / step_ms / 1e6, 1),
                              "frac": round(STEP_BYTES / step_ms / 1e6 / peak, 4)},
            "kernels": kernels,
            "gpu_launches": int(launches),
            "clocks": clk,
            "device": be.info,
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                out["cpu_baseline"] = cpu_baseline(path, args.cpu_tokens)
            except Exception as e:  # noqa: BLE001 - report, do not fail the GPU number
                out["cpu_baseline"] = {"unavailable": str(e)}
        print(json.dumps(out))
    dm.close()
    be.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
