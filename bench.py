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
  e2e          the same decode through the public C ABI with the host in the
               loop: every step's token goes in from and comes back to pinned
               host memory, and the host waits for it and checks the stop ids
               before the next step (wall clock)
  roofline     the dominant kernel: the persistent decode kernel (one launch
               runs up to 64 decode steps), each launch timed with CUDA
               events; algorithmic bytes = every weight byte of a step plus
               the K/V rows attention reads, per step times steps per launch
  cpu_baseline the reference's CPU library on this host (rank 0, N = 1)
  serving      config 3 on every GPU: 4096 requests sharded over the ranks,
               continuous batching of <= 256 sequences per GPU (generated tok/s)
  prefill_c2   config 2 (N = 1): 32 x 256-token Q4_K_M prefill on the tensor
               cores, with its int8 roofline and the reference CPU prefill
  decode_c1    config 1 (N = 1): Q2_0C bs1 decode after a 512-token prompt
  decode_c4    config 4's model whole on ONE GPU (N = 1): Q8_0 bs1 decode at
               KV length 4096, graph path
  decode_c4_tp config 4 as specified (N >= 2): the model split over the N
               GPUs (tensor parallelism), per-token latency (max over ranks)

`--impl reference` times the reference's own CPU implementation of the path
(oracle/_ref/libhymt2_ref.so, built from its sources) on the same config.
Multi-GPU: one process per GPU, independent replicas (no collective on the
data path); the process group only carries the barrier and the max-time.
"""
from __future__ import annotations

import argparse
import ctypes
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
    p.add_argument("--serve-requests", type=int, default=4096, help="config-3 requests (all GPUs); 0 skips")
    p.add_argument("--no-extra", action="store_true", help="skip the config 1 / config 2 lines (N = 1 only)")
    p.add_argument("--profile-pass", choices=["c0mega", "c2", "c3step", "c4step"],
                   help="for ncu --profile-from-start off: warm up, then run one persistent-kernel launch of "
                        "three config-0 decode steps, one batch pass of config 2 (32 x 256 prefill), one "
                        "config-3-shaped step (256 decode tokens at position 100) or two config-4 decode steps "
                        "(Q8_0, KV 4096) between cuProfilerStart/Stop, and exit")
    p.add_argument("--layers", type=int, default=32, help="model layers for --profile-pass")
    return p.parse_args()


def profile_pass(args):
    """One batch pass (c2, c3step) or two config-4 decode steps (c4step)
    bracketed by cuProfilerStart / cuProfilerStop."""
    import ctypes
    from hymt2_b200 import synth
    from hymt2_b200.device import Backend, DeviceModel
    if args.profile_pass == "c0mega":
        be = Backend(0)
        dm = DeviceModel(synth.ensure("c0_stq", args.model_dir), be, ctx=1024)
        lib, impl = be.lib, be.impl
        ids = prompt_ids()
        if lib.hyc_decode_begin(impl, ids.ctypes.data, PROMPT_LEN, 0, GEN_LEN, None, 0, dm.vocab_out) != 0 or \
                lib.hyc_decode_steps(impl, 3) != 0:
            raise RuntimeError(be.error())
        be.sync()
        cu = ctypes.CDLL("libcuda.so.1")
        cu.cuProfilerStart()
        if lib.hyc_decode_steps(impl, 3) != 0:
            raise RuntimeError(be.error())
        be.sync()
        cu.cuProfilerStop()
        dm.close()
        be.close()
        print("profiled one persistent-kernel launch of three decode steps")
        return
    if args.profile_pass == "c4step":
        be = Backend(0)
        dm = DeviceModel(synth.ensure("c4_q8_0", args.model_dir, layers=args.layers), be, ctx=C4_PROMPT + 128)
        lib, impl = be.lib, be.impl
        ids = np.random.default_rng(1).integers(0, VOCAB, C4_PROMPT).astype(np.int32)
        if lib.hyc_decode_begin(impl, ids.ctypes.data, C4_PROMPT, 0, 16, None, 0, dm.vocab_out) != 0 or \
                lib.hyc_decode_steps(impl, 3) != 0:
            raise RuntimeError(be.error())
        be.sync()
        cu = ctypes.CDLL("libcuda.so.1")
        cu.cuProfilerStart()
        if lib.hyc_decode_steps(impl, 2) != 0:
            raise RuntimeError(be.error())
        be.sync()
        cu.cuProfilerStop()
        dm.close()
        be.close()
        print("profiled two decode steps")
        return
    cfg = "c2_q4km" if args.profile_pass == "c2" else "c0_stq"
    be = Backend(0)
    dm = DeviceModel(synth.ensure(cfg, args.model_dir, layers=args.layers), be, ctx=512)
    rng = np.random.default_rng(0)
    if args.profile_pass == "c2":
        dm.batch_prepare(slots=C2_SEQS, slot_ctx=C2_LEN, max_tokens=C2_SEQS * C2_LEN, max_out=C2_SEQS)
        toks = rng.integers(0, VOCAB, C2_SEQS * C2_LEN)
        slots, pos = np.repeat(np.arange(C2_SEQS), C2_LEN), np.tile(np.arange(C2_LEN), C2_SEQS)
        rows = np.arange(C2_SEQS) * C2_LEN + C2_LEN - 1
    else:
        dm.batch_prepare(slots=SERVE_SLOTS, slot_ctx=256, max_tokens=SERVE_SLOTS, max_out=SERVE_SLOTS)
        toks, slots = rng.integers(0, VOCAB, SERVE_SLOTS), np.arange(SERVE_SLOTS)
        pos, rows = np.full(SERVE_SLOTS, 100), np.arange(SERVE_SLOTS)
    for _ in range(2):
        dm.batch_forward(toks, slots, pos, rows)
    cu = ctypes.CDLL("libcuda.so.1")
    cu.cuProfilerStart()
    dm.batch_forward(toks, slots, pos, rows)
    cu.cuProfilerStop()
    dm.close()
    be.close()
    print("profiled one pass")


def kernel_source_hash() -> str:
    """sha256 (first 16 hex digits) of the headers the kernels are built from (hy_*.cuh, hy_*.h)."""
    import hashlib
    h = hashlib.sha256()
    cdir = os.path.join(ROOT, "hymt2_b200", "csrc")
    for name in sorted(os.listdir(cdir)):
        if name.endswith((".cuh", ".h")):
            with open(os.path.join(cdir, name), "rb") as f:
                h.update(name.encode() + b"\0" + f.read())
    return h.hexdigest()[:16]


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


def int8_peak(torch) -> tuple[float, str]:
    """Dense int8 TOPS of this GPU: cuBLASLt int8 GEMM (torch._int_mm, 8192^3,
    best of 5); 2x the measured bf16 figure if that is unavailable."""
    try:
        n = 8192
        a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
        torch._int_mm(a, b)
        best = None
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1)
            best = t if best is None else min(best, t)
        del a, b
        return 2 * n ** 3 / (best / 1e3) / 1e12, "measured (torch._int_mm 8192^3 burst)"
    except Exception:  # noqa: BLE001
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                return 2 * float(json.load(f)["bf16_tflops"]), "2x measured bf16"
        except (OSError, KeyError, ValueError):
            return 2 * 1590.0, "2x fallback bf16"


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


SERVE_PREFIX, SERVE_MAX_NEW, SERVE_SLOTS, SERVE_STEP_TOKENS = 24, 64, 256, 512
SERVE_MAX_TOKENS = 4096  # pass capacity: prompt chunks may fill it while fewer than half the slots decode


def shard(items: list, rank: int, world: int) -> list:
    """This rank's share of independent requests: r, r + N, r + 2N, ..."""
    return items[rank::world]


def max_over_ranks_fn(dist, device):
    """Max of a per-rank float over the process group (identity without one)."""
    import torch

    def f(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return f


def serve_requests(n: int) -> list[list[int]]:
    """Config 3 requests: lengths uniform in [16, 128]; the first min(len, 24)
    ids are one shared prefix, the rest uniform over the vocab (seed 3)."""
    rng = np.random.default_rng(3)
    prefix = rng.integers(0, VOCAB, SERVE_PREFIX).tolist()
    out = []
    for _ in range(n):
        ln = int(rng.integers(16, 129))
        k = min(ln, SERVE_PREFIX)
        out.append(prefix[:k] + rng.integers(0, VOCAB, ln - k).tolist())
    return out


def bench_serving(dm, stream, torch, rank, world, nreq, max_over_ranks, barrier, tops=None, tops_kind="") -> dict:
    """Config 3 on this rank's shard (requests r, r + N, ...): continuous
    batching over 256 slots, 64 greedy tokens per request, device-timed
    around the whole serve call (host scheduling included)."""
    reqs = shard(serve_requests(nreq), rank, world)
    dm.batch_prepare(slots=SERVE_SLOTS, slot_ctx=128 + SERVE_MAX_NEW, max_tokens=SERVE_MAX_TOKENS,
                     max_out=SERVE_SLOTS)
    dm.serve(reqs[:min(len(reqs), 300)], 4, SERVE_STEP_TOKENS)  # warm-up: tensor-core weight tiles, clocks
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    out, st = dm.serve(reqs, SERVE_MAX_NEW, SERVE_STEP_TOKENS)
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = max_over_ranks(e0.elapsed_time(e1))
    total_gen = SERVE_MAX_NEW * nreq
    # useful int8 ops of this rank's run: every token (prefill or decode) through the layers, the head on each
    # generated token; the pass runs on the tensor cores (tcgen05 int8, >= 32 tokens per GEMM)
    ops = INT8_OPS_PER_TOKEN * (st["decode_tokens"] + st["prefill_tokens"]) + HEAD_OPS_PER_SEQ * st["decode_tokens"]
    roof = None
    if tops:
        achieved = ops / (ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tops, 1),
                "unit": "TOPS (int8, useful ops, rank 0's share over the max-over-ranks time)",
                "frac": round(achieved / tops, 4), "peak_kind": tops_kind, "ops_rank0": int(ops)}
    return {"value": round(total_gen / (ms / 1e3), 1), "unit": "generated tok/s", "n_gpus": world,
            "roofline": roof,
            "requests": nreq, "requests_per_gpu": len(reqs), "max_new": SERVE_MAX_NEW, "slots_per_gpu": SERVE_SLOTS,
            "step_token_budget": SERVE_STEP_TOKENS, "pass_capacity": SERVE_MAX_TOKENS,
            "mean_slot_occupancy_rank0": round(st["active_seq_steps"] / max(1, st["steps"] * SERVE_SLOTS), 3),
            "ms": round(ms, 2), "wall_s_rank0": round(wall, 3),
            "steps_rank0": st["steps"], "prefill_tokens_rank0": st["prefill_tokens"],
            "prefix_hits_rank0": st["prefix_hits"], "prefix_tokens_rank0": st["prefix_tokens"],
            "kv_pages_shared_rank0": st["shared_pages"], "kv_rows_copied_rank0": st["copied_rows"],
            "kv_pages_evicted_rank0": st["evictions"],
            "tokens_per_s_incl_prefill": round((st["decode_tokens"] + st["prefill_tokens"]) * world / (ms / 1e3), 1),
            "workload": "c3: c0_stq model, 4096 requests (prompt U[16,128] ids with a shared 24-token prefix), "
                        "64 greedy tokens each, continuous batching <= 256 sequences per GPU, requests sharded "
                        "round-robin over the GPUs with no collective; time = max over ranks"}


C2_SEQS, C2_LEN = 32, 256
INT8_OPS_PER_TOKEN = 2 * 1_543_503_872          # layer int8 MACs x 2 per token (c2 shapes)
HEAD_OPS_PER_SEQ = 2 * VOCAB * H                # the LM head runs on each sequence's last token


def ref_prefill_cpu(path: str, ntok: int) -> dict:
    """Reference CPU prefill of one ntok-token prompt (all physical cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    os.environ["HYMT2_DEVICE"] = "cpu"
    ref = O.Reference()
    cores = int(ref.lib.refh_physical_cores())
    m = ref.load(path, threads=cores, ctx=ntok + 8)
    try:
        ids = np.random.default_rng(2).integers(0, VOCAB, ntok).tolist()
        _, _, pre_ms, _, _ = m.greedy(ids, 1)
        threads = m.threads()
    finally:
        m.close()
    return {"value": round(ntok / (pre_ms / 1e3), 2), "unit": "prefill tok/s", "cores": threads,
            "kind": "reference", "sample": f"reference CPU ({ref.isa()}, {threads} threads): one {ntok}-token "
                                           f"prompt prefill (its 16-token chunks), {pre_ms:.0f} ms"}


def bench_prefill(args, be, torch, tops, tops_kind) -> dict:
    """Config 2: 32 independent sequences x 256 seeded ids (seed 2) through
    one ragged batch pass each (all 8192 tokens in every GEMM, LM head +
    argmax on each sequence's last token), CUDA events over 5 passes."""
    from hymt2_b200 import synth
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c2_q4km", args.model_dir)
    dm = DeviceModel(path, be, ctx=C2_LEN)
    try:
        rng = np.random.default_rng(2)
        toks = rng.integers(0, VOCAB, C2_SEQS * C2_LEN)
        slots = np.repeat(np.arange(C2_SEQS), C2_LEN)
        pos = np.tile(np.arange(C2_LEN), C2_SEQS)
        rows = np.arange(C2_SEQS) * C2_LEN + C2_LEN - 1
        dm.batch_prepare(slots=C2_SEQS, slot_ctx=C2_LEN, max_tokens=C2_SEQS * C2_LEN, max_out=C2_SEQS)
        stream = torch.cuda.ExternalStream(be.stream())
        for _ in range(3):
            dm.batch_forward(toks, slots, pos, rows)
        n = 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            dm.batch_forward(toks, slots, pos, rows)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        ntok = C2_SEQS * C2_LEN
        ops = INT8_OPS_PER_TOKEN * ntok + HEAD_OPS_PER_SEQ * C2_SEQS
        achieved = ops / (ms / 1e3) / 1e12
        out = {"value": round(ntok / (ms / 1e3), 1), "unit": "prefill tok/s", "ms_per_pass": round(ms, 3),
               "tokens_per_pass": ntok,
               "workload": "c2_q4km (Q4_K q/k/o/gate/up, Q6_K v/down/head): 32 sequences x 256 seeded ids, one "
                           "ragged pass (every projection one tcgen05 int8 GEMM over 8192 tokens), head + argmax on "
                           "each last token; host ids in, host ids out, synchronous",
               "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tops, 1),
                            "unit": "TOPS (int8, useful ops)", "frac": round(achieved / tops, 4),
                            "peak_kind": tops_kind, "ops_per_pass": ops,
                            "note": "Q4_K weights run as 3 exact int8 planes and Q6_K as 2, so the tensor pipe "
                                    "does ~2.7x the useful ops"}}
        if not args.no_cpu_baseline:
            try:
                out["cpu_baseline"] = ref_prefill_cpu(path, C2_LEN)
            except Exception as e:  # noqa: BLE001
                out["cpu_baseline"] = {"unavailable": str(e)}
        return out
    finally:
        dm.close()


C1_PROMPT, C1_GEN = 512, 128


def bench_c1(args, be, torch, peak) -> dict:
    """Config 1: Q2_0C layers, bs1 greedy decode of 128 tokens after a
    512-token seeded prompt (seed 1); CUDA events over the 127 decode steps."""
    from hymt2_b200 import synth
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c1_q2c", args.model_dir)
    dm = DeviceModel(path, be, ctx=1024)
    try:
        lib, impl = be.lib, be.impl
        ids = np.random.default_rng(1).integers(0, VOCAB, C1_PROMPT).astype(np.int32)
        stream = torch.cuda.ExternalStream(be.stream())
        for _ in range(2):
            if lib.hyc_decode_begin(impl, ids.ctypes.data, C1_PROMPT, 0, C1_GEN, None, 0, dm.vocab_out) != 0:
                raise RuntimeError("decode_begin: " + be.error())
            be.sync()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if lib.hyc_decode_steps(impl, C1_GEN - 1) != 0:
                raise RuntimeError("decode_steps: " + be.error())
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        out_ids = np.zeros(C1_GEN, dtype=np.int32)
        if lib.hyc_decode_read(impl, out_ids.ctypes.data, C1_GEN) != C1_GEN:
            raise RuntimeError("decode_read: " + be.error())
        # bytes per step: Q2_0C panel weights (same 68 B / 256 as STQ1_0) + Q6_K head + K/V rows at mean position
        kv = L * 2 * (C1_PROMPT + (C1_GEN - 1) / 2) * KVD * 2
        step_bytes = STEP_WEIGHT_BYTES + kv
        step_ms = ms / (C1_GEN - 1)
        out = {"value": round((C1_GEN - 1) / (ms / 1e3), 1), "unit": UNIT, "ms_per_step": round(step_ms, 4),
               "workload": "c1_q2c: Q2_0C layers (panel), Q6_K tied head; bs1 greedy decode, 512-token seeded "
                           "prompt, 128 tokens (positions 512..639), persistent decode kernel",
               "roofline_step": {"bytes_per_step": int(step_bytes),
                                 "achieved_gbs": round(step_bytes / step_ms / 1e6, 1),
                                 "frac": round(step_bytes / step_ms / 1e6 / peak, 4)}}
        if not args.no_cpu_baseline:
            try:
                sys.path.insert(0, os.path.join(ROOT, "oracle"))
                import oracle as O
                os.environ["HYMT2_DEVICE"] = "cpu"
                ref = O.Reference()
                cores = int(ref.lib.refh_physical_cores())
                m = ref.load(path, threads=cores, ctx=1024)
                _, _, pre_ms, dec_ms, _ = m.greedy(ids.tolist(), 9)
                thr = m.threads()
                m.close()
                out["cpu_baseline"] = {"value": round(8 / (dec_ms / 1e3), 2), "unit": UNIT, "cores": thr,
                                       "kind": "reference",
                                       "sample": f"reference CPU ({ref.isa()}, {thr} threads): 512-token prompt "
                                                 f"({pre_ms:.0f} ms), then 8 decode tokens"}
            except Exception as e:  # noqa: BLE001
                out["cpu_baseline"] = {"unavailable": str(e)}
        return out
    finally:
        dm.close()


NATIVE = 42 / 256  # native STQ1_0 bytes per weight (qs 32 + sign 8 + d 2 per 256)


def _graph_decode_ms(be, dm, torch, ids, n) -> float:
    """CUDA-event ms per step of n - 1 bs1 decode steps on the per-layer graph."""
    lib, impl = be.lib, be.impl
    stream = torch.cuda.ExternalStream(be.stream())
    if lib.hyc_set_decode_mode(impl, 1) != 0:
        raise RuntimeError("decode_mode: " + be.error())
    try:
        for _ in range(2):
            if lib.hyc_decode_begin(impl, ids.ctypes.data, len(ids), 0, n, None, 0, dm.vocab_out) != 0:
                raise RuntimeError("decode_begin: " + be.error())
            be.sync()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if lib.hyc_decode_steps(impl, n - 1) != 0:
                raise RuntimeError("decode_steps: " + be.error())
            e1.record(stream)
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (n - 1)
    finally:
        lib.hyc_set_decode_mode(impl, 0)


def bench_c0_native(args, be, torch, peak, path) -> dict:
    """The native STQ1_0 layout (the file's 42 B per 256 weights, the pattern
    table decoded in registers) on the config-0 model: the four layer GEMVs at
    one token, each cycling over the 32 layers' weights, bytes as stored; and
    bs1 decode on the per-layer graph (the persistent kernel takes panels
    only) beside the panel upload on the same graph."""
    from hymt2_b200.device import DeviceModel
    lib, impl = be.lib, be.impl
    stream = torch.cuda.ExternalStream(be.stream())
    ids = prompt_ids()
    out = {}
    for native in (True, False):
        be.set_stq_layout(native)
        try:
            dm = DeviceModel(path, be, ctx=1024)
        finally:
            be.set_stq_layout(False)
        try:
            step_ms = _graph_decode_ms(be, dm, torch, ids, GEN_LEN)
            key = "native" if native else "panel"
            out[f"graph_decode_{key}"] = {"tok_s": round(1e3 / step_ms, 1), "ms_per_step": round(step_ms, 4)}
            if native:
                kern = {}
                for op in (1, 2, 3, 4):
                    name = OPS[op][0].replace("_panel", "_native")
                    nbytes = int(OPS[op][2] / PANEL * NATIVE)
                    if lib.hyc_bench_op(impl, op, 4) != 0:
                        raise RuntimeError("bench_op: " + be.error())
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    if lib.hyc_bench_op(impl, op, 128) != 0:
                        raise RuntimeError("bench_op: " + be.error())
                    b.record(stream)
                    be.sync()
                    t = a.elapsed_time(b) / 128
                    kern[name] = {"ms_per_launch": round(t, 5), "bytes_per_launch": nbytes,
                                  "gbs": round(nbytes / (t / 1e3) / 1e9, 1),
                                  "gweights_s": round(nbytes / NATIVE / (t / 1e3) / 1e9, 1)}
                out["kernels"] = kern
        finally:
            dm.close()
    gu = out["kernels"]["gate_up_gemv_native"]
    out.update({"workload": "c0_stq with STQ1_0 layers uploaded native (hyc_set_stq_layout): gemv_panel_dec "
                            "<CPL, FMT_STQN> (row slice staged in shared memory, patterns decoded there), bs1 decode "
                            "positions 48..111 on the per-layer graph",
                "quant_gemv": {"kernel": "gate_up_gemv_native (2 x 6144 x 2048 native STQ1_0, nt 1)",
                               "gbs": gu["gbs"], "frac": round(gu["gbs"] / peak, 4),
                               "bytes_per_launch": gu["bytes_per_launch"], "ms_per_launch": gu["ms_per_launch"]}})
    return out


C4_PROMPT, C4_GEN = 4096, 64
# config 4 bytes per decode step: Q8_0 (34 B per 32 weights) layers and tied head as stored
C4_LAYER_BYTES = L * ((QD + 2 * KVD) * H + H * QD + 3 * FFN * H) * 34 // 32
C4_HEAD_BYTES = VOCAB * H * 34 // 32


def bench_c4(args, be, torch, peak) -> dict:
    """Config 4's model (Q8_0 everywhere, tied Q8_0 head) on one GPU: bs1
    greedy decode of 64 tokens after a 4096-token seeded prompt, so the
    attention reads K/V rows at positions 4096..4159; CUDA events over the 63
    decode steps (one CUDA graph of per-layer kernels per step).  The
    reference's tensor-parallel split of this config is not built here."""
    from hymt2_b200 import synth
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c4_q8_0", args.model_dir)
    dm = DeviceModel(path, be, ctx=C4_PROMPT + C4_GEN + 64)
    try:
        lib, impl = be.lib, be.impl
        ids = np.random.default_rng(1).integers(0, VOCAB, C4_PROMPT).astype(np.int32)
        stream = torch.cuda.ExternalStream(be.stream())
        for _ in range(2):
            if lib.hyc_decode_begin(impl, ids.ctypes.data, C4_PROMPT, 0, C4_GEN, None, 0, dm.vocab_out) != 0:
                raise RuntimeError("decode_begin: " + be.error())
            be.sync()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if lib.hyc_decode_steps(impl, C4_GEN - 1) != 0:
                raise RuntimeError("decode_steps: " + be.error())
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        import ctypes
        why = ctypes.create_string_buffer(128)
        lib.hyc_decode_path(impl, why, 128)
        path_why = why.value.decode()
        kv = L * 2 * (C4_PROMPT + (C4_GEN - 1) / 2) * KVD * 2
        step_bytes = C4_LAYER_BYTES + C4_HEAD_BYTES + kv
        step_ms = ms / (C4_GEN - 1)
        out = {"value": round((C4_GEN - 1) / (ms / 1e3), 1), "unit": UNIT, "ms_per_step": round(step_ms, 4),
               "workload": "c4_q8_0 on one GPU: Q8_0 layers and tied Q8_0 head (fp32 activations); bs1 greedy "
                           "decode, 4096-token seeded prompt, 64 tokens (positions 4096..4159); the model whole on one "
                           "GPU (its tensor-parallel split over N GPUs is the decode_c4_tp line at N >= 2)",
               "roofline_step": {"bytes_per_step": int(step_bytes),
                                 "achieved_gbs": round(step_bytes / step_ms / 1e6, 1),
                                 "frac": round(step_bytes / step_ms / 1e6 / peak, 4)},
               }
        if path_why:
            out["decode_path"] = path_why
        if not args.no_cpu_baseline:
            out["cpu_baseline"] = c4_cpu_baseline(path)
        return out
    finally:
        dm.close()


def c4_cpu_baseline(path: str) -> dict:
    """The reference's CPU decode of the config-4 model (scalar fp32 Q8_0
    rows, src/kernels.c:1097-1107) on all host cores.  Its prefill runs at
    ~0.3 s per token on 8 cores, so a 4096-token prompt would take tens of
    minutes: the sample is a 64-token prompt, then 4 decode tokens at KV
    64..67.  Attention over 4096 keys adds ~0.5 G multiply-adds per token to
    the ~1.9 G of the weights, so decode at KV 4096 is slower still."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        os.environ["HYMT2_DEVICE"] = "cpu"
        ref = O.Reference()
        cores = int(ref.lib.refh_physical_cores())
        m = ref.load(path, threads=cores, ctx=128)
        ids = np.random.default_rng(1).integers(0, VOCAB, 64).tolist()
        _, _, pre_ms, dec_ms, _ = m.greedy(ids, 5)
        thr = m.threads()
        m.close()
        return {"value": round(4 / (dec_ms / 1e3), 3), "unit": UNIT, "cores": thr, "kind": "reference",
                "sample": f"reference CPU ({ref.isa()}, {thr} threads): 64-token prompt ({pre_ms:.0f} ms), then 4 "
                          f"decode tokens at KV 64..67 (a 4096-token prefill is beyond the bench budget; KV 4096 "
                          f"decode is slower than this)"}
    except Exception as e:  # noqa: BLE001
        return {"unavailable": str(e)}


def bench_c4_tp(args, be, torch, dist, rank, world, max_over_ranks) -> dict:
    """Config 4 as specified: the Q8_0 model split over the N GPUs
    (tensor parallelism: heads and FFN columns per rank, o_proj / down
    row-parallel with the partial products summed by the backend's one-shot
    push over NVLink peer memory, vocabulary-split head).  Every rank prefills
    the 4096-token seeded prompt, then 63 greedy decode steps are timed with
    CUDA events on each rank's stream; the per-token latency is the max over
    ranks.  For comparison, the latency of one NCCL all-reduce of the same
    8 KB (2048 fp32, the exchange after o_proj and after down) is timed too."""
    from hymt2_b200 import synth
    from hymt2_b200.tp import TPDeviceModel
    if rank == 0:
        path = synth.ensure("c4_q8_0", args.model_dir)
        dist.barrier()
    else:
        dist.barrier()
        path = synth.ensure("c4_q8_0", args.model_dir)

    def allgather(b):
        out = [None] * world
        dist.all_gather_object(out, b)
        return out

    tm = TPDeviceModel(path, be, rank, world, allgather, ctx=C4_PROMPT + C4_GEN + 64)
    try:
        lib, impl = be.lib, be.impl
        ids = np.random.default_rng(1).integers(0, VOCAB, C4_PROMPT).astype(np.int32)
        stream = torch.cuda.ExternalStream(be.stream())
        ms = None
        for _ in range(2):
            if lib.hyc_decode_begin(impl, ids.ctypes.data, C4_PROMPT, 0, C4_GEN, None, 0, tm.vocab_out) != 0:
                raise RuntimeError("decode_begin: " + be.error())
            be.sync()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if lib.hyc_decode_steps(impl, C4_GEN - 1) != 0:
                raise RuntimeError("decode_steps: " + be.error())
            e1.record(stream)
            torch.cuda.synchronize()
            be.sync()
            ms = max_over_ranks(e0.elapsed_time(e1))
        out_ids = np.zeros(C4_GEN, dtype=np.int32)
        n = lib.hyc_decode_read(impl, out_ids.ctypes.data, C4_GEN)
        if n != C4_GEN:
            raise RuntimeError("decode_read: " + be.error())
        dist.barrier()  # every rank done with its peers' memory before any unmaps
    finally:
        tm.close()
    # the NCCL reference point: an all-reduce of 2048 fp32 (CUDA events, 200 iterations after warm-up)
    x = torch.zeros(2048, dtype=torch.float32, device="cuda")
    for _ in range(20):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(200):
        dist.all_reduce(x)
    b.record()
    torch.cuda.synchronize()
    nccl_us = max_over_ranks(a.elapsed_time(b) / 200 * 1e3)
    step_ms = ms / (C4_GEN - 1)
    per_rank_bytes = (C4_LAYER_BYTES + C4_HEAD_BYTES) / world + L * 2 * (C4_PROMPT + (C4_GEN - 1) / 2) * KVD * 2 / min(world, 4)
    return {"value": round((C4_GEN - 1) / (ms / 1e3), 1), "unit": "tok/s", "ms_per_token": round(step_ms, 4),
            "tp": world, "exchanges_per_token": 2 * L + 1, "nccl_allreduce_8kb_us": round(nccl_us, 2),
            "workload": "c4_q8_0 tensor-parallel over the GPUs: bs1 greedy decode after a 4096-token seeded prompt, "
                        "positions 4096..4159; per-token latency = max over ranks (CUDA events)",
            "roofline_step": {"bytes_per_rank_per_step": int(per_rank_bytes),
                              "achieved_gbs_per_rank": round(per_rank_bytes / step_ms / 1e6, 1)},
            "ids_head": out_ids[:8].tolist()}


def quant_gemv_entry(kernels, peak):
    """The quant-GEMV HBM figure: the STQ1_0 panel gate|up GEMV at one token
    (two 6144 x 2048 panels, the reference kernel benchmark's shape, in one
    launch), bytes as streamed / CUDA-event time per launch, cycling over the
    32 layers' weights (more than L2 holds)."""
    k = kernels.get("gate_up_gemv_panel")
    if not k:
        return None
    return {"kernel": "gate_up_gemv_panel (gemv_panel_dec, STQ1_0 panel 2 x 6144 x 2048, nt 1)",
            "gbs": k["gbs"], "frac": round(k["gbs"] / peak, 4), "bytes_per_launch": k["bytes_per_launch"],
            "ms_per_launch": k["ms_per_launch"]}


def c0_config(world: int) -> dict:
    """The `config` of the headline line, the same in both arms."""
    return {"workload": "c0_stq: Hy-MT2-1.8B shape, 32 layers STQ1_0 (panel) + Q6_K tied head, reference bench GGUF; "
                        "bs1 greedy decode after a 48-token prompt, positions 48..111",
            "global_batch": world, "seq_len": PROMPT_LEN + GEN_LEN, "parallelism": f"dp{world} replicas",
            "l2": "weights 613 MB per step > 126 MB L2 (no flush needed)"}


def reference_bench_gguf(model_dir: str) -> str:
    """The config-0 model written by the reference's own tool
    (tools/make_bench_gguf.c, compiled into oracle/_ref by its Makefile);
    the synthetic writer's byte-identical copy where the tool is not built."""
    tool = os.path.join(ROOT, "oracle", "_ref", "make_bench_gguf")
    if not os.path.exists(tool):
        from hymt2_b200 import synth
        return synth.ensure("c0_stq", model_dir)
    os.makedirs(model_dir, exist_ok=True)
    path = os.path.join(model_dir, "ref_make_bench_gguf_L32.gguf")
    if not os.path.exists(path):
        subprocess.run([tool, path + ".tmp"], check=True, stdout=subprocess.DEVNULL)
        os.replace(path + ".tmp", path)
    return path


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    path = reference_bench_gguf(args.model_dir)
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
        "config": c0_config(world),
        "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"reference CPU ({ref.isa()}, {threads} threads), {steps} decode steps after a "
                                   f"cached 48-token prompt"},
        "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    args = parse()
    rank, local, world = dist_env()
    if args.profile_pass:
        profile_pass(args)
        return
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
    # GGUF -> device: every weight through the pinned staging ring, STQ1_0 panels and the Q6_K head relaid out
    # on the device from the file's own bytes, then fused_prepare (the file is in the page cache: just written)
    t_load = time.perf_counter()
    dm = DeviceModel(path, be, ctx=1024)
    be.sync()
    load_s = time.perf_counter() - t_load
    load = {"s": round(load_s, 3), "file_bytes": os.path.getsize(path),
            "gbs": round(os.path.getsize(path) / load_s / 1e9, 2),
            "path": "mmap'd GGUF bytes through two 16 MB pinned staging slots (host copy of one chunk overlapping "
                    "the DMA of the previous), device-side repack to panels / Q6_K planes; includes fused_prepare"}
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

    max_over_ranks = max_over_ranks_fn(dist, "cuda")

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

    # ---- end to end with the host in the loop, as the reference's loop runs (src/model.c:943-954): every
    # step the host's token goes in from pinned memory, one decode step runs, the new token comes back, and the
    # host waits for it, reads it and checks it against the stop ids before it issues the next step
    host = lib.hyc_host_alloc(4 * 4)
    hp = ctypes.cast(host, ctypes.POINTER(ctypes.c_int))
    stop_ids = {-1}  # no id stops the benchmark stream; the membership test is the host loop's own work

    def host_loop(n):
        s = 0
        while s < n:
            check(lib.hyc_decode_rewind(impl, PROMPT_LEN, tok0), "rewind")
            for _ in range(min(GEN_LEN, n - s)):
                check(lib.hyc_decode_steps_host(impl, 1, host), "steps_host")
                check(lib.hyc_sync(impl), "sync")
                if hp[1] in stop_ids:
                    break
                s += 1

    host_loop(max(3, args.warmup))
    barrier()
    t0 = time.perf_counter()
    host_loop(args.steps)
    e2e_launch_s = max_over_ranks(time.perf_counter() - t0)

    # ---- the same host loop without a launch per token (hyc_decode_resident): one persistent launch per 64
    # steps; every step the host waits for the step's token in mapped pinned memory, reads it, checks the stop
    # ids and releases the next step with it as that step's input
    def resident_loop(n):
        s = 0
        t = ctypes.c_int()
        while s < n:
            m = min(GEN_LEN, n - s)
            check(lib.hyc_decode_rewind(impl, PROMPT_LEN, tok0), "rewind")
            lib.hyc_resident_go(host, 0, tok0)
            check(lib.hyc_decode_resident(impl, m, host, 0), "resident")
            for i in range(m):
                rc = lib.hyc_resident_wait(host, i, ctypes.byref(t), 5_000_000_000)
                if rc != 0:
                    lib.hyc_sync(impl)  # reports (and clears) the kernel's host-timeout word
                    raise RuntimeError(f"hyc_resident_wait returned {rc} at step {i}: {be.error()}")
                s += 1
                if t.value in stop_ids:
                    lib.hyc_resident_go(host, -1, 0)
                    break
                if i + 1 < m:
                    lib.hyc_resident_go(host, i + 1, t.value)
            check(lib.hyc_sync(impl), "sync")

    # under a profiler that serialises launches (ncu) the host cannot answer while the launch call blocks: the
    # kernel's bounded wait ends the loop, and e2e falls back to the launch-per-step loop
    e2e_s, e2e_how, e2e_note = e2e_launch_s, "launch", None
    if persistent:
        try:
            resident_loop(max(3, args.warmup))
            ok = 1
        except RuntimeError as ex:
            ok, e2e_note = 0, f"resident loop unavailable here ({ex}); e2e is the launch-per-step loop"
        if world > 1:
            flag = torch.tensor([ok], device="cuda")
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            ok = int(flag.item())
        barrier()
        if ok:
            t0 = time.perf_counter()
            resident_loop(args.steps)
            e2e_s, e2e_how = max_over_ranks(time.perf_counter() - t0), "resident"
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
    # per-layer kernels, each over all 32 layers' weights in turn (more bytes than L2 holds); the four
    # layer GEMVs always (the quant-GEMV HBM figure), the head and attention with --graph-breakdown or
    # when the step runs as a graph
    for op, (name, per_step, nbytes) in OPS.items():
        if op in (0, 5) and not (args.graph_breakdown or not persistent):
            continue
        iters = 20 if op == 0 else 128
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
    # DRAM bytes per step of one ncu capture of this kernel, scaled to a launch; only from a capture of the
    # same kernel sources (the file records their hash)
    traffic, traffic_note = None, "no capture of the current kernel sources"
    tfile = os.path.join(ROOT, "profiles", "dram_traffic_c0_stq.json")
    if os.path.exists(tfile):
        with open(tfile) as f:
            tj = json.load(f)
        ent = tj.get(dom)
        if ent and tj.get("source_sha16") == kernel_source_hash():
            traffic = int(ent["dram_bytes_per_step"] * dk.get("steps_per_launch", 1))
            traffic_note = f"ncu capture of {ent.get('kernel', dom)} ({tj.get('command', '')})"
        elif ent:
            traffic_note = "the committed capture is of other kernel sources: not used"

    # ---- config 3: continuous-batching serving on every GPU (bs256/GPU)
    serving = None
    if args.serve_requests > 0:
        stops, stops_kind = int8_peak(torch)
        serving = bench_serving(dm, stream, torch, rank, world, args.serve_requests, max_over_ranks, barrier,
                                stops, stops_kind)

    if rank == 0:
        step_ms = ms / args.steps
        value = world * args.steps / (ms / 1e3)
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8+fp32", "data": "synthetic",
            "config": c0_config(world),
            "e2e": {"value": round(world * args.steps / e2e_s, 2), "unit": UNIT,
                    "h2d_bytes_per_step": 8 if e2e_how == "resident" else 4,
                    "d2h_bytes_per_step": 8 if e2e_how == "resident" else 4,
                    "path": ("host loop through the C ABI, every step: hyc_resident_wait (the step's token and done "
                             "word from mapped pinned memory), the host checks the stop ids, hyc_resident_go (the "
                             "next step's go word and input token to mapped pinned memory); one persistent launch "
                             "(hyc_decode_resident) per 64 steps; wall clock, max over ranks")
                    if e2e_how == "resident" else
                            (f"host loop through the C ABI: hyc_decode_steps_host(1) (token in from pinned host, one "
                             f"decode step ({path_name}), token out), hyc_sync, the host reads the token and checks "
                             f"the stop ids; wall clock, max over ranks"),
                    "launch_per_step_value": round(world * args.steps / e2e_launch_s, 2),
                    **({"note": e2e_note} if e2e_note else {})},
            "decode_path": path_name,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": dk["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": round(dk["gbs"] / peak, 4), "traffic": traffic, "traffic_note": traffic_note,
                         "peak_kind": peak_kind,
                         "bytes_per_launch": dk["bytes_per_launch"], "ms_per_launch": dk["ms_per_launch"]},
            "roofline_step": {"bytes_per_step": STEP_BYTES, "achieved_gbs": round(STEP_BYTES / step_ms / 1e6, 1),
                              "frac": round(STEP_BYTES / step_ms / 1e6 / peak, 4)},
            "kernels": kernels,
            "quant_gemv": quant_gemv_entry(kernels, peak),
            "gpu_launches": int(launches),
            "load_c0": load,
            "clocks": clk,
            "device": be.info,
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                out["cpu_baseline"] = cpu_baseline(path, args.cpu_tokens)
            except Exception as e:  # noqa: BLE001 - report, do not fail the GPU number
                out["cpu_baseline"] = {"unavailable": str(e)}
        if serving:
            serving["cpu_baseline_note"] = ("the reference serves one request at a time: its rate is the bs1 "
                                            "cpu_baseline above")
            out["serving"] = serving
    dm.close()
    if world > 1 and not args.no_extra:
        try:
            c4tp = bench_c4_tp(args, be, torch, dist, rank, world, max_over_ranks)
        except Exception as e:  # noqa: BLE001 - report, do not lose the headline
            c4tp = {"unavailable": str(e)}
        if rank == 0:
            out["decode_c4_tp"] = c4tp
    if rank == 0 and world == 1 and not args.no_extra:
        tops, tops_kind = int8_peak(torch)
        for key, fn in (("prefill_c2", lambda: bench_prefill(args, be, torch, tops, tops_kind)),
                        ("decode_c0_native", lambda: bench_c0_native(args, be, torch, peak, path)),
                        ("decode_c1", lambda: bench_c1(args, be, torch, peak)),
                        ("decode_c4", lambda: bench_c4(args, be, torch, peak))):
            try:
                out[key] = fn()
            except Exception as e:  # noqa: BLE001 - report, do not lose the headline
                out[key] = {"unavailable": str(e)}
    if rank == 0:
        print(json.dumps(out))
    be.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
