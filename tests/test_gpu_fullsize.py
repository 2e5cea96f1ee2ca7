"""Full-size parity of the benchmark configurations 1-4 (needs a B200; slow).

The 32-layer Hy-MT2-1.8B-shaped models of the bench, on their own workloads,
against the reference's CPU library compiled from its sources (the reference
itself, oracle/_ref/libhymt2_ref.so, HYMT2_DEVICE=cpu):

  c1  Q2_0C, 512-token prompt, 32 greedy tokens (the persistent kernel);
  c2  Q4_K_M, the 32 x 256-token prefill as one batch pass on the tensor
      cores: against 8-sequence passes, sequence 0 against the reference
      (its spread over 256 tokens), the other sequences' errors printed;
  c3  the config-0 model served with continuous batching: 64 requests of the
      serving workload, 16 tokens each, against per-request greedy;
  c4  Q8_0, bs1 decode: a 128-token prompt and 8 steps (the reference's
      scalar Q8_0 prefill needs ~0.3 s per token here, so KV 4096 is out of
      the test budget; positions past 4096 are checked on the tiny Q8_0 model
      by test_gpu_model.py::test_long_context_decode_matches_oracle).

Logit tolerance, the reference's own rule (tests/test_model.py:353-364):
max(1e-5, 3 x spread), spread = max|l64 - l32| / max|l64| of the C
restatement in fp64 and fp32 on the same prompt.  The spread grows with the
prompt (config 2: 1e-5 after 48 tokens, 5e-3 after 256), so c2 and c4 measure
it on their whole prompts (c2 on its sequence 0); c1's 512-token prompt would take the fp64 oracle
many minutes, so c1 uses the first 48 tokens, whose spread is already 6 %
(the synthetic Q2_0C model is badly conditioned at 32 layers) and can only
understate the full one.  Where the tolerance is at most 1e-3 the north
star's 1e-3 bound applies on its own.  Greedy ids must agree up to the first
near-tie step (top-2 logits within 2 x tol of the largest).  Every test
prints the measured relative error.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
VOCAB = 120818


def _rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-12))


def _near_tie(lg, tol):
    top = np.sort(lg)[-2:]
    return (top[1] - top[0]) <= 2 * tol * np.abs(lg).max()


def _first_div(a, b):
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)


def _spread_tol(oracle, path, ids):
    import oracle as O
    om = O.OracleModel(oracle, path, ctx=len(ids) + 8)
    try:
        _, spread, tol = om.logits_spread(ids)
    finally:
        om.close()
    return spread, tol


def _ref_model(reference, path, ctx):
    os.environ["HYMT2_DEVICE"] = "cpu"
    cores = int(reference.lib.refh_physical_cores())
    return reference.load(path, threads=cores, ctx=ctx)


def test_c1_q2c_decode_full_size(backend, oracle, reference, synth, model_dir):
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c1_q2c", model_dir)
    ids = np.random.default_rng(1).integers(0, VOCAB, 512).tolist()
    dm = DeviceModel(path, backend, ctx=1024)
    try:
        got = dm.generate(ids, 32)
        dm.forward(ids[:256], 0, want_logits=False)  # the vtable's chunks hold 256 tokens at most
        _, lg_d = dm.forward(ids[256:], 256)
    finally:
        dm.close()
    rm = _ref_model(reference, path, 1024)
    try:
        want, steps, *_ = rm.greedy(ids, 32, step_logits=True)
    finally:
        rm.close()
    spread, tol = _spread_tol(oracle, path, ids[:48])
    rel = _rel(lg_d, steps[0])
    print(f"c1 full size: logits rel {rel:.3e}, spread {spread:.3e}, tol {tol:.3e}, ids {got[:8]}")
    assert rel <= tol and (tol > 1e-3 or rel <= 1e-3), (rel, tol)
    d = _first_div(got, want)
    assert d is None or _near_tie(steps[d], tol), (got, want)


def test_c2_q4km_prefill_pass_full_size(backend, oracle, reference, synth, model_dir):
    """The 32 x 256-token pass: within 1e-5 of the same sequences passed 8
    at a time, with the same greedy ids (the reference's batch-vs-step check,
    tests/test_model.py:369-399; the 32 last-token rows go through the head
    as one tensor-core GEMM, the 8-row passes through the dp4a GEMV, which
    add the block products in another float order), and
    sequence 0's last-token logits within the reference's rule, its spread
    measured over all 256 tokens.  The synthetic Q4_K_M model is chaotic on
    some prompts at 32 layers (on sequence 13 the reference library and its C
    restatement, both fp32, differ by 9 % and the fp64 spread is 22 %), so the
    errors of all 32 sequences are printed, not asserted."""
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c2_q4km", model_dir)
    seqs, length = 32, 256
    rng = np.random.default_rng(2)
    toks = rng.integers(0, VOCAB, seqs * length)
    dm = DeviceModel(path, backend, ctx=length)
    try:
        dm.batch_prepare(slots=seqs, slot_ctx=length, max_tokens=seqs * length, max_out=seqs)
        rows = np.arange(seqs) * length + length - 1
        gids, lg = dm.batch_forward(toks, np.repeat(np.arange(seqs), length), np.tile(np.arange(length), seqs), rows,
                                    want_logits=True)
        lg8 = np.zeros_like(lg)
        for s0 in range(0, seqs, 8):
            sl = np.arange(s0, s0 + 8)
            t = np.concatenate([toks[s * length:(s + 1) * length] for s in sl])
            _, l8 = dm.batch_forward(t, np.repeat(sl, length), np.tile(np.arange(length), 8),
                                     np.arange(8) * length + length - 1, want_logits=True)
            lg8[s0:s0 + 8] = l8
    finally:
        dm.close()
    batch_rel = max(_rel(lg[i], lg8[i]) for i in range(seqs))
    assert batch_rel <= 1e-5, batch_rel
    assert np.array_equal(lg.argmax(1), lg8.argmax(1))
    rm = _ref_model(reference, path, length + 8)
    errs = []
    try:
        for s in range(seqs):
            rm.reset_cache()
            want, steps, *_ = rm.greedy(toks[s * length:(s + 1) * length].tolist(), 1, step_logits=True)
            errs.append((_rel(lg[s][:steps.shape[1]], steps[0]), gids[s] == want[0]))
            if s == 0:
                l0, w0 = steps[0], want[0]
    finally:
        rm.close()
    spread, tol = _spread_tol(oracle, path, toks[:length].tolist())
    rel = errs[0][0]
    print(f"c2 full size: 32-pass vs 8-passes rel {batch_rel:.3e}; "
          f"sequence 0 logits rel {rel:.3e}, spread {spread:.3e}, tol {tol:.3e}; all 32: "
          f"median {np.median([e for e, _ in errs]):.3e}, argmax equal {sum(a for _, a in errs)}/32")
    assert rel <= tol and (tol > 1e-3 or rel <= 1e-3), (rel, tol)
    assert gids[0] == w0 or _near_tie(l0, tol), (gids[0], w0)


def test_c3_serving_full_size(backend, oracle, reference, synth, model_dir):
    sys.path.insert(0, ROOT)
    import bench
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c0_stq", model_dir)
    reqs = bench.serve_requests(64)
    max_new = 16
    dm = DeviceModel(path, backend, ctx=256)
    try:
        dm.batch_prepare(slots=bench.SERVE_SLOTS, slot_ctx=128 + max_new, max_tokens=bench.SERVE_MAX_TOKENS,
                         max_out=bench.SERVE_SLOTS)
        out, _ = dm.serve(reqs, max_new, bench.SERVE_STEP_TOKENS)
    finally:
        dm.close()
    rm = _ref_model(reference, path, 256)
    spread, tol = _spread_tol(oracle, path, (reqs[0] + reqs[1])[:48])
    bad = []
    try:
        for i, r in enumerate(reqs):
            rm.reset_cache()
            want, steps, *_ = rm.greedy(r, max_new, step_logits=True)
            got = out[i][:max_new].tolist()
            d = _first_div(got, want)
            if d is not None and not _near_tie(steps[d], tol):
                bad.append((i, d, got, want))
    finally:
        rm.close()
    print(f"c3 full size: 64 served requests, {len(bad)} streams part from the reference before a near tie "
          f"(tol {tol:.3e})")
    assert not bad, bad[:3]


def test_c4_q8_0_decode_full_size(backend, oracle, reference, synth, model_dir):
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c4_q8_0", model_dir)
    ids = np.random.default_rng(1).integers(0, VOCAB, 128).tolist()
    dm = DeviceModel(path, backend, ctx=256)
    try:
        got = dm.generate(ids, 8)
        _, lg_d = dm.forward(ids, 0)
    finally:
        dm.close()
    rm = _ref_model(reference, path, 256)
    try:
        want, steps, *_ = rm.greedy(ids, 8, step_logits=True)
    finally:
        rm.close()
    spread, tol = _spread_tol(oracle, path, ids)
    rel = _rel(lg_d, steps[0])
    print(f"c4 full size: logits rel {rel:.3e}, spread {spread:.3e}, tol {tol:.3e}, ids {got}")
    assert rel <= tol and (tol > 1e-3 or rel <= 1e-3), (rel, tol)
    d = _first_div(got, want)
    assert d is None or _near_tie(steps[d], tol), (got, want)


def test_c0_reference_loop_through_backend(backend, oracle, synth, model_dir):
    """The drop-in at full size: the reference's own model.c (oracle/_ref/
    libhymt2_dropin.so: its host C from its sources, linked with this backend
    in place of src/cuda.c) runs config 0 with HYMT2_DEVICE=cuda through the
    vtable (upload of host-built panels, fused_prepare, fused_forward per
    token with host h and logits, the host's own argmax, src/model.c:904-954).
    Its ids must be this backend's own on-device decode ids up to a near tie;
    the rate of that loop is printed (the path a reference user gets without
    the additive hyc_decode_* entry points)."""
    import oracle as O
    from hymt2_b200.device import DeviceModel
    if not os.path.exists(O.DROPIN_LIB):
        pytest.skip("drop-in not built")
    path = synth.ensure("c0_stq", model_dir)
    ids = np.random.default_rng(1).integers(0, VOCAB, 48).tolist()
    n = 33
    dm = DeviceModel(path, backend, ctx=256)
    try:
        own = dm.generate(ids, n)
    finally:
        dm.close()
    os.environ["HYMT2_DEVICE"] = "cuda"
    try:
        ref = O.Reference(O.DROPIN_LIB).load(path, threads=4, ctx=256)
        try:
            assert ref.uses_device(), ref.info()
            got, steps, *_ = ref.greedy(ids, n, step_logits=True)
            ref.reset_cache()
            _, _, pre_ms, dec_ms, _ = ref.greedy(ids, n)  # timed without the harness's logits copies
        finally:
            ref.close()
    finally:
        os.environ["HYMT2_DEVICE"] = "cpu"
    spread, tol = _spread_tol(oracle, path, ids)
    print(f"c0 reference loop through the backend: prompt {pre_ms:.1f} ms, {(n - 1) / (dec_ms / 1e3):.1f} decode "
          f"tok/s (fused_forward per token, host logits and argmax); ids {got[:8]}")
    d = _first_div(got, own)
    assert d is None or _near_tie(steps[d], tol), (got, own)
