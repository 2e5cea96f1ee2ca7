"""Pin the C restatement (oracle/hy_oracle.c) to the reference itself.

The reference library is compiled from the reference's own sources into
oracle/_ref (oracle/Makefile).  Every hot-path function the oracle restates is
compared here on seeded inputs with the edge cases the reference's tests use:
  - Q8_K quantiser: bit-identical 576-byte blocks (zeros, ties, outliers,
    exact .5 products, NaN/inf);
  - panel repack (STQ1_0, Q2_0C): identical bytes;
  - dequant_row for every format: identical floats (scalar in both);
  - matmul for every format: within 1e-5 of sum|term| (the reference's SIMD
    kernels sum in another order; reference tests/test_kernels.c:48-72);
  - exact per-block integers: checked independently against numpy integer
    arithmetic on dequantised codes;
  - model forward / greedy on tiny synthetic GGUFs: identical greedy ids and
    logits within the reference's own fp32-vs-fp64 spread rule.
"""
import os

import numpy as np
import pytest

from conftest import rand_act, rand_blocks

TYPES = {"STQ1_0": 43, "Q2_0C": 40, "Q4_K": 12, "Q6_K": 14, "Q8_0": 8, "F16": 1, "F32": 0}


def _edge_acts(rng, k):
    x = rand_act(rng, 6, k)
    x[1, :] = 0.0                       # all-zero blocks
    x[2, :256] = 1.0                    # every element ties for max |x|
    x[2, 256:512] = -1.0
    x[3, 5] = -7.0                      # signed max
    x[3, 9] = 7.0                       # tie in |x| after it: first index wins
    x[4, :] = np.arange(k, dtype=np.float32) * 0.5 - 100.0   # many exact halves after scaling
    x[5, 256:] = rng.standard_normal(k - 256) * 1e-30         # denormal-range block
    return x


def test_quantize_bit_identical(oracle, reference):
    rng = np.random.default_rng(5)
    for k in (256, 1536, 2048, 6144):
        x = _edge_acts(rng, k)
        a = oracle.quantize(x)
        b = reference.quantize(x)
        assert a.tobytes() == b.tobytes(), f"k={k}"


def test_quantize_nonfinite(oracle, reference):
    x = np.ones((1, 512), dtype=np.float32)
    x[0, 3] = np.nan
    x[0, 300] = np.inf
    x[0, 301] = -np.inf
    a, b = oracle.quantize(x), reference.quantize(x)
    assert a.tobytes() == b.tobytes()


@pytest.mark.parametrize("name", ["STQ1_0", "Q2_0C"])
def test_panel_repack_identical(oracle, reference, name):
    rng = np.random.default_rng(1)
    gt, rows, k = TYPES[name], 37, 1536
    raw = rand_blocks(rng, gt, rows, k)
    pk0, ps0 = oracle.panel(gt, raw, rows, k)
    pk1, ps1 = reference.panel(gt, raw, rows, k)
    assert pk0.tobytes() == pk1.tobytes()
    assert ps0.tobytes() == ps1.tobytes()


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_identical(oracle, reference, name):
    rng = np.random.default_rng(2)
    gt, rows, k = TYPES[name], 5, 1536
    raw = rand_blocks(rng, gt, rows, k)
    w = oracle.weight(gt, raw, rows, k, panel=False)
    for r in range(rows):
        a = oracle.dequant_row(w, r)
        b = reference.dequant_row(gt, raw, k, r)
        assert a.tobytes() == b.tobytes(), f"{name} row {r}"


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("panel", [0, 1])
def test_matmul_close(oracle, reference, name, panel):
    if panel and TYPES[name] not in (40, 43):
        pytest.skip("panel form only exists for STQ1_0 / Q2_0C")
    rng = np.random.default_rng(3)
    gt, rows, k, nt = TYPES[name], 7, 1536, 5
    raw = rand_blocks(rng, gt, rows, k)
    x = rand_act(rng, nt, k)
    w = oracle.weight(gt, raw, rows, k, panel=bool(panel))
    a = oracle.matmul(w, x)
    b = reference.matmul(gt, raw, rows, k, x, panel)
    # sum |term| from dequantised weights and (quantised) activations
    wd = np.stack([oracle.dequant_row(w, r) for r in range(rows)]).astype(np.float64)
    if gt in (0, 1, 8):
        xe = x.astype(np.float64)
    else:
        q = oracle.quantize(x)
        xe = (q["qs"].astype(np.float64) * q["d"][..., None]).reshape(nt, k)
    mag = np.abs(xe) @ np.abs(wd).T
    err = np.abs(a - b) / (mag + 1e-6)
    assert err.max() < 1e-5, f"{name} panel={panel}: {err.max():.3g}"
    want = xe @ wd.T
    assert (np.abs(a - want) / (mag + 1e-6)).max() < 1e-5


def _codes_int(oracle, gt, raw, rows, k, xq):
    """Independent exact block integers from dequantised integer codes."""
    nb = k // 256
    w = oracle.weight(gt, raw, rows, k, panel=False)
    qs = xq["qs"].astype(np.int64)          # [nt][nb][256]
    out = []
    for r in range(rows):
        deq = oracle.dequant_row(w, r).reshape(nb, 256).astype(np.float64)
        if gt == 43:
            d = np.array([np.frombuffer(raw[(r * nb + b) * 42 + 40:(r * nb + b) * 42 + 42].tobytes(), np.float16)[0]
                          for b in range(nb)], dtype=np.float64)
            codes = np.rint(deq / d[:, None]).astype(np.int64)          # -1, 0, +1
        else:  # Q2_0C: (2c-3)
            d = np.array([np.frombuffer(raw[(r * nb // 2 + b // 2) * 130:(r * nb // 2 + b // 2) * 130 + 2].tobytes(),
                                        np.float16)[0] for b in range(nb)], dtype=np.float64)
            codes = np.rint(deq / d[:, None]).astype(np.int64)
        out.append((codes[None] * qs).sum(-1))  # [nt][nb]
    return np.stack(out, 1)


@pytest.mark.parametrize("gt", [43, 40])
def test_block_ints_independent(oracle, gt):
    rng = np.random.default_rng(4)
    rows, k, nt = 9, 2048, 3
    raw = rand_blocks(rng, gt, rows, k)
    x = rand_act(rng, nt, k)
    xq = oracle.quantize(x)
    w = oracle.weight(gt, raw, rows, k, panel=True)
    got = oracle.block_ints(w, xq, nt)
    want = _codes_int(oracle, gt, raw, rows, k, xq)
    assert np.array_equal(got, want)


MODEL_CASES = ["t_stq", "t_q2c", "t_q4km", "t_q8_0", "t_f16head"]


@pytest.mark.parametrize("cfg", MODEL_CASES)
def test_model_greedy_matches_reference(oracle, reference, synth, model_dir, cfg, monkeypatch):
    """Greedy ids and logits of the restated forward vs the reference CPU path."""
    import oracle as O
    import np_forward
    monkeypatch.setenv("HYMT2_DEVICE", "cpu")
    path = synth.ensure(cfg, model_dir)
    rng = np.random.default_rng(1)
    om = O.OracleModel(oracle, path, ctx=256)
    ids = rng.integers(0, om.vocab, 20).tolist()
    rm = reference.load(path, threads=2, ctx=256)
    r_ids, r_lg, *_ = rm.greedy(ids, 6, step_logits=True)
    o_ids, o_lg = om.greedy(ids, 6, chunk=rm.batch, step_logits=True)
    r64, spread, tol = np_forward.spread_tolerance(oracle, path, ids)
    rel = np.abs(o_lg[0] - r_lg[0]).max() / np.abs(r_lg[0]).max()
    rel64 = np.abs(o_lg[0] - r64).max() / np.abs(r64).max()
    assert rel <= tol and rel64 <= tol, (cfg, rel, rel64, spread)
    assert o_ids == r_ids, (cfg, o_ids, r_ids)
    # KV cache of layer 0 is bit-identical after the same steps
    n = len(ids) + 5
    k0, v0 = om.kv(0, n)
    k1, v1 = rm.kv(0, n)
    assert (k0 != k1).mean() < 0.01 and (v0 != v1).mean() < 0.01
    rm.close()
    om.close()
