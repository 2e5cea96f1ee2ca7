"""Parity of the fused pieces of a decode layer (needs a B200), through the C ABI.

  - GEMV activation prologues: RMSNorm*w, SiLU(x)*up and plain input, each
    followed by the Q8_K quantiser (or fp32 for Q8_0/F16/F32) and the GEMV,
    against the oracle's host sequence (reference src/model.c:824-881);
    store and residual-add epilogues;
  - attention with its rope -> q/k RMSNorm -> bf16 KV-store prologue, decode
    (split-KV, any position) and prefill forms, against the oracle
    (reference src/model.c:768-795, 836-848): output within 1e-5 relative and
    KV cache rows bit-identical except for rare 1-ulp bf16 rounding flips.
"""
import ctypes

import numpy as np
import pytest

from conftest import rand_act, rand_blocks
from hymt2_b200 import _paths, abi

pytestmark = pytest.mark.gpu

TYPES = {"STQ1_0": 43, "Q2_0C": 40, "Q4_K": 12, "Q6_K": 14, "Q8_0": 8, "F16": 1}


def _rope(ctx, hd, base=10000.0, alpha=3.0):
    lib = abi.bind(ctypes.CDLL(_paths.BACKEND_LIB))
    cos = np.zeros(ctx * (hd // 2), dtype=np.float32)
    sin = np.zeros_like(cos)
    assert lib.hyc_rope_tables(base, alpha, hd, hd, ctx, cos.ctypes.data, sin.ctypes.data) == 0
    return cos, sin


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("act", [1, 2, 3])
@pytest.mark.parametrize("k", [512, 2048, 6144])
@pytest.mark.parametrize("nt", [1, 3])
def test_gemv_prologue(backend, oracle, name, act, k, nt):
    from hymt2_b200.device import weight_from_bytes
    gt = TYPES[name]
    rows = 96
    rng = np.random.default_rng(k + act * 7 + nt)
    raw = rand_blocks(rng, gt, rows, k)
    h = backend.upload(weight_from_bytes(gt, raw, rows, k))
    try:
        x = rand_act(rng, nt, k) * 3.0
        x2 = rand_act(rng, nt, k)
        nw = (1.0 + 0.2 * rng.standard_normal(k)).astype(np.float32)
        got = backend.gemv_test(h, act, x, rows, x2=x2 if act == 3 else None, norm_w=nw if act == 2 else None)
        w = oracle.weight(gt, raw, rows, k, panel=True)
        want = oracle.prologue_matmul(w, act, x, x2 if act == 3 else None, nw if act == 2 else None)
        err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-6)
        assert err < 2e-4, err
        base = rng.standard_normal((nt, rows)).astype(np.float32)
        got2 = backend.gemv_test(h, act, x, rows, x2=x2 if act == 3 else None, norm_w=nw if act == 2 else None,
                                 add_to=base)
        assert np.abs(got2 - (base + got)).max() <= 1e-5 * max(1.0, np.abs(got2).max())
    finally:
        backend.release(h)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("heads,kvh", [(4, 4), (4, 2), (16, 4), (16, 2)])
@pytest.mark.parametrize("pos0,nt", [(0, 1), (7, 1), (111, 1), (300, 1), (600, 1), (0, 5), (40, 17)])
def test_attention(backend, oracle, hd, heads, kvh, pos0, nt):
    _check_attention(backend, oracle, hd, heads, kvh, 1024, pos0, nt)


# Single-token decode past the persistent kernel's 64 units.  The kernel
# pair is fixed per context by the last position: with 4 KV heads up to
# ctx 4736 (37 chunks of 128 keys, 148 units) the per-layer chunk kernel,
# past it the split-KV kernel (ctx 8192).  Covered: chunk lengths 64, 96 and
# 128, merges of up to 141 chunks (kvh 1), a chunk holding only the current
# key (pos 4096), exactly 148 units (pos 4700).  Config 4's attention is
# (128, 16, 4) at KV 4096 in a 4224-row cache.
@pytest.mark.parametrize("hd,heads,kvh,ctx,pos0", [(128, 16, 4, 4736, 2100), (128, 16, 4, 4736, 4096),
                                                  (128, 16, 4, 4736, 4700), (128, 16, 4, 8192, 6000),
                                                  (64, 4, 2, 9472, 5000), (64, 8, 1, 10240, 9000)])
def test_attention_long_context(backend, oracle, hd, heads, kvh, ctx, pos0):
    _check_attention(backend, oracle, hd, heads, kvh, ctx, pos0, 1)


def _check_attention(backend, oracle, hd, heads, kvh, ctx, pos0, nt):
    rng = np.random.default_rng(hd + heads * 3 + kvh + pos0 + nt)
    qd, kvd = heads * hd, kvh * hd
    cos, sin = _rope(ctx, hd)
    kc = np.zeros((ctx, kvd), dtype=np.uint16)
    vc = np.zeros((ctx, kvd), dtype=np.uint16)
    # fill earlier positions with plausible bf16 keys / values
    if pos0:
        kc[:pos0] = (rng.standard_normal((pos0, kvd)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
        vc[:pos0] = (rng.standard_normal((pos0, kvd)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    qkv = (rng.standard_normal((nt, qd + 2 * kvd)) * 2.0).astype(np.float32)
    qn = (1.0 + 0.2 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1.0 + 0.2 * rng.standard_normal(hd)).astype(np.float32)
    kc_d, vc_d = kc.copy(), vc.copy()
    ao = backend.attention_test(heads, kvh, hd, ctx, qkv, pos0, kc_d, vc_d, qn, kn, cos, sin)
    kc_o, vc_o = kc.copy(), vc.copy()
    want = oracle.attention(heads, kvh, hd, qkv.copy(), pos0, kc_o, vc_o, qn, kn, cos, sin)
    rows = slice(pos0, pos0 + nt)
    assert np.array_equal(vc_d[rows], vc_o[rows])
    assert (kc_d[rows] != kc_o[rows]).mean() < 0.02
    assert np.array_equal(kc_d[:pos0], kc[:pos0]) and np.array_equal(kc_d[pos0 + nt:], kc[pos0 + nt:])
    err = np.abs(ao - want).max() / max(np.abs(want).max(), 1e-6)
    assert err < 1e-4, err
