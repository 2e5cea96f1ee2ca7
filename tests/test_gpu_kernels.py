"""Kernel-level parity of the CUDA backend, through its C ABI (needs a B200).

Bar (from the reference's own tests):
  - Q8_K quantiser: bit-identical blocks to the restated host quantiser;
  - per-block int32 accumulators of every Q8_K-format GEMV: bit-identical;
  - dequantised rows: bit-identical;
  - GEMV outputs vs the reference CPU library: max |gpu-cpu| / max |cpu| < 2e-4
    (reference tests/test_metal.py:42 uses the same bound for its GPU path),
    and within 1e-5 of sum|term| against the restated oracle.
"""
import numpy as np
import pytest

from conftest import rand_act, rand_blocks

pytestmark = pytest.mark.gpu

Q8_TYPES = {"STQ1_0": 43, "Q2_0C": 40, "Q4_K": 12, "Q6_K": 14}
FP_TYPES = {"Q8_0": 8, "F16": 1, "F32": 0}


def _edge_acts(rng, nt, k):
    x = rand_act(rng, nt, k)
    if nt > 2:
        x[1, :256] = 0.0
        x[2, :256] = 1.0
        x[2, 256:] = np.arange(k - 256, dtype=np.float32) * 0.5 - 50.0
    return x


@pytest.mark.parametrize("k", [256, 2048, 6144])
def test_quantize_bit_exact(backend, oracle, k):
    rng = np.random.default_rng(11)
    x = _edge_acts(rng, 7, k)
    x[0, 7] = np.nan
    got = backend.quantize_q8k(x)
    want = oracle.quantize(x)
    assert got.tobytes() == want.tobytes()


def _upload(backend, oracle, gt, raw, rows, k, host_panel=True):
    from hymt2_b200.device import weight_from_bytes
    pk = ps = None
    if host_panel and gt in (40, 43):
        pk, ps = oracle.panel(gt, raw, rows, k)
    w = weight_from_bytes(gt, raw, rows, k, pk, ps)
    return backend.upload(w), (pk, ps)


@pytest.mark.parametrize("name", list(Q8_TYPES))
@pytest.mark.parametrize("rows,k", [(37, 1536), (64, 2048), (300, 6144), (5, 512)])
@pytest.mark.parametrize("nt", [1, 3, 16])
@pytest.mark.parametrize("host_panel", [True, False])
def test_block_ints_exact(backend, oracle, name, rows, k, nt, host_panel):
    gt = Q8_TYPES[name]
    if not host_panel and gt not in (40, 43):
        pytest.skip("device-built panels only apply to STQ1_0 / Q2_0C")
    if gt == 40 and k % 512:
        pytest.skip("Q2_0C needs k % 512 == 0")
    rng = np.random.default_rng(rows * 7 + k + nt)
    raw = rand_blocks(rng, gt, rows, k)
    h, keep = _upload(backend, oracle, gt, raw, rows, k, host_panel)
    try:
        x = _edge_acts(rng, nt, k)
        xq = oracle.quantize(x)
        w = oracle.weight(gt, raw, rows, k, panel=True)
        want = oracle.block_ints(w, xq, nt)
        got = backend.block_ints(h, xq, nt, rows, want.shape[2])
        assert np.array_equal(got, want), f"{(got != want).sum()} block integers differ"
    finally:
        backend.release(h)


@pytest.mark.parametrize("name", list(Q8_TYPES))
@pytest.mark.parametrize("rows,nt", [(37, 1), (64, 3), (130, 16)])
def test_vtable_matmul_vs_reference(backend, oracle, reference, name, rows, nt):
    """hy_device_ops.matmul with host Q8_K blocks, as hymt2_debug_device_matmul does
    (reference src/model.c:1077-1108; test template tests/test_metal.py)."""
    gt, k = Q8_TYPES[name], 1536
    rng = np.random.default_rng(rows + nt)
    raw = rand_blocks(rng, gt, rows, k)
    h, keep = _upload(backend, oracle, gt, raw, rows, k)
    try:
        x = rand_act(rng, nt, k)
        xq = oracle.quantize(x).reshape(-1)
        gpu = np.zeros((nt, rows), dtype=np.float32)
        assert backend.matmul([h], [gpu], xq, nt)
        cpu = reference.matmul(gt, raw, rows, k, x, 1)
        err = np.abs(gpu - cpu).max() / max(np.abs(cpu).max(), 1e-6)
        assert err < 2e-4, err
        w = oracle.weight(gt, raw, rows, k, panel=True)
        orc = oracle.matmul(w, x, oracle.quantize(x))
        wd = np.stack([oracle.dequant_row(w, r) for r in range(rows)]).astype(np.float64)
        q = oracle.quantize(x)
        xe = (q["qs"].astype(np.float64) * q["d"][..., None]).reshape(nt, k)
        mag = np.abs(xe) @ np.abs(wd).T
        assert (np.abs(gpu - orc) / (mag + 1e-6)).max() < 1e-5
    finally:
        backend.release(h)


@pytest.mark.parametrize("name", list(Q8_TYPES) + list(FP_TYPES))
@pytest.mark.parametrize("nt", [1, 4, 9])
def test_matmul_f32_vs_reference(backend, oracle, reference, name, nt):
    """fp32 activations in; Q8_K formats quantise on the device first (the
    same sequence as the host's matmul_rows), Q8_0/F16/F32 use them as is."""
    gt = {**Q8_TYPES, **FP_TYPES}[name]
    rows, k = 77, 2048
    rng = np.random.default_rng(nt * 3 + gt)
    raw = rand_blocks(rng, gt, rows, k)
    h, keep = _upload(backend, oracle, gt, raw, rows, k)
    try:
        x = rand_act(rng, nt, k)
        gpu = backend.matmul_f32(h, x, rows)
        cpu = reference.matmul(gt, raw, rows, k, x, 1 if gt in (40, 43) else 0)
        err = np.abs(gpu - cpu).max() / max(np.abs(cpu).max(), 1e-6)
        assert err < 2e-4, err
    finally:
        backend.release(h)


@pytest.mark.parametrize("name", list(Q8_TYPES) + list(FP_TYPES))
def test_dequant_rows_exact(backend, oracle, name):
    gt = {**Q8_TYPES, **FP_TYPES}[name]
    rows, k = 9, 2048
    rng = np.random.default_rng(gt)
    raw = rand_blocks(rng, gt, rows, k)
    h, keep = _upload(backend, oracle, gt, raw, rows, k)
    try:
        w = oracle.weight(gt, raw, rows, k, panel=False)
        for r in (0, 4, rows - 1):
            assert backend.dequant_row(h, r, k).tobytes() == oracle.dequant_row(w, r).tobytes(), r
    finally:
        backend.release(h)


def test_head_shape_q6k_large(backend, oracle, reference):
    """LM-head shape (K=2048, many rows) through the Q6_K GEMV."""
    gt, rows, k = 14, 4099, 2048
    rng = np.random.default_rng(99)
    raw = rand_blocks(rng, gt, rows, k)
    h, keep = _upload(backend, oracle, gt, raw, rows, k)
    try:
        x = rand_act(rng, 1, k)
        gpu = backend.matmul_f32(h, x, rows)
        cpu = reference.matmul(gt, raw, rows, k, x, 0)
        assert np.abs(gpu - cpu).max() / np.abs(cpu).max() < 2e-4
    finally:
        backend.release(h)
