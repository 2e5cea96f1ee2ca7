"""Native STQ1_0 device layout (needs a B200), through the C ABI.

The weight keeps the file's 42 bytes per 256 weights (hyc_set_stq_layout):
per row the qs slots, the sign bits and the f16 scales as three planes,
decoded in registers by byte permutes over the format's pattern table.  The
parity row is the reference's native dot, stq1_0_dot_scalar
(src/kernels.c:202-215): sum over groups of (code - 1) * q8, times d * y.d.

  - per-block int32 sums of the dp4a GEMV (nt 1, 3, 16) and of the tcgen05
    GEMM (nt 32 .. 8192), host-made Q8_K blocks: bit-identical to the
    oracle's native restatement;
  - dequantised rows: bit-identical;
  - the vtable matmul: bit-identical to the same weight uploaded as a panel
    (same block integers, same scale products in the same order), within
    2e-4 of the reference library;
  - a whole model with native layers: prompt logits bit-identical to the
    panel upload's, greedy ids equal to the oracle's and the panel graph's up
    to a near tie.
"""
import numpy as np
import pytest

from conftest import rand_act, rand_blocks

pytestmark = pytest.mark.gpu

GT = 43


def _upload(backend, raw, rows, k, native):
    from hymt2_b200.device import weight_from_bytes
    backend.set_stq_layout(native)
    try:
        return backend.upload(weight_from_bytes(GT, raw, rows, k))
    finally:
        backend.set_stq_layout(False)


def _acts(rng, nt, k):
    x = rand_act(rng, nt, k) * 3.0
    x[0, :256] = 0.0                                   # an all-zero block
    if nt > 2:
        x[1, :256] = 1.0                               # ties for the first maximum
        x[2, 256:512] = np.linspace(-5.0, 5.0, 256)    # exact halves on the grid
    return x


@pytest.mark.parametrize("rows,k", [(37, 1536), (64, 2048), (300, 6144), (5, 512), (129, 8192)])
@pytest.mark.parametrize("nt", [1, 3, 16])
def test_native_block_ints_exact(backend, oracle, rows, k, nt):
    rng = np.random.default_rng(rows + k + nt)
    raw = rand_blocks(rng, GT, rows, k)
    h = _upload(backend, raw, rows, k, True)
    try:
        xq = oracle.quantize(_acts(rng, nt, k))
        want = oracle.block_ints(oracle.weight(GT, raw, rows, k, panel=False), xq, nt)
        got = backend.block_ints(h, xq, nt, rows, want.shape[2])
        assert np.array_equal(got, want), f"{(got != want).sum()} of {got.size} block integers differ"
    finally:
        backend.release(h)


@pytest.mark.parametrize("k,rows,nt", [(2048, 300, 32), (2048, 300, 256), (6144, 64, 37), (512, 640, 8192)])
def test_native_tc_block_ints_exact(backend, oracle, k, rows, nt):
    rng = np.random.default_rng(k + rows + nt)
    raw = rand_blocks(rng, GT, rows, k)
    h = _upload(backend, raw, rows, k, True)
    try:
        xq = oracle.quantize(_acts(rng, nt, k))
        want = oracle.block_ints(oracle.weight(GT, raw, rows, k, panel=False), xq, nt)
        got = backend.tc_block_ints(h, xq, nt, rows, want.shape[2])
        assert np.array_equal(got, want), f"{(got != want).sum()} of {got.size} block integers differ"
    finally:
        backend.release(h)


def test_native_dequant_rows_exact(backend, oracle):
    rows, k = 9, 2048
    rng = np.random.default_rng(5)
    raw = rand_blocks(rng, GT, rows, k)
    h = _upload(backend, raw, rows, k, True)
    try:
        w = oracle.weight(GT, raw, rows, k, panel=False)
        for r in range(rows):
            assert backend.dequant_row(h, r, k).tobytes() == oracle.dequant_row(w, r).tobytes(), r
    finally:
        backend.release(h)


@pytest.mark.parametrize("rows,nt", [(37, 1), (64, 3), (130, 16), (300, 8)])
def test_native_matmul_equals_panel(backend, oracle, reference, rows, nt):
    k = 2048
    rng = np.random.default_rng(rows * 3 + nt)
    raw = rand_blocks(rng, GT, rows, k)
    hn = _upload(backend, raw, rows, k, True)
    hp = _upload(backend, raw, rows, k, False)
    try:
        x = rand_act(rng, nt, k)
        xq = oracle.quantize(x).reshape(-1)
        got = np.zeros((nt, rows), dtype=np.float32)
        pan = np.zeros((nt, rows), dtype=np.float32)
        assert backend.matmul([hn], [got], xq, nt)
        assert backend.matmul([hp], [pan], xq, nt)
        assert got.tobytes() == pan.tobytes()
        cpu = reference.matmul(GT, raw, rows, k, x, 0)  # the reference's native rows
        assert np.abs(got - cpu).max() / max(np.abs(cpu).max(), 1e-6) < 2e-4
    finally:
        backend.release(hn)
        backend.release(hp)


def test_native_model_decode(backend, oracle, synth, model_dir):
    """t_stq with native layers on its own handle against the panel upload:
    the 24-token prompt pass runs the same GEMV templates on both layouts, so
    its logits are bit-identical; decode runs the per-layer graph on both
    (the persistent kernel takes panels only) and must give the oracle's ids
    up to a near tie."""
    import np_forward
    import oracle as O
    from hymt2_b200.device import Backend, DeviceModel
    path = synth.ensure("t_stq", model_dir)
    ids = np.random.default_rng(31).integers(0, 1000, 24).tolist()
    bn = Backend(0)
    try:
        bn.set_stq_layout(True)
        dn = DeviceModel(path, bn, ctx=256)
        try:
            _, ln = dn.forward(ids, 0)
            got = dn.generate(ids, 10)
        finally:
            dn.close()
    finally:
        bn.close()
    dp = DeviceModel(path, backend, ctx=256)
    try:
        assert backend.lib.hyc_set_decode_mode(backend.impl, 1) == 0
        _, lp = dp.forward(ids, 0)
        pan = dp.generate(ids, 10)
    finally:
        backend.lib.hyc_set_decode_mode(backend.impl, 0)
        dp.close()
    assert ln.tobytes() == lp.tobytes()
    om = O.OracleModel(oracle, path, ctx=256)
    try:
        want, steps = om.greedy(ids, 10, chunk=16, step_logits=True)
    finally:
        om.close()
    _, _, tol = np_forward.spread_tolerance(oracle, path, ids)
    for other in (want, pan):
        d = next((i for i, (a, b) in enumerate(zip(got, other)) if a != b), None)
        if d is not None:
            top = np.sort(steps[d])[-2:]
            assert top[1] - top[0] <= 2 * tol * np.abs(steps[d]).max(), (got, other)
