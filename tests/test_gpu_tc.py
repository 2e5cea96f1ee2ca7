"""The tcgen05 int8 tensor-core GEMM that multi-token chunks use (needs a
B200), through the C ABI.

  - one weight (STQ1_0, Q2_0C panels; Q4_K, Q6_K as int8 planes, also with
    extreme sub-scales so the 64*hi + lo split meets its bounds) on 1..200
    tokens with each activation
    prologue (plain, RMSNorm*w, SiLU*up): against the oracle's host sequence
    (Q8_K quantiser, panel rows; reference src/kernels.c:128-165, 565-581)
    within 1e-4 relative except for rare one-code Q8_K rounding flips of the
    prologue (in under 5 % of the tokens, each under 5e-3), and against the dp4a
    GEMV on the same inputs
    (same block integers, fp32 sums in another order) within 1e-5 where the
    GEMV hook takes the token count (<= 16);
  - whole prompts: a 150-token prefill through the tensor-core chunks gives
    the logits of the GEMV chunks (1e-4) and of the oracle (the reference's
    spread rule), and the same greedy ids.
"""
import numpy as np
import pytest

from conftest import rand_act, rand_blocks

pytestmark = pytest.mark.gpu

TYPES = {"STQ1_0": 43, "Q2_0C": 40, "Q4_K": 12, "Q6_K": 14, "Q4_K_ext": 12, "Q6_K_ext": 14}


def _extreme(raw: np.ndarray, gt: int, rng) -> np.ndarray:
    """Sub-scales at the ends of their ranges (Q6_K int8 -128 / 127, Q4_K 6-bit 63)."""
    raw = raw.copy()
    if gt == 14:
        blk = raw.reshape(-1, 210)
        blk[:, 192:208] = rng.choice(np.array([0x80, 0x7F, 0x81, 0x01], dtype=np.uint8), size=(blk.shape[0], 16))
    else:
        blk = raw.reshape(-1, 144)
        blk[:, 4:16] = 0xFF
    return raw


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("act", [1, 2, 3])
@pytest.mark.parametrize("k,rows", [(512, 48), (2048, 300), (6144, 512)])
@pytest.mark.parametrize("nt", [1, 37, 128, 200])
def test_tc_gemm(backend, oracle, name, act, k, rows, nt):
    from hymt2_b200.device import weight_from_bytes
    gt = TYPES[name]
    rng = np.random.default_rng(k + act * 7 + nt + rows)
    raw = rand_blocks(rng, gt, rows, k)
    if name.endswith("_ext"):
        raw = _extreme(raw, gt, rng)
    h = backend.upload(weight_from_bytes(gt, raw, rows, k))
    try:
        x = rand_act(rng, nt, k) * 3.0
        x2 = rand_act(rng, nt, k)
        nw = (1.0 + 0.2 * rng.standard_normal(k)).astype(np.float32)
        kw = dict(x2=x2 if act == 3 else None, norm_w=nw if act == 2 else None)
        got = backend.tc_test(h, act, x, rows, **kw)
        w = oracle.weight(gt, raw, rows, k, panel=True)
        want = oracle.prologue_matmul(w, act, x, x2 if act == 3 else None, nw if act == 2 else None)
        scale = max(np.abs(want).max(), 1e-6)
        # the device prologue (norm / SiLU order of operations) may round an
        # activation to the neighbouring Q8_K code where the oracle does not:
        # such flips are rare and bounded by one code step per block
        rel = np.abs(got - want) / scale
        flipped = (rel > 1e-4).any(axis=1).mean()  # a flip touches one token's whole row
        assert flipped < 0.05 and rel.max() < 5e-3, (rel.max(), flipped)
        if nt <= 16:  # the GEMV test hook takes the reference's MAX_BATCH tokens
            gemv = backend.gemv_test(h, act, x, rows, **kw)
            assert np.abs(got - gemv).max() / scale < 1e-5
    finally:
        backend.release(h)


@pytest.mark.parametrize("cfg", ["t_stq", "t_q2c"])
def test_tc_prefill(backend, oracle, synth, model_dir, cfg):
    import np_forward
    import oracle as O
    from hymt2_b200.device import DeviceModel
    path = synth.ensure(cfg, model_dir)
    dm = DeviceModel(path, backend, ctx=512)
    om = O.OracleModel(oracle, path, ctx=512)
    lib, impl = backend.lib, backend.impl
    try:
        ids = np.random.default_rng(44).integers(0, dm.vocab_out, 150).tolist()
        _, spread, tol = np_forward.spread_tolerance(oracle, path, ids)
        assert lib.hyc_set_tc(impl, 0) == 0
        _, lg_gemv = dm.forward(ids, 0)
        assert lib.hyc_set_tc(impl, 1) == 0
        _, lg_tc = dm.forward(ids, 0)
        _, lg_o = om.forward(ids, 0)
        scale = np.abs(lg_o).max()
        e_tc, e_gemv = np.abs(lg_tc - lg_o).max() / scale, np.abs(lg_gemv - lg_o).max() / scale
        assert e_tc <= tol and e_gemv <= tol, (cfg, e_tc, e_gemv, tol)
        assert np.abs(lg_tc - lg_gemv).max() / scale < max(1e-4, tol), cfg
        dm.cache = []
        got = dm.generate(ids, 8)
        om.reset()
        want, steps = om.greedy(ids, 8, chunk=16, step_logits=True)
        assert got == want or np.abs(np.sort(steps[0])[-1] - np.sort(steps[0])[-2]) <= 2 * tol * np.abs(steps[0]).max()
    finally:
        lib.hyc_set_tc(impl, 1)
        dm.close()
        om.close()


@pytest.mark.parametrize("name", ["STQ1_0", "Q6_K", "Q4_K"])
@pytest.mark.parametrize("k,rows,nt", [(512, 48, 40), (2048, 6144, 200), (512, 20480, 256)])
def test_tc_gemm_tile_widths(backend, oracle, name, k, rows, nt):
    """Every MMA width the launch picks (64-row slices while whole tiles
    would leave SMs idle, whole 256 / 128 / 64-row tiles otherwise) gives the
    oracle's result."""
    from hymt2_b200.device import weight_from_bytes
    gt = TYPES[name]
    rng = np.random.default_rng(k + rows + nt)
    raw = rand_blocks(rng, gt, rows, k)
    h = backend.upload(weight_from_bytes(gt, raw, rows, k))
    try:
        x = rand_act(rng, nt, k) * 3.0
        nw = (1.0 + 0.2 * rng.standard_normal(k)).astype(np.float32)
        got = backend.tc_test(h, 2, x, rows, norm_w=nw)
        want = oracle.prologue_matmul(oracle.weight(gt, raw, rows, k, panel=True), 2, x, None, nw)
        rel = np.abs(got - want) / max(np.abs(want).max(), 1e-6)
        flipped = (rel > 1e-4).any(axis=1).mean()
        assert flipped < 0.05 and rel.max() < 5e-3, (rel.max(), flipped)
    finally:
        backend.release(h)


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("k,rows,nt", [(2048, 300, 32), (2048, 300, 128), (512, 300, 200), (2048, 300, 256),
                                       (6144, 64, 37), (512, 128, 8192), (512, 640, 8192)])
def test_tc_block_ints_exact(backend, oracle, name, k, rows, nt):
    """The tcgen05 GEMM's per-block int32 accumulators (read back from TMEM
    by its epilogue) equal the reference's block integers bit for bit: the
    panel `(enc << shift) - off * sum` (src/kernels.c:565-581), Q6_K `acc`
    (:808-835), Q4_K `sumi` and `summ` (:861-877), for host-made Q8_K blocks
    (no device prologue).  The shapes reach both launch forms the product
    picks: 64-row slices of the weight tiles (few tiles) and whole tiles
    (8192 tokens x 640 rows)."""
    from hymt2_b200.device import weight_from_bytes
    gt = TYPES[name]
    rng = np.random.default_rng(k + rows + nt + gt)
    raw = rand_blocks(rng, gt, rows, k)
    if name.endswith("_ext"):
        raw = _extreme(raw, gt, rng)
    h = backend.upload(weight_from_bytes(gt, raw, rows, k))
    try:
        x = rand_act(rng, nt, k) * 3.0
        x[0, :256] = 0.0                                   # an all-zero block
        if nt > 2:
            x[1, :256] = 1.0                               # ties for the first maximum
            x[2, 256:512] = np.linspace(-5.0, 5.0, 256)    # exact halves on the grid
        xq = oracle.quantize(x)
        w = oracle.weight(gt, raw, rows, k, panel=True)
        want = oracle.block_ints(w, xq, nt)
        got = backend.tc_block_ints(h, xq, nt, rows, want.shape[2])
        assert np.array_equal(got, want), f"{(got != want).sum()} of {got.size} block integers differ"
    finally:
        backend.release(h)
