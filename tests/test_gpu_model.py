"""Model-level parity of the CUDA backend (needs a B200).

Against the restated oracle and the reference's own CPU library on identical
seeded GGUFs and prompts:
  - logits within the reference's rounding-spread rule tol = max(1e-5, 3*spread)
    (reference tests/test_model.py:353-364), for the vtable fused_forward
    (host h in / host logits out) in prefill and single-token form;
  - greedy ids identical on non-tie steps for on-device generation;
  - KV-prefix reuse gives the same ids as a cold start;
  - the reference's own host loop (model.c) driving this backend as its
    `HYMT2_DEVICE=cuda` device produces the reference CPU's greedy ids.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MODEL_CASES = ["t_stq", "t_q2c", "t_q4km", "t_q8_0", "t_f16head"]


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def _first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None


def _near_tie(logits, tol):
    top = np.sort(logits)[-2:]
    return (top[1] - top[0]) <= 2 * tol * np.abs(logits).max()


@pytest.fixture(scope="module")
def tiny_models(synth, model_dir):
    return {c: synth.ensure(c, model_dir) for c in MODEL_CASES}


@pytest.mark.parametrize("cfg", MODEL_CASES)
def test_fused_forward_logits(backend, oracle, tiny_models, cfg):
    import np_forward
    import oracle as O
    from hymt2_b200.device import DeviceModel
    path = tiny_models[cfg]
    rng = np.random.default_rng(21)
    dm = DeviceModel(path, backend, ctx=256)
    om = O.OracleModel(oracle, path, ctx=256)
    try:
        ids = rng.integers(0, dm.vocab_out, 20).tolist()
        _, spread, tol = np_forward.spread_tolerance(oracle, path, ids)
        h_d, lg_d = dm.forward(ids, 0)              # one 20-token prefill call
        h_o, lg_o = om.forward(ids, 0)
        assert _rel(lg_d, lg_o) <= tol, (cfg, _rel(lg_d, lg_o), tol)
        assert _rel(h_d, h_o) <= max(tol, 1e-4)
        # three single-token steps (graph path)
        for j, t in enumerate(rng.integers(0, dm.vocab_out, 3).tolist()):
            _, a = dm.forward([t], 20 + j)
            _, b = om.forward([t], 20 + j)
            assert _rel(a, b) <= tol, (cfg, j, _rel(a, b), tol)
        # device KV cache equals the oracle's bit for bit on (almost) every entry
        k_d, v_d = dm.kv(0, 23)
        k_o, v_o = om.kv(0, 23)
        assert (k_d != k_o).mean() < 0.01 and (v_d != v_o).mean() < 0.01
    finally:
        dm.close()
        om.close()


@pytest.mark.parametrize("cfg", MODEL_CASES)
def test_device_greedy_matches_oracle(backend, oracle, tiny_models, cfg):
    import np_forward
    import oracle as O
    from hymt2_b200.device import DeviceModel
    path = tiny_models[cfg]
    rng = np.random.default_rng(5)
    dm = DeviceModel(path, backend, ctx=256)
    om = O.OracleModel(oracle, path, ctx=256)
    try:
        ids = rng.integers(0, dm.vocab_out, 24).tolist()
        _, spread, tol = np_forward.spread_tolerance(oracle, path, ids)
        got = dm.generate(ids, 10)
        want, steps = om.greedy(ids, 10, chunk=16, step_logits=True)
        d = _first_divergence(got, want)
        assert d is None or _near_tie(steps[d], tol), (cfg, got, want)
        # prefix reuse: a second prompt sharing 16 tokens reuses the device KV
        ids2 = ids[:16] + rng.integers(0, dm.vocab_out, 6).tolist()
        warm = dm.generate(ids2, 6)
        om.reset()
        cold_o, steps2 = om.greedy(ids2, 6, chunk=16, step_logits=True)
        d2 = _first_divergence(warm, cold_o)
        assert d2 is None or _near_tie(steps2[d2], tol), (cfg, warm, cold_o)
    finally:
        dm.close()
        om.close()


@pytest.mark.parametrize("cfg", ["t_stq", "t_q8_0"])
def test_long_context_decode_matches_oracle(backend, oracle, tiny_models, cfg):
    """Greedy decode past position 4096 (the KV length of the Q8_0 config):
    a 4100-token prefill, then decode steps whose attention runs as 65
    chunks of 64 keys per KV head (130 units, past the persistent kernel's
    64), give the oracle's ids.  Near ties are judged with a fixed 1e-3
    relative margin (the fp64-vs-fp32 spread rule needs minutes of numpy at
    this length; it measures ~1e-5 for these models)."""
    import oracle as O
    from hymt2_b200.device import DeviceModel
    path = tiny_models[cfg]
    ctx, n = 4224, 4100
    dm = DeviceModel(path, backend, ctx=ctx)
    om = O.OracleModel(oracle, path, ctx=ctx)
    try:
        ids = np.random.default_rng(9).integers(0, dm.vocab_out, n).tolist()
        got = dm.generate(ids, 4)
        want, steps = om.greedy(ids, 4, chunk=16, step_logits=True)
        d = _first_divergence(got, want)
        assert d is None or _near_tie(steps[d], 1e-3), (cfg, got, want)
    finally:
        dm.close()
        om.close()


def test_decode_host_io_path_same_ids(backend, tiny_models):
    """The end-to-end form (each step's token through pinned host memory)
    yields the same stream as the device-resident loop."""
    import ctypes as C
    from hymt2_b200.device import DeviceModel
    dm = DeviceModel(tiny_models["t_stq"], backend, ctx=256)
    lib, impl = backend.lib, backend.impl
    try:
        ids = np.arange(3, 19, dtype=np.int32)
        a = dm.generate(ids.tolist(), 9)
        assert lib.hyc_decode_begin(impl, ids.ctypes.data, len(ids), 0, 9, None, 0, dm.vocab_out) == 0
        buf = lib.hyc_host_alloc(4 * 16)
        try:
            assert lib.hyc_decode_steps_host(impl, 8, buf) == 0
            out = np.zeros(9, dtype=np.int32)
            n = lib.hyc_decode_read(impl, out.ctypes.data, 9)
            tok = np.ctypeslib.as_array((C.c_int * 9).from_address(buf))
            assert n == 9 and out.tolist() == a
            assert tok[1:].tolist() == a[1:9]
        finally:
            lib.hyc_host_free(buf)
    finally:
        dm.close()


@pytest.mark.slow
def test_bench_model_greedy_full_size(backend, oracle, synth, model_dir):
    """Config 0 (reference bench GGUF, 32 layers): 48-token prompt.  Logits
    within tol = max(1e-5, 3*spread), spread = the oracle's fp64-vs-fp32
    deviation on the same prompt (the reference's rule, measured with the C
    oracle because the numpy model does not fit a 1.8B model in the test
    budget); greedy ids identical up to the first near-tie step."""
    import oracle as O
    from hymt2_b200.device import DeviceModel
    path = synth.ensure("c0_stq", model_dir)
    ids = np.random.default_rng(1).integers(0, 120818, 48).tolist()
    dm = DeviceModel(path, backend, ctx=1024)
    try:
        got = dm.generate(ids, 16)
        h_d, lg_d = dm.forward(ids, 0)
    finally:
        dm.close()
    om = O.OracleModel(oracle, path, ctx=1024)
    try:
        l32, spread, tol = om.logits_spread(ids)
        want, steps = om.greedy(ids, 16, chunk=16, step_logits=True)
    finally:
        om.close()
    rel = _rel(lg_d, l32)
    print(f"full-size logits rel {rel:.3e}, oracle spread {spread:.3e}, tol {tol:.3e}")
    assert rel <= tol, (rel, spread, tol)
    d = _first_divergence(got, want)
    assert d is None or _near_tie(steps[d], tol), (got, want)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref",
                                                    "libhymt2_dropin.so")), reason="drop-in not built")
@pytest.mark.parametrize("cfg", ["t_stq", "t_q4km", "t_q8_0"])
def test_reference_host_drives_backend(tiny_models, cfg, monkeypatch):
    """The reference's own model.c, linked with this backend in place of its
    src/cuda.c and forced to HYMT2_DEVICE=cuda, reproduces the reference CPU."""
    import oracle as O
    path = tiny_models[cfg]
    ids = np.random.default_rng(8).integers(0, 1000, 30).tolist()
    monkeypatch.setenv("HYMT2_DEVICE", "cpu")
    cpu = O.Reference(O.REF_LIB).load(path, threads=2, ctx=256)
    want, wl, *_ = cpu.greedy(ids, 8, step_logits=True)
    cpu.close()
    monkeypatch.setenv("HYMT2_DEVICE", "cuda")
    dev = O.Reference(O.DROPIN_LIB).load(path, threads=2, ctx=256)
    try:
        assert dev.uses_device(), dev.info()
        got, gl, *_ = dev.greedy(ids, 8, step_logits=True)
    finally:
        dev.close()
    assert _rel(gl[0], wl[0]) < 1e-3
    d = _first_divergence(got, want)
    assert d is None or _near_tie(wl[d], 1e-3), (got, want)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref",
                                                    "libhymt2_dropin.so")), reason="drop-in not built")
def test_reference_debug_device_matmul_cuda():
    """The reference's own device-parity hook (hymt2_debug_device_matmul,
    src/model.c:1077) with backend "cuda" — the CUDA port of tests/test_metal.py."""
    import oracle as O
    from conftest import rand_act, rand_blocks
    ref = O.Reference(O.DROPIN_LIB)
    rng = np.random.default_rng(11)
    for gt in (43, 40, 12, 14):
        for rows, nt in ((37, 1), (64, 3)):
            raw = rand_blocks(rng, gt, rows, 1536)
            x = rand_act(rng, nt, 1536)
            cpu = ref.matmul(gt, raw, rows, 1536, x, 1)
            gpu = np.zeros((nt, rows), dtype=np.float32)
            rc = ref.lib.hymt2_debug_device_matmul(b"cuda", gt, raw.ctypes.data, rows, 1536, x.ctypes.data, nt,
                                                   gpu.ctypes.data)
            assert rc == 0
            assert np.abs(gpu - cpu).max() / max(np.abs(cpu).max(), 1e-6) < 2e-4


@pytest.mark.parametrize("cfg", ["t_stq", "t_q8_0"])
def test_decode_stops_at_stop_id(backend, tiny_models, cfg):
    """On-device stop ids of a single sequence (hyc_decode_begin's stop list,
    the reference loop's break at src/model.c:947-949): with the k-th greedy
    id of an unstopped run as a stop id, the run ends there, hyc_decode_read
    returns the k ids before it, and later steps emit nothing.  t_stq runs the
    persistent kernel, t_q8_0 the per-layer graph."""
    from hymt2_b200.device import DeviceModel
    dm = DeviceModel(tiny_models[cfg], backend, ctx=256)
    lib, impl = backend.lib, backend.impl
    try:
        ids = np.random.default_rng(21).integers(0, dm.vocab_out, 20).astype(np.int32)

        def run(stops):
            st = np.asarray(stops or [0], dtype=np.int32)
            assert lib.hyc_decode_begin(impl, ids.ctypes.data, len(ids), 0, 12, st.ctypes.data, len(stops),
                                        dm.vocab_out) == 0, backend.error()
            assert lib.hyc_decode_steps(impl, 11) == 0, backend.error()
            out = np.zeros(12, dtype=np.int32)
            n = lib.hyc_decode_read(impl, out.ctypes.data, 12)
            assert n >= 0, backend.error()
            return out[:n].tolist()

        free = run([])
        assert len(free) == 12
        # the first id from position 2 on that has not appeared before it
        k = next((i for i in range(2, 12) if free[i] not in free[:i]), None)
        if k is None:
            pytest.skip("greedy stream repeats one id")
        stopped = run([free[k], dm.vocab_out + 5])
        assert stopped == free[:k], (free, k, stopped)
    finally:
        dm.close()
