"""The persistent decode kernel against the graph of per-layer launches
(needs a B200).

Both decode paths compute every step with the same arithmetic in the same
order, so on the same prompt they must agree bit for bit: the emitted ids,
the DecodeState they leave behind, and every KV-cache row of every layer.
The graph path itself is held to the oracle and the reference by
test_gpu_model.py.  Prompts of 120 tokens make the decode cross the
128-key split boundary, so the split-KV merge runs inside the persistent
kernel too; the persistent run is issued as several launches to check that
state carries over between them.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _decode(dm, backend, ids, max_new, mode, chunks):
    lib, impl = backend.lib, backend.impl
    assert lib.hyc_set_decode_mode(impl, mode) == 0
    pr = np.asarray(ids, dtype=np.int32)
    assert lib.hyc_decode_begin(impl, pr.ctypes.data, len(pr), 0, max_new, None, 0, dm.vocab_out) == 0, backend.error()
    why = C.create_string_buffer(128)
    path = lib.hyc_decode_path(impl, why, 128)
    for n in chunks:
        assert lib.hyc_decode_steps(impl, n) == 0, backend.error()
    out = np.zeros(max_new, dtype=np.int32)
    got = lib.hyc_decode_read(impl, out.ctypes.data, max_new)
    assert got == max_new, backend.error()
    npos = len(ids) + max_new - 1
    kv = [dm.kv(layer, npos) for layer in range(dm.hp.n_layer)]
    return out.tolist(), kv, path, why.value.decode()


def _compare(dm, backend, ids, max_new, chunks):
    try:
        ids_g, kv_g, path_g, _ = _decode(dm, backend, ids, max_new, 1, [max_new - 1])
        ids_m, kv_m, path_m, why = _decode(dm, backend, ids, max_new, 0, chunks)
    finally:
        backend.lib.hyc_set_decode_mode(backend.impl, 0)
    assert path_g == 0 and path_m == 1, why
    assert ids_m == ids_g
    for layer, ((kg, vg), (km, vm)) in enumerate(zip(kv_g, kv_m)):
        assert np.array_equal(kg, km) and np.array_equal(vg, vm), layer


@pytest.mark.parametrize("cfg", ["t_stq", "t_q2c"])
def test_persistent_matches_graph_tiny(backend, synth, model_dir, cfg):
    from hymt2_b200.device import DeviceModel
    dm = DeviceModel(synth.ensure(cfg, model_dir), backend, ctx=256)
    try:
        ids = np.random.default_rng(31).integers(0, dm.vocab_out, 120).tolist()
        _compare(dm, backend, ids, 24, [5, 1, 17])
    finally:
        dm.close()


def test_persistent_host_io_path(backend, synth, model_dir):
    """Per-step host token in / token out through the persistent kernel gives
    the stream of the device-resident loop."""
    from hymt2_b200.device import DeviceModel
    lib, impl = backend.lib, backend.impl
    dm = DeviceModel(synth.ensure("t_stq", model_dir), backend, ctx=256)
    try:
        assert lib.hyc_set_decode_mode(impl, 0) == 0
        ids = np.arange(3, 19, dtype=np.int32)
        a = dm.generate(ids.tolist(), 9)
        assert lib.hyc_decode_begin(impl, ids.ctypes.data, len(ids), 0, 9, None, 0, dm.vocab_out) == 0
        assert lib.hyc_decode_path(impl, None, 0) == 1
        buf = lib.hyc_host_alloc(4 * 16)
        try:
            assert lib.hyc_decode_steps_host(impl, 8, buf) == 0
            out = np.zeros(9, dtype=np.int32)
            assert lib.hyc_decode_read(impl, out.ctypes.data, 9) == 9
            tok = np.ctypeslib.as_array((C.c_int * 9).from_address(buf))
            assert out.tolist() == a and tok[1:].tolist() == a[1:9]
        finally:
            lib.hyc_host_free(buf)
    finally:
        dm.close()


def test_persistent_rejects_position_past_context(synth, model_dir):
    """Stepping past the context is caught by the kernel's own position check,
    reported through its error word, and leaves the handle marked broken."""
    from hymt2_b200.device import Backend, DeviceModel
    be = Backend(0)
    try:
        dm = DeviceModel(synth.ensure("t_stq", model_dir), be, ctx=64)
        ids = np.arange(1, 41, dtype=np.int32)
        assert be.lib.hyc_set_decode_mode(be.impl, 0) == 0
        assert be.lib.hyc_decode_begin(be.impl, ids.ctypes.data, 40, 0, 8, None, 0, dm.vocab_out) == 0
        assert be.lib.hyc_decode_steps(be.impl, 40) == 0      # enqueued; fails on the device at pos 64
        out = np.zeros(8, dtype=np.int32)
        assert be.lib.hyc_decode_read(be.impl, out.ctypes.data, 8) < 0
        assert "position outside the context" in be.error()
        dm.close()
    finally:
        be.close()


@pytest.mark.slow
def test_persistent_matches_graph_full_size(backend, synth, model_dir):
    """Config 0 (reference bench GGUF, 32 layers, Q6_K tied head)."""
    from hymt2_b200.device import DeviceModel
    dm = DeviceModel(synth.ensure("c0_stq", model_dir), backend, ctx=1024)
    try:
        ids = np.random.default_rng(1).integers(0, 120818, 120).tolist()
        _compare(dm, backend, ids, 20, [12, 7])
    finally:
        dm.close()


def test_bounded_waits_report_and_leave_the_handle_usable(backend, synth, model_dir):
    """The grid barrier of the persistent kernel and the mbarrier waits of
    the tensor-core GEMM give up after their limit (here 2 ms on targets
    that nothing reaches) and report it through status words the host reads;
    no trap, no fault, no hang, and the same handle then decodes normally."""
    import time
    from hymt2_b200.device import DeviceModel
    out = np.zeros(3, dtype=np.int32)
    t0 = time.perf_counter()
    assert backend.lib.hyc_wait_probe(backend.impl, 2_000_000, out.ctypes.data) == 0, backend.error()
    assert time.perf_counter() - t0 >= 0.004     # both waits ran out their 2 ms
    assert out.tolist() == [0, 1, 0]             # barrier gave up, raised the barrier timeout code; mbarrier gave up
    dm = DeviceModel(synth.ensure("t_stq", model_dir), backend, ctx=128)
    try:
        assert len(dm.generate([1, 2, 3, 4], 4)) == 4
    finally:
        dm.close()
