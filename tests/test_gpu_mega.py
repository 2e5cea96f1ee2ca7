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


def _resident_begin(lib, impl, dm, ids, max_new):
    pr = np.asarray(ids, dtype=np.int32)
    assert lib.hyc_decode_begin(impl, pr.ctypes.data, len(pr), 0, max_new, None, 0, dm.vocab_out) == 0
    first = np.zeros(1, dtype=np.int32)
    assert lib.hyc_decode_read(impl, first.ctypes.data, 1) == 1
    return int(first[0])


def test_resident_host_loop(backend, synth, model_dir):
    """The resident host loop (hyc_decode_resident): one persistent launch in
    which the host reads every step's token through mapped pinned memory and
    releases the next step with it, as the reference's loop does
    (src/model.c:943-954).  Its ids are the device-resident loop's; a host
    stop after five steps leaves the decode state after step five, and plain
    decode steps continue from there to the same stream."""
    from hymt2_b200.device import DeviceModel
    lib, impl = backend.lib, backend.impl
    dm = DeviceModel(synth.ensure("t_stq", model_dir), backend, ctx=256)
    io = lib.hyc_host_alloc(16)
    try:
        assert lib.hyc_set_decode_mode(impl, 0) == 0
        ids = np.arange(3, 19).tolist()
        want = dm.generate(ids, 12)
        t = C.c_int()
        # the whole stream
        tok = _resident_begin(lib, impl, dm, ids, 12)
        assert lib.hyc_resident_go(io, 0, tok) == 0
        assert lib.hyc_decode_resident(impl, 11, io, 0) == 0, backend.error()
        got = [tok]
        for s in range(11):
            assert lib.hyc_resident_wait(io, s, C.byref(t), 5_000_000_000) == 0
            got.append(t.value)
            if s + 1 < 11:
                lib.hyc_resident_go(io, s + 1, t.value)
        assert lib.hyc_sync(impl) == 0, backend.error()
        out = np.zeros(12, dtype=np.int32)
        assert lib.hyc_decode_read(impl, out.ctypes.data, 12) == 12
        assert got == want and out.tolist() == want
        # the host stops after five steps, then plain steps continue
        tok = _resident_begin(lib, impl, dm, ids, 12)
        lib.hyc_resident_go(io, 0, tok)
        assert lib.hyc_decode_resident(impl, 11, io, 0) == 0, backend.error()
        for s in range(5):
            assert lib.hyc_resident_wait(io, s, C.byref(t), 5_000_000_000) == 0
            lib.hyc_resident_go(io, s + 1 if s < 4 else -1, t.value)
        assert lib.hyc_sync(impl) == 0, backend.error()
        assert lib.hyc_decode_read(impl, out.ctypes.data, 12) == 6
        assert out[:6].tolist() == want[:6]
        assert lib.hyc_decode_steps(impl, 6) == 0
        assert lib.hyc_decode_read(impl, out.ctypes.data, 12) == 12
        assert out.tolist() == want
    finally:
        lib.hyc_host_free(io)
        dm.close()


def test_resident_host_timeout_reports_and_leaves_the_handle_usable(backend, synth, model_dir):
    """A host that never releases step 2 (limit 5 ms): the kernel gives up
    waiting, ends the loop cleanly and reports it once through hyc_sync; the
    waiting host sees the loop end (done < 0); the same handle decodes
    normally afterwards.  No trap, no fault, no hang."""
    from hymt2_b200.device import DeviceModel
    lib, impl = backend.lib, backend.impl
    dm = DeviceModel(synth.ensure("t_stq", model_dir), backend, ctx=256)
    io = lib.hyc_host_alloc(16)
    try:
        assert lib.hyc_set_decode_mode(impl, 0) == 0
        ids = np.arange(5, 21).tolist()
        want = dm.generate(ids, 8)
        t = C.c_int()
        tok = _resident_begin(lib, impl, dm, ids, 8)
        lib.hyc_resident_go(io, 0, tok)
        assert lib.hyc_decode_resident(impl, 7, io, 5_000_000) == 0, backend.error()
        for s in range(2):
            assert lib.hyc_resident_wait(io, s, C.byref(t), 5_000_000_000) == 0
            if s == 0:
                lib.hyc_resident_go(io, 1, t.value)
        assert lib.hyc_resident_wait(io, 2, C.byref(t), 5_000_000_000) == -1
        assert lib.hyc_sync(impl) == -1 and "host" in backend.error()
        assert lib.hyc_sync(impl) == 0                      # reported once; the handle is not broken
        out = np.zeros(8, dtype=np.int32)
        assert lib.hyc_decode_read(impl, out.ctypes.data, 8) == 3   # the prefill token and steps 0, 1
        assert out[:3].tolist() == want[:3]
        assert dm.generate(ids, 8) == want
    finally:
        lib.hyc_host_free(io)
        dm.close()
