"""The C-ABI library loads and exports every symbol its headers declare (CPU)."""
import ctypes
import os
import re
import subprocess

import pytest

from hymt2_b200 import _paths, abi

ROOT = _paths.ROOT


def _declared(header: str) -> set:
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = "\n".join(ln for ln in src.splitlines() if not ln.lstrip().startswith("#"))
    return set(re.findall(r"HYC_API[^;(]*?\b(\w+)\s*\(", src))


def _exported(lib: str) -> set:
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_library_exists():
    assert os.path.exists(_paths.BACKEND_LIB), "run __graft_entry__.build()"
    assert os.path.exists(_paths.BACKEND_ARCHIVE)


def test_exports_every_declared_symbol():
    decl = _declared("hymt2_cuda.h")
    assert {"hy_cuda_create", "hy_cuda_probe", "hyc_create", "hyc_generate"} <= decl
    exp = _exported(_paths.BACKEND_LIB)
    missing = decl - exp
    assert not missing, f"declared but not exported: {sorted(missing)}"
    # and the Python binding covers the same set
    assert decl == set(abi.SIGNATURES), sorted(decl ^ set(abi.SIGNATURES))


def test_loads_and_binds_without_gpu():
    lib = abi.bind(ctypes.CDLL(_paths.BACKEND_LIB))
    buf = ctypes.create_string_buffer(8)
    r = lib.hy_cuda_probe(buf, 8)          # no GPU here: "0"; on a GPU box: "1"
    assert buf.value in (b"0", b"1") and r in (0, 1)
    ops = lib.hyc_device_ops().contents
    for name, _ in abi.DeviceOps._fields_:
        assert getattr(ops, name), name   # every vtable slot is filled


def test_standalone_create_is_not_a_drop_in():
    """Without the host's device layer linked in, hy_cuda_create refuses
    (the host layer must own the wrapper); hyc_create is the standalone path."""
    lib = abi.bind(ctypes.CDLL(_paths.BACKEND_LIB))
    info = ctypes.create_string_buffer(256)
    assert not lib.hy_cuda_create(b"auto", info, 256)
    assert info.value


def test_resident_loop_host_words():
    """The host half of the resident decode loop (hyc_resident_go / wait)
    touches only the four host words [go, token in, done, token out], so it
    runs here: go writes the token before the go word (a negative step
    writes the stop value), wait returns the token once done reaches the
    step, -1 when the loop ended with an error (done < 0) and -2 after its
    limit."""
    import ctypes as C

    import numpy as np

    from hymt2_b200 import device
    lib = device.load_library()
    io = np.zeros(4, dtype=np.int32)
    p = io.ctypes.data
    assert lib.hyc_resident_go(p, 0, 77) == 0 and io.tolist() == [1, 77, 0, 0]
    assert lib.hyc_resident_go(p, 4, 5) == 0 and io[:2].tolist() == [5, 5]
    assert lib.hyc_resident_go(p, -1, 0) == 0 and io[0] == -1
    t = C.c_int(-9)
    assert lib.hyc_resident_wait(p, 0, C.byref(t), 2_000_000) == -2     # done = 0: nothing finished
    io[2], io[3] = 3, 1234
    assert lib.hyc_resident_wait(p, 2, C.byref(t), 2_000_000) == 0 and t.value == 1234
    assert lib.hyc_resident_wait(p, 3, C.byref(t), 2_000_000) == -2     # step 3 not done yet
    io[2] = -1
    assert lib.hyc_resident_wait(p, 3, C.byref(t), 2_000_000) == -1     # the loop ended with an error
    assert lib.hyc_resident_go(None, 0, 0) == -1 and lib.hyc_resident_wait(None, 0, C.byref(t), 1) == -1


def test_rope_tables_match_loader_formula():
    import numpy as np
    lib = abi.bind(ctypes.CDLL(_paths.BACKEND_LIB))
    cos = np.zeros(4 * 64, dtype=np.float32)
    sin = np.zeros_like(cos)
    assert lib.hyc_rope_tables(10000.0, 1000.0, 128, 128, 4, cos.ctypes.data, sin.ctypes.data) == 0
    libm = ctypes.CDLL(None)
    libm.powf.restype = libm.cosf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    libm.cosf.argtypes = [ctypes.c_float]
    base = np.float32(np.float32(10000.0) * np.float32(libm.powf(1000.0, float(np.float32(128) / np.float32(126)))))
    fr = np.float32(1.0) / np.float32(libm.powf(float(base), float(np.float32(5) / np.float32(64))))
    assert cos[3 * 64 + 5] == np.float32(libm.cosf(float(np.float32(3) * fr)))


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libhymt2_dropin.so")),
                    reason="drop-in build needs the reference sources")
def test_dropin_links_backend_in_place_of_reference_cuda():
    exp = _exported(os.path.join(ROOT, "oracle", "_ref", "libhymt2_dropin.so"))
    assert {"hy_cuda_create", "hy_cuda_probe", "hymt2_model_load", "hymt2_debug_device_matmul"} <= exp
