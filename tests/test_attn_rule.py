"""Host properties of the single-token decode attention's chunk rules
(hymt2_b200/csrc/hy_attn.cuh), on the CPU, through a shim nvcc compiles.

A decode position's keys 0..pos split into units of (KV head, chunk of cs
keys).  The persistent kernel uses attn_chunk_len (at most 64 units, its
merge holds two chunk weights per lane); the per-layer kernels use
attn_chunk_len_wide (the same answer wherever attn_chunk_len has one, else
up to min(units, 160) units).  The launch in hy_backend.cu attn_launch picks
the chunk kernel for a whole context when the rule has an answer at its last
position, ctx - 1, and launches min(attn_max_chunks(ctx), min(units, 160) /
kv_heads) chunk rows.  Checked here for every position of each context:

  - where the persistent rule has an answer the per-layer rule gives the same
    chunk length, so both paths split (and merge) that position identically;
  - chunk lengths are multiples of 32 up to 128, and kv_heads x chunks stays
    within the rule's unit limit (64, or min(units, 160)), so every chunk
    index is below the launched rows and the merges' lane capacity;
  - an answer at ctx - 1 implies one at every earlier position;
  - chunks <= attn_max_chunks(ctx), the partial buffer's rows per head.
"""
import ctypes as C
import os
import shutil
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def ar(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not found")
    so = str(tmp_path_factory.mktemp("attn_rule") / "libattnrule.so")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O1", "-shared",
                    "-Xcompiler", "-fPIC", "-o", so, os.path.join(HERE, "attn_rule_shim.cu")], check=True)
    L = C.CDLL(so)
    L.ar_rules.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    L.ar_rules.restype = None
    return L


def _rules(ar, kv, units, n):
    ln = np.zeros(n, dtype=np.int32)
    wd = np.zeros(n, dtype=np.int32)
    ar.ar_rules(kv, units, n, ln.ctypes.data, wd.ctypes.data)
    return ln, wd


@pytest.mark.parametrize("units", [148, 132, 64, 40])
@pytest.mark.parametrize("kv", [1, 2, 4, 8, 16])
def test_chunk_rules(ar, kv, units):
    lim_narrow = min(units, ar.ar_max_units())
    lim_wide = min(units, ar.ar_max_units_wide())
    cmax = ar.ar_chunk_max()
    n = 20480
    ln, wd = _rules(ar, kv, units, n)
    pos = np.arange(n)
    # the per-layer rule equals the persistent rule wherever the latter answers
    has = ln > 0
    assert np.array_equal(wd[has], ln[has])
    for cs, lim in ((ln, lim_narrow), (wd, lim_wide)):
        ok = cs > 0
        assert np.all(cs[ok] % 32 == 0) and np.all(cs[ok] <= cmax)
        nch = (pos[ok] + cs[ok]) // cs[ok]
        assert np.all(kv * nch <= lim)
        # the answers form a prefix of the positions
        if (~ok).any():
            assert not ok[np.argmax(~ok):].any()
    # the launch: rows for every context whose last position has a per-layer answer
    for ctx in (64, 1024, 2048, 4224, 4736, 8192, 9472, 10240, 18944, 20480):
        if wd[ctx - 1] == 0:
            continue
        rows = min(ar.ar_max_chunks(ctx), lim_wide // kv)
        cs = wd[:ctx]
        assert np.all(cs > 0)
        nch = (pos[:ctx] + cs) // cs
        assert nch.max() <= rows <= ar.ar_max_chunks(ctx), (ctx, nch.max(), rows)


def test_config4_split(ar):
    """Config 4 (4 KV heads, 148 SMs) at KV 4096..4159 in a 4224-row cache:
    the persistent rule has no answer, the per-layer rule gives 33 chunks of
    128 keys, 132 units, within the 37 launched rows."""
    ln, wd = _rules(ar, 4, 148, 4224)
    assert ln[4096] == 0 and wd[4223] > 0
    assert wd[4096] == 128 and (4096 + 128) // 128 == 33
    assert ar.ar_max_chunks(4224) == 132 and min(ar.ar_max_chunks(4224), min(148, ar.ar_max_units_wide()) // 4) == 37
