"""Shared fixtures.  `-m gpu` tests need a B200; everything else runs on CPU."""
import os
import sys
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

MODEL_DIR = os.environ.get("HYMT2_MODEL_DIR", os.path.join(tempfile.gettempdir(), "hymt2_models"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA backend")
    config.addinivalue_line("markers", "slow: full-size model (tens of seconds)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    return O.Oracle()


@pytest.fixture(scope="session")
def reference():
    import oracle as O
    ref = O.available_reference()
    if ref is None:
        pytest.skip("reference library oracle/_ref/libhymt2_ref.so not built")
    return ref


@pytest.fixture(scope="session")
def model_dir():
    os.makedirs(MODEL_DIR, exist_ok=True)
    return MODEL_DIR


@pytest.fixture(scope="session")
def synth():
    from hymt2_b200 import synth as S
    S.lib()
    return S


_BACKEND = []


@pytest.fixture
def backend():
    """One backend handle per session, replaced if a test left it broken
    (a failed launch marks a handle unusable, as the host contract requires)."""
    from hymt2_b200.device import Backend
    if _BACKEND and _BACKEND[0].error():
        _BACKEND.pop().close()
    if not _BACKEND:
        _BACKEND.append(Backend(0))
    return _BACKEND[0]


def rand_blocks(rng, gtype: int, rows: int, k: int) -> np.ndarray:
    """Random raw blocks of `gtype` with sane scales (style of the reference's
    own tests: tests/test_metal.py:13-29, tests/test_quants.py:19-34)."""
    f16 = lambda v: np.float16(v).tobytes()
    out = bytearray()
    if gtype == 43:
        for _ in range(rows * (k // 256)):
            out += rng.integers(0, 256, 40, dtype=np.uint8).tobytes() + f16(0.01 + 0.03 * rng.random())
    elif gtype == 40:
        for _ in range(rows * (k // 512)):
            out += f16(0.01 + 0.03 * rng.random()) + rng.integers(0, 256, 128, dtype=np.uint8).tobytes()
    elif gtype == 12:
        for _ in range(rows * (k // 256)):
            b = bytearray(rng.integers(0, 256, 144, dtype=np.uint8).tobytes())
            b[0:2] = f16(0.004 + 0.01 * rng.random())
            b[2:4] = f16(0.002 + 0.01 * rng.random())
            out += b
    elif gtype == 14:
        for _ in range(rows * (k // 256)):
            b = bytearray(rng.integers(0, 256, 210, dtype=np.uint8).tobytes())
            b[208:210] = f16(0.0008 + 0.001 * rng.random())
            for j in range(192, 208):
                b[j] = int(rng.integers(-24, 25)) & 0xFF
            out += b
    elif gtype == 8:
        for _ in range(rows * (k // 32)):
            b = bytearray(rng.integers(0, 256, 34, dtype=np.uint8).tobytes())
            b[0:2] = f16(0.01 + 0.02 * rng.random())
            out += b
    elif gtype == 1:
        out += (rng.standard_normal(rows * k) * 0.05).astype(np.float16).tobytes()
    elif gtype == 0:
        out += (rng.standard_normal(rows * k) * 0.05).astype(np.float32).tobytes()
    return np.frombuffer(bytes(out), dtype=np.uint8).copy()


def rand_act(rng, nt: int, k: int) -> np.ndarray:
    """Activations with occasional outliers (reference tests/test_metal.py:37)."""
    return (rng.standard_normal((nt, k)) * np.where(rng.random((nt, k)) < 0.02, 6.0, 1.0)).astype(np.float32)
