"""Seeded synthetic model files for the benchmark configurations.

There are no real Hy-MT2 weights on the machines this runs on; every parity test
and benchmark builds a GGUF of the right shape from a fixed seed with
`libhysynth.so` (synth/hysynth.c).  Config names follow the benchmark table:

  c0_stq   STQ1_0 layers + Q6_K tied head, byte-identical to the reference's
           own bench tool output (tools/make_bench_gguf.c)
  c1_q2c   Q2_0C layers (512-weight groups, d ~ |N(0,0.02)|)
  c2_q4km  Q4_K on q/k/o/gate/up, Q6_K on v/down, Q6_K tied head
  c4_q8_0  Q8_0 everywhere including the tied head (fp32-activation path)

`t_*` variants are tiny shapes for fast parity tests.
"""
from __future__ import annotations

import ctypes
import os

from . import _paths

GT = {"F32": 0, "F16": 1, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14, "Q2_0C": 40, "STQ1_0": 43}


class Spec(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int),
        ("n_layer", ctypes.c_int), ("hidden", ctypes.c_int), ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int),
        ("hdim", ctypes.c_int), ("ffn", ctypes.c_int), ("vocab", ctypes.c_int),
        ("layer_type", ctypes.c_int * 7), ("embd_type", ctypes.c_int), ("head_type", ctypes.c_int),
        ("freq_base", ctypes.c_float), ("rope_alpha", ctypes.c_float), ("eps", ctypes.c_float),
        ("seed", ctypes.c_uint64),
        ("scale_sigma", ctypes.c_double), ("kquant_sigma", ctypes.c_double), ("q8_code_sigma", ctypes.c_double),
        ("q8_scale_sigma", ctypes.c_double), ("f16_sigma", ctypes.c_double), ("norm_jitter", ctypes.c_double),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _paths.SYNTH_LIB
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built; run __graft_entry__.build()")
        _lib = ctypes.CDLL(path)
        _lib.hysynth_default_spec.argtypes = [ctypes.POINTER(Spec)]
        _lib.hysynth_write.argtypes = [ctypes.c_char_p, ctypes.POINTER(Spec)]
        _lib.hysynth_write.restype = ctypes.c_int
    return _lib


# projection order: q, k, v, o, gate, up, down
_MIX = {
    "stq": [GT["STQ1_0"]] * 7,
    "q2c": [GT["Q2_0C"]] * 7,
    "q4km": [GT["Q4_K"], GT["Q4_K"], GT["Q6_K"], GT["Q4_K"], GT["Q4_K"], GT["Q4_K"], GT["Q6_K"]],
    "q8_0": [GT["Q8_0"]] * 7,
    "f16": [GT["F16"]] * 7,
}

FULL = dict(n_layer=32, hidden=2048, heads=16, kv_heads=4, hdim=128, ffn=6144, vocab=120818)
TINY = dict(n_layer=2, hidden=256, heads=4, kv_heads=2, hdim=64, ffn=512, vocab=1000)
TINY512 = dict(n_layer=2, hidden=512, heads=8, kv_heads=2, hdim=64, ffn=1024, vocab=1000)
# splits over 2 / 4 / 8 ranks (heads, KV heads, FFN columns and vocabulary divide)
# tensor-parallel test model: 2-, 4- and 8-way splits keep whole 256-element
# blocks per rank (query dims 16 x 128 / 8, FFN 2048 / 8), and at 8 ranks every
# KV head sits on two ranks, as in the 1.8B shape
TINY_TP = dict(n_layer=2, hidden=512, heads=16, kv_heads=4, hdim=128, ffn=2048, vocab=1000)


def make_spec(mix: str, shape: dict, reftool: bool = False, seed: int = 0, embd: str = "Q6_K",
              head: str | None = None, alpha: float = 1000.0, norm_jitter: float = 0.0) -> Spec:
    sp = Spec()
    lib().hysynth_default_spec(ctypes.byref(sp))
    sp.mode = 0 if reftool else 1
    for k, v in shape.items():
        setattr(sp, k, v)
    if not reftool:
        for i, t in enumerate(_MIX[mix]):
            sp.layer_type[i] = t
        sp.embd_type = GT[embd]
        sp.head_type = GT[head] if head else -1
        sp.rope_alpha = alpha
        sp.seed = seed
        sp.norm_jitter = norm_jitter
    return sp


CONFIGS = {
    "c0_stq": lambda layers=32: make_spec("stq", dict(FULL, n_layer=layers), reftool=True),
    "c1_q2c": lambda layers=32: make_spec("q2c", dict(FULL, n_layer=layers), seed=0),
    "c2_q4km": lambda layers=32: make_spec("q4km", dict(FULL, n_layer=layers), seed=0),
    "c4_q8_0": lambda layers=32: make_spec("q8_0", dict(FULL, n_layer=layers), seed=0, embd="Q8_0"),
    "t_stq": lambda layers=2: make_spec("stq", dict(TINY, n_layer=layers), seed=7, alpha=3.0, norm_jitter=0.2),
    "t_q2c": lambda layers=2: make_spec("q2c", dict(TINY512, n_layer=layers), seed=7, alpha=3.0, norm_jitter=0.2),
    "t_q4km": lambda layers=2: make_spec("q4km", dict(TINY, n_layer=layers), seed=7, alpha=3.0, norm_jitter=0.2),
    "t_q8_0": lambda layers=2: make_spec("q8_0", dict(TINY, n_layer=layers), seed=7, embd="Q8_0", alpha=3.0,
                                         norm_jitter=0.2),
    "t_q8_0_tp16": lambda layers=2: make_spec("q8_0", dict(TINY_TP, n_layer=layers), seed=11, embd="Q8_0", alpha=3.0,
                                            norm_jitter=0.2),
    "t_f16head": lambda layers=2: make_spec("stq", dict(TINY, n_layer=layers), seed=7, embd="F16", alpha=3.0,
                                            norm_jitter=0.2),
}


def write(path: str, spec: Spec) -> str:
    rc = lib().hysynth_write(path.encode(), ctypes.byref(spec))
    if rc != 0:
        raise OSError(f"hysynth_write({path}) failed: {rc}")
    return path


def ensure(config: str, directory: str, layers: int | None = None) -> str:
    """Write `config` into `directory` once (cached by name) and return the path."""
    os.makedirs(directory, exist_ok=True)
    fn = CONFIGS[config]
    spec = fn() if layers is None else fn(layers)
    path = os.path.join(directory, f"{config}_L{spec.n_layer}.gguf")
    if not os.path.exists(path):
        tmp = path + ".tmp%d" % os.getpid()
        write(tmp, spec)
        os.replace(tmp, path)
    return path
