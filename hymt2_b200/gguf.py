"""Minimal read-only GGUF v2/v3 reader (memory-mapped, zero-copy).

Only what the host side of this backend needs to feed `hy_device_ops.upload`
from a model file: key/values and tensor byte ranges.  The hymt2 host library
has its own loader (src/gguf.c); this one exists so tests and the benchmark can
drive the CUDA backend without the reference's C host.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}

# bytes per block and weights per block of each ggml type used by hymt2
TYPE_BLOCK = {0: (4, 1), 1: (2, 1), 8: (34, 32), 12: (144, 256), 14: (210, 256), 40: (130, 512), 43: (42, 256)}


def row_bytes(gtype: int, k: int) -> int:
    b, w = TYPE_BLOCK[gtype]
    return (k // w) * b


@dataclass
class Tensor:
    name: str
    gtype: int
    dims: tuple
    offset: int  # absolute file offset
    nbytes: int

    @property
    def k(self) -> int:
        return int(self.dims[0])

    @property
    def n(self) -> int:
        return int(self.dims[1]) if len(self.dims) > 1 else 1


class GGUF:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self.mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.buf = np.frombuffer(self.mm, dtype=np.uint8)
        self.kv: dict = {}
        self.tensors: dict[str, Tensor] = {}
        self._parse()

    def close(self):
        """Close the mapping; if numpy views of it are still alive the
        mapping stays open until they are garbage-collected."""
        self.buf = None
        try:
            self.mm.close()
        except BufferError:
            pass
        self._f.close()

    def _parse(self):
        mm = self.mm
        if mm[:4] != b"GGUF":
            raise ValueError(f"{self.path}: not a GGUF file")
        version, n_t, n_kv = struct.unpack_from("<IQQ", mm, 4)
        if version not in (2, 3):
            raise ValueError(f"{self.path}: unsupported GGUF version {version}")
        pos = 24

        def rd_str(p):
            (n,) = struct.unpack_from("<Q", mm, p)
            return mm[p + 8:p + 8 + n].decode("utf-8", "replace"), p + 8 + n

        def rd_val(t, p):
            if t in _SCALAR:
                fmt = _SCALAR[t]
                return struct.unpack_from(fmt, mm, p)[0], p + struct.calcsize(fmt)
            if t == 8:
                return rd_str(p)
            if t == 9:
                at, n = struct.unpack_from("<IQ", mm, p)
                p += 12
                if at in _SCALAR:
                    sz = struct.calcsize(_SCALAR[at])
                    arr = np.frombuffer(mm, dtype=np.dtype(_SCALAR[at]), count=n, offset=p)
                    return arr, p + sz * n
                out = []
                for _ in range(n):
                    v, p = rd_val(at, p)
                    out.append(v)
                return out, p
            raise ValueError(f"unknown gguf value type {t}")

        for _ in range(n_kv):
            key, pos = rd_str(pos)
            (t,) = struct.unpack_from("<I", mm, pos)
            pos += 4
            val, pos = rd_val(t, pos)
            self.kv[key] = val
        infos = []
        for _ in range(n_t):
            name, pos = rd_str(pos)
            (nd,) = struct.unpack_from("<I", mm, pos)
            pos += 4
            dims = struct.unpack_from("<%dQ" % nd, mm, pos)
            pos += 8 * nd
            gtype, off = struct.unpack_from("<IQ", mm, pos)
            pos += 12
            infos.append((name, gtype, dims, off))
        align = int(self.kv.get("general.alignment", 32))
        data0 = (pos + align - 1) // align * align
        for name, gtype, dims, off in infos:
            k = int(dims[0])
            n = int(dims[1]) if len(dims) > 1 else 1
            nbytes = row_bytes(gtype, k) * n if gtype in TYPE_BLOCK else 0
            self.tensors[name] = Tensor(name, gtype, tuple(int(d) for d in dims), data0 + off, nbytes)

    def data(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self.buf[t.offset:t.offset + t.nbytes]

    def f32(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if t.gtype == 0:
            return np.frombuffer(self.mm, dtype=np.float32, count=t.k, offset=t.offset).copy()
        if t.gtype == 1:
            return np.frombuffer(self.mm, dtype=np.float16, count=t.k, offset=t.offset).astype(np.float32)
        raise ValueError(f"{name}: vector tensors must be F32/F16")


def _powf(x: float, y: float) -> float:
    import ctypes
    libm = ctypes.CDLL(None)
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    return libm.powf(x, y)


@dataclass
class HParams:
    n_layer: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    hdim: int
    rope_half: int
    rope_base: float  # effective base with rope.scaling.alpha folded in
    eps: float
    vocab: int


def hparams(g: GGUF) -> HParams:
    """Hyper-parameters as the hymt2 loader derives them (src/model.c:524-546)."""
    arch = g.kv.get("general.architecture", "hunyuan-dense")

    def ki(s, d=0):
        return int(g.kv.get(f"{arch}.{s}", d))

    def kf(s, d):
        return float(g.kv.get(f"{arch}.{s}", d))

    hidden = ki("embedding_length")
    heads = ki("attention.head_count")
    kvh = ki("attention.head_count_kv", heads)
    hdim = ki("attention.key_length") or hidden // heads
    rope_dim = ki("rope.dimension_count", hdim)
    base = np.float32(kf("rope.freq_base", 10000.0))
    alpha = np.float32(kf("rope.scaling.alpha", 0.0))
    if alpha > 0 and hdim > 2:
        # base *= powf(alpha, hdim/(hdim-2)) with the C library's powf, as the loader does
        base = np.float32(base * np.float32(_powf(float(alpha), float(np.float32(hdim) / np.float32(hdim - 2)))))
    return HParams(ki("block_count"), hidden, ki("feed_forward_length"), heads, kvh, hdim, rope_dim // 2,
                   float(base), float(np.float32(kf("attention.layer_norm_rms_epsilon", 1e-5))),
                   g.tensors["token_embd.weight"].n)
