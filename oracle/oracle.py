"""ctypes access to the test-only checkers (TEST INFRASTRUCTURE).

  Oracle       our C restatement (oracle/liborc.so, hy_oracle.c)
  Reference    the reference's own CPU library compiled from its sources
               (oracle/_ref/libhymt2_ref.so; absent when the reference was not
               available at build time)

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_LIB = os.path.join(HERE, "liborc.so")
REF_LIB = os.path.join(HERE, "_ref", "libhymt2_ref.so")
DROPIN_LIB = os.path.join(HERE, "_ref", "libhymt2_dropin.so")

P, I, F = C.c_void_p, C.c_int, C.c_float


def _import_abi():
    import sys
    root = os.path.dirname(HERE)
    if root not in sys.path:
        sys.path.insert(0, root)
    from hymt2_b200 import abi, gguf
    return abi, gguf


class Oracle:
    """Our restatement: formats, quantiser, exact block integers, forward."""

    def __init__(self, path: str = ORC_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle orc`")
        self.abi, self.gguf = _import_abi()
        L = self.lib = C.CDLL(path)
        W = C.POINTER(self.abi.WeightT)
        L.orc_quantize_rows.argtypes = [P, I, I, P]
        L.orc_panel_repack.argtypes = [I, P, C.c_size_t, I, I, P, P]
        L.orc_block_ints.argtypes = [W, P, I, P]
        L.orc_block_ints.restype = I
        L.orc_matmul.argtypes = [W, P, P, I, P]
        L.orc_dequant_row.argtypes = [W, I, P]
        L.orc_f32_to_bf16.argtypes = [F]
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_model_create.argtypes = [P]
        L.orc_model_create.restype = P
        L.orc_model_free.argtypes = [P]
        L.orc_model_reset.argtypes = [P]
        L.orc_forward.argtypes = [P, P, I, I, P, P]
        L.orc_greedy.argtypes = [P, P, I, I, I, P, P]
        L.orc_greedy.restype = I
        L.orc_kcache.argtypes = [P, I]
        L.orc_kcache.restype = P
        L.orc_vcache.argtypes = [P, I]
        L.orc_vcache.restype = P
        L.orc_set_threads.argtypes = [I]
        L.orc_set_f64.argtypes = [I]
        L.orc_attention.argtypes = [I, I, I, I, P, P, P, I, I, P, P, P, P, P, P, F, P]
        L.orc_prologue_matmul.argtypes = [W, I, P, P, P, F, I, P]

    def prologue_matmul(self, w, mode: int, x, x2=None, norm_w=None, eps: float = 1e-5) -> np.ndarray:
        """rmsnorm(x)*w (mode 2) / silu(x)*x2 (mode 3) / x (mode 1), then matmul."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt = x.shape[0]
        out = np.zeros((nt, w.n), dtype=np.float32)
        x2p = None if x2 is None else np.ascontiguousarray(x2, dtype=np.float32)
        nwp = None if norm_w is None else np.ascontiguousarray(norm_w, dtype=np.float32)
        self.lib.orc_prologue_matmul(C.byref(w), mode, x.ctypes.data, None if x2p is None else x2p.ctypes.data,
                                     None if nwp is None else nwp.ctypes.data, eps, nt, out.ctypes.data)
        return out

    def attention(self, heads, kv_heads, hd, qkv, pos0, kc, vc, q_norm, k_norm, cos, sin, eps=1e-5):
        """Rope + q/k norm + bf16 KV store + causal attention for qkv [nt][q|k|v];
        kc/vc [ctx][kvdim] updated in place.  Returns ao [nt][qdim]."""
        qkv = np.ascontiguousarray(qkv, dtype=np.float32)
        nt = qkv.shape[0]
        qd, kvd = heads * hd, kv_heads * hd
        q = np.ascontiguousarray(qkv[:, :qd])
        k = np.ascontiguousarray(qkv[:, qd:qd + kvd])
        v = np.ascontiguousarray(qkv[:, qd + kvd:])
        ao = np.zeros((nt, qd), dtype=np.float32)
        self.lib.orc_attention(heads, kv_heads, hd, hd // 2, q.ctypes.data, k.ctypes.data, v.ctypes.data, nt, pos0,
                               kc.ctypes.data, vc.ctypes.data, q_norm.ctypes.data, k_norm.ctypes.data,
                               cos.ctypes.data, sin.ctypes.data, eps, ao.ctypes.data)
        return ao

    def quantize(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt, k = x.shape
        y = self.abi.q8k_empty(nt * (k // 256))
        self.lib.orc_quantize_rows(x.ctypes.data, nt, k, y.ctypes.data)
        return y.reshape(nt, k // 256)

    def panel(self, gtype: int, data: np.ndarray, rows: int, k: int):
        nb = k // 256
        pk = np.zeros(rows * nb * 64 + 64, dtype=np.uint8)
        off = (-pk.ctypes.data) % 64
        pk = pk[off:off + rows * nb * 64]
        ps = np.zeros(rows * nb, dtype=np.float32)
        self.lib.orc_panel_repack(gtype, data.ctypes.data, self.gguf.row_bytes(gtype, k), rows, k, pk.ctypes.data,
                                  ps.ctypes.data)
        return pk, ps

    def weight(self, gtype, data, rows, k, panel=True):
        from hymt2_b200.device import weight_from_bytes
        pk = ps = None
        if panel and gtype in (40, 43):
            pk, ps = self.panel(gtype, data, rows, k)
        w = weight_from_bytes(gtype, data, rows, k, pk, ps)
        w._keep = (data, pk, ps)
        return w

    def block_ints(self, w, xq: np.ndarray, nt: int) -> np.ndarray:
        nb = w.k // 256
        per = 2 * nb if (w.type == 12 and not w.pk) else nb
        out = np.zeros((nt, w.n, per), dtype=np.int32)
        self.lib.orc_block_ints(C.byref(w), xq.ctypes.data, nt, out.ctypes.data)
        return out

    def matmul(self, w, x: np.ndarray, xq: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt = x.shape[0]
        if xq is None:
            xq = self.quantize(x) if w.k % 256 == 0 else self.abi.q8k_empty(1)
        out = np.zeros((nt, w.n), dtype=np.float32)
        self.lib.orc_matmul(C.byref(w), x.ctypes.data, xq.ctypes.data, nt, out.ctypes.data)
        return out

    def dequant_row(self, w, row: int) -> np.ndarray:
        out = np.zeros(w.k, dtype=np.float32)
        self.lib.orc_dequant_row(C.byref(w), row, out.ctypes.data)
        return out


def _make_desc_type():
    abi, _ = _import_abi()
    W = abi.WeightT

    class Desc(C.Structure):
        _fields_ = [("n_layer", I), ("hidden", I), ("ffn", I), ("heads", I), ("kv_heads", I), ("hdim", I),
                    ("ctx", I), ("rope_half", I), ("eps", F), ("rope_base", F), ("embd", W), ("outw", W),
                    ("out_norm", P), ("attn_norm", P), ("ffn_norm", P), ("q_norm", P), ("k_norm", P),
                    ("wq", P), ("wk", P), ("wv", P), ("wo", P), ("wg", P), ("wu", P), ("wd", P)]
    return Desc


class OracleModel:
    """The restated forward pass over a GGUF (panels built by the oracle)."""

    def __init__(self, orc: Oracle, path: str, ctx: int = 1024, threads: int = 0):
        abi, gg = orc.abi, orc.gguf
        self.orc = orc
        self.g = gg.GGUF(path)
        hp = self.hp = gg.hparams(self.g)
        Desc = _make_desc_type()
        d = self.desc = Desc()
        d.n_layer, d.hidden, d.ffn, d.heads, d.kv_heads, d.hdim = hp.n_layer, hp.hidden, hp.ffn, hp.heads, hp.kv_heads, hp.hdim
        d.ctx, d.rope_half, d.eps, d.rope_base = ctx, hp.rope_half, hp.eps, self._rope_base()
        keep = self._keep = []

        def wt(name):
            t = self.g.tensors[name]
            w = orc.weight(t.gtype, self.g.data(name), t.n, t.k)
            keep.append(w)
            return w

        d.embd = wt("token_embd.weight")
        d.outw = wt("output.weight") if "output.weight" in self.g.tensors else d.embd
        self.out_norm = self.g.f32("output_norm.weight")
        d.out_norm = self.out_norm.ctypes.data
        L = hp.n_layer
        arrs = {}
        for field, nm in (("attn_norm", "attn_norm"), ("ffn_norm", "ffn_norm"), ("q_norm", "attn_q_norm"),
                          ("k_norm", "attn_k_norm")):
            vecs = [self.g.f32(f"blk.{i}.{nm}.weight") for i in range(L)]
            keep.append(vecs)
            ptrs = (C.c_void_p * L)(*[v.ctypes.data for v in vecs])
            keep.append(ptrs)
            setattr(d, field, C.cast(ptrs, C.c_void_p))
        from hymt2_b200.device import PROJ
        for field, p in zip(("wq", "wk", "wv", "wo", "wg", "wu", "wd"), PROJ):
            ws = (abi.WeightT * L)()
            for i in range(L):
                ws[i] = wt(f"blk.{i}.{p}.weight")
            keep.append(ws)
            setattr(d, field, C.cast(ws, C.c_void_p))
        if threads:
            orc.lib.orc_set_threads(threads)
        self.m = orc.lib.orc_model_create(C.addressof(d))
        self.vocab = d.outw.n

    def _rope_base(self) -> float:
        return self.hp.rope_base

    def forward(self, tokens, pos0: int, logits: bool = True):
        t = np.asarray(tokens, dtype=np.int32)
        h = np.zeros((len(t), self.hp.hidden), dtype=np.float32)
        lg = np.zeros(self.vocab, dtype=np.float32) if logits else None
        self.orc.lib.orc_forward(self.m, t.ctypes.data, len(t), pos0, lg.ctypes.data if logits else None,
                                 h.ctypes.data)
        return h, lg

    def logits_spread(self, ids, chunk: int = 16):
        """(float32 logits, spread, tol) after the prompt: spread is the
        reference's own fp32-vs-fp64 deviation max|l64-l32|/max|l64|
        (tests/test_model.py:353-364), tol = max(1e-5, 3*spread)."""
        ids = list(ids)
        self.reset()
        self.orc.lib.orc_set_f64(1)
        try:
            l64 = self._prefill_logits(ids, chunk)
        finally:
            self.orc.lib.orc_set_f64(0)
        self.reset()
        l32 = self._prefill_logits(ids, chunk)
        spread = float(np.abs(l64 - l32).max() / np.abs(l64).max())
        return l32, spread, max(1e-5, 3 * spread)

    def _prefill_logits(self, ids, chunk):
        lg = None
        for i in range(0, len(ids), chunk):
            _, lg = self.forward(ids[i:i + chunk], i, logits=i + chunk >= len(ids))
        return lg

    def greedy(self, ids, ngen: int, chunk: int = 16, step_logits: bool = False):
        t = np.asarray(ids, dtype=np.int32)
        out = np.zeros(ngen, dtype=np.int32)
        sl = np.zeros((ngen, self.vocab), dtype=np.float32) if step_logits else None
        self.orc.lib.orc_greedy(self.m, t.ctypes.data, len(t), ngen, chunk, out.ctypes.data,
                                sl.ctypes.data if step_logits else None)
        return out.tolist(), sl

    def kv(self, layer: int, npos: int):
        kvd = self.hp.kv_heads * self.hp.hdim
        kp = self.orc.lib.orc_kcache(self.m, layer)
        vp = self.orc.lib.orc_vcache(self.m, layer)
        k = np.ctypeslib.as_array((C.c_uint16 * (npos * kvd)).from_address(kp)).reshape(npos, kvd).copy()
        v = np.ctypeslib.as_array((C.c_uint16 * (npos * kvd)).from_address(vp)).reshape(npos, kvd).copy()
        return k, v

    def reset(self):
        self.orc.lib.orc_model_reset(self.m)

    def close(self):
        if self.m:
            self.orc.lib.orc_model_free(self.m)
            self.m = None
        self.g.close()


class Reference:
    """The reference's CPU library (compiled from its sources) + id-level harness."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path = path
        L = self.lib = C.CDLL(path)
        L.refh_quantize_q8k.argtypes = [P, I, I, P]
        L.refh_panel_repack.argtypes = [C.c_uint, P, I, I, P, P]
        L.refh_panel_repack.restype = I
        L.hymt2_debug_matmul.argtypes = [C.c_uint, P, I, I, P, I, P, I]
        L.hymt2_debug_matmul.restype = I
        L.hymt2_debug_dequant_row.argtypes = [C.c_uint, P, I, I, P]
        L.hymt2_debug_dequant_row.restype = I
        L.hymt2_debug_device_matmul.argtypes = [C.c_char_p, C.c_uint, P, I, I, P, I, P]
        L.hymt2_debug_device_matmul.restype = I
        L.hymt2_model_load.argtypes = [C.c_char_p, I, I, C.c_char_p, I]
        L.hymt2_model_load.restype = P
        L.hymt2_model_free.argtypes = [P]
        L.hymt2_model_info.argtypes = [P, C.c_char_p, I]
        L.hymt2_isa.restype = C.c_char_p
        L.refh_dims.argtypes = [P, P]
        L.refh_forward.argtypes = [P, P, I, I, P, P]
        L.refh_forward.restype = I
        L.refh_greedy.argtypes = [P, P, I, I, P, P, P, P, P]
        L.refh_greedy.restype = I
        L.refh_reset_cache.argtypes = [P]
        L.refh_kv.argtypes = [P, I, I, P, P]
        L.refh_threads.argtypes = [P]
        L.refh_threads.restype = I
        L.refh_physical_cores.restype = I
        L.refh_uses_device.argtypes = [P]
        L.refh_uses_device.restype = I

    def isa(self) -> str:
        return self.lib.hymt2_isa().decode()

    def quantize(self, x: np.ndarray) -> np.ndarray:
        abi, _ = _import_abi()
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt, k = x.shape
        y = abi.q8k_empty(nt * (k // 256))
        self.lib.refh_quantize_q8k(x.ctypes.data, k, nt, y.ctypes.data)
        return y.reshape(nt, k // 256)

    def panel(self, gtype, data, rows, k):
        nb = k // 256
        pk = np.zeros(rows * nb * 64 + 64, dtype=np.uint8)
        off = (-pk.ctypes.data) % 64
        pk = pk[off:off + rows * nb * 64]
        ps = np.zeros(rows * nb, dtype=np.float32)
        assert self.lib.refh_panel_repack(gtype, data.ctypes.data, rows, k, pk.ctypes.data, ps.ctypes.data) == 0
        return pk, ps

    def matmul(self, gtype, data, rows, k, x, panel=1):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros((x.shape[0], rows), dtype=np.float32)
        rc = self.lib.hymt2_debug_matmul(gtype, data.ctypes.data, rows, k, x.ctypes.data, x.shape[0],
                                         out.ctypes.data, panel)
        assert rc == 0
        return out

    def dequant_row(self, gtype, data, k, row):
        out = np.zeros(k, dtype=np.float32)
        assert self.lib.hymt2_debug_dequant_row(gtype, data.ctypes.data, k, row, out.ctypes.data) == 0
        return out

    def load(self, path: str, threads: int = 0, ctx: int = 1024):
        err = C.create_string_buffer(512)
        m = self.lib.hymt2_model_load(path.encode(), threads, ctx, err, 512)
        if not m:
            raise RuntimeError("hymt2_model_load: " + err.value.decode())
        return RefModel(self, m)


class RefModel:
    def __init__(self, ref: Reference, m: int):
        self.ref, self.m = ref, m
        d = np.zeros(11, dtype=np.int32)
        ref.lib.refh_dims(m, d.ctypes.data)
        (self.n_layer, self.hidden, self.ffn, self.heads, self.kv_heads, self.hdim, self.ctx, self.rope_half,
         self.vocab_out, self.outw_rows, self.batch) = [int(v) for v in d]

    def info(self) -> str:
        buf = C.create_string_buffer(256)
        self.ref.lib.hymt2_model_info(self.m, buf, 256)
        return buf.value.decode()

    def forward(self, tokens, pos0: int, logits: bool = True):
        t = np.asarray(tokens, dtype=np.int32)
        h = np.zeros((self.batch, self.hidden), dtype=np.float32)
        lg = np.zeros(self.vocab_out, dtype=np.float32) if logits else None
        rows = self.ref.lib.refh_forward(self.m, t.ctypes.data, len(t), pos0, h.ctypes.data,
                                         lg.ctypes.data if logits else None)
        return h[:rows], lg

    def greedy(self, ids, ngen: int, step_logits: bool = False):
        t = np.asarray(ids, dtype=np.int32)
        out = np.zeros(ngen, dtype=np.int32)
        sl = np.zeros((ngen, self.vocab_out), dtype=np.float32) if step_logits else None
        pm, dm = C.c_double(), C.c_double()
        cached = C.c_int()
        rc = self.ref.lib.refh_greedy(self.m, t.ctypes.data, len(t), ngen, out.ctypes.data,
                                      sl.ctypes.data if step_logits else None, C.byref(pm), C.byref(dm),
                                      C.byref(cached))
        assert rc == ngen, rc
        return out.tolist(), sl, pm.value, dm.value, cached.value

    def reset_cache(self):
        self.ref.lib.refh_reset_cache(self.m)

    def kv(self, layer: int, npos: int):
        kvd = self.kv_heads * self.hdim
        k = np.zeros((npos, kvd), dtype=np.uint16)
        v = np.zeros_like(k)
        self.ref.lib.refh_kv(self.m, layer, npos, k.ctypes.data, v.ctypes.data)
        return k, v

    def threads(self) -> int:
        return self.ref.lib.refh_threads(self.m)

    def uses_device(self) -> bool:
        return bool(self.ref.lib.refh_uses_device(self.m))

    def close(self):
        if self.m:
            self.ref.lib.hymt2_model_free(self.m)
            self.m = None


def available_reference() -> Reference | None:
    try:
        return Reference()
    except (FileNotFoundError, OSError):
        return None
