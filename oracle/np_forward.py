"""Independent numpy forward pass (TEST INFRASTRUCTURE).

Restates the reference's own end-to-end test model (tests/test_model.py:255-302
of zhangbo8418/hymt2): dequantised weights, Q8_K round trip of every matmul
input, NeoX rope then per-head q/k RMSNorm, bf16 KV, softmax attention,
SiLU*up, tied/untied head.  Matmuls run in float64 (the reference value) or
float32 (to measure the reference's own rounding spread).  The tolerance rule
is the reference's: tol = max(1e-5, 3 * spread), spread =
max|ref64 - ref32| / max|ref64| (tests/test_model.py:353-364).

Only for small models: every weight is held dequantised in memory.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def bf16_round(x):
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def q8k_roundtrip(x):
    x = np.asarray(x, dtype=np.float32).reshape(-1, 256)
    out = np.zeros_like(x)
    for i, blk in enumerate(x):
        a = np.abs(blk)
        if a.max() == 0:
            continue
        mx = blk[int(np.argmax(a))]
        iscale = f32(-127.0) / f32(mx)
        q = np.clip(np.rint(blk * iscale), -127, 127).astype(np.float32)
        out[i] = q * (f32(1.0) / iscale)
    return out.reshape(-1)


class NumpyModel:
    def __init__(self, orc, path: str, dtype=np.float64):
        from hymt2_b200.device import PROJ
        from hymt2_b200.gguf import GGUF, hparams
        self.g = GGUF(path)
        hp = self.hp = hparams(self.g)
        self.dtype = dtype

        def deq(name):
            t = self.g.tensors[name]
            w = orc.weight(t.gtype, self.g.data(name), t.n, t.k, panel=False)
            return np.stack([orc.dequant_row(w, r) for r in range(t.n)])

        self.embd = deq("token_embd.weight")
        self.head = deq("output.weight") if "output.weight" in self.g.tensors else self.embd
        self.out_norm = self.g.f32("output_norm.weight")
        self.layers = []
        for i in range(hp.n_layer):
            L = {p: deq(f"blk.{i}.{p}.weight") for p in PROJ}
            for nm in ("attn_norm", "ffn_norm", "attn_q_norm", "attn_k_norm"):
                L[nm] = self.g.f32(f"blk.{i}.{nm}.weight")
            self.layers.append(L)
        import ctypes
        libm = ctypes.CDLL(None)
        libm.powf.restype = ctypes.c_float
        libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
        libm.cosf.restype = libm.sinf.restype = ctypes.c_float
        libm.cosf.argtypes = libm.sinf.argtypes = [ctypes.c_float]
        self._libm = libm
        self.base = f32(hp.rope_base)
        half = hp.rope_half
        self.freq = np.array([f32(1.0) / f32(libm.powf(float(self.base), float(f32(i) / f32(half)))) for i in range(half)],
                             dtype=np.float32)

    def rms(self, x, w):
        eps = self.hp.eps
        return (x * (f32(1) / np.sqrt(np.mean(x.astype(np.float64) ** 2) + eps).astype(np.float32)) * w).astype(np.float32)

    def mm(self, W, x):
        xq = q8k_roundtrip(x) if W.shape[1] % 256 == 0 else x
        if self.dtype == np.float64:
            return (W.astype(np.float64) @ xq.astype(np.float64)).astype(np.float32)
        return (W.astype(np.float32) @ xq.astype(np.float32)).astype(np.float32)

    def mm_fp(self, W, x, quant: bool):
        return self.mm(W, x) if quant else (W.astype(self.dtype) @ x.astype(self.dtype)).astype(np.float32)

    def logits(self, ids, quant_types=None):
        hp = self.hp
        HD, H, KV = hp.hdim, hp.heads, hp.kv_heads
        half = hp.rope_half
        libm = self._libm
        kc = [[] for _ in range(hp.n_layer)]
        vc = [[] for _ in range(hp.n_layer)]
        from hymt2_b200.device import PROJ
        qtypes = quant_types or {}
        last = None
        for pos, t in enumerate(ids):
            h = self.embd[t].copy()
            ang = [f32(pos) * fr for fr in self.freq]
            c = np.array([libm.cosf(float(a)) for a in ang], dtype=np.float32)
            s = np.array([libm.sinf(float(a)) for a in ang], dtype=np.float32)
            for li, L in enumerate(self.layers):
                q8 = lambda p: qtypes.get((li, p), True)
                xn = self.rms(h, L["attn_norm"])
                q = self.mm_fp(L["attn_q"], xn, q8("attn_q")).reshape(H, HD).copy()
                k = self.mm_fp(L["attn_k"], xn, q8("attn_k")).reshape(KV, HD).copy()
                v = self.mm_fp(L["attn_v"], xn, q8("attn_v"))
                for arr in (q, k):
                    x0, x1 = arr[:, :half].copy(), arr[:, half:2 * half].copy()
                    arr[:, :half] = x0 * c - x1 * s
                    arr[:, half:2 * half] = x0 * s + x1 * c
                q = np.stack([self.rms(r, L["attn_q_norm"]) for r in q])
                k = np.stack([self.rms(r, L["attn_k_norm"]) for r in k])
                kc[li].append(bf16_round(k))
                vc[li].append(bf16_round(v.reshape(KV, HD)))
                K = np.stack(kc[li])
                V = np.stack(vc[li])
                ao = np.zeros((H, HD), dtype=np.float32)
                for hh in range(H):
                    kvh = hh // (H // KV)
                    sc = (K[:, kvh, :].astype(np.float64) @ q[hh].astype(np.float64)) / np.sqrt(HD)
                    p = np.exp(sc - sc.max())
                    p /= p.sum()
                    ao[hh] = (p @ V[:, kvh, :].astype(np.float64)).astype(np.float32)
                h = h + self.mm_fp(L["attn_output"], ao.reshape(-1), q8("attn_output"))
                xn = self.rms(h, L["ffn_norm"])
                g = self.mm_fp(L["ffn_gate"], xn, q8("ffn_gate"))
                u = self.mm_fp(L["ffn_up"], xn, q8("ffn_up"))
                a = (g / (f32(1) + np.exp(-g)) * u).astype(np.float32)
                h = h + self.mm_fp(L["ffn_down"], a, q8("ffn_down"))
            last = h
        xn = self.rms(last, self.out_norm)
        return self.mm_fp(self.head, xn, qtypes.get("head", True))


def quant_map(g, n_layer: int) -> dict:
    """Which matmuls use Q8_K activations (K-quants, STQ1_0, Q2_0C) vs fp32 (Q8_0/F16/F32)."""
    from hymt2_b200.device import PROJ
    qm = {}
    for i in range(n_layer):
        for p in PROJ:
            qm[(i, p)] = g.tensors[f"blk.{i}.{p}.weight"].gtype not in (0, 1, 8)
    head = g.tensors.get("output.weight", g.tensors["token_embd.weight"])
    qm["head"] = head.gtype not in (0, 1, 8)
    return qm


def spread_tolerance(orc, path: str, ids) -> tuple[np.ndarray, float, float]:
    """(float64 reference logits, spread, tol) for the prompt `ids`."""
    m64 = NumpyModel(orc, path, np.float64)
    qm = quant_map(m64.g, m64.hp.n_layer)
    r64 = m64.logits(ids, qm)
    m64.dtype = np.float32
    r32 = m64.logits(ids, qm)
    spread = float(np.abs(r64 - r32).max() / np.abs(r64).max())
    return r64, spread, max(1e-5, 3 * spread)
