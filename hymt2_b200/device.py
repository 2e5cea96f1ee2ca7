"""Python host side of the B200 backend.

`Backend` is the vtable-level handle (the same operations the hymt2 host's
device layer dispatches, reference src/device.c:128-164).  `DeviceModel`
mirrors what the hymt2 loader and generation loop do around it (reference
src/model.c:510-631 and :914-958): read a GGUF, upload every weight, prepare
the fused state, then run prefill/decode — greedy, with longest-common-prefix
reuse of the device KV cache between calls.

The product path is the native library; there is no CPU fallback here: if
libhymt2_cuda.so is missing or the GPU is unusable, construction raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _paths, abi
from .gguf import GGUF, hparams

_lib = None


def load_library() -> C.CDLL:
    """The backend library; HYMT2_TRACE=1 selects the measurement build with
    the %globaltimer timelines (python -m hymt2_b200.build --trace)."""
    global _lib
    if _lib is None:
        path = _paths.TRACE_LIB if os.environ.get("HYMT2_TRACE") == "1" else _paths.BACKEND_LIB
        if not os.path.exists(path):
            raise RuntimeError(f"{path} not built: run __graft_entry__.build()")
        _lib = abi.bind(C.CDLL(path))
    return _lib


def _ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


class BackendError(RuntimeError):
    pass


class Backend:
    def __init__(self, device: int = 0):
        self.lib = load_library()
        info = C.create_string_buffer(256)
        self.impl = self.lib.hyc_create(device, info, 256)
        if not self.impl:
            raise BackendError(f"hyc_create({device}): {info.value.decode()}")
        self.info = info.value.decode()
        self.ops = self.lib.hyc_device_ops().contents
        self._keep = []

    # ---- vtable operations
    def error(self) -> str:
        buf = C.create_string_buffer(512)
        self.lib.hyc_last_error(self.impl, buf, 512)
        return buf.value.decode()

    def set_stq_layout(self, native: bool) -> None:
        """STQ1_0 weights uploaded from now on: panels (False) or the native
        42 B / 256 blocks decoded in registers (True)."""
        if self.lib.hyc_set_stq_layout(self.impl, 1 if native else 0) != 0:
            raise BackendError("hyc_set_stq_layout failed")

    def upload(self, w: abi.WeightT) -> int:
        h = self.ops.upload(self.impl, C.byref(w))
        if not h:
            raise BackendError("upload failed: " + self.error())
        return h

    def release(self, h: int) -> None:
        if h:
            self.ops.release(h)

    def matmul(self, handles, outs, xq: np.ndarray, nt: int) -> bool:
        n = len(handles)
        hs = (C.c_void_p * n)(*handles)
        os_ = (C.c_void_p * n)(*[o.ctypes.data for o in outs])
        return bool(self.ops.matmul(self.impl, hs, os_, n, xq.ctypes.data, nt))

    def weight_out(self, h: int) -> int:
        return self.ops.weight_out(h)

    def fused_prepare(self, args: abi.FusedArgs) -> bool:
        return bool(self.ops.fused_prepare(self.impl, C.byref(args)))

    def fused_forward(self, args: abi.FusedArgs) -> bool:
        return bool(self.ops.fused_forward(self.impl, C.byref(args)))

    def sync(self) -> None:
        if self.lib.hyc_sync(self.impl) != 0:
            raise BackendError(self.error())

    def stream(self) -> int:
        return self.lib.hyc_stream(self.impl)

    def launches(self) -> int:
        return int(self.lib.hyc_launch_count(self.impl))

    def close(self) -> None:
        if self.impl:
            self.ops.destroy_impl(self.impl)
            self.impl = None

    # ---- kernel-level hooks
    def quantize_q8k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt, k = x.shape
        y = abi.q8k_empty(nt * (k // 256))
        if self.lib.hyc_quantize_q8k(self.impl, x.ctypes.data, k, nt, y.ctypes.data) != 0:
            raise BackendError("quantize: " + self.error())
        return y.reshape(nt, k // 256)

    def block_ints(self, h: int, xq: np.ndarray, nt: int, rows: int, per: int) -> np.ndarray:
        out = np.zeros((nt, rows, per), dtype=np.int32)
        r = self.lib.hyc_block_ints(self.impl, h, xq.ctypes.data, nt, out.ctypes.data)
        if r != per:
            raise BackendError(f"block_ints returned {r}: " + self.error())
        return out

    def tc_block_ints(self, h: int, xq: np.ndarray, nt: int, rows: int, per: int) -> np.ndarray:
        """Per-block integers of the tensor-core GEMM (hyc_tc_block_ints)."""
        out = np.zeros((nt, rows, per), dtype=np.int32)
        r = self.lib.hyc_tc_block_ints(self.impl, h, xq.ctypes.data, nt, out.ctypes.data)
        if r != per:
            raise BackendError(f"tc_block_ints returned {r}: " + self.error())
        return out

    def matmul_f32(self, h: int, x: np.ndarray, rows: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros((x.shape[0], rows), dtype=np.float32)
        if self.lib.hyc_matmul_f32(self.impl, h, x.ctypes.data, x.shape[0], out.ctypes.data) != 0:
            raise BackendError("matmul_f32: " + self.error())
        return out

    def gemv_test(self, h: int, act: int, x, rows: int, x2=None, norm_w=None, eps: float = 1e-5,
                  add_to: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt = x.shape[0]
        out = np.zeros((nt, rows), dtype=np.float32) if add_to is None else np.ascontiguousarray(add_to).copy()
        x2p = None if x2 is None else np.ascontiguousarray(x2, dtype=np.float32)
        nwp = None if norm_w is None else np.ascontiguousarray(norm_w, dtype=np.float32)
        rc = self.lib.hyc_gemv_test(self.impl, h, act, x.ctypes.data, None if x2p is None else x2p.ctypes.data,
                                    None if nwp is None else nwp.ctypes.data, eps, nt, int(add_to is not None),
                                    out.ctypes.data)
        if rc != 0:
            raise BackendError("gemv_test: " + self.error())
        return out

    def tc_test(self, h: int, act: int, x, rows: int, x2=None, norm_w=None, eps: float = 1e-5) -> np.ndarray:
        """One panel weight through the tensor-core GEMM path (hyc_tc_test)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt = x.shape[0]
        out = np.zeros((nt, rows), dtype=np.float32)
        x2p = None if x2 is None else np.ascontiguousarray(x2, dtype=np.float32)
        nwp = None if norm_w is None else np.ascontiguousarray(norm_w, dtype=np.float32)
        rc = self.lib.hyc_tc_test(self.impl, h, act, x.ctypes.data, None if x2p is None else x2p.ctypes.data,
                                  None if nwp is None else nwp.ctypes.data, eps, nt, out.ctypes.data)
        if rc != 0:
            raise BackendError("tc_test: " + self.error())
        return out

    def attention_test(self, heads, kv_heads, hd, ctx, qkv, pos0, kc, vc, q_norm, k_norm, cos, sin, eps=1e-5):
        qkv = np.ascontiguousarray(qkv, dtype=np.float32)
        nt = qkv.shape[0]
        ao = np.zeros((nt, heads * hd), dtype=np.float32)
        rc = self.lib.hyc_attention_test(self.impl, heads, kv_heads, hd, ctx, nt, pos0, eps, qkv.ctypes.data,
                                         kc.ctypes.data, vc.ctypes.data, q_norm.ctypes.data, k_norm.ctypes.data,
                                         cos.ctypes.data, sin.ctypes.data, ao.ctypes.data)
        if rc != 0:
            raise BackendError("attention_test: " + self.error())
        return ao

    def dequant_row(self, h: int, row: int, k: int) -> np.ndarray:
        out = np.zeros(k, dtype=np.float32)
        if self.lib.hyc_dequant_row(self.impl, h, row, out.ctypes.data) != 0:
            raise BackendError("dequant_row: " + self.error())
        return out


def weight_from_bytes(gtype: int, data: np.ndarray, rows: int, k: int, pk: np.ndarray | None = None,
                      ps: np.ndarray | None = None) -> abi.WeightT:
    from .gguf import row_bytes
    w = abi.WeightT()
    w.data = data.ctypes.data
    w.type = gtype
    w.k = k
    w.n = rows
    w.row_bytes = row_bytes(gtype, k)
    if pk is not None:
        w.pk = pk.ctypes.data
        w.ps = ps.ctypes.data
        w.pshift = 1 if gtype == abi.GT_Q2_0C else 0
        w.poff = 3 if gtype == abi.GT_Q2_0C else 1
    return w


PROJ = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


class DeviceModel:
    """A GGUF model resident on one GPU behind the backend vtable."""

    def __init__(self, path: str, backend: Backend | None = None, ctx: int = 1024, panel_fn=None):
        self.be = backend or Backend()
        self.g = GGUF(path)
        self.hp = hp = hparams(self.g)
        self.ctx = ctx
        self._keep = []
        self.handles = []

        def up(name):
            t = self.g.tensors[name]
            data = self.g.data(name)
            pk = ps = None
            if panel_fn is not None and t.gtype in (abi.GT_STQ1_0, abi.GT_Q2_0C):
                pk, ps = panel_fn(t.gtype, data, t.n, t.k)
                self._keep += [pk, ps]
            h = self.be.upload(weight_from_bytes(t.gtype, data, t.n, t.k, pk, ps))
            self.handles.append(h)
            return h

        self.embd_h = up("token_embd.weight")
        self.head_h = up("output.weight") if "output.weight" in self.g.tensors else self.embd_h
        head_t = self.g.tensors.get("output.weight", self.g.tensors["token_embd.weight"])
        self.vocab_out = head_t.n
        self.layers = (abi.FusedLayer * hp.n_layer)()
        self.norms = []
        for i in range(hp.n_layer):
            L = self.layers[i]
            hs = [up(f"blk.{i}.{p}.weight") for p in PROJ]
            L.wq, L.wk, L.wv, L.wo, L.wg, L.wu, L.wd = hs
            for field, nm in (("attn_norm", "attn_norm"), ("ffn_norm", "ffn_norm"), ("q_norm", "attn_q_norm"),
                              ("k_norm", "attn_k_norm")):
                v = self.g.f32(f"blk.{i}.{nm}.weight")
                self.norms.append(v)
                setattr(L, field, v.ctypes.data)
        self.out_norm = self.g.f32("output_norm.weight")
        arch = self.g.kv.get("general.architecture", "hunyuan-dense")
        base = float(self.g.kv.get(f"{arch}.rope.freq_base", 10000.0))
        alpha = float(self.g.kv.get(f"{arch}.rope.scaling.alpha", 0.0))
        rope_dim = int(self.g.kv.get(f"{arch}.rope.dimension_count", hp.hdim))
        self.rope_cos = np.zeros(ctx * (rope_dim // 2), dtype=np.float32)
        self.rope_sin = np.zeros_like(self.rope_cos)
        rc = self.be.lib.hyc_rope_tables(base, alpha, hp.hdim, rope_dim, ctx, self.rope_cos.ctypes.data,
                                         self.rope_sin.ctypes.data)
        assert rc == 0
        self.shape = self._args()
        if not self.be.fused_prepare(self.shape):
            raise BackendError("fused_prepare: " + self.be.error())
        if self.be.lib.hyc_set_embedding(self.be.impl, self.embd_h) != 0:
            raise BackendError("set_embedding")
        self.cache: list[int] = []

    def _args(self) -> abi.FusedArgs:
        hp = self.hp
        a = abi.FusedArgs()
        a.n_layer, a.hidden, a.ffn = hp.n_layer, hp.hidden, hp.ffn
        a.heads, a.kv_heads, a.hdim = hp.heads, hp.kv_heads, hp.hdim
        a.qdim, a.kvdim, a.ctx, a.rope_half = hp.heads * hp.hdim, hp.kv_heads * hp.hdim, self.ctx, hp.rope_half
        a.eps = hp.eps
        a.layers = self.layers
        a.outw = self.head_h
        a.out_norm = self.out_norm.ctypes.data
        a.rope_cos = self.rope_cos.ctypes.data
        a.rope_sin = self.rope_sin.ctypes.data
        return a

    def embed(self, tokens) -> np.ndarray:
        """Host embedding rows, as the host loop does before fused_forward (src/model.c:802)."""
        return np.stack([self.be.dequant_row(self.embd_h, int(t), self.hp.hidden) for t in tokens])

    def forward(self, tokens, pos0: int, want_logits: bool = True):
        """The reference-facing call: hy_device_fused_forward with host buffers."""
        h = np.ascontiguousarray(self.embed(tokens), dtype=np.float32)
        logits = np.zeros(self.g.tensors["token_embd.weight"].n if self.head_h == self.embd_h
                          else self.g.tensors["output.weight"].n, dtype=np.float32)
        a = self._args()
        a.nt, a.pos0, a.want_logits = len(tokens), pos0, int(want_logits)
        a.h = h.ctypes.data
        a.logits = logits.ctypes.data
        if not self.be.fused_forward(a):
            raise BackendError("fused_forward: " + self.be.error())
        return h, (logits if want_logits else None)

    def generate(self, prompt, max_new: int, stop=()) -> list[int]:
        """Greedy ids with on-device argmax and KV prefix reuse (src/model.c:930-954)."""
        ids = [int(t) for t in prompt]
        n = len(ids)
        keep = 0
        while keep < len(self.cache) and keep < n - 1 and self.cache[keep] == ids[keep]:
            keep += 1
        pr = np.asarray(ids, dtype=np.int32)
        st = np.asarray(list(stop) or [0], dtype=np.int32)
        out = np.zeros(max_new, dtype=np.int32)
        ng = self.be.lib.hyc_generate(self.be.impl, pr.ctypes.data, n, keep, max_new, st.ctypes.data, len(stop),
                                      self.vocab_out, out.ctypes.data)
        if ng < 0:
            raise BackendError("generate: " + self.be.error())
        gen = out[:ng].tolist()
        fed = gen if ng < max_new else gen[:-1]
        self.cache = ids + fed
        return gen

    # ---- ragged multi-sequence batches and the continuous-batching server
    def batch_prepare(self, slots: int, slot_ctx: int, max_tokens: int, max_out: int | None = None) -> None:
        mo = slots if max_out is None else max_out
        if self.be.lib.hyc_batch_prepare(self.be.impl, slots, slot_ctx, max_tokens, mo) != 0:
            raise BackendError("batch_prepare: " + self.be.error())
        self.batch_vocab = self.g.tensors.get("output.weight", self.g.tensors["token_embd.weight"]).n

    def batch_forward(self, tokens, slots, positions, out_rows, want_logits: bool = False):
        """One pass over a ragged batch; argmax ids of the out_rows tokens (and their logits)."""
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        sl = np.ascontiguousarray(slots, dtype=np.int32)
        ps = np.ascontiguousarray(positions, dtype=np.int32)
        rows = np.ascontiguousarray(out_rows, dtype=np.int32)
        ids = np.zeros(max(len(rows), 1), dtype=np.int32)
        lg = np.zeros((len(rows), self.batch_vocab), dtype=np.float32) if want_logits else None
        rc = self.be.lib.hyc_batch_forward(self.be.impl, tk.ctypes.data, sl.ctypes.data, ps.ctypes.data, len(tk),
                                           rows.ctypes.data, len(rows), self.vocab_out, ids.ctypes.data, _ptr(lg))
        if rc != 0:
            raise BackendError("batch_forward: " + self.be.error())
        return ids[:len(rows)], lg

    def batch_kv(self, slot: int, layer: int, npos: int):
        kvd = self.hp.kv_heads * self.hp.hdim
        k = np.zeros(npos * kvd, dtype=np.uint16)
        v = np.zeros_like(k)
        if self.be.lib.hyc_batch_kv_read(self.be.impl, slot, layer, npos, k.ctypes.data, v.ctypes.data) != 0:
            raise BackendError("batch_kv_read")
        return k.reshape(npos, kvd), v.reshape(npos, kvd)

    def serve(self, prompts, max_new: int, step_tokens: int, stop=()):
        """Greedy generation for many requests with continuous batching.

        Returns ([nreq][max_new] ids: the ids before a stop id, the stop id, then -1; stats with
        "lengths", the ids per request before its stop id)."""
        if len(prompts) == 0:
            return np.zeros((0, max_new), dtype=np.int32), {"lengths": np.zeros(0, dtype=np.int32)}
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.int32) for p in prompts]))
        off = np.zeros(len(prompts) + 1, dtype=np.int32)
        off[1:] = np.cumsum([len(p) for p in prompts])
        out = np.zeros((len(prompts), max_new), dtype=np.int32)
        lens = np.zeros(len(prompts), dtype=np.int32)
        stops = np.asarray(list(stop) or [0], dtype=np.int32)
        st = abi.ServeStats()
        rc = self.be.lib.hyc_serve(self.be.impl, flat.ctypes.data, off.ctypes.data, len(prompts), max_new,
                                   stops.ctypes.data, len(stop), self.vocab_out, step_tokens, out.ctypes.data,
                                   lens.ctypes.data, C.byref(st))
        if rc != 0:
            raise BackendError("serve: " + self.be.error())
        stats = {f: getattr(st, f) for f, _ in abi.ServeStats._fields_}
        stats["lengths"] = lens
        return out, stats

    def kv(self, layer: int, npos: int):
        kvd = self.hp.kv_heads * self.hp.hdim
        k = np.zeros(npos * kvd, dtype=np.uint16)
        v = np.zeros_like(k)
        if self.be.lib.hyc_kv_read(self.be.impl, layer, npos, k.ctypes.data, v.ctypes.data) != 0:
            raise BackendError("kv_read")
        return k.reshape(npos, kvd), v.reshape(npos, kvd)

    def close(self):
        seen = set()
        for h in self.handles:
            if h not in seen:
                self.be.release(h)
                seen.add(h)
        self.handles = []
        self.g.close()
