"""Tensor-parallel split of the decoder across GPUs (one process per GPU).

The split of the reference's layer loop (src/model.c:824-882) and head
(:884-900, argmax :945-948) that config 4 asks for:

  - q/k/v column-parallel by heads: rank r owns query heads
    [r*heads/world, (r+1)*heads/world) and the KV heads they use (replicated
    when world > kv_heads);
  - gate/up column-parallel, down row-parallel over FFN slice r;
  - o_proj row-parallel over the rank's query-head columns;
  - the LM head split by vocabulary rows; the embedding table whole.

After o_proj and after down the residual stream gets the sum over ranks of
the partial products (hyc_tp_* in the backend: a one-shot push over NVLink
peer memory); the greedy token is the largest argmax key over the ranks.

`shard_plan`, `slice_rows` and `slice_cols` are plain byte arithmetic on the
GGUF tensors (tested on the CPU with gloo ranks); `TPDeviceModel` uploads a
rank's share and connects it to its peers through an all-gather of the IPC
handles supplied by the caller (e.g. torch.distributed.all_gather_object).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import abi
from .gguf import GGUF, TYPE_BLOCK, hparams, row_bytes

PROJ = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


@dataclass
class Shard:
    rank: int
    world: int
    q0: int       # query heads [q0, q1)
    q1: int
    kv0: int      # KV heads [kv0, kv1) those query heads use
    kv1: int
    f0: int       # FFN columns [f0, f1)
    f1: int
    v0: int       # vocabulary rows [v0, v1) of the head
    v1: int

    @property
    def heads(self) -> int:
        return self.q1 - self.q0

    @property
    def kv_heads(self) -> int:
        return self.kv1 - self.kv0


def shard_plan(heads: int, kv_heads: int, ffn: int, vocab: int, rank: int, world: int) -> Shard:
    """Rank `rank`'s share of the split.  Needs heads % world == 0, every
    rank's query heads inside one run of whole KV groups (world divides
    kv_heads, or kv_heads divides world), and ffn % world == 0."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    if heads % world or ffn % world:
        raise ValueError(f"heads {heads} and ffn {ffn} must divide by world {world}")
    g = heads // kv_heads
    hl = heads // world
    q0, q1 = rank * hl, (rank + 1) * hl
    kv0, kv1 = q0 // g, (q1 - 1) // g + 1
    if hl % g and g % hl:
        raise ValueError("a rank's query heads must cover whole KV groups or lie inside one")
    fl = ffn // world
    vl = -(-vocab // world)
    v0, v1 = min(vocab, rank * vl), min(vocab, (rank + 1) * vl)
    return Shard(rank, world, q0, q1, kv0, kv1, rank * fl, (rank + 1) * fl, v0, v1)


def slice_rows(data: np.ndarray, gtype: int, n: int, k: int, r0: int, r1: int) -> np.ndarray:
    """Rows [r0, r1) of a row-major quantised tensor (raw bytes)."""
    rb = row_bytes(gtype, k)
    return np.ascontiguousarray(np.asarray(data).reshape(n, rb)[r0:r1]).reshape(-1)


def slice_cols(data: np.ndarray, gtype: int, n: int, k: int, k0: int, k1: int) -> np.ndarray:
    """Input columns [k0, k1) of every row (whole quantisation blocks)."""
    bb, be = TYPE_BLOCK[gtype]
    if k0 % be or k1 % be:
        raise ValueError(f"columns [{k0}, {k1}) cut a {be}-element block")
    blk = np.asarray(data).reshape(n, k // be, bb)
    return np.ascontiguousarray(blk[:, k0 // be:k1 // be]).reshape(-1)


def _weight(gtype: int, data: np.ndarray, n: int, k: int) -> abi.WeightT:
    w = abi.WeightT()
    w.data = data.ctypes.data
    w.type = gtype
    w.k = k
    w.n = n
    w.row_bytes = row_bytes(gtype, k)
    return w


class TPDeviceModel:
    """Rank `rank` of a `world`-way split of a GGUF model on one GPU.

    allgather(bytes) -> list[bytes] (one per rank, in rank order) exchanges
    the exchange areas' IPC handles and doubles as the barrier between every
    rank's hyc_tp_init and hyc_tp_connect."""

    def __init__(self, path: str, backend, rank: int, world: int, allgather, ctx: int = 1024):
        self.be = backend
        self.g = GGUF(path)
        self.hp = hp = hparams(self.g)
        self.ctx = ctx
        head_t = self.g.tensors.get("output.weight", self.g.tensors["token_embd.weight"])
        self.vocab_out = head_t.n
        self.sh = sh = shard_plan(hp.heads, hp.kv_heads, hp.ffn, head_t.n, rank, world)
        self._keep = []
        self.handles = []
        hd = hp.hdim

        def up(gtype, data, n, k):
            self._keep.append(data)
            h = self.be.upload(_weight(gtype, data, n, k))
            self.handles.append(h)
            return h

        def tensor(name):
            t = self.g.tensors[name]
            return t, self.g.data(name)

        t, d = tensor("token_embd.weight")
        self.embd_h = up(t.gtype, d, t.n, t.k)
        self.head_h = up(head_t.gtype, slice_rows(self.g.data(head_t.name), head_t.gtype, head_t.n, head_t.k,
                                                  sh.v0, sh.v1), sh.v1 - sh.v0, head_t.k)
        self.layers = (abi.FusedLayer * hp.n_layer)()
        self.norms = []
        for i in range(hp.n_layer):
            L = self.layers[i]
            hs = []
            for p in PROJ:
                t, d = tensor(f"blk.{i}.{p}.weight")
                if p == "attn_q":
                    hs.append(up(t.gtype, slice_rows(d, t.gtype, t.n, t.k, sh.q0 * hd, sh.q1 * hd), sh.heads * hd, t.k))
                elif p in ("attn_k", "attn_v"):
                    hs.append(up(t.gtype, slice_rows(d, t.gtype, t.n, t.k, sh.kv0 * hd, sh.kv1 * hd),
                                 sh.kv_heads * hd, t.k))
                elif p == "attn_output":
                    hs.append(up(t.gtype, slice_cols(d, t.gtype, t.n, t.k, sh.q0 * hd, sh.q1 * hd), t.n, sh.heads * hd))
                elif p in ("ffn_gate", "ffn_up"):
                    hs.append(up(t.gtype, slice_rows(d, t.gtype, t.n, t.k, sh.f0, sh.f1), sh.f1 - sh.f0, t.k))
                else:  # ffn_down
                    hs.append(up(t.gtype, slice_cols(d, t.gtype, t.n, t.k, sh.f0, sh.f1), t.n, sh.f1 - sh.f0))
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
        rope_dim = int(self.g.kv.get(f"{arch}.rope.dimension_count", hd))
        self.rope_cos = np.zeros(ctx * (rope_dim // 2), dtype=np.float32)
        self.rope_sin = np.zeros_like(self.rope_cos)
        assert self.be.lib.hyc_rope_tables(base, alpha, hd, rope_dim, ctx, self.rope_cos.ctypes.data,
                                           self.rope_sin.ctypes.data) == 0
        a = abi.FusedArgs()
        a.n_layer, a.hidden, a.ffn = hp.n_layer, hp.hidden, sh.f1 - sh.f0
        a.heads, a.kv_heads, a.hdim = sh.heads, sh.kv_heads, hd
        a.qdim, a.kvdim, a.ctx, a.rope_half = sh.heads * hd, sh.kv_heads * hd, ctx, hp.rope_half
        a.eps = hp.eps
        a.layers = self.layers
        a.outw = self.head_h
        a.out_norm = self.out_norm.ctypes.data
        a.rope_cos = self.rope_cos.ctypes.data
        a.rope_sin = self.rope_sin.ctypes.data
        self.shape = a
        from .device import BackendError
        if not self.be.fused_prepare(a):
            raise BackendError("fused_prepare: " + self.be.error())
        if self.be.lib.hyc_set_embedding(self.be.impl, self.embd_h) != 0:
            raise BackendError("set_embedding")
        hdl = (C.c_ubyte * 64)()
        if self.be.lib.hyc_tp_init(self.be.impl, rank, world, sh.v0, hdl) != 64:
            raise BackendError("tp_init: " + self.be.error())
        allh = allgather(bytes(hdl))
        buf = (C.c_ubyte * (64 * world)).from_buffer_copy(b"".join(allh))
        if self.be.lib.hyc_tp_connect(self.be.impl, buf) != 0:
            raise BackendError("tp_connect: " + self.be.error())
        self.cache: list[int] = []

    def generate(self, prompt, max_new: int, stop=()) -> list[int]:
        """Greedy ids (every rank returns the same ids)."""
        ids = [int(t) for t in prompt]
        pr = np.asarray(ids, dtype=np.int32)
        st = np.asarray(list(stop) or [0], dtype=np.int32)
        out = np.zeros(max_new, dtype=np.int32)
        ng = self.be.lib.hyc_generate(self.be.impl, pr.ctypes.data, len(ids), 0, max_new, st.ctypes.data, len(stop),
                                      self.vocab_out, out.ctypes.data)
        if ng < 0:
            from .device import BackendError
            raise BackendError("generate: " + self.be.error())
        return out[:ng].tolist()

    def close(self):
        seen = set()
        for h in self.handles:
            if h not in seen:
                self.be.release(h)
                seen.add(h)
        self.handles = []
        self.g.close()
