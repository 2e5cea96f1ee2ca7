"""The tensor-parallel split's host arithmetic on CPU (no GPU): two gloo ranks.

The split (hymt2_b200/tp.py) cuts the reference's layer loop
(src/model.c:824-882) into column-parallel q/k/v and gate/up, row-parallel
o_proj and down, and a vocabulary split of the head (:884-900, 945-948).
These tests check, with the C restatement of the reference as the
arithmetic, that the byte slices of the GGUF tensors and the exchanges
recombine to the unsplit products: the sum over ranks of the row-parallel
partial products equals the full product (within 1e-5 of its largest
magnitude: fp32 sums in another order), the column-
parallel rows are the full rows, and the maximum over ranks of the
(logit, first index) keys is the full argmax.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import rand_blocks

Q8_0 = 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_plan_partitions_heads_ffn_and_vocab():
    from hymt2_b200.tp import shard_plan
    for world in (1, 2, 4, 8):
        plans = [shard_plan(16, 4, 6144, 120818, r, world) for r in range(world)]
        assert [p.q0 for p in plans] == [r * 16 // world for r in range(world)]
        assert plans[-1].q1 == 16 and plans[-1].f1 == 6144 and plans[-1].v1 == 120818
        for p in plans:
            # the KV heads a rank holds are exactly those its query heads use (group of 4)
            assert (p.kv0, p.kv1) == (p.q0 // 4, (p.q1 - 1) // 4 + 1)
            assert p.heads == 16 // world and p.f1 - p.f0 == 6144 // world
        assert sum(p.v1 - p.v0 for p in plans) == 120818
    # eight ranks: two query heads each, every KV head on two ranks
    p8 = [shard_plan(16, 4, 6144, 120818, r, 8) for r in range(8)]
    assert [p.kv0 for p in p8] == [0, 0, 1, 1, 2, 2, 3, 3] and all(p.kv_heads == 1 for p in p8)
    with pytest.raises(ValueError):
        shard_plan(16, 4, 6144, 1000, 0, 3)


def _rank_main(rank, world, port, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "oracle"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import torch

        import oracle as O
        from hymt2_b200.tp import shard_plan, slice_cols, slice_rows
        orc = O.Oracle()
        rng = np.random.default_rng(5)            # the same tensors on every rank
        H, heads, kvh, hd, F, V = 512, 8, 4, 64, 1024, 1000
        sh = shard_plan(heads, kvh, F, V, rank, world)
        x_h = rng.standard_normal((1, H)).astype(np.float32)
        x_q = rng.standard_normal((1, heads * hd)).astype(np.float32)
        x_f = rng.standard_normal((1, F)).astype(np.float32)
        wo = rand_blocks(rng, Q8_0, H, heads * hd)
        wd = rand_blocks(rng, Q8_0, H, F)
        wq = rand_blocks(rng, Q8_0, heads * hd, H)
        wh = rand_blocks(rng, Q8_0, V, H)
        res = {}
        # row-parallel o_proj and down: partial products over the rank's K columns, summed over ranks
        for name, w, k, x, k0, k1 in (("o", wo, heads * hd, x_q, sh.q0 * hd, sh.q1 * hd),
                                      ("down", wd, F, x_f, sh.f0, sh.f1)):
            part = orc.matmul(orc.weight(Q8_0, slice_cols(w, Q8_0, H, k, k0, k1), H, k1 - k0), x[:, k0:k1])
            t = torch.from_numpy(part.copy())
            dist.all_reduce(t)
            full = orc.matmul(orc.weight(Q8_0, w, H, k), x)
            res[name] = float(np.abs(t.numpy() - full).max() / max(np.abs(full).max(), 1e-6))
        # column-parallel q rows: the rank's rows of the full product
        part = orc.matmul(orc.weight(Q8_0, slice_rows(wq, Q8_0, heads * hd, H, sh.q0 * hd, sh.q1 * hd),
                                     sh.heads * hd, H), x_h)
        full = orc.matmul(orc.weight(Q8_0, wq, heads * hd, H), x_h)
        res["q_rows_equal"] = bool(np.array_equal(part, full[:, sh.q0 * hd:sh.q1 * hd]))
        # vocabulary split of the head: local argmax keys (logit, first index), maximum over ranks
        lg = orc.matmul(orc.weight(Q8_0, slice_rows(wh, Q8_0, V, H, sh.v0, sh.v1), sh.v1 - sh.v0, H), x_h)[0]
        j = int(np.argmax(lg))                    # numpy: the first maximum
        keys = [None] * world
        dist.all_gather_object(keys, (float(lg[j]), -(sh.v0 + j)))
        best = max(keys)
        full = orc.matmul(orc.weight(Q8_0, wh, V, H), x_h)[0]
        res["argmax"] = (-best[1], int(np.argmax(full)))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_row_parallel_sums_and_vocab_argmax_recombine(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        res = out[r]
        assert res["o"] < 1e-5 and res["down"] < 1e-5, res
        assert res["q_rows_equal"], res
        got, want = res["argmax"]
        assert got == want, res
