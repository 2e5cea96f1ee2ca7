"""Tensor-parallel decode across GPUs (needs 2, 4 or 8 B200s; skipped otherwise).

One process per GPU, each holding its rank's share of a Q8_0 model
(hymt2_b200/tp.py): query heads and the KV heads they use, FFN columns,
o_proj / down K-columns and a vocabulary slice of the tied head.  The ranks
exchange the o_proj and down partial products and the argmax keys through
the backend's one-shot pushes over NVLink peer memory (hyc_tp_*); a gloo
process group on the CPU only carries the IPC handles.

Checked: every rank produces the same greedy ids; they equal the single-GPU
path's ids and the oracle's (reference CPU restatement, src/model.c:914-958),
except after a near-tie step (two top logits within the reference's own
fp64-vs-fp32 spread rule), where the paths may legitimately part.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG, PROMPT, GEN = "t_q8_0_tp16", 40, 12


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path, prompt, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from hymt2_b200.device import Backend
        from hymt2_b200.tp import TPDeviceModel

        def allgather(b):
            out = [None] * world
            dist.all_gather_object(out, b)
            return out

        be = Backend(rank)
        try:
            tm = TPDeviceModel(path, be, rank, world, allgather, ctx=256)
            try:
                ids = tm.generate(prompt, GEN)
                dist.barrier()               # every rank done with its peers' memory before unmapping
            finally:
                tm.close()
        finally:
            be.close()
        q.put((rank, ids, None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_single_gpu_and_oracle(oracle, synth, model_dir, world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import np_forward
    import oracle as O
    import torch.multiprocessing as mp

    from hymt2_b200.device import Backend, DeviceModel
    path = synth.ensure(CFG, model_dir)
    prompt = np.random.default_rng(9).integers(0, 1000, PROMPT).tolist()
    # the unsplit model on one GPU and the oracle
    be = Backend(0)
    try:
        dm = DeviceModel(path, be, ctx=256)
        try:
            single = dm.generate(prompt, GEN)
        finally:
            dm.close()
    finally:
        be.close()
    om = O.OracleModel(oracle, path, ctx=256)
    try:
        want, steps = om.greedy(prompt, GEN, chunk=16, step_logits=True)
    finally:
        om.close()
    _, _, tol = np_forward.spread_tolerance(oracle, path, prompt)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, path, prompt, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, ids, err = q.get(timeout=300)
        res[r] = (ids, err)
    for p in ps:
        p.join(timeout=60)
    for r in range(world):
        assert res[r][1] is None, (r, res[r][1])
    got = res[0][0]
    assert all(res[r][0] == got for r in range(world)), res

    def first_div(a, b):
        return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)

    def near_tie(lg):
        top = np.sort(lg)[-2:]
        return (top[1] - top[0]) <= 2 * tol * np.abs(lg).max()

    for other in (want, single):
        d = first_div(got, other)
        assert d is None or near_tie(steps[d]), (world, got, want, single)
