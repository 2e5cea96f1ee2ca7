"""The N > 1 host path on CPU: two gloo ranks (no GPU).

Multi-GPU runs are data-parallel with no collective on the data path: each
rank serves a round-robin share of the independent requests (config 3) or
runs its own batch-1 replica (config 0), and the process group carries only
barriers and the max-over-ranks time.  These tests run that host logic of
bench.py with the gloo backend: the shares partition the request list, the
max over ranks is the slowest rank's time, and the reference arm does its
work on rank 0 only.
"""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, nreq, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        reqs = bench.serve_requests(nreq)
        mine = bench.shard(list(range(nreq)), rank, world)
        shares = [None] * world
        dist.all_gather_object(shares, mine)
        # every rank's share holds the same prompts bench would serve there
        assert [reqs[i] for i in mine] == bench.shard(reqs, rank, world)
        mx = bench.max_over_ranks_fn(dist, "cpu")(10.0 * (rank + 1))
        # the reference arm: rank 0 alone runs it, the others return at once
        class A:
            pass
        skipped = bench.run_reference_arm(A(), rank, world) if rank != 0 else None
        dist.barrier()
        q.put((rank, shares, mx, skipped))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,nreq", [(2, 4096), (2, 7)])
def test_request_shards_and_max_over_ranks(world, nreq):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, nreq, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, shares, mx, skipped in results:
        flat = sorted(i for s in shares for i in s)
        assert flat == list(range(nreq))            # a partition: each request served exactly once
        assert max(len(s) for s in shares) - min(len(s) for s in shares) <= 1
        assert mx == 10.0 * world                   # the slowest rank's time
        assert skipped is None


def test_serve_requests_follow_the_config():
    """Config 3: prompt lengths in [16, 128], a shared 24-token prefix."""
    import bench
    reqs = bench.serve_requests(512)
    assert all(16 <= len(r) <= 128 for r in reqs)
    assert all(r[:16] == reqs[0][:16] for r in reqs)
    assert all(r[:24] == reqs[0][:24] for r in reqs if len(r) >= 24)
    longer = [tuple(r) for r in reqs if len(r) > 24]  # shorter ones are all prefix, so some repeat
    assert len(set(longer)) == len(longer)
