"""Multi-rank host logic on CPU (gloo, world size 2): the sharding of independent
prompts over ranks and the max-over-ranks device time the benchmark reports."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        lo, hi = bench.shard_range(32, world, rank)
        t = bench.max_over_ranks(1.0 + 2.0 * rank, world)
        shards = [None] * world
        dist.all_gather_object(shards, (lo, hi))
        out[rank] = (lo, hi, t, shards)
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_prompts_and_take_max_time():
    world, port = 2, _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    assert res[0][:2] == (0, 16) and res[1][:2] == (16, 32)
    assert res[0][2] == res[1][2] == 3.0          # both ranks report the slowest rank's time
    assert res[0][3] == [(0, 16), (16, 32)]       # disjoint shards covering all prompts


def test_shard_range_rejects_uneven_split():
    import bench
    with pytest.raises(ValueError):
        bench.shard_range(32, 3, 0)
    assert bench.shard_range(64, 8, 7) == (56, 64)
