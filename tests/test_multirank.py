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


# ---- vocabulary-sharded LM head: the per-step protocol over two gloo ranks ------------------

class _FakeShardBatch:
    """Stands in for a Batch on CPU (numpy for the device work, the library's rules
    restated): deterministic hidden rows per (rank, sequence, step), a shared vocabulary
    table with duplicated rows so that exact ties straddle the slice boundary, each rank's
    slice argmax (ties: lowest index), and the merge over the ranks' candidates."""

    def __init__(self, rank, world, B=3, H=8, V=41):
        import numpy as np
        self.np = np
        self.rank, self.world, self.batch, self.H, self.V = rank, world, B, H, V
        rng = np.random.Generator(np.random.PCG64(7))
        table = rng.standard_normal((V, H)).astype(np.float32)
        self.tie = V // 2                  # the slice boundary of two ranks
        table[self.tie] = table[self.tie - 1]
        self.table = table
        rows = world * B
        self._shard = (rank, world, {
            "gather_hi": torch.zeros((rows, H)), "gather_lo": torch.zeros((rows, H)),
            "pairs_local": torch.zeros((rows, 2), dtype=torch.int64),
            "pairs_all": torch.zeros((world, rows, 2), dtype=torch.int64)})
        self.tokens = [rank * 100 + b for b in range(B)]
        self.ids, self.step = [], 0

    def hidden(self, rank, b, step, token):
        np = self.np
        h = np.random.Generator(np.random.PCG64(1000 * rank + 10 * b + step)).standard_normal(self.H)
        h = h.astype(np.float32)
        if b == 0:                          # steer row 0 of every rank onto the tied pair
            h = self.table[self.tie].copy() * 10
        return h

    def step_layers(self):
        bufs = self._shard[2]
        for b in range(self.batch):
            h = torch.from_numpy(self.hidden(self.rank, b, self.step, self.tokens[b]))
            bufs["gather_hi"][self.rank * self.batch + b] = h
            bufs["gather_lo"][self.rank * self.batch + b] = 0.0

    def step_lm_slice(self):
        np = self.np
        bufs = self._shard[2]
        v0, v1 = self.V * self.rank // self.world, self.V * (self.rank + 1) // self.world
        x = (bufs["gather_hi"] + bufs["gather_lo"]).numpy()
        logits = x @ self.table[v0:v1].T
        for r in range(logits.shape[0]):
            i = int(np.argmax(logits[r]))           # first maximum: lowest index
            bufs["pairs_local"][r, 0] = v0 + i
            bufs["pairs_local"][r, 1] = int(np.float32(logits[r, i]).view(np.int32))

    def step_merge(self):
        np = self.np
        bufs = self._shard[2]
        out = []
        for b in range(self.batch):
            best_v, best_i = None, None
            for w in range(self.world):
                i = int(bufs["pairs_all"][w, self.rank * self.batch + b, 0])
                v = float(np.int32(int(bufs["pairs_all"][w, self.rank * self.batch + b, 1])).view(np.float32))
                if best_v is None or v > best_v or (v == best_v and i < best_i):
                    best_v, best_i = v, i
            out.append(best_i)
        self.tokens = out
        self.ids.append(out)
        self.step += 1

    def shard_sync(self, n):
        ids, self.ids = self.np.array(self.ids[-n:], self.np.int32), self.ids[:-n]
        return ids


def _gather(out, inp):
    parts = [torch.zeros_like(inp) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, inp.contiguous())
    out.copy_(torch.stack(parts).reshape(out.shape))


def _shard_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kernel_optimization_webgpu_b200 import runtime as R
        fake = _FakeShardBatch(rank, world)
        ids = R.sharded_decode(fake, 3, _gather)
        # reference: the full-vocabulary argmax of the same hidden rows, on this rank alone
        ref = _FakeShardBatch(rank, 1)
        ref.table = fake.table
        want = []
        for step in range(3):
            row = []
            for b in range(fake.batch):
                logits = fake.table @ ref.hidden(rank, b, step, 0)
                row.append(int(fake.np.argmax(logits)))
            want.append(row)
        out[rank] = (ids.tolist(), want)
    finally:
        dist.destroy_process_group()


def test_two_ranks_vocab_sharded_lm_head_protocol():
    """R.sharded_decode over two gloo ranks: each rank's merged ids equal the
    full-vocabulary argmax of its own rows, including an exact tie across the slice
    boundary (the lower index wins)."""
    world, port = 2, _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_shard_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for rank in range(world):
        got, want = res[rank]
        assert got == want, rank
        tied = _FakeShardBatch(0, world).tie - 1
        assert got[0][0] == tied            # the tie resolved to the lower index
