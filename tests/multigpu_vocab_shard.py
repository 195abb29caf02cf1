"""Vocabulary-sharded LM head over NCCL, one rank per GPU (launched by
tests/test_zy_multigpu.py through torchrun): each rank decodes its own batch of
the small seeded model with the replicated LM head, then the same batch with the
LM head split by vocabulary across the ranks (all-gathers over NCCL); the ids must
be identical. Prints one line per rank; exits non-zero on a mismatch."""
import os
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from kernel_optimization_webgpu_b200 import runtime as R  # noqa: E402
from kernel_optimization_webgpu_b200 import synth  # noqa: E402


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    B, ctx, steps = 4, 40, 6
    with tempfile.TemporaryDirectory() as d:
        synth.write_runtime(d, synth.TINY, seed=2)
        stream = torch.cuda.Stream()
        with R.Engine(d, device=local, max_seq=64) as eng:
            eng.set_stream(stream)
            tokens = np.random.Generator(np.random.PCG64(100 + rank)).integers(0, synth.TINY.vocab, size=B)
            with R.Batch(eng, B, ctx + steps + 1) as bt:
                bt.fill_context(ctx, 30 + rank)
                bt.set_tokens(tokens, [ctx] * B)
                want = bt.decode(steps)
            with R.Batch(eng, B, ctx + steps + 1) as bt, torch.cuda.stream(stream):
                bt.fill_context(ctx, 30 + rank)
                bt.set_tokens(tokens, [ctx] * B)
                bt.set_vocab_shard(rank, world)
                got = bt.decode_sharded(steps, lambda out, inp: dist.all_gather_into_tensor(out, inp))
            eng.set_stream(None)
    ok = got.tolist() == want.tolist()
    print(f"rank {rank}/{world}: sharded {got[:, 0].tolist()} replicated {want[:, 0].tolist()} {'OK' if ok else 'MISMATCH'}",
          flush=True)
    flags = [None] * world
    dist.all_gather_object(flags, ok)
    dist.destroy_process_group()
    return 0 if all(flags) else 1


if __name__ == "__main__":
    sys.exit(main())
