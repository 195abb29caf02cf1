"""Multi-GPU checks that need two or more GPUs (skipped on a single-GPU box):
the vocabulary-sharded LM head over NCCL against the replicated one."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_vocab_sharded_lm_head_over_nccl_two_ranks():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29517",
           os.path.join(ROOT, "tests", "multigpu_vocab_shard.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert res.stdout.count(" OK") == 2, res.stdout
