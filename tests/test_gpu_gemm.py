"""tcgen05 q4 GEMM (qd_q4_gemm) vs the oracle's per-row matvecs (needs a B200)."""
import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import runtime as R
from kernel_optimization_webgpu_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (3, 3072, 1024), (64, 1024, 3072), (64, 2048, 1024),
                                   (100, 200, 128), (300, 1024, 2048), (1000, 384, 1024)])
def test_q4_gemm_matches_oracle_rows(m, n, k):
    _, w, s = synth.matvec_case(n, k, seed=11)
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    y = R.q4_gemm(torch.from_numpy(x).cuda(), torch.from_numpy(w.view(np.int32)).cuda(),
                  torch.from_numpy(s.astype(np.float16)).cuda())
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    want = np.stack([O.q4_matvec(x[i], w, s) for i in range(m)])
    assert rel(y, want) < 1e-5
