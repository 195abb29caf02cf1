"""qd_gqa_decode_noalloc: decode attention for callers that cannot allocate.

Some hosts cannot call cudaMalloc when they call into the library (their own pool
owns the device memory, or they cannot take the synchronisation a cudaFree may
cause). For them the library keeps the split-KV partials in a fixed device array
of QD_NOALLOC_SCRATCH_BYTES instead of a caller-allocated workspace. These tests
call it through the C ABI and check it against qd_gqa_decode, on two calls in a
row with different sizes (the shared array keeps the previous call's contents),
and check that a size whose partials do not fit is refused with a clear error.
The file is named to be collected last; it also passes on its own.
"""
import ctypes as C

import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import _lib

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-4  # same bound as the other parity tests: max |diff| / max |reference|


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def _inputs(seq, kv_dtype, seed):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal(16 * 128).astype(np.float32)).cuda()
    dt = np.float16 if kv_dtype == _lib.QD_KV_F16 else np.float32
    k = torch.from_numpy(rng.standard_normal((seq, 8, 128)).astype(dt)).cuda()
    v = torch.from_numpy(rng.standard_normal((seq, 8, 128)).astype(dt)).cuda()
    return q, k, v


def _with_workspace(L, q, k, v, seq, kv_dtype):
    y = torch.empty(16 * 128, device="cuda")
    ws = torch.empty(L.qd_gqa_decode_workspace_bytes(seq, 16), dtype=torch.uint8, device="cuda")
    rc = L.qd_gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_dtype, y.data_ptr(), seq, 16, 8, 128,
                         ws.data_ptr(), None)
    assert rc == 0, L.qd_last_error(None)
    return y


def _no_alloc(L, q, k, v, seq, kv_dtype):
    y = torch.empty(16 * 128, device="cuda")
    rc = L.qd_gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_dtype, y.data_ptr(), seq, 16, 8,
                                 128, None)
    assert rc == 0, L.qd_last_error(None)
    return y


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    L = _lib.load()
    cases = [(700, _lib.QD_KV_F16, 1), (37, _lib.QD_KV_F32, 2)]  # 3 splits, then 1
    for seq, kv_dtype, seed in cases:
        q, k, v = _inputs(seq, kv_dtype, seed)
        got = _no_alloc(L, q, k, v, seq, kv_dtype)
        want = _with_workspace(L, q, k, v, seq, kv_dtype)
        torch.cuda.synchronize()
        assert _rel(got.cpu().numpy(), want.cpu().numpy()) < TOL, (seq, kv_dtype)


def test_noalloc_refuses_sizes_beyond_its_fixed_scratch():
    L = _lib.load()
    p = C.c_void_p(256)
    # 16 query heads need about 8.3 KB of partials per 256 positions: 20000 positions do not fit.
    rc = L.qd_gqa_decode_noalloc(p, p, p, _lib.QD_KV_F16, p, 20000, 16, 8, 128, None)
    assert rc == _lib.QD_E_RANGE
    assert b"QD_NOALLOC_SCRATCH_BYTES" in L.qd_last_error(None)
