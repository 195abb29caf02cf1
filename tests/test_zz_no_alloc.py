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
import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import _lib

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-4  # same bound as the other parity tests: max |diff| / max |reference|


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def _inputs(seq, kv_dtype, seed, q_heads=16, kv_heads=8):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal(q_heads * 128).astype(np.float32)).cuda()
    dt = np.float16 if kv_dtype == _lib.QD_KV_F16 else np.float32
    k = torch.from_numpy(rng.standard_normal((seq, kv_heads, 128)).astype(dt)).cuda()
    v = torch.from_numpy(rng.standard_normal((seq, kv_heads, 128)).astype(dt)).cuda()
    return q, k, v


def _with_workspace(L, q, k, v, seq, kv_dtype, q_heads=16, kv_heads=8):
    y = torch.empty(q_heads * 128, device="cuda")
    ws = torch.empty(L.qd_gqa_decode_workspace_bytes(seq, q_heads), dtype=torch.uint8, device="cuda")
    rc = L.qd_gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_dtype, y.data_ptr(), seq, q_heads, kv_heads,
                         128, ws.data_ptr(), None)
    assert rc == 0, L.qd_last_error(None)
    return y


def _no_alloc(L, q, k, v, seq, kv_dtype, q_heads=16, kv_heads=8):
    y = torch.empty(q_heads * 128, device="cuda")
    rc = L.qd_gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_dtype, y.data_ptr(), seq, q_heads,
                                 kv_heads, 128, None)
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


@pytest.mark.parametrize("q_heads,kv_heads", [(8, 8), (16, 8), (16, 4), (16, 2)])
def test_noalloc_matches_the_oracle_for_every_group_size(q_heads, kv_heads):
    """Query heads per KV head 1, 2, 4 and 8, against the CPU restatement of
    gqa_decode.wgsl (f16 cache values read back as f32, as the kernel reads them)."""
    from oracle import oracle as O
    L = _lib.load()
    for seq, kv_dtype, seed in ((300, _lib.QD_KV_F16, 5), (513, _lib.QD_KV_F32, 6)):
        q, k, v = _inputs(seq, kv_dtype, seed, q_heads, kv_heads)
        got = _no_alloc(L, q, k, v, seq, kv_dtype, q_heads, kv_heads)
        torch.cuda.synchronize()
        want = O.gqa_decode(q.cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), seq, q_heads,
                            kv_heads, 128)
        assert _rel(got.cpu().numpy(), want) < TOL, (q_heads, kv_heads, seq)


def test_noalloc_at_the_edge_of_its_fixed_scratch():
    """16 query heads fill the 512 KiB exactly at 16128 positions (63 splits of 256:
    8 KiB of (max, sum) pairs, then 63 * 16 * 512 bytes of outputs); 16129 positions
    need a 64th split and are refused before any launch."""
    L = _lib.load()
    q, k, v = _inputs(16129, _lib.QD_KV_F16, 7)
    got = _no_alloc(L, q, k, v, 16128, _lib.QD_KV_F16)
    want = _with_workspace(L, q, k, v, 16128, _lib.QD_KV_F16)
    torch.cuda.synchronize()
    assert _rel(got.cpu().numpy(), want.cpu().numpy()) < TOL
    y = torch.empty(16 * 128, device="cuda")
    rc = L.qd_gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.QD_KV_F16, y.data_ptr(), 16129,
                                 16, 8, 128, None)
    assert rc == _lib.QD_E_RANGE
    assert b"QD_NOALLOC_SCRATCH_BYTES" in L.qd_last_error(None)


def test_noalloc_refuses_sizes_beyond_its_fixed_scratch():
    L = _lib.load()
    # Real tensors of the requested size, so nothing can reach an invalid address
    # whatever order the entry checks and launches in.
    q, k, v = _inputs(20000, _lib.QD_KV_F16, 3)
    y = torch.empty(16 * 128, device="cuda")
    rc = L.qd_gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.QD_KV_F16, y.data_ptr(), 20000,
                                 16, 8, 128, None)
    assert rc == _lib.QD_E_RANGE
    assert b"QD_NOALLOC_SCRATCH_BYTES" in L.qd_last_error(None)
