"""Failure detection on the GPU without a fault.

Every device-side wait of the decode kernels has a deadline. These tests make one
wait run out on purpose through the library's test hooks (a result that is never
published, so nothing the waiting threads poll for ever arrives), then check that
the call reports QD_E_TIMEOUT within a few seconds and that the same engine or
batch decodes correctly afterwards. Nothing here traps, faults or hangs a GPU: the
waits end by their own deadlines (200 ms in the persistent decode kernel, 1 s in the
tensor-core GEMM) and every kernel returns.

The reference's counterpart is the A/B page's error guard, which refuses to report
results after a device error (src/bench/ab-page.js:158-161,181-187).
"""
import time

import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import _lib
from kernel_optimization_webgpu_b200 import runtime as R

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_persistent_decode_wait_runs_out_and_the_engine_recovers(tiny_runtime):
    prompt = [17, 4000, 3, 999]
    with R.Engine(tiny_runtime, max_seq=32, persistent=1) as eng:
        assert eng.token_kernel == 1
        want, _ = eng.generate_greedy(prompt, 5)
        eng.inject_stall()
        t0 = time.monotonic()
        with pytest.raises(_lib.QdError) as ex:
            eng.generate_greedy(prompt, 5)
        assert ex.value.code == _lib.QD_E_TIMEOUT
        assert time.monotonic() - t0 < 20.0
        for _ in range(2):  # the repair holds for every later launch
            ids, _ = eng.generate_greedy(prompt, 5)
            assert ids == want


def test_persistent_stall_hook_needs_the_persistent_kernel(tiny_runtime):
    with R.Engine(tiny_runtime, max_seq=32, persistent=0) as eng:
        with pytest.raises(_lib.QdError) as ex:
            eng.inject_stall()
        assert ex.value.code == _lib.QD_E_INVALID


def test_gemm_wait_runs_out_and_the_batch_recovers(tiny_runtime):
    rng = np.random.Generator(np.random.PCG64(11))
    with R.Engine(tiny_runtime, max_seq=64) as eng, R.Batch(eng, 3, 96) as bt:
        tokens = rng.integers(0, eng.profile["vocab"], size=3).astype(np.int32)
        bt.fill_context(40, 5)
        bt.set_tokens(tokens, [40, 40, 40])
        want = bt.decode(4)
        bt.set_tokens(tokens, [40, 40, 40])
        bt.inject_stall()
        t0 = time.monotonic()
        with pytest.raises(_lib.QdError) as ex:
            bt.decode(4)
        assert ex.value.code == _lib.QD_E_TIMEOUT
        assert time.monotonic() - t0 < 30.0
        # the failed steps wrote rows 40..43; the retry rewrites each before reading it
        bt.set_tokens(tokens, [40, 40, 40])
        assert np.array_equal(bt.decode(4), want)
        # and a prefill afterwards is unaffected as well
        first = bt.prefill(rng.integers(0, eng.profile["vocab"], size=(3, 20)).astype(np.int32))
        assert first.shape == (3,)
