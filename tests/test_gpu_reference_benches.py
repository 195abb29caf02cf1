"""The reference's benchmark exports (runKernelBenchmarks, runFullDecoderStackBenchmark,
webgpu-runtime.js:62-163) through the C ABI on the GPU: the same result fields, finite
timings, and each kernel's result close to the double-precision CPU evaluation of its
math (the reference reports these errors; here they are also bounded)."""
import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import runtime as R
from kernel_optimization_webgpu_b200 import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

KERNEL_FIELDS = {"baselineMatvecMs", "optimizedMatvecMs", "matvecSpeedup", "baselineBytes", "optimizedBytes",
                 "memoryReduction", "maxAbsError", "meanAbsError", "blockDefaultMs", "blockOptimizedMs",
                 "blockSpeedup", "blockMaxAbsError", "blockMeanAbsError", "realQ4Ms", "realQ4MaxAbsError",
                 "realQ4MeanAbsError", "gqaMs", "gqaMaxAbsError", "gqaMeanAbsError", "gqaSeqLen",
                 "layer0DecodeMs", "layer0Finite", "layer0MeanAbs", "rmsMs", "estimatedGbps"}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("shape", ["tiny", "qwen"])
def test_run_kernel_benchmarks(shape, tiny_runtime, qwen_runtime):
    rt, sh = (tiny_runtime, synth.TINY) if shape == "tiny" else (qwen_runtime, synth.QWEN3_0_6B)
    ctx = R.createWebGpuContext(rt)
    prof = dict(R.qwenProfile, hiddenSize=sh.hidden, intermediateSize=sh.intermediate, attentionHeads=sh.heads,
                kvHeads=sh.kv_heads)
    res = R.runKernelBenchmarks(ctx["device"], prof)
    assert set(res) == KERNEL_FIELDS
    for key in ("baselineMatvecMs", "optimizedMatvecMs", "blockDefaultMs", "blockOptimizedMs", "realQ4Ms", "gqaMs",
                "layer0DecodeMs", "rmsMs"):
        assert 0.0 < res[key] < 50.0, (key, res[key])
    # bounds at ~1e-5 of each output's peak magnitude (q8 matvec ~14, MLP block ~4400)
    assert res["maxAbsError"] < 2e-4 and res["blockMaxAbsError"] < 5e-2
    assert res["realQ4MaxAbsError"] < 1e-4 and res["gqaMaxAbsError"] < 1e-5
    assert res["gqaSeqLen"] == 128
    assert res["layer0Finite"] == sh.hidden and res["layer0MeanAbs"] > 0.0
    assert res["baselineBytes"] == res["optimizedBytes"] == sh.hidden * 4 + sh.hidden * sh.intermediate + \
        sh.intermediate * 4
    assert res["memoryReduction"] == 1.0
    # the engine decodes as before after the benchmarks overwrote its state
    eng = ctx["device"].engine(1, "optimized")
    ids, _ = eng.generate_greedy([5, 6, 7], 4)
    with R.Engine(rt, max_seq=64) as fresh:
        want, _ = fresh.generate_greedy([5, 6, 7], 4)
    assert ids == want
    ctx["device"].close()


def test_run_full_decoder_stack_benchmark(tiny_runtime):
    ctx = R.createWebGpuContext(tiny_runtime)
    res = R.runFullDecoderStackBenchmark(ctx["device"], {"hiddenSize": synth.TINY.hidden})
    assert set(res) == {"ms", "warmupMs", "layers", "finite", "meanAbs"}
    assert res["layers"] == synth.TINY.layers and res["finite"] == synth.TINY.hidden
    assert res["ms"] > 0.0 and res["warmupMs"] > 0.0 and np.isfinite(res["meanAbs"]) and res["meanAbs"] > 0.0
    with pytest.raises(ValueError):
        R.runFullDecoderStackBenchmark(ctx["device"], {"hiddenSize": 1024})
    ctx["device"].close()
