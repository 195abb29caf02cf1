import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def tiny_runtime(tmp_path_factory):
    """The small seeded model in the reference's runtime layout."""
    from kernel_optimization_webgpu_b200 import synth
    d = str(tmp_path_factory.mktemp("tiny_runtime"))
    synth.write_runtime(d, synth.TINY, seed=2)
    return d


@pytest.fixture(scope="session")
def qwen_runtime(tmp_path_factory):
    """Qwen3-0.6B-shape random-init weights (seed 2) in the reference's runtime layout."""
    from kernel_optimization_webgpu_b200 import synth
    d = str(tmp_path_factory.mktemp("qwen_seed2"))
    synth.write_runtime(d, synth.QWEN3_0_6B, seed=2)
    return d


@pytest.fixture(scope="session")
def qwen_runtime_centered(tmp_path_factory):
    """Qwen3-0.6B-shape random-init weights (seed 5) with nibbles centred on the zero
    point: a model whose greedy ids change from step to step."""
    from kernel_optimization_webgpu_b200 import synth
    d = str(tmp_path_factory.mktemp("qwen_seed5_centered"))
    synth.write_runtime(d, synth.QWEN3_0_6B, seed=5, nibbles="centered")
    return d
