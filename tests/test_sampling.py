"""Sampling beyond greedy (top-k / top-p with a seeded counter-based draw).

The oracle's qo_sample states the library's definition in C; these CPU tests pin it
against a plain-Python statement of the same definition and check its properties
(greedy limits, the top-k and top-p cuts, the empirical distribution). The GPU tests
compare the CUDA sampler with it through the C ABI, kernel by kernel and for whole
generations."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def splitmix64(x):
    x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return x ^ (x >> 31)


def py_sample(logits, temperature, top_k, top_p, seed, step):
    """The definition in plain Python (f32 arithmetic through numpy scalars)."""
    logits = np.asarray(logits, np.float32)
    greedy = not (temperature > 0) or top_k == 1
    K = 1 if greedy else (top_k if 1 <= top_k <= 64 else 64)
    K = min(K, logits.size)
    t = np.float32(1.0 if greedy else temperature)
    key = lambda i: (1 if math.isnan(logits[i]) else 0, -float(logits[i]) if not math.isnan(logits[i]) else 0.0, i)  # noqa: E731
    cand = sorted(range(logits.size), key=key)[:K]
    v0 = logits[cand[0]]
    cum, s = [], np.float32(0.0)
    for i, c in enumerate(cand):
        v = logits[c]
        if not math.isnan(v) and not math.isnan(v0):
            p = np.float32(np.exp(np.float32((v - v0) / t), dtype=np.float32))
        else:
            p = np.float32(1.0 if i == 0 else 0.0)
        s = np.float32(s + p)
        cum.append(s)
    m = len(cand) - 1
    if top_p < 1.0:
        for i in range(len(cand)):
            if cum[i] >= np.float32(top_p) * s:
                m = i
                break
    h = splitmix64(seed ^ ((step * 0xD1B54A32D192ED03) & 0xFFFFFFFFFFFFFFFF))
    u = np.float32((h >> 40) * 5.9604644775390625e-08)
    target = np.float32(u * cum[m])
    for i in range(m + 1):
        if cum[i] > target:
            return cand[i]
    return cand[m]


@pytest.mark.parametrize("case", range(40))
def test_oracle_sampler_matches_the_python_statement(case):
    rng = np.random.default_rng(case)
    logits = (rng.standard_normal(int(rng.integers(2, 300))) * rng.uniform(0.2, 4)).astype(np.float32)
    if case % 5 == 0:
        logits[rng.integers(0, logits.size, 3)] = logits.max()          # ties at the top
    params = (float(rng.choice([0.0, 0.5, 1.0, 1.7])), int(rng.choice([0, 1, 5, 40, 64, 100])),
              float(rng.choice([0.3, 0.9, 1.0])), int(rng.integers(0, 2**63)), int(rng.integers(0, 10**6)))
    assert O.sample(logits, *params) == py_sample(logits, *params)


def test_greedy_limits_are_the_argmax_with_the_lowest_index():
    logits = np.array([0.5, 2.0, -1.0, 2.0, 1.9], np.float32)
    for temperature, top_k in ((0.0, 0), (-1.0, 10), (1.0, 1)):
        assert O.sample(logits, temperature, top_k, 1.0, 123, 7) == 1


def test_top_k_and_top_p_cut_the_candidates():
    rng = np.random.default_rng(5)
    logits = rng.standard_normal(5000).astype(np.float32)
    order = np.argsort(-logits, kind="stable")
    top5 = set(order[:5].tolist())
    got = {O.sample(logits, 1.5, 5, 1.0, 11, s) for s in range(400)}
    assert got <= top5 and len(got) > 1
    # a peaked distribution: top_p = 0.5 keeps only the most likely token
    peaked = logits.copy()
    peaked[order[0]] += 10.0
    assert {O.sample(peaked, 1.0, 0, 0.5, 3, s) for s in range(200)} == {int(order[0])}


def test_draws_follow_the_softmax():
    logits = np.array([1.0, 0.2, -0.5, 2.0, 0.0], np.float32)
    n = 20000
    counts = np.bincount([O.sample(logits, 0.8, 0, 1.0, 99, s) for s in range(n)], minlength=5)
    p = np.exp((logits - logits.max()) / 0.8)
    p /= p.sum()
    assert np.all(np.abs(counts / n - p) < 0.015), (counts / n, p)


def test_nan_ranks_below_every_number():
    logits = np.array([np.nan, -1e30, np.nan, -3.0], np.float32)
    assert O.sample(logits, 0.0, 0, 1.0, 0, 0) == 3
    assert {O.sample(logits, 1.0, 2, 1.0, 4, s) for s in range(50)} <= {1, 3}


# ---- the CUDA sampler through the C ABI --------------------------------------------

def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [1, 3, 7, 63])
def test_cuda_sampler_vocab_below_the_candidate_count(vocab):
    """Fewer tokens than candidates (K = 64): the padding candidates of the short chunk
    are never drawn and the draw matches the oracle, whatever the seed."""
    torch = _cuda()
    from kernel_optimization_webgpu_b200 import runtime as R
    rng = np.random.default_rng(100 + vocab)
    for case in range(60):
        logits = (rng.standard_normal(vocab) * 2.0).astype(np.float32)
        params = (float(rng.choice([0.5, 1.0, 3.0])), int(rng.choice([0, 64, 100])), float(rng.choice([0.5, 1.0])),
                  int(rng.integers(0, 2**63)), int(rng.integers(0, 10**6)))
        got = R.sample_logits(torch.from_numpy(logits).cuda(), *params)
        assert 0 <= got < vocab, (vocab, case, params, got)
        assert got == O.sample(logits, *params), (vocab, case, params)


@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [7, 1000, 4099, 151936])
def test_cuda_sampler_matches_the_oracle(vocab):
    torch = _cuda()
    from kernel_optimization_webgpu_b200 import runtime as R
    rng = np.random.default_rng(vocab)
    for case in range(40):
        logits = (rng.standard_normal(vocab) * rng.uniform(0.2, 4)).astype(np.float32)
        if case % 4 == 0:
            logits[rng.integers(0, vocab, 3)] = logits.max()   # ties at the top
        if case % 7 == 0:
            logits[rng.integers(0, vocab, 2)] = np.nan
        params = (float(rng.choice([0.0, 0.5, 1.0, 1.7])), int(rng.choice([0, 1, 5, 40, 64, 100])),
                  float(rng.choice([0.3, 0.9, 1.0])), int(rng.integers(0, 2**63)), int(rng.integers(0, 10**6)))
        got = R.sample_logits(torch.from_numpy(logits).cuda(), *params)
        assert got == O.sample(logits, *params), (vocab, case, params)


@pytest.mark.gpu
@pytest.mark.parametrize("persistent", [1, 0])
def test_engine_sampled_generation_matches_the_oracle(tiny_runtime, persistent):
    _cuda()
    from kernel_optimization_webgpu_b200 import runtime as R
    prompt = [17, 4000, 3, 999]
    model = O.Model(tiny_runtime)
    with R.Engine(tiny_runtime, max_seq=64, persistent=persistent) as eng:
        for temperature, top_k, top_p, seed in ((0.9, 40, 0.9, 7), (1.3, 0, 0.95, 12345), (0.6, 5, 1.0, 3)):
            ids, st = eng.generate_sample(prompt, 16, temperature, top_k, top_p, seed)
            want = model.session(max_seq=64, kv_f16=True).sample(prompt, 16, temperature, top_k, top_p, seed)
            assert ids == want, (temperature, top_k, top_p, seed)
            assert st["generated_tokens"] == 16
        greedy, _ = eng.generate_greedy(prompt, 10)
        assert eng.generate_sample(prompt, 10, 0.0, 0, 1.0, 5)[0] == greedy
        assert eng.generate_sample(prompt, 10, 1.0, 1, 1.0, 5)[0] == greedy
        with pytest.raises(R.QdError):
            eng.generate_sample(prompt, 4, 1.0, 0, 1.5, 5)   # top_p beyond 1
