"""CUDA path vs the CPU oracle through the C ABI (needs a B200).

Tolerances: the contract allows 1e-2 relative for logits and matvec outputs; the
kernels accumulate in f32 like the reference, so these tests hold them to a
tighter 1e-4 (max |diff| / max |reference|) and greedy ids to bit-exact.
"""
import json
import math
import os

import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import runtime as R
from kernel_optimization_webgpu_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-4


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def run_matvec(x, w, s, in_size=None):
    y = R.q4_matvec(dev(x), dev(w.view(np.int32)), dev(s.astype(np.float16)), in_size=in_size)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("n,k", [(3072, 1024), (2048, 1024), (1024, 2048), (1024, 3072),
                                 (4096, 1024), (6144, 1024)])
def test_q4_matvec_config0_shapes(n, k):
    x, w, s = synth.matvec_case(n, k, seed=0)
    assert rel(run_matvec(x, w, s), O.q4_matvec(x, w, s)) < TOL


def test_q4_matvec_matches_golden_js_port():
    refs = np.load(os.path.join(GOLDEN, "js_cpu_refs.npz"))
    for name, (n, k) in {"gate": (3072, 1024), "q": (2048, 1024), "o": (1024, 2048),
                         "down": (1024, 3072)}.items():
        x, w, s = synth.matvec_case(n, k, seed=0)
        assert rel(run_matvec(x, w, s), refs[f"q4_{name}_y"]) < TOL, name


@pytest.mark.parametrize("n,k,in_size", [(1, 1024, 1024), (7, 512, 512), (33, 256, 250),
                                         (129, 4096, 4096), (5000, 96, 90)])
def test_q4_matvec_ragged_shapes(n, k, in_size):
    x, w, s = synth.matvec_case(n, k, seed=7)
    assert rel(run_matvec(x, w, s, in_size), O.q4_matvec(x, w, s, in_size=in_size)) < TOL


def lm_head(table, h, norm_weight=None, eps=1e-6):
    logits = torch.empty(table.shape[0], dtype=torch.float32, device="cuda")
    nw = dev(norm_weight) if norm_weight is not None else None
    r = R.lm_head_argmax(dev(h), dev(table.view(np.uint16), torch.float16), nw, eps, logits=logits)
    torch.cuda.synchronize()
    r = r.cpu().numpy().view(np.uint32)
    return int(r[0]), float(r[1:2].view(np.float32)[0]), logits.cpu().numpy()


def test_lm_head_argmax_config1():
    table, x, eps = synth.lm_head_case()
    ones = np.ones(1024, np.float32)
    idx, val, logits = lm_head(table, x, ones, eps)
    h = O.rms_norm(x, ones, eps)
    want = O.lm_head_f16(h, table)
    assert rel(logits, want) < TOL
    oi, ov = O.argmax(want)
    assert idx == oi
    assert val == logits[idx]
    # the winner must be clear of the numerical noise for an exact index match to mean anything
    srt = np.sort(want)
    assert srt[-1] - srt[-2] > 1e-4


@pytest.mark.parametrize("case", ["all_ties", "last_wins", "dup_far_apart", "nan_row", "all_neg_inf"])
def test_lm_head_argmax_adversarial(case):
    V, H = 151936, 1024
    h = np.ones(H, np.float32)
    table = np.zeros((V, H), np.float16)
    if case == "last_wins":
        table[-1] = 1.0
    elif case == "dup_far_apart":
        table[[90001, 3, 151935, 77777]] = 0.5
    elif case == "nan_row":
        table[5] = np.nan
        table[6] = 0.25
    elif case == "all_neg_inf":
        table[:] = -np.inf
    idx, val, logits = lm_head(table, h)
    want = {"all_ties": 0, "last_wins": V - 1, "dup_far_apart": 3, "nan_row": 6, "all_neg_inf": 0}[case]
    assert idx == want
    oi, ov = O.argmax(logits)
    assert idx == oi and val == ov
    if case == "all_neg_inf":
        assert val == float(np.float32(-3.4028234e38))


@pytest.mark.parametrize("seq", [1, 7, 128, 256, 257, 700, 2049])
@pytest.mark.parametrize("kv", ["f16", "f32"])
def test_gqa_decode_vs_oracle(seq, kv):
    rng = np.random.default_rng(seq)
    q = rng.standard_normal(16 * 128).astype(np.float32)
    k = rng.standard_normal((seq, 8, 128)).astype(np.float32)
    v = rng.standard_normal((seq, 8, 128)).astype(np.float32)
    if kv == "f16":
        k, v = k.astype(np.float16), v.astype(np.float16)
    y = R.gqa_decode(dev(q), dev(k), dev(v), seq, 16, 8)
    torch.cuda.synchronize()
    want = O.gqa_decode(q, k.astype(np.float32), v.astype(np.float32), seq, 16, 8, 128)
    assert rel(y.cpu().numpy(), want) < TOL


def test_gqa_decode_matches_golden_js_port():
    refs = np.load(os.path.join(GOLDEN, "js_cpu_refs.npz"))
    cv = lambda n, step, fn: np.array([fn(i * step) for i in range(n)], np.float64).astype(np.float32)  # noqa
    q = cv(16 * 128, 0.011, math.sin)
    k = cv(128 * 8 * 128, 0.007, math.cos)
    v = cv(128 * 8 * 128, 0.013, math.sin)
    y = R.gqa_decode(dev(q), dev(k), dev(v), 128, 16, 8)
    torch.cuda.synchronize()
    assert rel(y.cpu().numpy(), refs["gqa_y"]) < TOL


# ---- whole engine ---------------------------------------------------------------

@pytest.fixture(scope="module")
def tiny_model(tiny_runtime):
    return O.Model(tiny_runtime)


@pytest.mark.parametrize("kv", ["f16", "f32"])
def test_engine_layer_trace_matches_oracle(tiny_runtime, tiny_model, kv):
    with R.Engine(tiny_runtime, max_seq=64, kv_dtype=kv) as eng:
        sess = tiny_model.session(max_seq=64, kv_f16=(kv == "f16"))
        for pos, tok in enumerate([11, 4000, 7, 123]):
            got = eng.forward_trace(tok, pos)
            want = sess.forward(tok, pos, trace=True)
            for layer in range(got.shape[0]):
                assert rel(got[layer], want[layer]) < TOL, (pos, layer)


# persistent: 1 = the persistent kernel, 0 = one kernel per stage
@pytest.mark.parametrize("use_graph,persistent", [(True, 1), (False, 1), (True, 0), (False, 0)])
def test_engine_greedy_tiny_matches_oracle_f16_kv(tiny_runtime, tiny_model, use_graph, persistent):
    with open(os.path.join(GOLDEN, "tiny_seed2_greedy.json")) as f:
        g = json.load(f)
    with R.Engine(tiny_runtime, max_seq=64, use_graph=use_graph, persistent=persistent) as eng:
        assert eng.token_kernel == persistent
        ids, st = eng.generate_greedy(g["prompt"], g["max_new"])
        sess = tiny_model.session(max_seq=64, kv_f16=True)
        want, margins = sess.greedy(g["prompt"], g["max_new"])
        assert ids == want
        assert st["generated_tokens"] == g["max_new"]
        # final hidden state after the last fed token, and the last step's logits
        _, logits, _ = sess.next_token()
        assert rel(eng.logits(), logits) < TOL
        assert rel(eng.hidden(), sess.hidden()) < TOL


@pytest.mark.parametrize("persistent", [1, 0])
def test_engine_greedy_tiny_f32_kv_matches_js_port_golden(tiny_runtime, persistent):
    with open(os.path.join(GOLDEN, "tiny_seed2_greedy.json")) as f:
        g = json.load(f)
    with R.Engine(tiny_runtime, max_seq=64, kv_dtype="f32", persistent=persistent) as eng:
        assert eng.token_kernel == persistent
        ids, _ = eng.generate_greedy(g["prompt"], 1)
        first = np.load(os.path.join(GOLDEN, "tiny_seed2_first_logits.npy"))
        assert rel(eng.logits(), first) < TOL
        ids, _ = eng.generate_greedy(g["prompt"], g["max_new"])
        assert ids == g["generated"]


@pytest.mark.parametrize("persistent", [1, 0])
def test_engine_long_prompt_matches_oracle(tiny_runtime, tiny_model, persistent):
    """A 300-token prompt: each attention warp walks ~19 cached positions (the K/V
    prefetch pipeline refills in the loop)."""
    rng = np.random.Generator(np.random.PCG64(8))
    prompt = rng.integers(0, tiny_model.vocab, size=300).tolist()
    with R.Engine(tiny_runtime, max_seq=320, persistent=persistent) as eng:
        assert eng.token_kernel == persistent
        ids, _ = eng.generate_greedy(prompt, 6)
        sess = tiny_model.session(max_seq=320, kv_f16=True)
        want, margins = sess.greedy(prompt, 6)
        assert ids == want, (ids, want, margins.tolist())
        _, logits, _ = sess.next_token()
        assert rel(eng.logits(), logits) < TOL


def test_engine_callback_order_and_early_stop(tiny_runtime):
    seen = []
    with R.Engine(tiny_runtime, max_seq=64) as eng:
        full, _ = eng.generate_greedy([1, 2, 3], 10)
        ids, st = eng.generate_greedy([1, 2, 3], 10, on_token=seen.append)
        assert seen == ids == full
        seen2 = []
        ids2, _ = eng.generate_greedy([1, 2, 3], 10, on_token=lambda t: (seen2.append(t), len(seen2) < 4)[1])
        assert ids2 == full[:4] and seen2 == full[:4]


def test_engine_rejects_bad_requests(tiny_runtime):
    with R.Engine(tiny_runtime, max_seq=16) as eng:
        with pytest.raises(R.QdError) as ex:
            eng.generate_greedy(list(range(10)), 8)          # 10 + 8 - 1 > 16
        assert ex.value.code == -5
        with pytest.raises(R.QdError):
            eng.generate_greedy([synth.TINY.vocab], 1)        # id outside the vocabulary
        ids, _ = eng.generate_greedy(list(range(10)), 7)      # exactly fits
        assert len(ids) == 7


def test_reference_api_mirror(tiny_runtime):
    ctx = R.createWebGpuContext(tiny_runtime)
    prof = dict(R.qwenProfile, hiddenSize=synth.TINY.hidden, intermediateSize=synth.TINY.intermediate,
                attentionHeads=synth.TINY.heads, kvHeads=synth.TINY.kv_heads)
    toks, progress = [], []
    out = R.runCustomQwenGreedyPrompt(device=ctx["device"], profile=prof, inputIds=[5, 6, 7], maxNewTokens=4,
                                      onToken=toks.append, onProgress=progress.append)
    assert set(out) == {"generated", "generatedTokens", "generateMs", "firstTokenMs", "outputText"}
    assert out["generatedTokens"] == 4 and toks == [str(t) for t in out["generated"]]
    assert out["outputText"] == " ".join(toks) and out["firstTokenMs"] <= out["generateMs"]
    ctx["device"].close()


@pytest.mark.parametrize("persistent", [1, 0])
def test_engine_qwen_shape_greedy_config2(qwen_runtime, persistent):
    """Config 2: 28 layers, 8 seeded prompt ids, 24 generated tokens, f16 KV."""
    rng = np.random.Generator(np.random.PCG64(2))
    prompt = rng.integers(0, 151936, size=8).tolist()
    model = O.Model(qwen_runtime)
    want, margins = model.session(max_seq=64, kv_f16=True).greedy(prompt, 24)
    with R.Engine(qwen_runtime, max_seq=64, persistent=persistent) as eng:
        assert eng.token_kernel == persistent
        ids, _ = eng.generate_greedy(prompt, 24)
        assert ids == want, (ids, want, margins.tolist())
        got_h = eng.forward_trace(want[-1], 8 + 23)[-1]
    sess = model.session(max_seq=64, kv_f16=True)
    for i, t in enumerate(prompt + want[:-1]):
        sess.forward(t, i)
    want_h = sess.forward(want[-1], 8 + 23, trace=True)[-1]
    assert rel(got_h, want_h) < 1e-3


def test_stepping_interface_matches_generate_and_flags_overrun(tiny_runtime):
    prompt = [9, 8, 7, 6]
    with R.Engine(tiny_runtime, max_seq=16) as eng:
        want, _ = eng.generate_greedy(prompt, 6)
        stream = torch.cuda.Stream()
        eng.set_stream(stream)
        eng.decode_begin(prompt, 6)
        for _ in range(6):
            eng.decode_step()
        assert eng.decode_sync(6) == want
        # replay from a seek: same positions, same tokens
        eng.decode_seek(len(prompt) - 1)
        for _ in range(6):
            eng.decode_step()
        eng.decode_sync(0)
        # stepping past max_seq is caught on the device and reported, never out of bounds
        eng.decode_begin(prompt, 6)
        for _ in range(16):
            eng.decode_step()
        with pytest.raises(R.QdError) as ex:
            eng.decode_sync(0)
        assert ex.value.code == -6
        eng.set_stream(None)
        ids, _ = eng.generate_greedy(prompt, 6)   # the engine stays usable
        assert ids == want


# ---- every step's logits, varied ids, variants, the RoPE stride option ------------

def _engine_step_logits(eng, prompt, n):
    """Greedy ids and each step's logits through the stepping entry points."""
    eng.decode_begin(prompt, n)
    logits = []
    for _ in range(n):
        eng.decode_step()
        logits.append(eng.logits())
    return eng.decode_sync(n), logits


def _oracle_step_logits(model, prompt, n, **session_kw):
    sess = model.session(**session_kw)
    for i, t in enumerate(prompt[:-1]):
        sess.forward(t, i)
    tok, ids, logits, margins = prompt[-1], [], [], []
    for step in range(n):
        sess.forward(tok, len(prompt) - 1 + step)
        tok, lg, margin = sess.next_token()
        ids.append(tok)
        logits.append(lg)
        margins.append(margin)
    return ids, logits, margins


def _check_steps(got_ids, got_logits, want_ids, want_logits, margins, tol=TOL):
    for step, (g, w) in enumerate(zip(got_logits, want_logits)):
        err = rel(g, w)
        print(f"step {step}: id {want_ids[step]} top-2 margin {margins[step]:.4g} logits rel err {err:.2e}")
        assert err < tol, (step, err)
    assert got_ids == want_ids, (got_ids, want_ids, margins)


@pytest.mark.parametrize("persistent", [1, 0])
def test_engine_qwen_shape_config2_every_step_logits(qwen_runtime, persistent):
    """Config 2 at the Qwen3-0.6B shape: all 24 steps' logits against the oracle at
    1e-4 (this seed-2 model emits one id at every step, so the ids alone say little)."""
    rng = np.random.Generator(np.random.PCG64(2))
    prompt = rng.integers(0, 151936, size=8).tolist()
    want_ids, want_logits, margins = _oracle_step_logits(O.Model(qwen_runtime), prompt, 24, max_seq=64,
                                                         kv_f16=True)
    with R.Engine(qwen_runtime, max_seq=64, persistent=persistent) as eng:
        got_ids, got_logits = _engine_step_logits(eng, prompt, 24)
    _check_steps(got_ids, got_logits, want_ids, want_logits, margins)


@pytest.mark.parametrize("persistent", [1, 0])
def test_engine_qwen_shape_varied_ids(qwen_runtime_centered, persistent):
    """A Qwen3-0.6B-shape model whose greedy ids change from step to step (seed 5,
    nibbles centred on the zero point): bit-exact ids and every step's logits."""
    rng = np.random.Generator(np.random.PCG64(2))
    prompt = rng.integers(0, 151936, size=8).tolist()
    want_ids, want_logits, margins = _oracle_step_logits(O.Model(qwen_runtime_centered), prompt, 24, max_seq=64,
                                                         kv_f16=True)
    assert len(set(want_ids)) >= 12, want_ids
    with R.Engine(qwen_runtime_centered, max_seq=64, persistent=persistent) as eng:
        got_ids, got_logits = _engine_step_logits(eng, prompt, 24)
        ids, _ = eng.generate_greedy(prompt, 24)
    # 1e-3 (still 10x inside the 1e-2 contract): in this model the K/V values that the
    # GPU and the oracle round to f16 differ by one f16 ulp now and then (their f32
    # sums differ in the last bits), and 28 layers carry that to ~1.1e-4 of the logits.
    _check_steps(got_ids, got_logits, want_ids, want_logits, margins, tol=1e-3)
    assert ids == want_ids


def test_variants_emit_identical_ids(tiny_runtime):
    """The reference's own bar: every variant emits the same greedy ids
    (docs/05-reproduce.md:98-100, src/bench/ab-page.js:95-97)."""
    # the reference's fallback prompt (src/bench/ab-page.js:18), folded into TINY's vocabulary
    prompt = [t % synth.TINY.vocab for t in (3838, 374, 279, 6722, 315, 9625, 30)]
    got = {}
    for variant in R.VARIANTS:
        with R.Engine(tiny_runtime, max_seq=64, variant=variant) as eng:
            got[variant], _ = eng.generate_greedy(prompt, 12)
    ctx = R.createWebGpuContext(tiny_runtime)
    for variant in R.VARIANTS:
        out = R.runCustomQwenGreedyPrompt(device=ctx["device"], profile={}, inputIds=prompt, maxNewTokens=12,
                                          variant=variant)
        assert out["generated"] == got["optimized"], variant
    ctx["device"].close()
    assert got["original"] == got["mixed"] == got["optimized"]
    want, _ = O.Model(tiny_runtime).session(max_seq=64, kv_f16=True).greedy(prompt, 12)
    assert got["optimized"] == want


@pytest.mark.parametrize("n,k", [(3072, 1024), (1024, 3072)])
def test_q4_matvec_matches_the_original_variant_oracle(n, k):
    """The CUDA matvec against the restatement of baseline/matmul_nbits_q4.wgsl
    (the 'original' variant's kernel and its summation order)."""
    x, w, s = synth.matvec_case(n, k, seed=0)
    assert rel(run_matvec(x, w, s), O.q4_matvec(x, w, s, original=True)) < TOL


@pytest.mark.parametrize("persistent", [1, 0])
def test_engine_rope_row_stride_option(tiny_runtime, tiny_model, persistent):
    """rope_row_stride = 64 reads table row p at position p (rope.wgsl:27 reads row
    2p with the reference's stride 128); the engine follows the oracle either way."""
    prompt = [11, 4000, 7, 123, 9]
    with R.Engine(tiny_runtime, max_seq=64, rope_row_stride=64, persistent=persistent) as eng:
        got_ids, got_logits = _engine_step_logits(eng, prompt, 8)
    want_ids, want_logits, margins = _oracle_step_logits(tiny_model, prompt, 8, max_seq=64, kv_f16=True,
                                                         rope_row_stride=64)
    _check_steps(got_ids, got_logits, want_ids, want_logits, margins)
    # the option changes the math: the default stride gives other logits
    _, default_logits, _ = _oracle_step_logits(tiny_model, prompt, 8, max_seq=64, kv_f16=True)
    assert any(rel(a, b) > 1e-3 for a, b in zip(want_logits, default_logits))


def test_prompt_pass_rope_row_stride(tiny_runtime, tiny_model):
    """The batched prompt pass reads the RoPE table with the engine's row stride too:
    a 12-token prompt at rope_row_stride = 64, pass on and off, against the oracle."""
    prompt = [11, 4000, 7, 123, 9, 77, 3000, 5, 19, 2048, 1, 400]
    want_ids, want_logits, margins = _oracle_step_logits(tiny_model, prompt, 6, max_seq=64, kv_f16=True,
                                                         rope_row_stride=64)
    for pp in (True, False):
        with R.Engine(tiny_runtime, max_seq=64, rope_row_stride=64, prompt_pass=pp) as eng:
            got_ids, got_logits = _engine_step_logits(eng, prompt, 6)
            ids, _ = eng.generate_greedy(prompt, 6)
        _check_steps(got_ids, got_logits, want_ids, want_logits, margins)
        assert ids == want_ids, pp


# ---- the batched prompt pass --------------------------------------------------------

@pytest.mark.parametrize("persistent", [1, 0])
def test_prompt_pass_matches_token_by_token_and_oracle(tiny_runtime, tiny_model, persistent):
    """Prompts of 5..258 tokens with the batched prompt pass on and off: identical
    greedy ids, and every step's logits within 1e-4 of the oracle either way. Through
    the stepping calls the pass covers a prompt's first 5..256 tokens (the last one
    goes through the decode kernel): 5 tokens (4 < 5: no pass), 6 (the shortest pass),
    257 (the longest) and 258 (too long: token by token). qd_generate_greedy with two
    or more ids also takes a whole prompt of 5..256 tokens and the first id from the
    pass (5 and 256 are its edges; 257 falls back to the 256-token pass). One engine
    takes every length in turn (graphs cached per length, nine lengths evict the
    oldest)."""
    rng = np.random.Generator(np.random.PCG64(11))
    lengths = [5, 6, 9, 33, 64, 65, 129, 256, 257, 258, 9, 6]
    prompts = {n: rng.integers(0, tiny_model.vocab, size=n).tolist() for n in set(lengths)}
    with R.Engine(tiny_runtime, max_seq=320, persistent=persistent) as on, \
            R.Engine(tiny_runtime, max_seq=320, persistent=persistent, prompt_pass=False) as off:
        for n in lengths:
            got_ids, got_logits = _engine_step_logits(on, prompts[n], 4)
            ref_ids, ref_logits = _engine_step_logits(off, prompts[n], 4)
            assert got_ids == ref_ids, n
            for g, r in zip(got_logits, ref_logits):
                assert rel(g, r) < TOL, n
            if n in (6, 257):
                want_ids, want_logits, margins = _oracle_step_logits(tiny_model, prompts[n], 4, max_seq=320,
                                                                     kv_f16=True)
                _check_steps(got_ids, got_logits, want_ids, want_logits, margins)
            ids, _ = on.generate_greedy(prompts[n], 4)
            assert ids == ref_ids, n
            if n in (5, 256):  # two ids (the first from the pass), and one (no head in the pass)
                assert on.generate_greedy(prompts[n], 2)[0] == ref_ids[:2], n
                assert on.generate_greedy(prompts[n], 1)[0] == ref_ids[:1], n
                assert rel(on.logits(), ref_logits[0]) < TOL, n


# ---- the argmax-only LM head (int8 coarse pass + exact recompute of candidates) ------

def test_argmax_head_ties_and_nan_rows(tiny_runtime, tmp_path):
    """Every embedding row present twice (exact ties at every logit) plus NaN rows: the
    argmax-only head picks the lower index of the best pair and never a NaN row, the
    same ids as the oracle and as the full head (greedy through the sampler); the logits
    asked for afterwards are the oracle's."""
    import shutil
    d = str(tmp_path / "ties")
    shutil.copytree(tiny_runtime, d)
    path = os.path.join(d, "shared", "embed_tokens.f16")
    s = synth.TINY
    emb = np.fromfile(path, dtype=np.float16).reshape(s.vocab, s.hidden)
    half = s.vocab // 2
    emb[half:2 * half] = emb[:half]
    emb[[7, 7 + half, s.vocab - 1]] = np.nan
    emb.tofile(path)
    prompt = [5, 77, 1000, 3]
    sess = O.Model(d).session(max_seq=64, kv_f16=True)
    want, margins = sess.greedy(prompt, 12)
    _, want_logits, _ = sess.next_token()
    with R.Engine(d, max_seq=64, persistent=1) as eng:
        assert eng.token_kernel == 1
        ids, _ = eng.generate_greedy(prompt, 12)
        logits = eng.logits()
        full, _ = eng.generate_sample(prompt, 12, temperature=1.0, top_k=1)
    assert ids == want, (ids, want, margins)
    assert full == want
    assert all(i < half and i != 7 for i in ids)
    nan = np.isnan(want_logits)
    assert np.array_equal(np.isnan(logits), nan)
    assert rel(logits[~nan], want_logits[~nan]) < TOL
