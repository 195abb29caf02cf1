"""The CPU oracle pinned against the golden fixtures (ported JS CPU check functions)."""
import json
import math
import os

import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import synth
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def refs():
    return np.load(os.path.join(GOLDEN, "js_cpu_refs.npz"))


def create_vector(size, step, fn):
    return np.array([fn(i * step) for i in range(size)], dtype=np.float64).astype(np.float32)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def js_half_to_float(h):
    sign = -1 if (h & 0x8000) else 1
    e, frac = (h >> 10) & 0x1F, h & 0x3FF
    if e == 0:
        return sign * 2.0 ** -14 * (frac / 1024)
    if e == 0x1F:
        return float("nan") if frac else sign * float("inf")
    return sign * 2.0 ** (e - 15) * (1 + frac / 1024)


def test_half_to_float_all_65536_codes():
    for h in range(0, 65536, 7):
        got, want = O.half_to_float(h), js_half_to_float(h)
        assert (math.isnan(got) and math.isnan(want)) or got == want, h
    for h in (0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x7E00):
        got, want = O.half_to_float(h), js_half_to_float(h)
        assert (math.isnan(got) and math.isnan(want)) or got == want, h


def test_float_to_half_round_to_nearest_even_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e-8, 2.0 ** -24, 2.0 ** -25,
                  2.0 ** -25 * 1.0001, 3 * 2.0 ** -26, np.inf, -np.inf], np.float32)]).astype(np.float32)
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    got = np.array([O.float_to_half(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, want)


def test_q4_matvec_matches_js_cpu_ref_on_reference_fixture_x(refs):
    _, w, s = synth.matvec_case(3072, 1024, seed=0)
    x = create_vector(1024, 0.017, math.sin)
    y = O.q4_matvec(x, w, s)
    assert rel_err(y, refs["q4_createvector_y"]) < 1e-5


@pytest.mark.parametrize("name,n,k", [("gate", 3072, 1024), ("q", 2048, 1024), ("o", 1024, 2048),
                                      ("down", 3072 // 3, 3072)])
def test_q4_matvec_config0_shapes(refs, name, n, k):
    x, w, s = synth.matvec_case(n, k, seed=0)
    y = O.q4_matvec(x, w, s)
    assert rel_err(y, refs[f"q4_{name}_y"]) < 1e-5
    y0 = O.q4_matvec(x, w, s, original=True)
    assert rel_err(y0, refs[f"q4_{name}_y"]) < 1e-5


def test_q4_matvec_tail_in_size_not_multiple_of_8():
    # dot_word_tail path: in_size smaller than blocks_per_row * block_size.
    x, w, s = synth.matvec_case(64, 64, seed=3)
    y = O.q4_matvec(x, w, s, in_size=61)
    nib = np.stack([(w.astype(np.uint64) >> np.uint64(4 * i)) & np.uint64(15) for i in range(8)], -1)
    deq = (nib.reshape(64, -1).astype(np.float64) - 8) * np.repeat(s.reshape(64, 2), 32, axis=1)
    want = deq[:, :61] @ x[:61].astype(np.float64)
    assert rel_err(y, want) < 1e-5


def test_gqa_decode_matches_js_cpu_ref(refs):
    q = create_vector(16 * 128, 0.011, math.sin)
    kc = create_vector(128 * 8 * 128, 0.007, math.cos)
    vc = create_vector(128 * 8 * 128, 0.013, math.sin)
    y = O.gqa_decode(q, kc, vc, 128, 16, 8, 128)
    assert rel_err(y, refs["gqa_y"]) < 1e-5


def test_gqa_decode_uncapped_matches_float64_softmax():
    rng = np.random.default_rng(1)
    seq = 700  # above the shader's 256-position cap
    q = rng.standard_normal(16 * 128).astype(np.float32)
    kc = rng.standard_normal((seq, 8, 128)).astype(np.float32)
    vc = rng.standard_normal((seq, 8, 128)).astype(np.float32)
    y = O.gqa_decode(q, kc, vc, seq, 16, 8, 128).reshape(16, 128)
    for h in range(16):
        s = kc[:, h // 2, :].astype(np.float64) @ q[h * 128:(h + 1) * 128] / math.sqrt(128)
        p = np.exp(s - s.max())
        p /= p.sum()
        want = p @ vc[:, h // 2, :].astype(np.float64)
        assert rel_err(y[h], want) < 1e-4


def test_rms_norm_matches_js_cpu_ref(refs):
    x = np.array([math.cos(i * 0.013) for i in range(1024)], np.float64).astype(np.float32)
    y = O.rms_norm(x, np.ones(1024, np.float32))
    assert rel_err(y, refs["rms_y"]) < 1e-6


def test_rope_reads_row_two_p_of_the_half_width_table():
    shape = synth.Shape(rope_rows=64)
    cos, sin = synth.rope_tables(shape)
    cos, sin = cos.astype(np.float32), sin.astype(np.float32)
    x = np.random.default_rng(2).standard_normal(2 * 128).astype(np.float32)
    p = 5
    y = O.rope(x, cos, sin, 2, 128, p)
    c, s = cos[2 * p], sin[2 * p]          # row 2p: position * head_dim into a 64-wide table
    for h in range(2):
        lo, hi = x[h * 128:h * 128 + 64], x[h * 128 + 64:(h + 1) * 128]
        assert np.allclose(y[h * 128:h * 128 + 64], lo * c - hi * s, atol=1e-6)
        assert np.allclose(y[h * 128 + 64:(h + 1) * 128], hi * c + lo * s, atol=1e-6)
    y1 = O.rope(x, cos, sin, 2, 128, p, row_stride=64)   # "fixed" indexing: row p
    assert np.allclose(y1[:64], x[:64] * cos[p] - x[64:128] * sin[p], atol=1e-6)


def host_scan(logits):
    best, tok = -math.inf, 0
    for i, v in enumerate(logits.tolist()):
        if v > best:
            best, tok = v, i
    return tok


ARGMAX_CASES = {
    "all_ties": lambda n: np.zeros(n, np.float32),
    "winner_last_index": lambda n: np.concatenate([np.zeros(n - 1, np.float32), [1.0]]).astype(np.float32),
    "duplicate_maxima": lambda n: np.where(np.arange(n) % 977 == 3, 5.0, 0.0).astype(np.float32),
    "dup_across_stride_span": lambda n: np.where(np.isin(np.arange(n), [65536 + 7, 7, 131072 + 7]),
                                                 2.0, -1.0).astype(np.float32),
    "winner_first": lambda n: np.concatenate([[3.0], np.full(n - 1, 2.9)]).astype(np.float32),
    "negative_values": lambda n: -np.abs(np.random.default_rng(3).standard_normal(n)).astype(np.float32) - 1,
    "random": lambda n: np.random.default_rng(4).standard_normal(n).astype(np.float32),
}


@pytest.mark.parametrize("case", sorted(ARGMAX_CASES))
def test_argmax_adversarial_cases_match_host_scan(case):
    n = 151936
    logits = ARGMAX_CASES[case](n)
    idx, val = O.argmax(logits)
    assert idx == host_scan(logits)
    assert val == logits[idx]


def test_argmax_nan_never_wins_and_all_neg_inf_gives_zero():
    logits = np.full(1000, -np.inf, np.float32)
    assert O.argmax(logits) == (0, float(np.float32(-3.4028234e38)))
    logits[10] = np.nan
    logits[500] = -5.0
    assert O.argmax(logits)[0] == 500


def test_lm_head_f16_matches_float64():
    table, x, eps = synth.lm_head_case(vocab=5000, hidden=1024, seed=1)
    h = O.rms_norm(x, np.ones(1024, np.float32), eps)
    logits = O.lm_head_f16(h, table)
    want = table.astype(np.float64) @ h.astype(np.float64)
    assert rel_err(logits, want) < 1e-5


def test_tiny_model_greedy_matches_js_port(tiny_runtime):
    with open(os.path.join(GOLDEN, "tiny_seed2_greedy.json")) as f:
        g = json.load(f)
    model = O.Model(tiny_runtime)
    sess = model.session(max_seq=64, kv_f16=False)
    ids, margins = sess.greedy(g["prompt"], g["max_new"])
    assert ids == g["generated"]
    first = np.load(os.path.join(GOLDEN, "tiny_seed2_first_logits.npy"))
    sess2 = model.session(max_seq=64, kv_f16=False)
    for i, t in enumerate(g["prompt"]):
        sess2.forward(t, i)
    tok, logits, _ = sess2.next_token()
    assert tok == g["generated"][0]
    assert rel_err(logits, first) < 1e-4


def test_tiny_model_f16_kv_mode_runs_and_reports_margins(tiny_runtime):
    model = O.Model(tiny_runtime)
    ids, margins = model.session(max_seq=64, kv_f16=True).greedy([1, 2, 3, 4], 6)
    assert len(ids) == 6 and all(0 <= t < synth.TINY.vocab for t in ids)
    assert np.all(margins >= 0)


def test_oracle_rejects_out_of_range_token_and_position(tiny_runtime):
    model = O.Model(tiny_runtime)
    sess = model.session(max_seq=4)
    with pytest.raises(ValueError):
        sess.forward(synth.TINY.vocab, 0)
    with pytest.raises(ValueError):
        sess.forward(0, 4)
