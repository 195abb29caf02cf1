"""Batched decode (B sequences per step, tcgen05 GEMMs) against the CPU oracle.

The oracle runs each sequence on its own (one session per sequence, the
reference's single-sequence flow) from the same cached context rows, so greedy
ids must agree exactly and logits to f32 rounding.
"""
import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import runtime as R
from kernel_optimization_webgpu_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-4


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


# ---- the context generator, restated (kb_ctx_hidden / ctx_normal) -------------------
def _hash(x):
    x = x.astype(np.uint32)
    x ^= x >> np.uint32(16)
    x *= np.uint32(0x7FEB352D)
    x ^= x >> np.uint32(15)
    x *= np.uint32(0x846CA68B)
    x ^= x >> np.uint32(16)
    return x


def ctx_hidden(seed, layer, row, H):
    """Hidden row `row` (= seq * ctx + position) of `layer`: f32 [H]."""
    with np.errstate(over="ignore"):
        key = _hash(np.array([(seed * 0x9E3779B9 + layer * 0x85EBCA6B + 0x632BE5AB) & 0xFFFFFFFF], np.uint32))[0]
        d = np.arange(H, dtype=np.uint64)
        base = ((np.uint64(row) * np.uint64(H) + d) * np.uint64(4)) & np.uint64(0xFFFFFFFF)
        s = np.zeros(H, np.int64)
        for j in range(4):
            s += (_hash((base + np.uint64(j)).astype(np.uint32) ^ key) >> np.uint32(8)).astype(np.int64)
    s -= 2 << 24
    return (s.astype(np.float32) * np.float32(5.9604644775390625e-08)) * np.float32(1.7320508)


def oracle_kv_row(model, seed, layer, row, pos, row_stride=128):
    norms, w, s = model.layers[layer]
    H, NKV, hd = model.hidden, model.kv_heads, model.head_dim
    x = O.rms_norm(ctx_hidden(seed, layer, row, H), norms["input"], model.eps)
    k = O.q4_matvec(x, w[1], s[1], H, NKV * hd)
    v = O.q4_matvec(x, w[2], s[2], H, NKV * hd)
    k = O.head_rms_norm(k, norms["k"], hd, NKV, model.eps)
    k = O.rope(k, model.cos, model.sin, NKV, hd, pos, row_stride)
    return k.astype(np.float16).astype(np.float32), v.astype(np.float16).astype(np.float32)


def oracle_decode(model, batch, seq, pos, tok, steps, max_seq):
    """One sequence from the batch's cached rows [0, pos), decoded alone by the oracle."""
    sess = model.session(max_seq=max_seq, kv_f16=True)
    for layer in range(len(model.layers)):
        if pos:
            k, v = batch.read_kv(layer, seq, 0, pos)
            sess.set_kv(layer, 0, k, v)
    ids, margins = [], []
    logits = None
    for i in range(steps):
        sess.forward(int(tok), pos + i)
        tok, logits, margin = sess.next_token()
        ids.append(tok)
        margins.append(margin)
    return ids, logits, margins


@pytest.fixture(scope="module")
def tiny(tiny_runtime):
    eng = R.Engine(tiny_runtime, max_seq=64)
    yield eng, O.Model(tiny_runtime)
    eng.close()


def test_context_fill_matches_oracle_projection(tiny):
    eng, model = tiny
    B, ctx, seed = 3, 70, 3
    with R.Batch(eng, B, 160) as bt:
        bt.fill_context(ctx, seed)
        assert bt.positions().tolist() == [ctx] * B
        for layer in range(len(model.layers)):
            for seq, pos in [(0, 0), (0, 69), (1, 33), (2, 64), (2, 5)]:
                gk, gv = bt.read_kv(layer, seq, pos, 1)
                wk, wv = oracle_kv_row(model, seed, layer, seq * ctx + pos, pos)
                for g, w in ((gk[0], wk), (gv[0], wv)):
                    assert np.allclose(g, w, rtol=2.0 ** -10, atol=1e-4), (layer, seq, pos)
                    assert np.mean(g == w) > 0.97
        # rows beyond the context stay zero
        k, v = bt.read_kv(0, 1, ctx, 4)
        assert not k.any() and not v.any()


def _decode_case(eng, model, B, max_seq, positions, steps, seed=3, ctx=None, logits=True):
    rng = np.random.Generator(np.random.PCG64(seed))
    tokens = rng.integers(0, model.vocab, size=B).astype(np.int32)
    with R.Batch(eng, B, max_seq) as bt:
        bt.fill_context(ctx if ctx is not None else max(positions), seed)
        bt.set_tokens(tokens, positions)
        if logits:
            bt.keep_logits(True)
        ids = bt.decode(steps)
        assert ids.shape == (steps, B)
        assert bt.positions().tolist() == [p + steps for p in positions]
        got_logits = bt.logits() if logits else None
        for s in range(B):
            want, want_logits, margins = oracle_decode(model, bt, s, positions[s], tokens[s], steps, max_seq)
            assert ids[:, s].tolist() == want, (s, ids[:, s].tolist(), want, margins)
            if logits:
                assert rel(got_logits[s], want_logits) < TOL, s


def test_batch_decode_matches_oracle(tiny):
    eng, model = tiny
    _decode_case(eng, model, B=4, max_seq=160, positions=[70] * 4, steps=6)


def test_batch_decode_ragged_positions(tiny):
    """Each sequence at its own position: tile edges (64), a short one, one near max_seq."""
    eng, model = tiny
    _decode_case(eng, model, B=5, max_seq=160, positions=[70, 5, 64, 150, 0], steps=6, ctx=150)


def test_batch_decode_multi_split_context(tiny):
    """1100 cached positions: three 512-position attention splits, ragged last tile."""
    eng, model = tiny
    _decode_case(eng, model, B=2, max_seq=1200, positions=[1100, 1037], steps=3, ctx=1100)


def test_batch_decode_chunks_and_step_accounting(tiny):
    eng, model = tiny
    with R.Batch(eng, 2, 400) as bt:
        assert bt.step_kernels == len(model.layers) * 10 + 4
        bt.fill_context(10, 1)
        bt.set_tokens([5, 6], [10, 10])
        a = bt.decode(300)             # more steps than one id chunk (256)
        bt.set_tokens([5, 6], [10, 10])
        b1 = bt.decode(100)
        b2 = bt.decode(200)
        assert np.array_equal(a, np.concatenate([b1, b2]))
        assert bt.decode(0).shape == (0, 2)


def test_batch_rejects_bad_requests(tiny):
    eng, model = tiny
    with R.Batch(eng, 2, 32) as bt:
        bt.fill_context(30, 1)
        with pytest.raises(R.QdError) as ex:
            bt.decode(3)                           # 30 + 3 > 32
        assert ex.value.code == -5
        with pytest.raises(R.QdError) as ex:
            bt.set_tokens([0, model.vocab], None)  # token outside the vocabulary
        assert ex.value.code == -5
        with pytest.raises(R.QdError) as ex:
            bt.read_kv(0, 2, 0, 1)                 # sequence outside the batch
        assert ex.value.code == -5
        with pytest.raises(R.QdError):
            bt.logits()                            # logits not kept
        ids = bt.decode(2)                         # exactly fits
        assert ids.shape == (2, 2)
    with pytest.raises(R.QdError):
        R.Batch(eng, 0, 32)


def test_batch_qwen_shape_config3(qwen_runtime):
    """Config 3 shape: 64 sequences, 2048 cached positions each, Qwen3-0.6B layers;
    two sequences checked against the oracle for 3 steps."""
    model = O.Model(qwen_runtime)
    B, ctx, steps = 64, 2048, 3
    rng = np.random.Generator(np.random.PCG64(3))
    tokens = rng.integers(0, model.vocab, size=B).astype(np.int32)
    with R.Engine(qwen_runtime, max_seq=64) as eng, R.Batch(eng, B, ctx + 8) as bt:
        bt.fill_context(ctx, 3)
        bt.set_tokens(tokens, [ctx] * B)
        ids = bt.decode(steps)
        for s in (0, B - 1):
            want, _, margins = oracle_decode(model, bt, s, ctx, tokens[s], steps, ctx + 8)
            assert ids[:, s].tolist() == want, (s, ids[:, s].tolist(), want, margins)
        # the context rows of one sequence against the oracle's projection
        for layer, pos in [(0, 0), (27, 2047)]:
            gk, gv = bt.read_kv(layer, 17, pos, 1)
            wk, wv = oracle_kv_row(model, 3, layer, 17 * ctx + pos, pos)
            assert np.allclose(gk[0], wk, rtol=2.0 ** -10, atol=1e-4)
            assert np.allclose(gv[0], wv, rtol=2.0 ** -10, atol=1e-4)


# ---- prefill (config 4 flow) -------------------------------------------------------

def _oracle_greedy(model, prompt, max_new, max_seq):
    sess = model.session(max_seq=max_seq, kv_f16=True)
    ids, margins = sess.greedy(prompt, max_new)
    return ids, margins, sess


@pytest.mark.parametrize("n", [1, 64, 70, 130])
def test_prefill_then_decode_matches_oracle(tiny, n):
    """Prompts of n ids (a single id, exactly one tile, ragged tiles) prefilled as one
    GEMM pass with causal attention, then 4 decode steps."""
    eng, model = tiny
    B, steps = 3, 4
    rng = np.random.Generator(np.random.PCG64(4))
    ids = rng.integers(0, model.vocab, size=(B, n)).astype(np.int32)
    with R.Batch(eng, B, n + steps + 2) as bt:
        first = bt.prefill(ids)
        assert bt.positions().tolist() == [n] * B
        more = bt.decode(steps)
        for s in range(B):
            want, margins, sess = _oracle_greedy(model, ids[s].tolist(), steps + 1, n + steps + 2)
            got = [int(first[s])] + more[:, s].tolist()
            assert got == want, (s, got, want, margins)
        # the prompt's cached rows against the oracle's (f16 rounding of nearby values)
        sess = model.session(max_seq=n + 1, kv_f16=True)
        for i, t in enumerate(ids[1].tolist()):
            sess.forward(t, i)
        for layer in range(len(model.layers)):
            gk, gv = bt.read_kv(layer, 1, 0, n)
            wk, wv = sess.kv(layer, 0, n)
            assert np.allclose(gk, wk, rtol=2.0 ** -9, atol=1e-3), layer
            assert np.allclose(gv, wv, rtol=2.0 ** -9, atol=1e-3), layer


def test_generate_batch_wrapper(tiny):
    eng, model = tiny
    rng = np.random.Generator(np.random.PCG64(5))
    ids = rng.integers(0, model.vocab, size=(2, 9)).astype(np.int32)
    out = R.generate_batch(eng, ids, 5)
    assert out.shape == (2, 5)
    for s in range(2):
        want, _, _ = _oracle_greedy(model, ids[s].tolist(), 5, 16)
        assert out[s].tolist() == want


def test_prefill_rejects_bad_requests(tiny):
    eng, model = tiny
    with R.Batch(eng, 2, 16) as bt:
        with pytest.raises(R.QdError) as ex:
            bt.prefill(np.zeros((2, 17), np.int32))        # longer than max_seq
        assert ex.value.code == -5
        bad = np.zeros((2, 4), np.int32)
        bad[1, 2] = model.vocab
        with pytest.raises(R.QdError) as ex:
            bt.prefill(bad)                                # id outside the vocabulary
        assert ex.value.code == -5
        with pytest.raises(ValueError):
            bt.prefill(np.zeros((3, 4), np.int32))         # wrong batch


def test_prefill_qwen_shape_config4(qwen_runtime):
    """Config 4 shape: 32 prompts of 512 ids (seed 4), prefill then 16 decode tokens;
    the last prompt checked end to end against the oracle's sequential greedy."""
    model = O.Model(qwen_runtime)
    B, n, steps = 32, 512, 16
    rng = np.random.Generator(np.random.PCG64(4))
    ids = rng.integers(0, model.vocab, size=(B, n)).astype(np.int32)
    with R.Engine(qwen_runtime, max_seq=64) as eng, R.Batch(eng, B, n + steps) as bt:
        first = bt.prefill(ids)
        more = bt.decode(steps - 1)
        for s in (B - 1,):
            want, margins, _ = _oracle_greedy(model, ids[s].tolist(), steps, n + steps)
            got = [int(first[s])] + more[:, s].tolist()
            assert got == want, (s, got, want, margins)


# ---- vocabulary-sharded LM head (config 3 across GPUs), ranks emulated on one GPU ---------

def _emulated_shard_decode(eng, model, world, B, steps, ctx=40, max_seq=64):
    """`world` batches on one GPU play the ranks: the all-gathers are copies between their
    buffers, in rank order, on the engine's stream. Returns each rank's ids and the ids the
    same batches give with the replicated LM head."""
    stream = torch.cuda.Stream()  # the library and the copies below share this stream
    eng.set_stream(stream)
    rng = np.random.Generator(np.random.PCG64(11))
    tokens = [rng.integers(0, model.vocab, size=B).astype(np.int32) for _ in range(world)]
    want = []
    for r in range(world):
        with R.Batch(eng, B, max_seq) as bt:
            bt.fill_context(ctx, 20 + r)
            bt.set_tokens(tokens[r], [ctx] * B)
            want.append(bt.decode(steps))
    batches = [R.Batch(eng, B, max_seq) for _ in range(world)]
    try:
        bufs = []
        for r, bt in enumerate(batches):
            bt.fill_context(ctx, 20 + r)
            bt.set_tokens(tokens[r], [ctx] * B)
            bufs.append(bt.set_vocab_shard(r, world))
        with torch.cuda.stream(stream):
            for _ in range(steps):
                for bt in batches:
                    bt.step_layers()
                for key in ("gather_hi", "gather_lo"):
                    for dst in bufs:
                        for r, src in enumerate(bufs):
                            dst[key][r * B:(r + 1) * B].copy_(src[key][r * B:(r + 1) * B])
                for bt in batches:
                    bt.step_lm_slice()
                for dst in bufs:
                    for r, src in enumerate(bufs):
                        dst["pairs_all"][r].copy_(src["pairs_local"])
                for bt in batches:
                    bt.step_merge()
        got = [bt.shard_sync(steps) for bt in batches]
        pos = [bt.positions().tolist() for bt in batches]
    finally:
        for bt in batches:
            bt.close()
        eng.set_stream(None)
    return got, want, pos


@pytest.mark.parametrize("world", [1, 3])
def test_vocab_sharded_lm_head_matches_replicated(tiny, world):
    """Each rank scores a vocabulary slice (uneven for 3 ranks: 4099 rows) for every rank's
    rows; the merged ids equal the replicated LM head's, bit for bit."""
    eng, model = tiny
    B, steps, ctx = 2, 5, 40
    got, want, pos = _emulated_shard_decode(eng, model, world, B, steps, ctx)
    for r in range(world):
        assert got[r].tolist() == want[r].tolist(), r
        assert pos[r] == [ctx + steps] * B


def test_vocab_shard_rejects_bad_requests(tiny):
    eng, model = tiny
    with R.Batch(eng, 2, 32) as bt:
        with pytest.raises(R.QdError):
            bt.step_layers()                      # no shard set
        with pytest.raises(R.QdError):
            bt.set_vocab_shard(2, 2)              # rank outside 0..world-1
        bt.fill_context(4, 1)
        bt.set_tokens([1, 2], [4, 4])
        bt.set_vocab_shard(0, 1)
        with pytest.raises(R.QdError):
            bt.shard_sync(1)                      # no merged step to sync
