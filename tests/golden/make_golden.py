"""Generate the golden fixtures in this directory.

The reference (JavaScript + WGSL) cannot execute here: it needs a WebGPU device
and a JavaScript runtime, and neither exists on these machines. Its repository
ships no golden vectors either. What it does ship are CPU check functions that
state the decode math in plain JavaScript; this script ports them literally to
Python (JavaScript numbers are float64 and `Float32Array` stores round to f32,
so the port computes in float64 and rounds where the JS stores into a
Float32Array) and evaluates them on the reference's own fixture inputs:

* cpuQ4MatMulNBits   src/bench/webgpu-runtime.js:1028-1056
* cpuGqaDecode       src/bench/webgpu-runtime.js:943-982
* cpuRmsNorm         src/bench/webgpu-runtime.js:1423-1430
* createVector       src/bench/webgpu-runtime.js:1432-1436
* halfToFloat        src/bench/webgpu-runtime.js:1732-1739
* the greedy flow    src/bench/webgpu-runtime.js:165-214, 471-604 (layer order :498-562)
* the host argmax    src/bench/webgpu-runtime.js:353-357 (strict >, first index wins)

Fixture inputs: the GQA check's q/k/v (runGqaDecodeComparison :902-941), the
q4 check's x (runRealQwenQ4Projection :984-1026; its real layer-0 weights are
not in the reference checkout, so seeded synthetic weights stand in), the RMS
check's x (runRmsNorm :1636-1641) and a small seeded synthetic model.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from kernel_optimization_webgpu_b200 import synth  # noqa: E402

f32 = np.float32


def create_vector(size: int, step: float, fn) -> np.ndarray:
    return np.array([fn(i * step) for i in range(size)], dtype=np.float64).astype(f32)


def half_to_float(h: int) -> float:
    sign = -1 if (h & 0x8000) else 1
    exp = (h >> 10) & 0x1F
    frac = h & 0x03FF
    if exp == 0:
        return sign * 2.0 ** -14 * (frac / 1024)
    if exp == 0x1F:
        return float("nan") if frac else sign * float("inf")
    return sign * 2.0 ** (exp - 15) * (1 + frac / 1024)


def cpu_q4_matmul_nbits(in_size, out_size, blocks_per_row, block_size, x, weights, scales):
    """Vectorised cpuQ4MatMulNBits: float64 products ((nib-8)*scale)*x summed in float64."""
    words = weights.reshape(out_size, -1).astype(np.uint64)
    nib = np.stack([(words >> np.uint64(4 * i)) & np.uint64(0xF) for i in range(8)], axis=-1)
    vals = nib.reshape(out_size, -1).astype(np.float64) - 8.0
    sc = np.repeat(scales.reshape(out_size, blocks_per_row).astype(np.float64), block_size, axis=1)
    w = (vals * sc)[:, :in_size]
    return (w @ x.astype(np.float64)[:in_size]).astype(f32)


def cpu_gqa_decode(q, k_cache, v_cache, seq_len, q_heads, kv_heads, head_dim):
    y = np.zeros(q_heads * head_dim, f32)
    heads_per_kv = q_heads // kv_heads
    scale = 1 / math.sqrt(head_dim)
    k = k_cache.reshape(-1, kv_heads, head_dim).astype(np.float64)
    v = v_cache.reshape(-1, kv_heads, head_dim).astype(np.float64)
    for q_head in range(q_heads):
        kv_head = q_head // heads_per_kv
        qv = q[q_head * head_dim:(q_head + 1) * head_dim].astype(np.float64)
        score = (k[:seq_len, kv_head, :] @ qv) * scale          # float64
        scores = score.astype(f32)                              # Float32Array store
        max_score = float(np.max(score))                        # Math.max over float64 scores
        e = np.exp(scores.astype(np.float64) - max_score)
        scores = e.astype(f32)                                  # stored back into Float32Array
        s = float(np.sum(e))                                    # sum of float64 e
        w = scores.astype(np.float64) / s
        y[q_head * head_dim:(q_head + 1) * head_dim] = (w @ v[:seq_len, kv_head, :]).astype(f32)
    return y


def cpu_rms_norm(x, weight, eps):
    x64 = x.astype(np.float64)
    inv = 1 / math.sqrt(float(np.sum(x64 * x64)) / x.size + eps)
    return (x64 * inv * weight.astype(np.float64)).astype(f32)


def rope_f64(x, cos_tab, sin_tab, heads, head_dim, position, row_stride):
    half = head_dim // 2
    xx = x.reshape(heads, head_dim).astype(np.float64)
    base = position * row_stride
    c = cos_tab[base:base + half].astype(np.float64)
    s = sin_tab[base:base + half].astype(np.float64)
    lo, hi = xx[:, :half], xx[:, half:]
    return np.concatenate([lo * c - hi * s, hi * c + lo * s], axis=1).reshape(-1).astype(f32)


def host_argmax(logits):
    best_token, best = 0, -math.inf
    for i, v in enumerate(logits.tolist()):
        if v > best:
            best, best_token = v, i
    return best_token


class JsPortModel:
    """The reference's per-token flow with the JS CPU functions above."""

    def __init__(self, runtime_dir):
        with open(os.path.join(runtime_dir, "manifest.json")) as f:
            m = json.load(f)
        rd = lambda e, dt: np.fromfile(os.path.join(runtime_dir, e["file"]), dtype=dt)  # noqa: E731
        table = np.array([half_to_float(h) for h in range(65536)], dtype=np.float64).astype(f32)
        h2f = lambda e: table[rd(e, np.uint16)]  # noqa: E731
        self.m = m
        self.H, self.I = m["hiddenSize"], m["intermediateSize"]
        self.nh, self.nkv, self.hd = m["attentionHeads"], m["kvHeads"], m["headDim"]
        self.eps = m["normEpsilon"]
        self.embed = h2f(m["shared"]["embedTokens"]).reshape(-1, self.H)
        self.cos = h2f(m["shared"]["cosCache"]).reshape(-1)
        self.sin = h2f(m["shared"]["sinCache"]).reshape(-1)
        self.final_norm = h2f(m["finalNorm"])
        self.layers = []
        for le in m["layers"]:
            norms = {k: h2f(v) for k, v in le["norms"].items()}
            projs = {}
            for k, p in le["projections"].items():
                d = p["matmulNBits"]
                projs[k] = (d, rd(p["weight"], np.uint32), rd(p["scales"], np.float32))
            self.layers.append((norms, projs))

    def proj(self, projs, name, x):
        d, w, s = projs[name]
        return cpu_q4_matmul_nbits(d["inSize"], d["outSize"], d["blocksPerRow"], d["blockSize"], x, w, s)

    def greedy(self, ids, max_new, max_seq):
        kv = self.nkv * self.hd
        k_cache = [np.zeros((max_seq, kv), f32) for _ in self.layers]
        v_cache = [np.zeros((max_seq, kv), f32) for _ in self.layers]
        state = {}

        def forward(token, pos):
            h = self.embed[token].copy()
            for li, (norms, projs) in enumerate(self.layers):
                n = cpu_rms_norm(h, norms["input"], self.eps)
                q, k, v = (self.proj(projs, p, n) for p in ("q", "k", "v"))
                qn = np.concatenate([cpu_rms_norm(q[i * self.hd:(i + 1) * self.hd], norms["q"], self.eps)
                                     for i in range(self.nh)])
                kn = np.concatenate([cpu_rms_norm(k[i * self.hd:(i + 1) * self.hd], norms["k"], self.eps)
                                     for i in range(self.nkv)])
                qr = rope_f64(qn, self.cos, self.sin, self.nh, self.hd, pos, self.hd)
                kr = rope_f64(kn, self.cos, self.sin, self.nkv, self.hd, pos, self.hd)
                k_cache[li][pos] = kr
                v_cache[li][pos] = v
                attn = cpu_gqa_decode(qr, k_cache[li].reshape(-1), v_cache[li].reshape(-1), pos + 1,
                                      self.nh, self.nkv, self.hd)
                o = self.proj(projs, "o", attn)
                ar = (h.astype(np.float64) + o).astype(f32)
                post = cpu_rms_norm(ar, norms["postAttention"], self.eps)
                g, u = self.proj(projs, "gate", post), self.proj(projs, "up", post)
                g64 = g.astype(np.float64)
                act = ((g64 / (1 + np.exp(-g64))) * u.astype(np.float64)).astype(f32)
                down = self.proj(projs, "down", act)
                h = (ar.astype(np.float64) + down).astype(f32)
            state["final"] = cpu_rms_norm(h, self.final_norm, self.eps)

        def next_token():
            logits = (self.embed.astype(np.float64) @ state["final"].astype(np.float64)).astype(f32)
            srt = np.sort(logits)
            return host_argmax(logits), float(srt[-1] - srt[-2]), logits

        for i, t in enumerate(ids):
            forward(int(t), i)
        out, margins, first_logits = [], [], None
        for step in range(max_new):
            if step > 0:
                forward(out[-1], len(ids) + step - 1)
            tok, margin, logits = next_token()
            if first_logits is None:
                first_logits = logits
            out.append(tok)
            margins.append(margin)
        return out, margins, first_logits


def main():
    out = {}
    # GQA check inputs (runGqaDecodeComparison :902-909)
    q = create_vector(16 * 128, 0.011, math.sin)
    kc = create_vector(128 * 8 * 128, 0.007, math.cos)
    vc = create_vector(128 * 8 * 128, 0.013, math.sin)
    out["gqa_y"] = cpu_gqa_decode(q, kc, vc, 128, 16, 8, 128)
    # q4 check x (runRealQwenQ4Projection :992) on a seeded synthetic gate projection
    x, w, s = synth.matvec_case(3072, 1024, seed=0)
    xcv = create_vector(1024, 0.017, math.sin)
    out["q4_createvector_y"] = cpu_q4_matmul_nbits(1024, 3072, 32, 32, xcv, w, s)
    # config-0 shapes (seed 0 for each shape)
    for name, (n, k) in {"gate": (3072, 1024), "q": (2048, 1024), "o": (1024, 2048),
                         "down": (1024, 3072)}.items():
        x, w, s = synth.matvec_case(n, k, seed=0)
        out[f"q4_{name}_y"] = cpu_q4_matmul_nbits(k, n, k // 32, 32, x, w, s)
    # RMS check (runRmsNorm :1636-1641)
    xr = np.array([math.cos(i * 0.013) for i in range(1024)], dtype=np.float64).astype(f32)
    out["rms_y"] = cpu_rms_norm(xr, np.ones(1024, f32), 1e-6)
    np.savez_compressed(os.path.join(HERE, "js_cpu_refs.npz"), **out)

    # Whole-model greedy flow on the tiny synthetic model (f32 KV cache, as the reference).
    with tempfile.TemporaryDirectory() as d:
        synth.write_runtime(d, synth.TINY, seed=2)
        model = JsPortModel(d)
        rng = np.random.Generator(np.random.PCG64(5))
        prompt = rng.integers(0, synth.TINY.vocab, size=8).tolist()
        ids, margins, first_logits = model.greedy(prompt, 12, 64)
    np.save(os.path.join(HERE, "tiny_seed2_first_logits.npy"), first_logits)
    with open(os.path.join(HERE, "tiny_seed2_greedy.json"), "w") as f:
        json.dump({"shape": "TINY", "seed": 2, "prompt": prompt, "max_new": 12,
                   "generated": ids, "top2_margins": margins}, f, indent=1)
        f.write("\n")
    print("prompt", prompt, "generated", ids, "min margin", min(margins))


if __name__ == "__main__":
    main()
