"""Seeded synthetic Qwen3-shaped weights in the reference's extracted runtime layout.

The on-disk layout is the one `scripts/extract-qwen-runtime-assets.mjs` writes
(manifest schema :14-25, shared tensors :27-34, per-layer norms :44-53,
projections :55-65 and `extractProjection` :74-102):

    manifest.json
    shared/embed_tokens.f16      [vocab][hidden] f16 (tied: input gather + LM head)
    shared/cos_cache.f16         [rope_rows][head_dim/2] f16
    shared/sin_cache.f16         [rope_rows][head_dim/2] f16
    shared/final_norm.f16        [hidden] f16
    layers/<i>/norm_{input,q,k,postAttention}.f16
    layers/<i>/<proj>_weight_q4.bin   [out][in/32][16 bytes] (ONNX MatMulNBits, bits=4, block 32)
    layers/<i>/<proj>_scales_f32.bin  [out * in/32] f32 (values originate as f16)

Block scales are drawn as |N(0, scale_std)|, rounded to f16 first and then
stored as f32, so the f32 file holds exactly what the ONNX f16 initializer
would have held (the extractor's `float16TensorToFloat32`, :133-143).

The RoPE tables follow the ONNX export: `[40960, 64]` f16 with
angle(row, j) = row * theta^(-2j/head_dim).
"""
from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass

import numpy as np

PROJECTIONS = ("q", "k", "v", "o", "gate", "up", "down")
NORMS = ("input", "q", "k", "postAttention")
BLOCK_SIZE = 32


@dataclass(frozen=True)
class Shape:
    """Model dimensions (the reference's `qwenProfile`, src/model/qwen3-0.6b.js:1-15)."""

    layers: int = 28
    hidden: int = 1024
    intermediate: int = 3072
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151936
    rope_rows: int = 40960
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6

    def proj_dims(self, name: str) -> tuple[int, int]:
        """(out_size, in_size) of a projection."""
        q = self.heads * self.head_dim
        kv = self.kv_heads * self.head_dim
        return {
            "q": (q, self.hidden),
            "k": (kv, self.hidden),
            "v": (kv, self.hidden),
            "o": (self.hidden, q),
            "gate": (self.intermediate, self.hidden),
            "up": (self.intermediate, self.hidden),
            "down": (self.hidden, self.intermediate),
        }[name]


QWEN3_0_6B = Shape()
# Small shape used by the fast parity tests; same kernels, fewer bytes.
TINY = Shape(layers=2, hidden=512, intermediate=1024, heads=4, kv_heads=2, head_dim=128,
             vocab=4099, rope_rows=4096)


def f16_round(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def q4_projection(rng: np.random.Generator, out_size: int, in_size: int,
                  scale_std: float = 0.02, nibbles: str = "uniform") -> tuple[np.ndarray, np.ndarray]:
    """Random MatMulNBits weight: u32 words [out][in/8] of random nibbles, f16-valued f32 scales.

    nibbles "uniform": every nibble uniform on 0..15 (mean 7.5, so each weight
    carries a -0.5 * scale bias against the zero point 8); "centered": uniform on
    1..15, symmetric around the zero point."""
    if in_size % BLOCK_SIZE:
        raise ValueError("in_size must be a multiple of the block size")
    if nibbles == "uniform":
        words = rng.integers(0, 2**32, size=(out_size, in_size // 8), dtype=np.uint64).astype(np.uint32)
    elif nibbles == "centered":
        nib = rng.integers(1, 16, size=(out_size, in_size // 8, 8), dtype=np.uint32)
        words = np.zeros((out_size, in_size // 8), np.uint32)
        for i in range(8):
            words |= nib[:, :, i] << np.uint32(4 * i)
    else:
        raise ValueError(f"unknown nibble distribution {nibbles!r}")
    scales = np.abs(rng.standard_normal(out_size * (in_size // BLOCK_SIZE))) * scale_std
    scales = f16_round(scales).astype(np.float32)
    return words, scales


def rope_tables(shape: Shape) -> tuple[np.ndarray, np.ndarray]:
    half = shape.head_dim // 2
    inv_freq = shape.rope_theta ** (-(np.arange(half, dtype=np.float64) * 2.0) / shape.head_dim)
    ang = np.arange(shape.rope_rows, dtype=np.float64)[:, None] * inv_freq[None, :]
    return f16_round(np.cos(ang)), f16_round(np.sin(ang))


def _norm_weight(rng: np.random.Generator, n: int, mode: str) -> np.ndarray:
    if mode == "ones":
        return np.ones(n, dtype=np.float16)
    return f16_round(1.0 + 0.1 * rng.standard_normal(n))


def _write(path: str, arr: np.ndarray) -> int:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    data = np.ascontiguousarray(arr)
    data.tofile(path)
    return data.nbytes


def write_runtime(out_dir: str, shape: Shape = QWEN3_0_6B, seed: int = 2,
                  norm_mode: str = "random", embed_std: float = 0.02,
                  scale_std: float = 0.02, nibbles: str = "uniform") -> dict:
    """Write a complete runtime directory and return its manifest.

    norm_mode "random" draws every RMSNorm weight as f16(1 + 0.1 N(0,1)) so that
    a wrong weight index shows up in parity; "ones" gives unit weights.
    nibbles: see q4_projection. With "uniform" nibbles the per-weight bias drives
    a random-init Qwen3-0.6B-shape model to emit one id over and over; "centered"
    nibbles give a model whose greedy ids change from step to step.
    Draw order (fixed, part of the format): embedding, then per layer the four
    norms followed by q, k, v, o, gate, up, down; the final norm last.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    manifest: dict = {
        "source": f"synthetic seed={seed}",
        "dtype": "q4f16",
        "hiddenSize": shape.hidden,
        "intermediateSize": shape.intermediate,
        "attentionHeads": shape.heads,
        "kvHeads": shape.kv_heads,
        "headDim": shape.head_dim,
        "vocabSize": shape.vocab,
        "normEpsilon": shape.eps,
        "ropeTheta": shape.rope_theta,
        "layers": [],
        "shared": {},
        "finalNorm": None,
    }

    def entry(name: str, file: str, dims: list[int], nbytes: int, data_type: int = 10) -> dict:
        return {"name": name, "file": file, "dims": dims, "dataType": data_type, "bytes": nbytes}

    embed = f16_round(rng.standard_normal((shape.vocab, shape.hidden), dtype=np.float32) * embed_std)
    n = _write(os.path.join(out_dir, "shared/embed_tokens.f16"), embed)
    manifest["shared"]["embedTokens"] = entry("model.embed_tokens.weight", "shared/embed_tokens.f16",
                                              [shape.vocab, shape.hidden], n)
    del embed
    cos, sin = rope_tables(shape)
    n = _write(os.path.join(out_dir, "shared/cos_cache.f16"), cos)
    manifest["shared"]["cosCache"] = entry("cos_cache", "shared/cos_cache.f16", list(cos.shape), n)
    n = _write(os.path.join(out_dir, "shared/sin_cache.f16"), sin)
    manifest["shared"]["sinCache"] = entry("sin_cache", "shared/sin_cache.f16", list(sin.shape), n)

    for layer in range(shape.layers):
        d = f"layers/{layer}"
        le: dict = {"layer": layer, "norms": {}, "projections": {}}
        for key in NORMS:
            size = shape.head_dim if key in ("q", "k") else shape.hidden
            w = _norm_weight(rng, size, norm_mode)
            f = f"{d}/norm_{key}.f16"
            n = _write(os.path.join(out_dir, f), w)
            le["norms"][key] = entry(f"model.layers.{layer}.{key}_norm.weight", f, [size], n)
        for key in PROJECTIONS:
            out_size, in_size = shape.proj_dims(key)
            words, scales = q4_projection(rng, out_size, in_size, scale_std, nibbles)
            wf, sf = f"{d}/{key}_weight_q4.bin", f"{d}/{key}_scales_f32.bin"
            nw = _write(os.path.join(out_dir, wf), words)
            ns = _write(os.path.join(out_dir, sf), scales)
            bpr = in_size // BLOCK_SIZE
            prefix = f"model.layers.{layer}.{key}_proj.MatMul"
            le["projections"][key] = {
                "prefix": prefix,
                "weight": entry(f"{prefix}.weight_Q4", wf, [out_size, bpr, BLOCK_SIZE // 2], nw, 2),
                "scales": {**entry(f"{prefix}.weight_scales", sf, [out_size * bpr], out_size * bpr * 2),
                           "sourceDataType": 10, "dataType": "float32", "bytes": ns},
                "matmulNBits": {"outSize": out_size, "blocksPerRow": bpr,
                                "bytesPerBlock": BLOCK_SIZE // 2, "blockSize": BLOCK_SIZE,
                                "inSize": in_size},
            }
        manifest["layers"].append(le)

    fn = _norm_weight(rng, shape.hidden, norm_mode)
    n = _write(os.path.join(out_dir, "shared/final_norm.f16"), fn)
    manifest["finalNorm"] = entry("model.norm.weight", "shared/final_norm.f16", [shape.hidden], n)
    manifest["synthetic"] = {"seed": seed, "normMode": norm_mode, "embedStd": embed_std,
                             "scaleStd": scale_std, "nibbles": nibbles, "shape": asdict(shape)}
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=2)
        f.write("\n")
    return manifest


def ensure_runtime(out_dir: str, shape: Shape = QWEN3_0_6B, seed: int = 2,
                   norm_mode: str = "random", nibbles: str = "uniform") -> dict:
    """Write the runtime directory unless a matching one already exists there."""
    path = os.path.join(out_dir, "manifest.json")
    if os.path.exists(path):
        with open(path) as f:
            m = json.load(f)
        syn = m.get("synthetic", {})
        if (syn.get("seed") == seed and syn.get("normMode") == norm_mode and syn.get("shape") == asdict(shape)
                and syn.get("nibbles", "uniform") == nibbles):
            return m
    return write_runtime(out_dir, shape, seed, norm_mode, nibbles=nibbles)


# ---- single-kernel workloads -------------------------------------------------

def matvec_case(out_size: int, in_size: int, seed: int = 0):
    """q4 matvec inputs: x ~ N(0,1) f32, uniform nibbles, |N(0,0.02)| f16 scales."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal(in_size, dtype=np.float32)
    words, scales = q4_projection(rng, out_size, in_size)
    return x, words, scales


def lm_head_case(vocab: int = 151936, hidden: int = 1024, seed: int = 1, eps: float = 1e-6):
    """LM-head inputs: f16 table ~ N(0,0.02), x ~ N(0,1) then RMSNorm (unit weight)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    table = f16_round(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.02)
    x = rng.standard_normal(hidden, dtype=np.float32)
    return table, x, eps
