"""ctypes wrapper of the CPU oracle. TEST INFRASTRUCTURE ONLY.

Only the tests, the smoke check and the benchmark's CPU-baseline leg import this
module, as the checker. The product library never calls it. See oracle.h for
what each function restates and for the parity status ("parity unpinned"
against an executed reference; pinned against the reference's own JavaScript
CPU check functions, ported literally in tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        srcs = [os.path.join(HERE, f) for f in ("oracle.c", "oracle.h")]
        if not os.path.exists(LIB_PATH) or any(os.path.getmtime(f) > os.path.getmtime(LIB_PATH) for f in srcs):
            build()
        L = C.CDLL(LIB_PATH)
        u32, i32, f32, vp = C.c_uint32, C.c_int, C.c_float, C.c_void_p
        L.qo_half_to_float.argtypes = [C.c_uint16]; L.qo_half_to_float.restype = f32
        L.qo_float_to_half.argtypes = [f32]; L.qo_float_to_half.restype = C.c_uint16
        L.qo_q4_matvec.argtypes = [_f32p, _u32p, _f32p, _f32p, u32, u32, u32, u32]
        L.qo_q4_matvec_original.argtypes = [_f32p, _u32p, _f32p, _f32p, u32, u32, u32, u32]
        L.qo_rms_norm.argtypes = [_f32p, _f32p, _f32p, u32, f32]
        L.qo_head_rms_norm.argtypes = [_f32p, _f32p, _f32p, u32, u32, f32]
        L.qo_rope.argtypes = [_f32p, _f32p, _f32p, _f32p, u32, u32, u32, u32]
        L.qo_cache_write.argtypes = [_f32p, _f32p, u32, u32, i32]
        L.qo_gqa_decode.argtypes = [_f32p, _f32p, _f32p, _f32p, u32, u32, u32, u32]
        L.qo_silu_mul.argtypes = [_f32p, _f32p, _f32p, u32]
        L.qo_residual_add.argtypes = [_f32p, _f32p, _f32p, u32]
        L.qo_lm_head_f16.argtypes = [_f32p, _u16p, _f32p, u32, u32]
        L.qo_argmax.argtypes = [_f32p, u32, _u32p]
        L.qo_model_new.argtypes = [i32] * 8 + [f32]; L.qo_model_new.restype = vp
        L.qo_model_free.argtypes = [vp]
        L.qo_model_set_shared.argtypes = [vp, vp, vp, vp, vp]
        L.qo_model_set_layer.argtypes = [vp, i32, vp, vp, vp, vp, C.POINTER(vp), C.POINTER(vp)]
        L.qo_session_new.argtypes = [vp, i32, i32, i32]; L.qo_session_new.restype = vp
        L.qo_session_free.argtypes = [vp]
        L.qo_session_set_trace.argtypes = [vp, vp]
        L.qo_session_kv.argtypes = [vp, i32, i32]; L.qo_session_kv.restype = C.POINTER(f32)
        L.qo_session_set_kv.argtypes = [vp, i32, i32, i32, _f32p, _f32p]; L.qo_session_set_kv.restype = i32
        L.qo_forward.argtypes = [vp, i32, i32]; L.qo_forward.restype = i32
        L.qo_session_final_hidden.argtypes = [vp]; L.qo_session_final_hidden.restype = C.POINTER(f32)
        L.qo_session_hidden.argtypes = [vp]; L.qo_session_hidden.restype = C.POINTER(f32)
        L.qo_next_token.argtypes = [vp, vp, _u32p, vp]; L.qo_next_token.restype = i32
        L.qo_greedy.argtypes = [vp, vp, i32, i32, vp, vp]; L.qo_greedy.restype = i32
        L.qo_sample.argtypes = [vp, C.c_uint32, C.c_float, i32, C.c_float, C.c_uint64, C.c_uint32]
        L.qo_sample.restype = C.c_int32
        L.qo_generate_sample.argtypes = [vp, vp, i32, i32, C.c_float, i32, C.c_float, C.c_uint64, vp]
        L.qo_generate_sample.restype = i32
        L.qo_num_threads.restype = i32
        L.qo_set_num_threads.argtypes = [i32]
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def half_to_float(bits: int) -> float:
    return lib().qo_half_to_float(bits)


def float_to_half(x: float) -> int:
    return lib().qo_float_to_half(x)


def q4_matvec(x, words, scales, in_size=None, out_size=None, block_size=32, original=False):
    x = _c(x, np.float32)
    words = _c(words, np.uint32)
    scales = _c(scales, np.float32)
    out_size = out_size or words.shape[0]
    blocks_per_row = scales.size // out_size
    in_size = in_size or blocks_per_row * block_size
    y = np.zeros(out_size, np.float32)
    fn = lib().qo_q4_matvec_original if original else lib().qo_q4_matvec
    fn(x, words.reshape(-1), scales.reshape(-1), y, in_size, out_size, blocks_per_row, block_size)
    return y


def rms_norm(x, w, eps=1e-6):
    x = _c(x, np.float32)
    y = np.zeros_like(x)
    lib().qo_rms_norm(x, _c(w, np.float32), y, x.size, eps)
    return y


def head_rms_norm(x, w, head_dim, heads, eps=1e-6):
    x = _c(x, np.float32)
    y = np.zeros_like(x)
    lib().qo_head_rms_norm(x, _c(w, np.float32), y, head_dim, heads, eps)
    return y


def rope(x, cos_tab, sin_tab, heads, head_dim, position, row_stride=None):
    x = _c(x, np.float32)
    y = np.zeros_like(x)
    lib().qo_rope(x, _c(cos_tab, np.float32).reshape(-1), _c(sin_tab, np.float32).reshape(-1), y,
                  heads, head_dim, position, row_stride or head_dim)
    return y


def gqa_decode(q, k_cache, v_cache, seq_len, q_heads, kv_heads, head_dim):
    y = np.zeros(q_heads * head_dim, np.float32)
    lib().qo_gqa_decode(_c(q, np.float32), _c(k_cache, np.float32).reshape(-1),
                        _c(v_cache, np.float32).reshape(-1), y, seq_len, q_heads, kv_heads, head_dim)
    return y


def silu_mul(g, u):
    g = _c(g, np.float32)
    y = np.zeros_like(g)
    lib().qo_silu_mul(g, _c(u, np.float32), y, g.size)
    return y


def lm_head_f16(hidden, table_f16):
    t = _c(table_f16, np.float16)
    rows, hs = t.shape
    logits = np.zeros(rows, np.float32)
    lib().qo_lm_head_f16(_c(hidden, np.float32), t.view(np.uint16).reshape(-1), logits, hs, rows)
    return logits


def sample(logits, temperature: float, top_k: int, top_p: float, seed: int, step: int) -> int:
    """qo_sample: one draw from logits with the library's top-k / top-p definition."""
    logits = _c(logits, np.float32)
    return int(lib().qo_sample(logits.ctypes.data, logits.size, temperature, top_k, top_p,
                               seed & 0xFFFFFFFFFFFFFFFF, step))


def argmax(logits):
    logits = _c(logits, np.float32)
    r = np.zeros(2, np.uint32)
    lib().qo_argmax(logits, logits.size, r)
    return int(r[0]), float(r[1:2].view(np.float32)[0])


PROJ_ORDER = ("q", "k", "v", "o", "gate", "up", "down")


class Model:
    """A runtime directory (reference layout) loaded for the oracle."""

    def __init__(self, runtime_dir: str):
        with open(os.path.join(runtime_dir, "manifest.json")) as f:
            m = json.load(f)
        self.manifest = m
        rd = lambda e, dt: np.fromfile(os.path.join(runtime_dir, e["file"]), dtype=dt)  # noqa: E731
        f16f32 = lambda e: rd(e, np.float16).astype(np.float32)  # noqa: E731
        self.hidden = m["hiddenSize"]
        self.inter = m["intermediateSize"]
        self.heads = m["attentionHeads"]
        self.kv_heads = m["kvHeads"]
        self.head_dim = m["headDim"]
        self.eps = float(m.get("normEpsilon", 1e-6))
        self.embed = rd(m["shared"]["embedTokens"], np.uint16)
        self.vocab = m["shared"]["embedTokens"]["dims"][0]
        self.cos = f16f32(m["shared"]["cosCache"])
        self.sin = f16f32(m["shared"]["sinCache"])
        self.rope_rows = m["shared"]["cosCache"]["dims"][0]
        self.final_norm = f16f32(m["finalNorm"])
        self.layers = []
        for le in m["layers"]:
            norms = {k: f16f32(le["norms"][k]) for k in ("input", "q", "k", "postAttention")}
            w = [rd(le["projections"][p]["weight"], np.uint32) for p in PROJ_ORDER]
            s = [rd(le["projections"][p]["scales"], np.float32) for p in PROJ_ORDER]
            self.layers.append((norms, w, s))
        L = lib()
        self._h = L.qo_model_new(len(self.layers), self.hidden, self.inter, self.heads, self.kv_heads,
                                 self.head_dim, self.vocab, self.rope_rows, self.eps)
        L.qo_model_set_shared(self._h, self.embed.ctypes.data, self.cos.ctypes.data,
                              self.sin.ctypes.data, self.final_norm.ctypes.data)
        for i, (norms, w, s) in enumerate(self.layers):
            wp = (C.c_void_p * 7)(*[a.ctypes.data for a in w])
            sp = (C.c_void_p * 7)(*[a.ctypes.data for a in s])
            L.qo_model_set_layer(self._h, i, norms["input"].ctypes.data, norms["q"].ctypes.data,
                                 norms["k"].ctypes.data, norms["postAttention"].ctypes.data, wp, sp)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().qo_model_free(self._h)
            self._h = None

    def session(self, max_seq: int = 256, kv_f16: bool = True, rope_row_stride: int = 0) -> "Session":
        return Session(self, max_seq, kv_f16, rope_row_stride)


class Session:
    def __init__(self, model: Model, max_seq: int, kv_f16: bool, rope_row_stride: int):
        self.model = model
        self.max_seq = max_seq
        self._h = lib().qo_session_new(model._h, max_seq, int(kv_f16), rope_row_stride)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().qo_session_free(self._h)
            self._h = None

    def kv(self, layer: int, pos0: int, count: int):
        """Cached K and V rows [pos0, pos0 + count) of `layer` (copies)."""
        kvs = self.model.kv_heads * self.model.head_dim
        out = []
        for which in (0, 1):
            p = lib().qo_session_kv(self._h, layer, which)
            a = np.ctypeslib.as_array(p, shape=(self.max_seq, kvs))
            out.append(a[pos0:pos0 + count].copy())
        return out[0], out[1]

    def set_kv(self, layer: int, pos0: int, k, v) -> None:
        """Cached K/V rows [pos0, pos0 + len(k)) of `layer` ([n][kv_heads * head_dim] f32)."""
        k = _c(k, np.float32)
        v = _c(v, np.float32)
        if lib().qo_session_set_kv(self._h, layer, pos0, k.shape[0], k.reshape(-1), v.reshape(-1)):
            raise ValueError("oracle set_kv: rows outside the cache")

    def forward(self, token: int, position: int, trace: bool = False):
        tr = None
        if trace:
            tr = np.zeros((len(self.model.layers), self.model.hidden), np.float32)
            lib().qo_session_set_trace(self._h, tr.ctypes.data)
        rc = lib().qo_forward(self._h, token, position)
        if trace:
            lib().qo_session_set_trace(self._h, None)
        if rc:
            raise ValueError(f"oracle forward failed: {rc}")
        return tr

    def final_hidden(self) -> np.ndarray:
        p = lib().qo_session_final_hidden(self._h)
        return np.ctypeslib.as_array(p, shape=(self.model.hidden,)).copy()

    def hidden(self) -> np.ndarray:
        """Residual stream after the last layer (before the final RMSNorm)."""
        p = lib().qo_session_hidden(self._h)
        return np.ctypeslib.as_array(p, shape=(self.model.hidden,)).copy()

    def next_token(self):
        logits = np.zeros(self.model.vocab, np.float32)
        r = np.zeros(2, np.uint32)
        margin = C.c_float()
        lib().qo_next_token(self._h, logits.ctypes.data, r, C.addressof(margin))
        return int(r[0]), logits, float(margin.value)

    def sample(self, ids, max_new: int, temperature: float, top_k: int, top_p: float, seed: int):
        """qo_generate_sample: the greedy flow with each token drawn by sample()."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        rc = lib().qo_generate_sample(self._h, ids.ctypes.data, ids.size, max_new, temperature, top_k, top_p,
                                      seed & 0xFFFFFFFFFFFFFFFF, out.ctypes.data)
        if rc:
            raise ValueError(f"oracle sample failed: {rc}")
        return out[:max_new].tolist()

    def greedy(self, ids, max_new: int):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(max_new, np.int32)
        margins = np.zeros(max_new, np.float32)
        rc = lib().qo_greedy(self._h, ids.ctypes.data, ids.size, max_new, out.ctypes.data,
                             margins.ctypes.data)
        if rc:
            raise ValueError(f"oracle greedy failed: {rc}")
        return out.tolist(), margins
