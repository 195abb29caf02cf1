"""ctypes binding of libqdecode.so (the C ABI declared in include/qdecode.h).

There is no fallback: if the CUDA library cannot be built or loaded, every call
raises. The library is built in-tree (kernel_optimization_webgpu_b200/libqdecode.so).
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

QD_OK = 0
QD_E_INVALID = -1
QD_E_IO = -2
QD_E_CUDA = -3
QD_E_NOMEM = -4
QD_E_RANGE = -5
QD_E_DEVICE = -6
QD_E_TIMEOUT = -7
QD_KV_F16 = 0
QD_KV_F32 = 1

# Every function include/qdecode.h declares (checked by the tests).
EXPORTS = (
    "qd_options_default", "qd_engine_create", "qd_engine_destroy", "qd_last_error",
    "qd_engine_profile", "qd_generate_greedy", "qd_engine_logits", "qd_engine_hidden",
    "qd_engine_forward_trace", "qd_engine_uses_persistent", "qd_engine_timeline",
    "qd_q4_matvec",
    "qd_q4_gemm_workspace_bytes", "qd_q4_gemm", "qd_lm_head_argmax_workspace_bytes",
    "qd_lm_head_argmax", "qd_gqa_decode_workspace_bytes", "qd_gqa_decode",
    "qd_engine_set_stream", "qd_decode_begin", "qd_decode_step", "qd_decode_seek", "qd_decode_sync",
    "qd_decode_step_kernels", "qd_gqa_decode_noalloc",
    "qd_batch_create", "qd_batch_destroy", "qd_batch_size", "qd_batch_fill_context", "qd_batch_set_tokens",
    "qd_batch_positions", "qd_batch_decode", "qd_batch_prefill", "qd_batch_keep_logits", "qd_batch_logits",
    "qd_batch_read_kv", "qd_batch_write_kv", "qd_batch_step_kernels", "qd_generate_batch",
    "qd_batch_set_vocab_shard", "qd_batch_step_layers", "qd_batch_step_lm_slice", "qd_batch_step_merge",
    "qd_batch_shard_sync", "qd_engine_inject_stall", "qd_batch_inject_stall",
    "qd_run_kernel_benchmarks", "qd_run_full_decoder_stack_benchmark",
    "qd_generate_sample", "qd_sample_workspace_bytes", "qd_sample_logits",
)


class QdOptions(C.Structure):
    _fields_ = [("device", C.c_int), ("max_seq", C.c_int), ("kv_dtype", C.c_int),
                ("rope_row_stride", C.c_int), ("variant", C.c_char_p), ("use_graph", C.c_int),
                ("persistent", C.c_int), ("timeline", C.c_int), ("prompt_pass", C.c_int)]


class QdProfile(C.Structure):
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("intermediate", C.c_int),
                ("heads", C.c_int), ("kv_heads", C.c_int), ("head_dim", C.c_int),
                ("vocab", C.c_int), ("rope_rows", C.c_int), ("eps", C.c_float)]


class QdStats(C.Structure):
    _fields_ = [("generate_ms", C.c_double), ("first_token_ms", C.c_double),
                ("steady_ms_per_token", C.c_double), ("generated_tokens", C.c_int),
                ("prompt_tokens", C.c_int)]


class QdSampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("seed", C.c_uint64)]


class QdKernelBench(C.Structure):
    _fields_ = [(n, C.c_double) for n in (
        "baseline_matvec_ms", "optimized_matvec_ms", "matvec_speedup", "baseline_bytes", "optimized_bytes",
        "memory_reduction", "max_abs_error", "mean_abs_error", "block_default_ms", "block_optimized_ms",
        "block_speedup", "block_max_abs_error", "block_mean_abs_error", "real_q4_ms", "real_q4_max_abs_error",
        "real_q4_mean_abs_error", "gqa_ms", "gqa_max_abs_error", "gqa_mean_abs_error")] + [
        ("gqa_seq_len", C.c_int), ("layer0_finite", C.c_int), ("layer0_decode_ms", C.c_double),
        ("layer0_mean_abs", C.c_double), ("rms_ms", C.c_double), ("estimated_gbps", C.c_double)]


class QdStackBench(C.Structure):
    _fields_ = [("ms", C.c_double), ("warmup_ms", C.c_double), ("layers", C.c_int), ("finite", C.c_int),
                ("mean_abs", C.c_double)]


TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)


class QdError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"qdecode error {code}: {msg}")
        self.code = code


_lib = None


def lib_path() -> str:
    return _build.LIB


def load(build_if_stale: bool = True):
    """Load libqdecode.so (building it first when sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if build_if_stale:
        _build.build()
    if not os.path.exists(_build.LIB):
        raise QdError(QD_E_INVALID, f"CUDA library missing: {_build.LIB}")
    L = C.CDLL(_build.LIB)
    vp, i32, u32, f32 = C.c_void_p, C.c_int, C.c_uint32, C.c_float
    L.qd_options_default.argtypes = [C.POINTER(QdOptions)]
    L.qd_options_default.restype = None
    L.qd_engine_create.argtypes = [C.c_char_p, C.POINTER(QdOptions), C.POINTER(vp)]
    L.qd_engine_create.restype = i32
    L.qd_engine_destroy.argtypes = [vp]
    L.qd_engine_destroy.restype = None
    L.qd_last_error.argtypes = [vp]
    L.qd_last_error.restype = C.c_char_p
    L.qd_engine_profile.argtypes = [vp, C.POINTER(QdProfile)]
    L.qd_engine_profile.restype = i32
    L.qd_generate_greedy.argtypes = [vp, vp, i32, i32, vp, TOKEN_CB, vp, C.POINTER(QdStats)]
    L.qd_generate_greedy.restype = i32
    L.qd_engine_logits.argtypes = [vp, vp]
    L.qd_engine_logits.restype = i32
    L.qd_engine_hidden.argtypes = [vp, vp]
    L.qd_engine_hidden.restype = i32
    L.qd_engine_forward_trace.argtypes = [vp, C.c_int32, i32, vp]
    L.qd_engine_forward_trace.restype = i32
    L.qd_engine_uses_persistent.argtypes = [vp]
    L.qd_engine_uses_persistent.restype = i32
    L.qd_engine_timeline.argtypes = [vp, vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.qd_engine_timeline.restype = i32
    L.qd_engine_set_stream.argtypes = [vp, vp]
    L.qd_engine_set_stream.restype = i32
    L.qd_decode_begin.argtypes = [vp, vp, i32, i32]
    L.qd_decode_begin.restype = i32
    L.qd_decode_step.argtypes = [vp]
    L.qd_decode_step.restype = i32
    L.qd_decode_seek.argtypes = [vp, i32]
    L.qd_decode_seek.restype = i32
    L.qd_decode_sync.argtypes = [vp, vp, i32]
    L.qd_decode_sync.restype = i32
    L.qd_decode_step_kernels.argtypes = [vp]
    L.qd_decode_step_kernels.restype = i32
    L.qd_q4_matvec.argtypes = [vp, vp, vp, vp, u32, u32, u32, u32, vp]
    L.qd_q4_matvec.restype = i32
    L.qd_q4_gemm_workspace_bytes.argtypes = [u32, u32]
    L.qd_q4_gemm_workspace_bytes.restype = C.c_size_t
    L.qd_q4_gemm.argtypes = [vp, vp, vp, vp, u32, u32, u32, u32, vp, vp]
    L.qd_q4_gemm.restype = i32
    L.qd_lm_head_argmax_workspace_bytes.argtypes = [u32]
    L.qd_lm_head_argmax_workspace_bytes.restype = C.c_size_t
    L.qd_lm_head_argmax.argtypes = [vp, vp, f32, vp, vp, vp, u32, u32, vp, vp]
    L.qd_lm_head_argmax.restype = i32
    L.qd_gqa_decode_workspace_bytes.argtypes = [u32, u32]
    L.qd_gqa_decode_workspace_bytes.restype = C.c_size_t
    L.qd_gqa_decode.argtypes = [vp, vp, vp, i32, vp, u32, u32, u32, u32, vp, vp]
    L.qd_gqa_decode.restype = i32
    L.qd_gqa_decode_noalloc.argtypes = [vp, vp, vp, i32, vp, u32, u32, u32, u32, vp]
    L.qd_gqa_decode_noalloc.restype = i32
    ip = C.POINTER(C.c_int)
    L.qd_batch_create.argtypes = [vp, i32, i32, C.POINTER(vp)]
    L.qd_batch_create.restype = i32
    L.qd_batch_destroy.argtypes = [vp]
    L.qd_batch_destroy.restype = None
    L.qd_batch_size.argtypes = [vp, ip, ip]
    L.qd_batch_size.restype = i32
    L.qd_batch_fill_context.argtypes = [vp, i32, u32]
    L.qd_batch_fill_context.restype = i32
    L.qd_batch_set_tokens.argtypes = [vp, vp, vp]
    L.qd_batch_set_tokens.restype = i32
    L.qd_batch_positions.argtypes = [vp, vp]
    L.qd_batch_positions.restype = i32
    L.qd_batch_decode.argtypes = [vp, i32, vp]
    L.qd_batch_decode.restype = i32
    L.qd_batch_prefill.argtypes = [vp, vp, i32, vp]
    L.qd_batch_prefill.restype = i32
    L.qd_batch_keep_logits.argtypes = [vp, i32]
    L.qd_batch_keep_logits.restype = i32
    L.qd_batch_logits.argtypes = [vp, vp]
    L.qd_batch_logits.restype = i32
    L.qd_batch_read_kv.argtypes = [vp, i32, i32, i32, i32, vp, vp]
    L.qd_batch_read_kv.restype = i32
    L.qd_batch_write_kv.argtypes = [vp, i32, i32, i32, i32, vp, vp]
    L.qd_batch_write_kv.restype = i32
    L.qd_batch_step_kernels.argtypes = [vp]
    L.qd_batch_step_kernels.restype = i32
    L.qd_generate_batch.argtypes = [vp, i32, vp, i32, i32, vp]
    L.qd_generate_batch.restype = i32
    L.qd_batch_set_vocab_shard.argtypes = [vp, i32, i32, vp, vp, vp, vp]
    L.qd_batch_set_vocab_shard.restype = i32
    for name in ("qd_batch_step_layers", "qd_batch_step_lm_slice", "qd_batch_step_merge"):
        getattr(L, name).argtypes = [vp]
        getattr(L, name).restype = i32
    L.qd_batch_shard_sync.argtypes = [vp, i32, vp]
    L.qd_batch_shard_sync.restype = i32
    L.qd_generate_sample.argtypes = [vp, vp, i32, i32, C.POINTER(QdSampling), vp, TOKEN_CB, vp,
                                     C.POINTER(QdStats)]
    L.qd_generate_sample.restype = i32
    L.qd_sample_workspace_bytes.argtypes = [u32]
    L.qd_sample_workspace_bytes.restype = C.c_size_t
    L.qd_sample_logits.argtypes = [vp, u32, C.POINTER(QdSampling), u32, vp, vp, vp]
    L.qd_sample_logits.restype = i32
    L.qd_run_kernel_benchmarks.argtypes = [vp, C.POINTER(QdKernelBench)]
    L.qd_run_kernel_benchmarks.restype = i32
    L.qd_run_full_decoder_stack_benchmark.argtypes = [vp, C.POINTER(QdStackBench)]
    L.qd_run_full_decoder_stack_benchmark.restype = i32
    L.qd_engine_inject_stall.argtypes = [vp]
    L.qd_engine_inject_stall.restype = i32
    L.qd_batch_inject_stall.argtypes = [vp]
    L.qd_batch_inject_stall.restype = i32
    _lib = L
    return L


def check(rc: int, engine=None) -> None:
    if rc != QD_OK:
        msg = load().qd_last_error(engine)
        raise QdError(rc, msg.decode() if msg else "")
