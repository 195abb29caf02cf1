"""Host-side API over libqdecode.so.

Two layers:

* `Engine` and the kernel-level functions (`q4_matvec`, `lm_head_argmax`,
  `gqa_decode`) - thin, typed wrappers of the C ABI.
* `createWebGpuContext` / `runCustomQwenGreedyPrompt` - the reference's own
  JavaScript entry points (src/bench/webgpu-runtime.js:43-60 and :165-214),
  same argument names, same result object and the same error on an over-long
  request, so callers of the reference switch by changing the import.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Callable, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import QD_KV_F16, QD_KV_F32, QdError, QdOptions, QdProfile, QdStats, check

# qwenProfile, src/model/qwen3-0.6b.js:1-15.
qwen_profile = {
    "modelId": "Qwen/Qwen3-0.6B",
    "parameters": "0.6B",
    "nonEmbeddingParameters": "0.44B",
    "layers": 28,
    "hiddenSize": 1024,
    "intermediateSize": 3072,
    "attentionHeads": 16,
    "kvHeads": 8,
    "headDim": 128,
    "contextLength": 32768,
    "vocabSize": 151936,
    "normEpsilon": 1e-6,
    "quantizationTarget": "weight-only Q4 MatMulNBits for projection and MLP matvecs",
}
qwenProfile = qwen_profile

VARIANTS = ("original", "mixed", "optimized")


class Engine:
    """One model resident on one GPU (qd_engine_create / qd_generate_greedy)."""

    def __init__(self, runtime_dir: str, device: int = 0, max_seq: int = 256, kv_dtype: str = "f16",
                 rope_row_stride: int = 0, variant: str = "optimized", use_graph: bool = True,
                 persistent: "bool | int" = True, timeline: bool = False, prompt_pass: bool = True):
        L = _lib.load()
        opt = QdOptions()
        L.qd_options_default(C.byref(opt))
        opt.device = device
        opt.max_seq = max_seq
        opt.kv_dtype = {"f16": QD_KV_F16, "f32": QD_KV_F32}[kv_dtype]
        opt.rope_row_stride = rope_row_stride
        self._variant = variant.encode()
        opt.variant = self._variant
        opt.use_graph = int(use_graph)
        # True/nonzero: one persistent kernel per token (one CTA per SM); False/0: one
        # kernel per fused stage.
        opt.persistent = int(persistent)
        opt.timeline = int(timeline)
        # True: a prompt's first 5..256 tokens take one batched pass (f16 KV cache);
        # False: every prompt token goes through the decode kernel.
        opt.prompt_pass = int(prompt_pass)
        h = C.c_void_p()
        check(L.qd_engine_create(os.fsencode(runtime_dir), C.byref(opt), C.byref(h)))
        self._h = h
        self.max_seq = max_seq
        self.variant = variant
        p = QdProfile()
        check(L.qd_engine_profile(self._h, C.byref(p)), self._h)
        self.profile = {f: getattr(p, f) for f, _ in QdProfile._fields_}

    def close(self) -> None:
        if getattr(self, "_h", None) and _lib is not None and _lib._lib is not None:
            _lib._lib.qd_engine_destroy(self._h)
        self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def generate_greedy(self, ids: Sequence[int], max_new: int,
                        on_token: Optional[Callable[[int], object]] = None):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        st = QdStats()
        err: list = []

        def _cb(tok, _user):
            try:
                return 1 if (on_token and on_token(int(tok)) is False) else 0
            except BaseException as ex:  # surface callback errors after the C call returns
                err.append(ex)
                return 1

        cb = _lib.TOKEN_CB(_cb)
        rc = _lib.load().qd_generate_greedy(self._h, ids.ctypes.data, int(ids.size), int(max_new),
                                            out.ctypes.data, cb, None, C.byref(st))
        check(rc, self._h)
        if err:
            raise err[0]
        stats = {f: getattr(st, f) for f, _ in QdStats._fields_}
        return out[:st.generated_tokens].tolist(), stats

    def generate_sample(self, ids: Sequence[int], max_new: int, temperature: float = 1.0, top_k: int = 0,
                        top_p: float = 1.0, seed: int = 0, on_token: Optional[Callable[[int], object]] = None):
        """qd_generate_sample: the greedy flow with each token drawn by top-k / top-p
        sampling (temperature <= 0 or top_k == 1: greedy)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        st = QdStats()
        err: list = []

        def _cb(tok, _user):
            try:
                return 1 if (on_token and on_token(int(tok)) is False) else 0
            except BaseException as ex:
                err.append(ex)
                return 1

        cb = _lib.TOKEN_CB(_cb)
        sp = _lib.QdSampling(float(temperature), int(top_k), float(top_p), int(seed) & 0xFFFFFFFFFFFFFFFF)
        rc = _lib.load().qd_generate_sample(self._h, ids.ctypes.data, int(ids.size), int(max_new), C.byref(sp),
                                            out.ctypes.data, cb, None, C.byref(st))
        check(rc, self._h)
        if err:
            raise err[0]
        stats = {f: getattr(st, f) for f, _ in QdStats._fields_}
        return out[:st.generated_tokens].tolist(), stats

    # stepping interface (enqueue only)
    def set_stream(self, stream=None) -> None:
        """Enqueue on a torch.cuda.Stream (None: the engine's own stream). The legacy
        default stream (handle 0) is refused: the C ABI reads a NULL stream as the
        engine's own stream, which would not be ordered with work on the default one."""
        if stream is not None and stream.cuda_stream == 0:
            raise ValueError("pass a created torch.cuda.Stream(), not the legacy default stream")
        ptr = C.c_void_p(stream.cuda_stream) if stream is not None else None
        check(_lib.load().qd_engine_set_stream(self._h, ptr), self._h)

    def decode_begin(self, ids: Sequence[int], max_new: int) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        check(_lib.load().qd_decode_begin(self._h, ids.ctypes.data, int(ids.size), int(max_new)), self._h)

    def decode_step(self) -> None:
        check(_lib.load().qd_decode_step(self._h), self._h)

    def decode_seek(self, position: int) -> None:
        check(_lib.load().qd_decode_seek(self._h, int(position)), self._h)

    def decode_sync(self, n: int = 0) -> list:
        out = np.zeros(max(n, 1), np.int32)
        check(_lib.load().qd_decode_sync(self._h, out.ctypes.data, int(n)), self._h)
        return out[:n].tolist()

    def timeline(self) -> np.ndarray:
        """Stage stamps (ns) of the last persistent launch, shape [ctas][events]."""
        L = _lib.load()
        ctas, ev = C.c_int(), C.c_int()
        check(L.qd_engine_timeline(self._h, None, C.byref(ctas), C.byref(ev)), self._h)
        out = np.zeros((ctas.value, ev.value), np.uint64)
        check(L.qd_engine_timeline(self._h, out.ctypes.data, None, None), self._h)
        return out

    @property
    def persistent(self) -> bool:
        return bool(_lib.load().qd_engine_uses_persistent(self._h))

    @property
    def token_kernel(self) -> int:
        """1: the persistent kernel, 0: one kernel per stage."""
        return int(_lib.load().qd_engine_uses_persistent(self._h))

    @property
    def step_kernels(self) -> int:
        return int(_lib.load().qd_decode_step_kernels(self._h))

    def logits(self) -> np.ndarray:
        out = np.zeros(self.profile["vocab"], np.float32)
        check(_lib.load().qd_engine_logits(self._h, out.ctypes.data), self._h)
        return out

    def inject_stall(self) -> None:
        """Test hook: the next persistent decode launch withholds layer 0's q/k/v
        results, so its bounded waits run out (qd_engine_inject_stall)."""
        check(_lib.load().qd_engine_inject_stall(self._h), self._h)

    def hidden(self) -> np.ndarray:
        out = np.zeros(self.profile["hidden"], np.float32)
        check(_lib.load().qd_engine_hidden(self._h, out.ctypes.data), self._h)
        return out

    def forward_trace(self, token: int, position: int) -> np.ndarray:
        out = np.zeros((self.profile["layers"], self.profile["hidden"]), np.float32)
        check(_lib.load().qd_engine_forward_trace(self._h, int(token), int(position), out.ctypes.data), self._h)
        return out


class Batch:
    """B independent sequences decoded together on an engine's weights (qd_batch_*).

    The batch owns its KV cache ([layer][seq][kv_head][max_seq][128] f16); the
    engine must outlive it."""

    def __init__(self, engine: Engine, batch: int, max_seq: int):
        L = _lib.load()
        h = C.c_void_p()
        check(L.qd_batch_create(engine._h, int(batch), int(max_seq), C.byref(h)))
        self._h = h
        self.engine = engine
        self.batch = batch
        self.max_seq = max_seq

    def close(self) -> None:
        if getattr(self, "_h", None) and _lib is not None and _lib._lib is not None:
            _lib._lib.qd_batch_destroy(self._h)
        self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def fill_context(self, ctx: int, seed: int) -> None:
        check(_lib.load().qd_batch_fill_context(self._h, int(ctx), int(seed) & 0xFFFFFFFF))

    def set_tokens(self, tokens=None, positions=None) -> None:
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        p = None if positions is None else np.ascontiguousarray(positions, dtype=np.int32)
        for a in (t, p):
            if a is not None and a.size != self.batch:
                raise ValueError(f"expected {self.batch} entries")
        check(_lib.load().qd_batch_set_tokens(self._h, None if t is None else t.ctypes.data,
                                              None if p is None else p.ctypes.data))

    def positions(self) -> np.ndarray:
        out = np.zeros(self.batch, np.int32)
        check(_lib.load().qd_batch_positions(self._h, out.ctypes.data))
        return out

    def decode(self, steps: int, want_ids: bool = True) -> Optional[np.ndarray]:
        """`steps` greedy steps of every sequence; ids [steps][batch]."""
        out = np.zeros((max(steps, 1), self.batch), np.int32) if want_ids else None
        check(_lib.load().qd_batch_decode(self._h, int(steps), None if out is None else out.ctypes.data))
        return None if out is None else out[:steps]

    def prefill(self, ids) -> np.ndarray:
        """Prompts [batch][n] at positions 0..n-1; returns each sequence's first generated id."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        if ids.ndim != 2 or ids.shape[0] != self.batch:
            raise ValueError(f"ids must be [{self.batch}][n_prompt]")
        out = np.zeros(self.batch, np.int32)
        check(_lib.load().qd_batch_prefill(self._h, ids.ctypes.data, int(ids.shape[1]), out.ctypes.data))
        return out

    def keep_logits(self, keep: bool = True) -> None:
        check(_lib.load().qd_batch_keep_logits(self._h, int(keep)))

    def logits(self) -> np.ndarray:
        out = np.zeros((self.batch, self.engine.profile["vocab"]), np.float32)
        check(_lib.load().qd_batch_logits(self._h, out.ctypes.data))
        return out

    def read_kv(self, layer: int, seq: int, pos0: int, count: int):
        kvs = self.engine.profile["kv_heads"] * self.engine.profile["head_dim"]
        k = np.zeros((count, kvs), np.float32)
        v = np.zeros((count, kvs), np.float32)
        check(_lib.load().qd_batch_read_kv(self._h, int(layer), int(seq), int(pos0), int(count),
                                           k.ctypes.data, v.ctypes.data))
        return k, v

    def write_kv(self, layer: int, seq: int, pos0: int, k, v) -> None:
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        check(_lib.load().qd_batch_write_kv(self._h, int(layer), int(seq), int(pos0), int(k.shape[0]),
                                            k.ctypes.data, v.ctypes.data))

    @property
    def step_kernels(self) -> int:
        return int(_lib.load().qd_batch_step_kernels(self._h))

    def inject_stall(self) -> None:
        """Test hook: one CTA of the next tensor-core GEMM withholds its first
        activation tiles, so its bounded waits run out (qd_batch_inject_stall)."""
        check(_lib.load().qd_batch_inject_stall(self._h))

    # ---- vocabulary-sharded LM head (qd_batch_set_vocab_shard) ----------------------------
    def set_vocab_shard(self, rank: int, world: int, device=None) -> dict:
        """Split the LM head by vocabulary over `world` ranks (this batch is rank `rank`).
        Allocates the exchange buffers as torch CUDA tensors and returns them:
        gather_hi / gather_lo f16 [world*batch][hidden] (this rank's rows at rank*batch),
        pairs_local int32 [world*batch][2], pairs_all int32 [world][world*batch][2]."""
        import torch

        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        rows, H = world * self.batch, self.engine.profile["hidden"]
        bufs = {
            "gather_hi": torch.zeros((rows, H), dtype=torch.float16, device=dev),
            "gather_lo": torch.zeros((rows, H), dtype=torch.float16, device=dev),
            "pairs_local": torch.zeros((rows, 2), dtype=torch.int32, device=dev),
            "pairs_all": torch.zeros((world, rows, 2), dtype=torch.int32, device=dev),
        }
        check(_lib.load().qd_batch_set_vocab_shard(self._h, int(rank), int(world),
                                                   *(C.c_void_p(bufs[k].data_ptr()) for k in
                                                     ("gather_hi", "gather_lo", "pairs_local", "pairs_all"))))
        self._shard = (int(rank), int(world), bufs)
        return bufs

    def step_layers(self) -> None:
        check(_lib.load().qd_batch_step_layers(self._h))

    def step_lm_slice(self) -> None:
        check(_lib.load().qd_batch_step_lm_slice(self._h))

    def step_merge(self) -> None:
        check(_lib.load().qd_batch_step_merge(self._h))

    def shard_sync(self, steps: int) -> np.ndarray:
        out = np.zeros((max(steps, 1), self.batch), np.int32)
        check(_lib.load().qd_batch_shard_sync(self._h, int(steps), out.ctypes.data))
        return out[:steps]

    def decode_sharded(self, steps: int, all_gather) -> np.ndarray:
        """`steps` greedy steps with the vocabulary-sharded LM head; ids [steps][batch]
        (see sharded_decode)."""
        return sharded_decode(self, steps, all_gather)


def sharded_decode(batch, steps: int, all_gather) -> np.ndarray:
    """The per-step flow of the vocabulary-sharded LM head on one rank: layers, all-gather
    of the final-norm rows, this rank's vocabulary slice for every row, all-gather of the
    (index, value) pairs, merge of this rank's rows. all_gather(out, inp) gathers every
    rank's `inp` into `out` in rank order and must be ordered on the engine's stream
    (torch.distributed.all_gather_into_tensor on an NCCL group, called with the engine's
    stream as torch's current stream, for instance). Returns ids [steps][batch]."""
    rank, world, bufs = batch._shard
    B = batch.batch
    parts = []
    done = 0
    while done < steps:
        n = min(steps - done, 256)
        for _ in range(n):
            batch.step_layers()
            for key in ("gather_hi", "gather_lo"):
                all_gather(bufs[key], bufs[key][rank * B:(rank + 1) * B])
            batch.step_lm_slice()
            all_gather(bufs["pairs_all"], bufs["pairs_local"])
            batch.step_merge()
        parts.append(batch.shard_sync(n))
        done += n
    return np.concatenate(parts) if parts else np.zeros((0, B), np.int32)


def generate_batch(engine: Engine, ids, max_new: int) -> np.ndarray:
    """qd_generate_batch: prompts [batch][n] -> generated ids [batch][max_new]."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.zeros((ids.shape[0], max(max_new, 1)), np.int32)
    check(_lib.load().qd_generate_batch(engine._h, int(ids.shape[0]), ids.ctypes.data, int(ids.shape[1]),
                                        int(max_new), out.ctypes.data))
    return out[:, :max_new]


# ---- the reference's JavaScript API --------------------------------------------

class CudaDevice:
    """What createWebGpuContext().device stands for: a GPU plus the runtime files.

    Engines are created on first use and kept (the reference builds a runtime on
    every call and never frees it, docs/04-results.md:43-54)."""

    def __init__(self, runtime_dir: str, ordinal: int = 0, kv_dtype: str = "f16"):
        self.runtime_dir = runtime_dir
        self.ordinal = ordinal
        self.kv_dtype = kv_dtype
        self._engines: dict = {}

    def engine(self, needed_positions: int, variant: str) -> Engine:
        cap = max(256, needed_positions)
        for (c, v), eng in self._engines.items():
            if c >= needed_positions and v == variant:
                return eng
        eng = Engine(self.runtime_dir, self.ordinal, max_seq=cap, kv_dtype=self.kv_dtype, variant=variant)
        self._engines[(cap, variant)] = eng
        return eng

    def close(self) -> None:
        for eng in self._engines.values():
            eng.close()
        self._engines.clear()


def createWebGpuContext(runtime_dir: Optional[str] = None, device: int = 0, kv_dtype: str = "f16"):
    """createWebGpuContext (webgpu-runtime.js:43-60): {adapter, device}.

    runtime_dir defaults to $QDECODE_RUNTIME (the reference fetches /qwen/runtime)."""
    runtime_dir = runtime_dir or os.environ.get("QDECODE_RUNTIME")
    if not runtime_dir or not os.path.exists(os.path.join(runtime_dir, "manifest.json")):
        raise RuntimeError("No qwen runtime directory was found (set QDECODE_RUNTIME).")
    try:
        import torch  # noqa: F401  (only for the adapter description)
        name = torch.cuda.get_device_name(device) if torch.cuda.is_available() else "cuda"
    except Exception:  # pragma: no cover
        name = "cuda"
    return {"adapter": {"info": {"vendor": "nvidia", "architecture": "sm_100a", "device": name}},
            "device": CudaDevice(runtime_dir, device, kv_dtype)}


create_web_gpu_context = createWebGpuContext


def runCustomQwenGreedyPrompt(*, device: CudaDevice, profile: dict, inputIds: Sequence[int],
                              maxNewTokens: int, onToken=None, decodeToken=None, onProgress=None,
                              variant: str = "optimized", maxSeqLen: int = 256) -> dict:
    """runCustomQwenGreedyPrompt (webgpu-runtime.js:165-214) on the B200 engine.

    Raises like the reference when prompt + generation exceeds the capacity
    (256 positions by default, the reference's cap; pass maxSeqLen for more)."""
    if len(inputIds) + maxNewTokens > maxSeqLen:
        raise ValueError(f"Custom CUDA path currently supports prompt + generation length up to "
                         f"{maxSeqLen} tokens.")
    eng = device.engine(len(inputIds) + maxNewTokens, variant)
    p = eng.profile
    for key, ours in (("hiddenSize", "hidden"), ("intermediateSize", "intermediate"),
                      ("attentionHeads", "heads"), ("kvHeads", "kv_heads"), ("headDim", "head_dim")):
        if key in profile and int(profile[key]) != p[ours]:
            raise ValueError(f"profile.{key}={profile[key]} does not match the runtime ({p[ours]})")
    if onProgress:
        onProgress(f"Custom prefill {len(inputIds)}/{len(inputIds)}")
    count = [0]

    def _tok(t):
        count[0] += 1
        if onProgress:
            onProgress(f"Custom decode {count[0]}/{maxNewTokens}")
        if onToken:
            onToken(decodeToken([t]) if decodeToken else str(t))

    generated, st = eng.generate_greedy(list(inputIds), maxNewTokens, _tok)
    return {
        "generated": generated,
        "generatedTokens": len(generated),
        "generateMs": st["generate_ms"],
        "firstTokenMs": st["first_token_ms"] if generated else None,
        "outputText": decodeToken(generated) if decodeToken else " ".join(str(t) for t in generated),
    }


run_custom_qwen_greedy_prompt = runCustomQwenGreedyPrompt

# result field -> qd_kernel_bench member (runKernelBenchmarks, webgpu-runtime.js:62-96)
_KERNEL_BENCH_FIELDS = {
    "baselineMatvecMs": "baseline_matvec_ms", "optimizedMatvecMs": "optimized_matvec_ms",
    "matvecSpeedup": "matvec_speedup", "baselineBytes": "baseline_bytes", "optimizedBytes": "optimized_bytes",
    "memoryReduction": "memory_reduction", "maxAbsError": "max_abs_error", "meanAbsError": "mean_abs_error",
    "blockDefaultMs": "block_default_ms", "blockOptimizedMs": "block_optimized_ms",
    "blockSpeedup": "block_speedup", "blockMaxAbsError": "block_max_abs_error",
    "blockMeanAbsError": "block_mean_abs_error", "realQ4Ms": "real_q4_ms",
    "realQ4MaxAbsError": "real_q4_max_abs_error", "realQ4MeanAbsError": "real_q4_mean_abs_error",
    "gqaMs": "gqa_ms", "gqaMaxAbsError": "gqa_max_abs_error", "gqaMeanAbsError": "gqa_mean_abs_error",
    "gqaSeqLen": "gqa_seq_len", "layer0DecodeMs": "layer0_decode_ms", "layer0Finite": "layer0_finite",
    "layer0MeanAbs": "layer0_mean_abs", "rmsMs": "rms_ms", "estimatedGbps": "estimated_gbps",
}


def _check_profile(eng: Engine, profile: dict) -> None:
    p = eng.profile
    for key, ours in (("hiddenSize", "hidden"), ("intermediateSize", "intermediate"),
                      ("attentionHeads", "heads"), ("kvHeads", "kv_heads"), ("headDim", "head_dim")):
        if key in profile and int(profile[key]) != p[ours]:
            raise ValueError(f"profile.{key}={profile[key]} does not match the runtime ({p[ours]})")


def runKernelBenchmarks(device: CudaDevice, profile: dict) -> dict:
    """runKernelBenchmarks (webgpu-runtime.js:62-96) on the B200 engine: the same
    result fields (qd_run_kernel_benchmarks)."""
    eng = device.engine(1, "optimized")
    _check_profile(eng, profile)
    out = _lib.QdKernelBench()
    check(_lib.load().qd_run_kernel_benchmarks(eng._h, C.byref(out)), eng._h)
    return {js: getattr(out, c) for js, c in _KERNEL_BENCH_FIELDS.items()}


def runFullDecoderStackBenchmark(device: CudaDevice, profile: dict) -> dict:
    """runFullDecoderStackBenchmark (webgpu-runtime.js:98-163): {ms, warmupMs, layers,
    finite, meanAbs} (qd_run_full_decoder_stack_benchmark)."""
    eng = device.engine(1, "optimized")
    _check_profile(eng, profile)
    out = _lib.QdStackBench()
    check(_lib.load().qd_run_full_decoder_stack_benchmark(eng._h, C.byref(out)), eng._h)
    return {"ms": out.ms, "warmupMs": out.warmup_ms, "layers": out.layers, "finite": out.finite,
            "meanAbs": out.mean_abs}


run_kernel_benchmarks = runKernelBenchmarks
run_full_decoder_stack_benchmark = runFullDecoderStackBenchmark


# ---- kernel level (torch CUDA tensors as device memory) -------------------------

def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def q4_matvec(x, weights, scales_f16, y=None, in_size: Optional[int] = None, stream=None):
    """y = dequant(weights) . x on the GPU (qd_q4_matvec). weights: uint32/int32 [N][K/8]."""
    import torch
    n = weights.shape[0]
    bpr = scales_f16.numel() // n
    in_size = in_size or bpr * 32
    if y is None:
        y = torch.empty(n, dtype=torch.float32, device=x.device)
    check(_lib.load().qd_q4_matvec(x.data_ptr(), weights.data_ptr(), scales_f16.data_ptr(), y.data_ptr(),
                                   in_size, n, bpr, 32, _stream(stream)))
    return y


def q4_gemm(x, weights, scales_f16, y=None, stream=None):
    """Y[m] = dequant(weights) . x[m] for every row of x [M][K] on tcgen05 (qd_q4_gemm)."""
    import torch
    M, K = x.shape
    n = weights.shape[0]
    if y is None:
        y = torch.empty(M, n, dtype=torch.float32, device=x.device)
    ws = torch.empty(_lib.load().qd_q4_gemm_workspace_bytes(M, K), dtype=torch.uint8, device=x.device)
    check(_lib.load().qd_q4_gemm(x.data_ptr(), weights.data_ptr(), scales_f16.data_ptr(), y.data_ptr(), M, K, n,
                                 32, ws.data_ptr(), _stream(stream)))
    return y


class LmHeadWorkspace:
    def __init__(self, vocab: int, device):
        import torch
        n = _lib.load().qd_lm_head_argmax_workspace_bytes(vocab)
        self.buf = torch.zeros(n, dtype=torch.uint8, device=device)


def lm_head_argmax(hidden, embed_f16, norm_weight=None, eps: float = 1e-6, logits=None,
                   workspace: Optional[LmHeadWorkspace] = None, result=None, stream=None):
    """logits = embed . rms_norm(hidden) and the (index, value) argmax (qd_lm_head_argmax)."""
    import torch
    vocab, hs = embed_f16.shape
    ws = workspace or LmHeadWorkspace(vocab, hidden.device)
    if result is None:
        result = torch.zeros(2, dtype=torch.int32, device=hidden.device)
    lp = logits.data_ptr() if logits is not None else None
    nw = norm_weight.data_ptr() if norm_weight is not None else None
    check(_lib.load().qd_lm_head_argmax(hidden.data_ptr(), nw, eps, embed_f16.data_ptr(), lp,
                                        result.data_ptr(), hs, vocab, ws.buf.data_ptr(), _stream(stream)))
    return result


def sample_logits(logits, temperature: float, top_k: int, top_p: float, seed: int, step: int, stream=None) -> int:
    """One draw from device logits (qd_sample_logits); returns the id."""
    import torch
    vocab = logits.numel()
    ws = torch.empty(_lib.load().qd_sample_workspace_bytes(vocab), dtype=torch.uint8, device=logits.device)
    tok = torch.zeros(1, dtype=torch.int32, device=logits.device)
    sp = _lib.QdSampling(float(temperature), int(top_k), float(top_p), int(seed) & 0xFFFFFFFFFFFFFFFF)
    check(_lib.load().qd_sample_logits(logits.data_ptr(), vocab, C.byref(sp), int(step), ws.data_ptr(),
                                       tok.data_ptr(), _stream(stream)))
    return int(tok.item())


def gqa_decode(q, k_cache, v_cache, seq_len: int, q_heads: int, kv_heads: int, y=None, stream=None):
    """Decode attention over [0, seq_len) (qd_gqa_decode); caches f16 or f32 [seq][kv][128]."""
    import torch
    kv_dtype = QD_KV_F16 if k_cache.dtype == torch.float16 else QD_KV_F32
    if y is None:
        y = torch.empty(q_heads * 128, dtype=torch.float32, device=q.device)
    n = _lib.load().qd_gqa_decode_workspace_bytes(seq_len, q_heads)
    ws = torch.empty(n, dtype=torch.uint8, device=q.device)
    check(_lib.load().qd_gqa_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), kv_dtype,
                                    y.data_ptr(), seq_len, q_heads, kv_heads, 128, ws.data_ptr(),
                                    _stream(stream)))
    return y


__all__ = ["Engine", "QdError", "createWebGpuContext", "runCustomQwenGreedyPrompt", "runKernelBenchmarks",
           "runFullDecoderStackBenchmark", "qwen_profile",
           "qwenProfile", "q4_matvec", "lm_head_argmax", "gqa_decode", "LmHeadWorkspace"]
