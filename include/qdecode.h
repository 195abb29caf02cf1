/*
 * qdecode: B200 (sm_100a) decode engine for the Qwen3-0.6B q4 stack of
 * kernel_optimization_webgpu, behind a plain C ABI.
 *
 * Conventions: every call returns 0 (QD_OK) or a negative QD_E_* code and never
 * throws. qd_last_error() gives the message. An engine is driven by one host
 * thread at a time; different engines (one per GPU) may run concurrently.
 * Kernel-level entry points take DEVICE pointers and a cudaStream_t (as void*,
 * NULL = the legacy default stream) and return after enqueueing.
 *
 * Reference interfaces replaced (paths within the reference project):
 *   qd_engine_create    createWebGpuContext + createAutoregressiveQwenRuntime
 *                       (src/bench/webgpu-runtime.js:43-60, :223-314), reading the
 *                       runtime directory written by scripts/extract-qwen-runtime-assets.mjs
 *   qd_generate_greedy  runCustomQwenGreedyPrompt (src/bench/webgpu-runtime.js:165-214)
 *   qd_q4_matvec        matmul_nbits_q4.wgsl (src/kernels/matmul_nbits_q4.wgsl:43-92),
 *                       bound by createQ4RuntimeProjection (webgpu-runtime.js:1191-1207)
 *   qd_lm_head_argmax   lm_head_f16.wgsl + argmax_stage1/2.wgsl, dispatched by
 *                       greedyNextTokenResident (webgpu-runtime.js:580-604)
 *   qd_gqa_decode       gqa_decode.wgsl (src/kernels/gqa_decode.wgsl:17-90) without its
 *                       256-position cap
 *   qd_batch_*          the same per-token flow (webgpu-runtime.js:471-604) for B
 *                       independent sequences at once; the reference runs one sequence
 *   qd_generate_batch   runCustomQwenGreedyPrompt over B prompts of equal length
 */
#ifndef QDECODE_H
#define QDECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QD_OK 0
#define QD_E_INVALID (-1)     /* bad argument or shape the kernels do not support */
#define QD_E_IO (-2)          /* runtime directory: missing, short or malformed file */
#define QD_E_CUDA (-3)        /* CUDA runtime error (message has the CUDA error string) */
#define QD_E_NOMEM (-4)       /* device or pinned allocation failed */
#define QD_E_RANGE (-5)       /* prompt + generation beyond max_seq, token id beyond vocab */
#define QD_E_DEVICE (-6)      /* a kernel flagged a bad token or position (status word) */
#define QD_E_TIMEOUT (-7)     /* a device-side wait expired; the launch was abandoned */

#define QD_KV_F16 0           /* f16 KV cache (default) */
#define QD_KV_F32 1           /* f32 KV cache, as the reference (cache_write.wgsl) */

typedef struct qd_engine qd_engine;

typedef struct qd_options {
  int device;            /* CUDA device ordinal */
  int max_seq;           /* KV capacity in positions (the reference sizes it prompt + new) */
  int kv_dtype;          /* QD_KV_F16 or QD_KV_F32 */
  int rope_row_stride;   /* cos/sin offset = position * stride + pair; 0 = head_dim (reference) */
  const char* variant;   /* "optimized" | "mixed" | "original": accepted, one B200 path */
  int use_graph;         /* 1 (default): each token is one CUDA graph launch */
  int persistent;        /* nonzero (default 1): one persistent kernel per token, one CTA per
                            SM, where the shape allows; 0: one kernel per fused stage */
  int timeline;          /* 1: record per-CTA stage timestamps of each persistent launch */
  int prompt_pass;       /* 1 (default): with an f16 KV cache, a prompt's first 5..256 tokens
                            take one batched pass through the layers (tensor-core GEMMs over
                            all of them, causal attention among them) before decoding; a
                            greedy generation of two or more ids whose whole prompt is
                            5..256 tokens also takes its first id from that pass (LM head on
                            the last prompt row); 0: every prompt token goes through the
                            decode kernel, one at a time, as runCustomQwenGreedyPrompt
                            feeds them */
} qd_options;

typedef struct qd_profile {
  int layers, hidden, intermediate, heads, kv_heads, head_dim, vocab, rope_rows;
  float eps;
} qd_profile;

typedef struct qd_stats {
  double generate_ms;          /* prefill + every decode step (generateMs) */
  double first_token_ms;       /* firstTokenMs */
  double steady_ms_per_token;  /* (generate_ms - first_token_ms) / (generated - 1) */
  int generated_tokens;
  int prompt_tokens;
} qd_stats;

/* Called on the calling thread once per generated token, in order
 * (onToken in runCustomQwenGreedyPrompt). Return non-zero to stop early. */
typedef int (*qd_token_cb)(int32_t token, void* user);

void qd_options_default(qd_options* opt);
int qd_engine_create(const char* runtime_dir, const qd_options* opt, qd_engine** out);
void qd_engine_destroy(qd_engine* e);
/* Message of the last failed call on this engine; with e == NULL, of the last
 * failed qd_engine_create or kernel-level call on this thread. */
const char* qd_last_error(const qd_engine* e);
int qd_engine_profile(const qd_engine* e, qd_profile* out);

/* Greedy generation: prompt ids at positions 0..n_prompt-1, then max_new_tokens
 * tokens, each fed back at the next position. out_ids (host) receives the
 * generated ids. Requires n_prompt >= 1 and n_prompt + max_new_tokens - 1 <= max_seq. */
int qd_generate_greedy(qd_engine* e, const int32_t* input_ids, int n_prompt, int max_new_tokens,
                       int32_t* out_ids, qd_token_cb on_token, void* user, qd_stats* stats);

/* Sampling beyond greedy (no counterpart in the reference, which decodes greedily only,
 * README.md:172-173): the token of each step is drawn from the LM head's logits.
 *  - candidates: the top_k largest logits (1..64; 0 or more than 64: the 64 largest),
 *    ordered by value with ties to the lower index, NaN below every number;
 *  - p_i = exp((v_i - v_max) / temperature) over the candidates;
 *  - top_p in (0, 1]: the shortest prefix of candidates whose sum reaches top_p of the
 *    candidates' sum is kept (with top_k = 0 this is top-p over the 64 most likely
 *    tokens, the same as full-vocabulary top-p whenever that nucleus has <= 64 tokens);
 *  - u = (splitmix64(seed ^ (step * 0xD1B54A32D192ED03)) >> 40) * 2^-24, step = the index
 *    of the generated token; the first kept candidate whose running sum exceeds
 *    u * (kept sum) is the token.
 * temperature <= 0 or top_k == 1 is greedy decoding (qd_generate_greedy's ids).
 * QD_E_INVALID for top_p outside (0, 1], top_k < 0 or a non-finite temperature. */
typedef struct qd_sampling {
  float temperature;
  int top_k;
  float top_p;
  uint64_t seed;
} qd_sampling;
/* runCustomQwenGreedyPrompt's flow (prompt, then max_new_tokens generated) with the
 * tokens drawn as above; arguments and stats as qd_generate_greedy. */
int qd_generate_sample(qd_engine* e, const int32_t* input_ids, int n_prompt, int max_new_tokens,
                       const qd_sampling* sampling, int32_t* out_ids, qd_token_cb on_token, void* user,
                       qd_stats* stats);
/* Kernel level: one draw from logits[vocab] (device) at RNG step `step`; the id goes to
 * token[0] (device). workspace: qd_sample_workspace_bytes(vocab) bytes of device memory. */
size_t qd_sample_workspace_bytes(uint32_t vocab);
int qd_sample_logits(const float* logits, uint32_t vocab, const qd_sampling* sampling, uint32_t step,
                     void* workspace, int32_t* token, void* stream);

/* Parity and inspection helpers. */
int qd_engine_logits(qd_engine* e, float* host_logits);       /* logits of the last generated step */
int qd_engine_hidden(qd_engine* e, float* host_hidden);       /* residual stream after the last layer */
/* Token kernel in use: 1 = the persistent kernel, 0 = one kernel per stage. */
int qd_engine_uses_persistent(const qd_engine* e);
/* Stage timestamps (ns, globaltimer) of the last persistent launch: host_out[cta][event]
 * (needs qd_options.timeline = 1). Pass host_out NULL to query the sizes. Per CTA: start;
 * per layer 19 events (0 layer input ready, 1 QKV weights ready, 2 QKV stored, 3 attention
 * + O stage done, 4 h_attn ready, 5 attention softmax done, 6 gate/up stage start, 7
 * gate/up done, 8 down weights ready, 9 down partial issued, 10 QKV input weighted, 11
 * attention scores done, 12 gate/up input weighted, 13 down partial start, 14 q/k/v
 * arrived, 15 head norm + RoPE done, 16 weighted sum done, 17 O weights ready, 18 O slice
 * dots done; events 5, 11 and 14-18 only in the attention CTAs); LM-head input ready, LM
 * head done, merged. */
int qd_engine_timeline(qd_engine* e, uint64_t* host_out, int* ctas, int* events_per_cta);
/* One token through the layers at `position` (no LM head), with the residual
 * stream after every layer copied to host_trace[layers][hidden]. */
int qd_engine_forward_trace(qd_engine* e, int32_t token, int position, float* host_trace);

/* Stepping interface (enqueue only; used to time steady-state decode on a
 * caller's stream). qd_decode_begin copies the prompt, resets the position and
 * enqueues the prefill of ids[0 .. n_prompt-2]; each qd_decode_step enqueues one
 * token (layers at the current position + LM head + argmax, token fed back);
 * qd_decode_seek enqueues a position change (KV rows below it are kept);
 * qd_decode_sync waits, checks the device status word and copies up to n
 * generated ids. These replace the per-token loop of runCustomQwenGreedyPrompt
 * (webgpu-runtime.js:195-205) for callers that drive the loop themselves. */
int qd_engine_set_stream(qd_engine* e, void* stream);   /* NULL: the engine's own stream */
int qd_decode_begin(qd_engine* e, const int32_t* input_ids, int n_prompt, int max_new_tokens);
int qd_decode_step(qd_engine* e);
int qd_decode_seek(qd_engine* e, int position);
int qd_decode_sync(qd_engine* e, int32_t* out_ids, int n);
/* Kernels one qd_decode_step launches (for launch accounting). */
int qd_decode_step_kernels(const qd_engine* e);

/* ---- batched decode and prefill -------------------------------------------- */

/* B independent sequences on the engine's device and stream. Every step advances
 * all of them by one token; projections and the LM head run as tcgen05 GEMMs over
 * the B rows. The batch owns a KV cache [layer][seq][kv_head][max_seq][128] f16
 * (layers * B * kv_heads * max_seq * 512 bytes) and its step buffers. A batch
 * borrows the engine's weights: destroy it before the engine. */
typedef struct qd_batch qd_batch;

int qd_batch_create(qd_engine* e, int batch, int max_seq, qd_batch** out);
void qd_batch_destroy(qd_batch* b);
int qd_batch_size(const qd_batch* b, int* batch, int* max_seq);
/* Seeded synthetic context: for every sequence, layer and position p < ctx, the K
 * and V rows of a synthetic hidden state pushed through the layer's input RMSNorm,
 * k/v projections, k head-RMSNorm and RoPE at position p (tcgen05 GEMMs). Hidden
 * value d of row r = seq * ctx + p in layer l is the Irwin-Hall sum of four hashed
 * 24-bit uniforms (see kb_ctx_hidden), reproducible on any host. Every sequence's
 * position becomes ctx; input tokens are left as they are. */
int qd_batch_fill_context(qd_batch* b, int ctx, uint32_t seed);
/* Next input token and position of every sequence (host arrays of `batch` entries). */
int qd_batch_set_tokens(qd_batch* b, const int32_t* tokens, const int32_t* positions);
int qd_batch_positions(qd_batch* b, int32_t* positions);
/* `steps` greedy steps for every sequence (one CUDA graph launch per step): each
 * sequence's token is run at its position, the argmax (ties: lowest index) is fed
 * back and the position advanced. out_ids [steps][batch] (host) may be NULL.
 * Requires position + steps <= max_seq for every sequence. */
int qd_batch_decode(qd_batch* b, int steps, int32_t* out_ids);
/* Prefill: prompt ids [batch][n_prompt] at positions 0..n_prompt-1 of every
 * sequence (cache rows rewritten), run as GEMMs over batch * n_prompt rows with
 * causal attention inside each prompt; first_ids [batch] (host, may be NULL)
 * receives each sequence's first generated token, which becomes its next input
 * at position n_prompt. */
int qd_batch_prefill(qd_batch* b, const int32_t* ids, int n_prompt, int32_t* first_ids);
/* Keep the f32 logits [batch][vocab] of each step for qd_batch_logits (off by
 * default: the LM head then writes only 8 bytes per sequence and CTA). */
int qd_batch_keep_logits(qd_batch* b, int keep);
int qd_batch_logits(qd_batch* b, float* host_logits);
/* Cached K and V rows of one sequence and layer, positions [pos0, pos0 + count),
 * as f32 [count][kv_heads * 128] on the host (the cache holds f16). */
int qd_batch_read_kv(qd_batch* b, int layer, int seq, int pos0, int count, float* k, float* v);
int qd_batch_write_kv(qd_batch* b, int layer, int seq, int pos0, int count, const float* k, const float* v);
/* Kernels one qd_batch_decode step launches (for launch accounting). */
int qd_batch_step_kernels(const qd_batch* b);

/* Vocabulary-sharded LM head of a batched step across `world` ranks (config 3 with the LM head
 * split by vocabulary over GPUs; one batch per rank, every rank the same batch size). Per step:
 * each rank runs its layers (qd_batch_step_layers), the ranks all-gather their final-norm rows,
 * each rank scores its vocabulary slice [V*rank/world, V*(rank+1)/world) for every rank's rows
 * and reduces each row to one (index, value) pair (qd_batch_step_lm_slice), the ranks all-gather
 * the pairs, and each rank keeps the best candidate of its own rows, ties to the lowest index
 * (qd_batch_step_merge). The collectives are the caller's (NCCL all-gather on the engine's
 * stream, for instance); the buffers are the caller's device memory:
 *   gather_hi, gather_lo  f16 [world * batch][hidden], 16-byte aligned; this rank's rows start at
 *                         rank * batch (qd_batch_step_layers writes them): the all-gather's buffers
 *   pairs_local           u32 [world * batch][2] = {index, f32 bits of the max} of this rank's slice
 *   pairs_all             u32 [world][world * batch][2]: the all-gather of every rank's pairs_local
 * The three step calls only enqueue on the engine's stream; qd_batch_shard_sync waits and returns
 * the ids [steps][batch] of the steps merged since the previous sync (at most 256).
 * Replaces, for the batch, the replicated LM head + argmax of greedyNextTokenResident
 * (webgpu-runtime.js:580-604). */
int qd_batch_set_vocab_shard(qd_batch* b, int rank, int world, void* gather_hi, void* gather_lo,
                             void* pairs_local, void* pairs_all);
int qd_batch_step_layers(qd_batch* b);
int qd_batch_step_lm_slice(qd_batch* b);
int qd_batch_step_merge(qd_batch* b);
int qd_batch_shard_sync(qd_batch* b, int steps, int32_t* out_ids);

/* ---- the reference's benchmark exports -------------------------------------------
 * runKernelBenchmarks(device, profile) (webgpu-runtime.js:62-96): each field is the
 * reference's result field of the same name (camelCase there). Timings are CUDA-event
 * milliseconds per launch over back-to-back launches on the engine's stream (the
 * reference: wall clock per submit). Error fields compare the GPU result with a
 * double-precision CPU evaluation of the same math (the reference's cpu* checks,
 * errorStats :1540-1552). Inputs are the reference's own fixtures:
 *  - q8 matvec hidden -> intermediate (runQ8Comparison :1438, createQ8Inputs :1464):
 *    baseline = one thread per row, optimized = one warp per row with 128-bit loads;
 *  - q8 MLP block rms -> gate/up -> silu*up -> down (runQwenMlpBlockComparison :1058);
 *  - layer 0's resident q4 gate projection on sin(0.017 i) (runRealQwenQ4Projection :984);
 *  - decode attention over 128 positions of createVector data (runGqaDecodeComparison :902);
 *  - one decode layer (layer 0, position 0, input sin(0.013 i)) (runRealQwenLayer0Decode :614);
 *  - RMSNorm of cos(0.013 i) (runRmsNorm :1636).
 * The layer runs overwrite the engine's hidden state and KV row 0; the next
 * generation starts from its own prompt as always. */
typedef struct qd_kernel_bench {
  double baseline_matvec_ms, optimized_matvec_ms, matvec_speedup;
  double baseline_bytes, optimized_bytes, memory_reduction;
  double max_abs_error, mean_abs_error;
  double block_default_ms, block_optimized_ms, block_speedup, block_max_abs_error, block_mean_abs_error;
  double real_q4_ms, real_q4_max_abs_error, real_q4_mean_abs_error;
  double gqa_ms, gqa_max_abs_error, gqa_mean_abs_error;
  int gqa_seq_len;
  int layer0_finite;
  double layer0_decode_ms, layer0_mean_abs;
  double rms_ms, estimated_gbps;
} qd_kernel_bench;
int qd_run_kernel_benchmarks(qd_engine* e, qd_kernel_bench* out);

/* runFullDecoderStackBenchmark(device, profile) (webgpu-runtime.js:98-163): every
 * layer plus the final RMSNorm for one token whose hidden input is sin(0.013 i),
 * at position 0 (attention over its own K/V only, as the reference's stack bench
 * without a cache). warmup_ms is the first run, ms the second (CUDA events);
 * finite / mean_abs describe the final-norm output. */
typedef struct qd_stack_bench {
  double ms, warmup_ms;
  int layers, finite;
  double mean_abs;
} qd_stack_bench;
int qd_run_full_decoder_stack_benchmark(qd_engine* e, qd_stack_bench* out);

/* ---- failure-path test hooks ------------------------------------------------------
 * The reference's only failure detection is the A/B page's uncapturederror guard
 * (src/bench/ab-page.js:158-161,181-187), which refuses results after a device error.
 * Here every device-side wait is bounded and a wait that runs out makes the call
 * return QD_E_TIMEOUT with the engine still usable. These two calls let a test make
 * one such wait run out on purpose, without any fault:
 *  - qd_engine_inject_stall: the next persistent decode launch withholds layer 0's
 *    q/k/v results, so its attention CTAs wait until their 200 ms deadline, raise the
 *    abort flag and every CTA returns; the generation that contains it returns
 *    QD_E_TIMEOUT and the next one runs normally. QD_E_INVALID unless the engine
 *    runs the persistent kernel (qd_engine_uses_persistent == 1).
 *  - qd_batch_inject_stall: CTA (0, 0, 0) of the next tensor-core GEMM the batch
 *    launches withholds its first activation tiles, so its MMA issuer waits until
 *    its 1 s deadline; the decode or prefill call that contains it returns
 *    QD_E_TIMEOUT. Both only enqueue (on the engine's stream). */
int qd_engine_inject_stall(qd_engine* e);
int qd_batch_inject_stall(qd_batch* b);

/* runCustomQwenGreedyPrompt over `batch` prompts of n_prompt ids each: prefill,
 * then max_new_tokens greedy tokens per prompt. ids [batch][n_prompt], out_ids
 * [batch][max_new_tokens] (host). Uses a temporary batch of max_seq
 * n_prompt + max_new_tokens. */
int qd_generate_batch(qd_engine* e, int batch, const int32_t* ids, int n_prompt, int max_new_tokens,
                      int32_t* out_ids);

/* ---- kernel level (device pointers) ---------------------------------------- */

/* y[out_size] = dequant(weights) . x. weights: u32 words [out_size][blocks_per_row*block_size/8]
 * (ONNX MatMulNBits bits=4), scales_f16: [out_size][blocks_per_row], implicit zero point 8.
 * Only block_size 32 is supported; in_size <= blocks_per_row * 32. */
int qd_q4_matvec(const float* x, const uint32_t* weights, const uint16_t* scales_f16, float* y,
                 uint32_t in_size, uint32_t out_size, uint32_t blocks_per_row,
                 uint32_t block_size, void* stream);

/* Batched q4 MatMulNBits on the tcgen05 tensor cores: y[m][out_size] = dequant(weights) . x[m]
 * for m < M (x: [M][in_size] f32, same weight layout as qd_q4_matvec). The MMA inputs are
 * f16 hi/lo splits of the exact f32 weights and of x (three MMAs per step), so results agree
 * with f32 arithmetic to ~1e-6 relative. in_size must be a multiple of 64 (<= 4096). The
 * workspace holds the split x (qd_q4_gemm_workspace_bytes). Replaces M dispatches of
 * matmul_nbits_q4.wgsl (matmul_nbits_q4.wgsl:43-92). */
size_t qd_q4_gemm_workspace_bytes(uint32_t M, uint32_t in_size);
int qd_q4_gemm(const float* x, const uint32_t* weights, const uint16_t* scales_f16, float* y, uint32_t M,
               uint32_t in_size, uint32_t out_size, uint32_t block_size, void* workspace, void* stream);

/* Workspace (device, zeroed once by the caller; left zeroed by each call). */
size_t qd_lm_head_argmax_workspace_bytes(uint32_t vocab);
/* logits[vocab] = embed_f16 . h where h = rms_norm(hidden) * norm_weight when norm_weight
 * is non-NULL (eps), else hidden. result[2] = {argmax index (ties: lowest), f32 bits of the
 * max}. logits may be NULL. hidden_size must be a multiple of 256, at most 1024. */
int qd_lm_head_argmax(const float* hidden, const float* norm_weight, float eps,
                      const uint16_t* embed_f16, float* logits, uint32_t* result,
                      uint32_t hidden_size, uint32_t vocab, void* workspace, void* stream);

/* Decode attention over positions [0, seq_len): q [q_heads][128] f32 (final, after RoPE),
 * caches [seq][kv_heads][128] of kv_dtype, y [q_heads][128]. head_dim must be 128. */
size_t qd_gqa_decode_workspace_bytes(uint32_t seq_len, uint32_t q_heads);
int qd_gqa_decode(const float* q, const void* k_cache, const void* v_cache, int kv_dtype, float* y,
                  uint32_t seq_len, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                  void* workspace, void* stream);

/* ---- decode attention without device allocation ---------------------------- */

/* Bytes of the fixed device array that qd_gqa_decode_noalloc keeps its scratch in
 * (512 KiB: split-KV partials for 16 query heads up to 16128 positions). */
#define QD_NOALLOC_SCRATCH_BYTES (512u * 1024u)

/* No counterpart in the reference: its WebGPU runtime allocates every buffer up
 * front and never frees one. This is qd_gqa_decode for callers that cannot
 * allocate device memory when they call: a host whose own pool takes all device
 * memory at start-up and forbids driver allocations afterwards, or a
 * latency-critical loop that cannot take the device-wide synchronisation a
 * cudaFree may cause. Same arguments and results as qd_gqa_decode, minus the
 * workspace: the split-KV partials live in one array of QD_NOALLOC_SCRATCH_BYTES
 * in device global memory owned by the library, which every GPU that loads the
 * library holds until the process exits. The call allocates and frees nothing.
 *  - Sizes whose partials do not fit (ceil(seq_len/256) * q_heads * 520 bytes,
 *    about) are rejected with QD_E_RANGE; use qd_gqa_decode for those.
 *  - The first call on each device looks up that array's device address (a CUDA
 *    symbol query, with the device current); make that first call before any
 *    stream capture begins. The address is kept per device together with the id
 *    of the CUDA context it belongs to; the first call in a new context (after
 *    cudaDeviceReset, say) looks it up again, so it too belongs outside a capture.
 *  - All calls on a device share the one array and it keeps the last call's
 *    contents. Nothing in it needs to start at zero: each call writes every
 *    partial it reads. Calls whose kernels overlap on the GPU (other streams,
 *    other host threads) race on it: order them on one stream or serialise them. */
int qd_gqa_decode_noalloc(const float* q, const void* k_cache, const void* v_cache, int kv_dtype,
                          float* y, uint32_t seq_len, uint32_t q_heads, uint32_t kv_heads,
                          uint32_t head_dim, void* stream);

#ifdef __cplusplus
}
#endif
#endif
