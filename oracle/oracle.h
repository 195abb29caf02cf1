/*
 * CPU oracle for the Qwen3 q4 greedy-decode path. TEST INFRASTRUCTURE ONLY:
 * only the tests, the smoke check and the CPU-baseline leg of the benchmark use
 * it, as the checker. It is never linked into the product library.
 *
 * Each function restates one WGSL shader of the reference (reference file:line
 * given beside it) in plain C, keeping the shader's lane decomposition and its
 * shared-memory tree-reduction order, so that the f32 rounding sequence is the
 * shader's own (compiled with -ffp-contract=off: no fused multiply-adds).
 *
 * Parity status: the reference is JavaScript + WGSL and needs a WebGPU device,
 * which no machine here has, and it ships no golden vectors. The oracle is
 * therefore "parity unpinned" against an executed reference; it is pinned
 * instead against a literal float64 port of the reference's own JavaScript CPU
 * check functions (cpuQ4MatMulNBits, cpuGqaDecode, cpuRmsNorm, halfToFloat in
 * src/bench/webgpu-runtime.js) on the reference's own createVector fixtures.
 */
#ifndef QDECODE_ORACLE_H
#define QDECODE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float qo_half_to_float(uint16_t h);
uint16_t qo_float_to_half(float f);

void qo_q4_matvec(const float* x, const uint32_t* weights, const float* scales, float* y,
                  uint32_t in_size, uint32_t out_size, uint32_t blocks_per_row,
                  uint32_t block_size);
void qo_q4_matvec_original(const float* x, const uint32_t* weights, const float* scales,
                           float* y, uint32_t in_size, uint32_t out_size,
                           uint32_t blocks_per_row, uint32_t block_size);
void qo_rms_norm(const float* x, const float* weight, float* y, uint32_t n, float eps);
void qo_head_rms_norm(const float* x, const float* weight, float* y, uint32_t head_dim,
                      uint32_t heads, float eps);
void qo_rope(const float* x, const float* cos_tab, const float* sin_tab, float* y,
             uint32_t heads, uint32_t head_dim, uint32_t position, uint32_t row_stride);
void qo_cache_write(const float* src, float* cache, uint32_t size, uint32_t position,
                    int round_f16);
void qo_gqa_decode(const float* q, const float* k_cache, const float* v_cache, float* y,
                   uint32_t seq_len, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim);
void qo_silu_mul(const float* gate, const float* up, float* y, uint32_t n);
void qo_residual_add(const float* a, const float* b, float* y, uint32_t n);
void qo_lm_head_f16(const float* hidden, const uint16_t* embed, float* logits,
                    uint32_t hidden_size, uint32_t rows);
void qo_argmax(const float* logits, uint32_t count, uint32_t result[2]);

/* ---- whole model ---------------------------------------------------------- */
typedef struct qo_model qo_model;
typedef struct qo_session qo_session;

enum { QO_Q = 0, QO_K, QO_V, QO_O, QO_GATE, QO_UP, QO_DOWN, QO_NPROJ };

qo_model* qo_model_new(int layers, int hidden, int inter, int heads, int kv_heads,
                       int head_dim, int vocab, int rope_rows, float eps);
void qo_model_free(qo_model* m);
void qo_model_set_shared(qo_model* m, const uint16_t* embed, const float* cos_tab,
                         const float* sin_tab, const float* final_norm);
void qo_model_set_layer(qo_model* m, int layer, const float* norm_input, const float* norm_q,
                        const float* norm_k, const float* norm_post,
                        const uint32_t* const* weights, const float* const* scales);

qo_session* qo_session_new(const qo_model* m, int max_seq, int kv_f16, int rope_row_stride);
void qo_session_free(qo_session* s);
/* Optional per-layer dump of the hidden state after each layer: [layers][hidden]. */
void qo_session_set_trace(qo_session* s, float* trace);
/* The session's K (which = 0) or V (which = 1) cache of a layer: [max_seq][kv_heads * head_dim]. */
const float* qo_session_kv(const qo_session* s, int layer, int which);
/* Overwrite cached K/V rows [pos0, pos0 + count) of a layer: [count][kv_heads * head_dim]. */
int qo_session_set_kv(qo_session* s, int layer, int pos0, int count, const float* k, const float* v);
/* One token through all layers plus the final norm (enqueueAutoregressiveToken). */
int qo_forward(qo_session* s, int32_t token, int position);
const float* qo_session_final_hidden(const qo_session* s);
/* Residual stream after the last layer of the last forward (before the final norm). */
const float* qo_session_hidden(const qo_session* s);
/* LM head + argmax on the last forward's final hidden (greedyNextTokenResident). */
int qo_next_token(qo_session* s, float* logits_out, uint32_t result[2], float* top2_margin);
/* runCustomQwenGreedyPrompt's token flow. Returns 0 or a negative error. */
int32_t qo_sample(const float* logits, uint32_t vocab, float temperature, int top_k, float top_p, uint64_t seed,
                  uint32_t step);
int qo_generate_sample(qo_session* s, const int32_t* ids, int n_prompt, int max_new, float temperature, int top_k,
                       float top_p, uint64_t seed, int32_t* out_ids);
int qo_greedy(qo_session* s, const int32_t* ids, int n_prompt, int max_new, int32_t* out_ids,
              float* top2_margins);

int qo_num_threads(void);
void qo_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
