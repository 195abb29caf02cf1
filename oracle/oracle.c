/*
 * CPU oracle for the Qwen3 q4 greedy-decode path. TEST INFRASTRUCTURE ONLY
 * (checker for the tests, the smoke check and the benchmark's CPU-baseline leg;
 * never part of the product library). See oracle.h for the parity status.
 *
 * Build: gcc -O3 -fopenmp -ffp-contract=off -fPIC -shared (recipe in oracle/Makefile).
 * Row-parallel loops use OpenMP; every row keeps the shader's own lane order,
 * so results do not depend on the thread count.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Most negative finite f32 the shaders use as -inf (argmax_stage1.wgsl:16). */
#define QO_NEG_INF (-3.4028234e38f)
/* gqa_decode.wgsl:42 pads masked lanes with this value. */
#define QO_GQA_PAD (-3.402823e38f)

int qo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Threads of the parallel loops from now on (n >= 1; a no-op without OpenMP). */
void qo_set_num_threads(int n) {
#ifdef _OPENMP
  if (n >= 1) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* halfToFloat, src/bench/webgpu-runtime.js:1732-1739 (exact f16 -> f32). */
float qo_half_to_float(uint16_t h) {
  const float sign = (h & 0x8000u) ? -1.0f : 1.0f;
  const int e = (h >> 10) & 0x1f;
  const int frac = h & 0x3ff;
  if (e == 0) return sign * ldexpf((float)frac, -24);
  if (e == 0x1f) return frac ? NAN : sign * INFINITY;
  return sign * ldexpf((float)(1024 + frac), e - 25);
}

/* f32 -> f16, round to nearest even (the engine's f16 KV-cache store). */
uint16_t qo_float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520: inf */
  if (ax < 0x38800000u) {                                   /* below 2^-14: subnormal half */
    if (ax < 0x33000000u) return (uint16_t)sign;            /* below 2^-25: zero */
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126 - e;                         /* 14 - (e - 127) + 13 */
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((ax >> 13) - (112u << 10));
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

/* ---- matmul_nbits_q4.wgsl ------------------------------------------------- */

/* dot_word, matmul_nbits_q4.wgsl:20-31. */
static float dot_word(uint32_t packed, const float* x, uint32_t base) {
  float sum = 0.0f;
  for (uint32_t i = 0; i < 8; ++i)
    sum = sum + (float)((int)((packed >> (4u * i)) & 0xfu) - 8) * x[base + i];
  return sum;
}

/* dot_word_tail, matmul_nbits_q4.wgsl:33-41. */
static float dot_word_tail(uint32_t packed, const float* x, uint32_t base, uint32_t in_size) {
  float sum = 0.0f;
  for (uint32_t i = 0; i < 8; ++i)
    if (base + i < in_size)
      sum = sum + (float)((int)((packed >> (4u * i)) & 0xfu) - 8) * x[base + i];
  return sum;
}

/* main, matmul_nbits_q4.wgsl:43-92: 64 lanes per row, one word per lane, strided. */
void qo_q4_matvec(const float* x, const uint32_t* weights, const float* scales, float* y,
                  uint32_t in_size, uint32_t out_size, uint32_t blocks_per_row,
                  uint32_t block_size) {
  const uint32_t words_per_block = block_size / 8u;
  const uint32_t words_per_row = blocks_per_row * words_per_block;
#pragma omp parallel for schedule(static)
  for (long row = 0; row < (long)out_size; ++row) {
    float partial[64];
    const uint64_t row_word_offset = (uint64_t)row * words_per_row;
    const uint64_t row_scale_offset = (uint64_t)row * blocks_per_row;
    for (uint32_t tid = 0; tid < 64; ++tid) {
      float acc = 0.0f;
      for (uint32_t w = tid; w < words_per_row; w += 64) {
        const uint32_t packed = weights[row_word_offset + w];
        const float scale = scales[row_scale_offset + w / words_per_block];
        const uint32_t col = w * 8u;
        if (col + 8u <= in_size) acc = acc + dot_word(packed, x, col) * scale;
        else acc = acc + dot_word_tail(packed, x, col, in_size) * scale;
      }
      partial[tid] = acc;
    }
    for (uint32_t stride = 32; stride >= 1; stride /= 2)
      for (uint32_t tid = 0; tid < stride; ++tid) partial[tid] = partial[tid] + partial[tid + stride];
    y[row] = partial[0];
  }
}

/* baseline/matmul_nbits_q4.wgsl:25-79 ("original" variant): 256 lanes over blocks. */
void qo_q4_matvec_original(const float* x, const uint32_t* weights, const float* scales,
                           float* y, uint32_t in_size, uint32_t out_size,
                           uint32_t blocks_per_row, uint32_t block_size) {
  const uint32_t words_per_block = block_size / 8u;
#pragma omp parallel for schedule(static)
  for (long row = 0; row < (long)out_size; ++row) {
    float partial[256];
    const uint64_t row_word_offset = (uint64_t)row * blocks_per_row * words_per_block;
    const uint64_t row_scale_offset = (uint64_t)row * blocks_per_row;
    for (uint32_t tid = 0; tid < 256; ++tid) {
      float acc = 0.0f;
      for (uint32_t block = tid; block < blocks_per_row; block += 256) {
        const float scale = scales[row_scale_offset + block];
        const uint32_t col_base = block * block_size;
        const uint64_t block_word_offset = row_word_offset + (uint64_t)block * words_per_block;
        for (uint32_t wi = 0; wi < words_per_block; ++wi) {
          const uint32_t packed = weights[block_word_offset + wi];
          for (uint32_t lane = 0; lane < 4; ++lane) {
            const uint32_t b = (packed >> (lane * 8u)) & 0xffu;
            const uint32_t pair_base = col_base + wi * 8u + lane * 2u;
            if (pair_base < in_size)
              acc = acc + (float)((int)(b & 0xfu) - 8) * scale * x[pair_base];
            if (pair_base + 1u < in_size)
              acc = acc + (float)((int)((b >> 4) & 0xfu) - 8) * scale * x[pair_base + 1u];
          }
        }
      }
      partial[tid] = acc;
    }
    for (uint32_t stride = 128; stride >= 1; stride /= 2)
      for (uint32_t tid = 0; tid < stride; ++tid) partial[tid] = partial[tid] + partial[tid + stride];
    y[row] = partial[0];
  }
}

/* ---- norms, rope, cache ---------------------------------------------------- */

static float tree256(float* p) {
  for (uint32_t stride = 128; stride >= 1; stride /= 2)
    for (uint32_t tid = 0; tid < stride; ++tid) p[tid] = p[tid] + p[tid + stride];
  return p[0];
}

/* rms_norm.wgsl:15-44 (256 lanes, strided sum of squares, tree). */
void qo_rms_norm(const float* x, const float* weight, float* y, uint32_t n, float eps) {
  float partial[256];
  for (uint32_t tid = 0; tid < 256; ++tid) {
    float sum = 0.0f;
    for (uint32_t i = tid; i < n; i += 256) sum = sum + x[i] * x[i];
    partial[tid] = sum;
  }
  const float total = tree256(partial);
  const float inv_rms = 1.0f / sqrtf(total / (float)n + eps);
  for (uint32_t i = 0; i < n; ++i) y[i] = x[i] * inv_rms * weight[i];
}

/* head_rms_norm.wgsl:15-52: one 256-lane group per head, shared [head_dim] weight. */
void qo_head_rms_norm(const float* x, const float* weight, float* y, uint32_t head_dim,
                      uint32_t heads, float eps) {
  for (uint32_t head = 0; head < heads; ++head) {
    const uint32_t base = head * head_dim;
    float partial[256];
    for (uint32_t tid = 0; tid < 256; ++tid) {
      float sum = 0.0f;
      for (uint32_t i = tid; i < head_dim; i += 256) sum = sum + x[base + i] * x[base + i];
      partial[tid] = sum;
    }
    const float total = tree256(partial);
    const float inv_rms = 1.0f / sqrtf(total / (float)head_dim + eps);
    for (uint32_t i = 0; i < head_dim; ++i) y[base + i] = x[base + i] * inv_rms * weight[i];
  }
}

/* rope.wgsl:14-31: rotate-half RoPE. The table offset is position * row_stride +
 * pair_d; the reference passes row_stride = head_dim (uniform [heads, headDim,
 * position] at webgpu-runtime.js:477-478) into a table that is head_dim/2 wide,
 * so position p reads table row 2p. */
void qo_rope(const float* x, const float* cos_tab, const float* sin_tab, float* y,
             uint32_t heads, uint32_t head_dim, uint32_t position, uint32_t row_stride) {
  const uint32_t total = heads * head_dim;
  const uint32_t half_dim = head_dim / 2u;
  for (uint32_t index = 0; index < total; ++index) {
    const uint32_t d = index % head_dim;
    const uint32_t pair_d = d % half_dim;
    const uint32_t peer = d >= half_dim ? index - half_dim : index + half_dim;
    const float sign = d >= half_dim ? 1.0f : -1.0f;
    const uint64_t off = (uint64_t)position * row_stride + pair_d;
    const float c = cos_tab[off];
    const float s = sin_tab[off];
    y[index] = x[index] * c + sign * x[peer] * s;
  }
}

/* cache_write.wgsl:12-18. round_f16 != 0 stores f16(src) (the engine's f16 cache),
 * read back as f32 by the attention. */
void qo_cache_write(const float* src, float* cache, uint32_t size, uint32_t position,
                    int round_f16) {
  float* dst = cache + (uint64_t)position * size;
  for (uint32_t i = 0; i < size; ++i)
    dst[i] = round_f16 ? qo_half_to_float(qo_float_to_half(src[i])) : src[i];
}

/* gqa_decode.wgsl:17-90, with the seq_len <= 256 cap lifted: lane t covers
 * positions t, t+256, ... (for seq_len <= 256 this is exactly the shader). */
void qo_gqa_decode(const float* q, const float* k_cache, const float* v_cache, float* y,
                   uint32_t seq_len, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim) {
  const uint32_t heads_per_kv = q_heads / kv_heads;
  const float scale = 1.0f / sqrtf((float)head_dim);
  float* scores = (float*)malloc(sizeof(float) * (seq_len ? seq_len : 1));
  for (uint32_t q_head = 0; q_head < q_heads; ++q_head) {
    const uint32_t kv_head = q_head / heads_per_kv;
    const uint32_t q_offset = q_head * head_dim;
    for (uint32_t pos = 0; pos < seq_len; ++pos) {
      float dot = 0.0f;
      const uint64_t k_offset = ((uint64_t)pos * kv_heads + kv_head) * head_dim;
      for (uint32_t d = 0; d < head_dim; ++d) dot = dot + q[q_offset + d] * k_cache[k_offset + d];
      scores[pos] = dot * scale;
    }
    float scratch[256];
    for (uint32_t tid = 0; tid < 256; ++tid) {
      float m = QO_GQA_PAD;
      for (uint32_t pos = tid; pos < seq_len; pos += 256) m = fmaxf(m, scores[pos]);
      scratch[tid] = m;
    }
    for (uint32_t stride = 128; stride >= 1; stride /= 2)
      for (uint32_t tid = 0; tid < stride; ++tid)
        scratch[tid] = fmaxf(scratch[tid], scratch[tid + stride]);
    const float max_score = scratch[0];
    for (uint32_t pos = 0; pos < seq_len; ++pos) scores[pos] = expf(scores[pos] - max_score);
    for (uint32_t tid = 0; tid < 256; ++tid) {
      float s = 0.0f;
      for (uint32_t pos = tid; pos < seq_len; pos += 256) s = s + scores[pos];
      scratch[tid] = s;
    }
    const float inv_sum = 1.0f / tree256(scratch);
    for (uint32_t d = 0; d < head_dim; ++d) {
      float acc = 0.0f;
      for (uint32_t pos = 0; pos < seq_len; ++pos) {
        const float weight = scores[pos] * inv_sum;
        const uint64_t v_offset = ((uint64_t)pos * kv_heads + kv_head) * head_dim;
        acc = acc + weight * v_cache[v_offset + d];
      }
      y[q_head * head_dim + d] = acc;
    }
  }
  free(scores);
}

/* silu_mul.wgsl:13-23. */
void qo_silu_mul(const float* gate, const float* up, float* y, uint32_t n) {
  for (uint32_t i = 0; i < n; ++i) {
    const float g = gate[i];
    const float silu = g / (1.0f + expf(-g));
    y[i] = silu * up[i];
  }
}

/* residual_add.wgsl:13-19. */
void qo_residual_add(const float* a, const float* b, float* y, uint32_t n) {
  for (uint32_t i = 0; i < n; ++i) y[i] = a[i] + b[i];
}

/* ---- LM head + argmax ------------------------------------------------------ */

/* Exact f16 -> f32 for all 65536 codes (the values qo_half_to_float gives). */
static float g_h2f[65536];
static int g_h2f_ready = 0;
static const float* h2f_table(void) {
  if (!g_h2f_ready) {
#pragma omp critical(qo_h2f)
    if (!g_h2f_ready) {
      for (uint32_t h = 0; h < 65536u; ++h) g_h2f[h] = qo_half_to_float((uint16_t)h);
      __atomic_store_n(&g_h2f_ready, 1, __ATOMIC_RELEASE);
    }
  }
  return g_h2f;
}

/* lm_head_f16.wgsl:19-58: 64 lanes per vocab row, one f16 pair (u32 word) per lane. */
void qo_lm_head_f16(const float* hidden, const uint16_t* embed, float* logits,
                    uint32_t hidden_size, uint32_t rows) {
  const uint32_t words_per_row = hidden_size / 2u;
  const float* h2f = h2f_table();
#pragma omp parallel for schedule(static)
  for (long row = 0; row < (long)rows; ++row) {
    const uint16_t* e = embed + (uint64_t)row * hidden_size;
    float partial[64];
    for (uint32_t tid = 0; tid < 64; ++tid) {
      float acc = 0.0f;
      for (uint32_t w = tid; w < words_per_row; w += 64) {
        const uint32_t col = w * 2u;
        const float px = h2f[e[col]];
        const float py = h2f[e[col + 1]];
        acc = acc + px * hidden[col] + py * hidden[col + 1];
      }
      partial[tid] = acc;
    }
    for (uint32_t stride = 32; stride >= 1; stride /= 2)
      for (uint32_t tid = 0; tid < stride; ++tid) partial[tid] = partial[tid] + partial[tid + stride];
    logits[row] = partial[0];
  }
}

static void argmax_tree(float* v, uint32_t* idx) {
  for (uint32_t stride = 128; stride >= 1; stride /= 2)
    for (uint32_t tid = 0; tid < stride; ++tid) {
      const float ov = v[tid + stride];
      const uint32_t oi = idx[tid + stride];
      if (ov > v[tid] || (ov == v[tid] && oi < idx[tid])) {
        v[tid] = ov;
        idx[tid] = oi;
      }
    }
}

/* argmax_stage1.wgsl:21-69 (256 groups x 256 lanes, strided) followed by
 * argmax_stage2.wgsl:22-58. result = {index, f32 bits of the winning value}. */
void qo_argmax(const float* logits, uint32_t count, uint32_t result[2]) {
  enum { GROUPS = 256, WG = 256 };
  float best_value[GROUPS];
  uint32_t best_index[GROUPS];
  const uint32_t stride_span = GROUPS * WG;
  for (uint32_t group = 0; group < GROUPS; ++group) {
    float sv[WG];
    uint32_t si[WG];
    for (uint32_t tid = 0; tid < WG; ++tid) {
      float value = QO_NEG_INF;
      uint32_t index = 0;
      for (uint32_t i = group * WG + tid; i < count; i += stride_span) {
        const float c = logits[i];
        if (c > value) {
          value = c;
          index = i;
        }
      }
      sv[tid] = value;
      si[tid] = index;
    }
    argmax_tree(sv, si);
    best_value[group] = sv[0];
    best_index[group] = si[0];
  }
  argmax_tree(best_value, best_index);
  result[0] = best_index[0];
  memcpy(&result[1], &best_value[0], 4);
}

/* ---- whole model ----------------------------------------------------------- */

typedef struct {
  const float *norm_input, *norm_q, *norm_k, *norm_post;
  const uint32_t* w[QO_NPROJ];
  const float* s[QO_NPROJ];
} qo_layer;

struct qo_model {
  int layers, hidden, inter, heads, kv_heads, head_dim, vocab, rope_rows;
  float eps;
  const uint16_t* embed;
  const float *cos_tab, *sin_tab, *final_norm;
  qo_layer* layer;
};

struct qo_session {
  const qo_model* m;
  int max_seq, kv_f16, rope_row_stride;
  float **k_cache, **v_cache;
  float *h, *h2, *norm, *q, *k, *v, *qn, *kn, *qr, *kr, *attn, *o, *attn_res, *post, *gate, *up,
      *act, *down, *final_out, *logits;
  float* trace;
};

qo_model* qo_model_new(int layers, int hidden, int inter, int heads, int kv_heads,
                       int head_dim, int vocab, int rope_rows, float eps) {
  qo_model* m = (qo_model*)calloc(1, sizeof(qo_model));
  m->layers = layers; m->hidden = hidden; m->inter = inter; m->heads = heads;
  m->kv_heads = kv_heads; m->head_dim = head_dim; m->vocab = vocab;
  m->rope_rows = rope_rows; m->eps = eps;
  m->layer = (qo_layer*)calloc((size_t)layers, sizeof(qo_layer));
  return m;
}

void qo_model_free(qo_model* m) {
  if (!m) return;
  free(m->layer);
  free(m);
}

void qo_model_set_shared(qo_model* m, const uint16_t* embed, const float* cos_tab,
                         const float* sin_tab, const float* final_norm) {
  m->embed = embed; m->cos_tab = cos_tab; m->sin_tab = sin_tab; m->final_norm = final_norm;
}

void qo_model_set_layer(qo_model* m, int layer, const float* norm_input, const float* norm_q,
                        const float* norm_k, const float* norm_post,
                        const uint32_t* const* weights, const float* const* scales) {
  qo_layer* l = &m->layer[layer];
  l->norm_input = norm_input; l->norm_q = norm_q; l->norm_k = norm_k; l->norm_post = norm_post;
  for (int i = 0; i < QO_NPROJ; ++i) { l->w[i] = weights[i]; l->s[i] = scales[i]; }
}

static float* fz(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

qo_session* qo_session_new(const qo_model* m, int max_seq, int kv_f16, int rope_row_stride) {
  qo_session* s = (qo_session*)calloc(1, sizeof(qo_session));
  const size_t H = (size_t)m->hidden, I = (size_t)m->inter;
  const size_t QS = (size_t)m->heads * m->head_dim, KV = (size_t)m->kv_heads * m->head_dim;
  s->m = m; s->max_seq = max_seq; s->kv_f16 = kv_f16;
  s->rope_row_stride = rope_row_stride > 0 ? rope_row_stride : m->head_dim;
  s->k_cache = (float**)calloc((size_t)m->layers, sizeof(float*));
  s->v_cache = (float**)calloc((size_t)m->layers, sizeof(float*));
  for (int l = 0; l < m->layers; ++l) {
    s->k_cache[l] = fz((size_t)max_seq * KV);
    s->v_cache[l] = fz((size_t)max_seq * KV);
  }
  s->h = fz(H); s->h2 = fz(H); s->norm = fz(H); s->q = fz(QS); s->k = fz(KV); s->v = fz(KV);
  s->qn = fz(QS); s->kn = fz(KV); s->qr = fz(QS); s->kr = fz(KV); s->attn = fz(QS);
  s->o = fz(H); s->attn_res = fz(H); s->post = fz(H); s->gate = fz(I); s->up = fz(I);
  s->act = fz(I); s->down = fz(H); s->final_out = fz(H); s->logits = fz((size_t)m->vocab);
  return s;
}

void qo_session_free(qo_session* s) {
  if (!s) return;
  for (int l = 0; l < s->m->layers; ++l) { free(s->k_cache[l]); free(s->v_cache[l]); }
  free(s->k_cache); free(s->v_cache);
  float* bufs[] = {s->h, s->h2, s->norm, s->q, s->k, s->v, s->qn, s->kn, s->qr, s->kr, s->attn,
                   s->o, s->attn_res, s->post, s->gate, s->up, s->act, s->down, s->final_out,
                   s->logits};
  for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); ++i) free(bufs[i]);
  free(s);
}

void qo_session_set_trace(qo_session* s, float* trace) { s->trace = trace; }

/* The session's K (which = 0) or V (which = 1) cache of a layer: [max_seq][kv_heads * head_dim]. */
const float* qo_session_kv(const qo_session* s, int layer, int which) {
  if (layer < 0 || layer >= s->m->layers) return 0;
  return which ? s->v_cache[layer] : s->k_cache[layer];
}

/* Cache rows set from outside (a context built elsewhere): rows are stored as
 * given, in the [pos][kv_head * head_dim] layout cache_write.wgsl:12-18 writes. */
int qo_session_set_kv(qo_session* s, int layer, int pos0, int count, const float* k, const float* v) {
  const qo_model* m = s->m;
  const size_t KV = (size_t)m->kv_heads * m->head_dim;
  if (layer < 0 || layer >= m->layers || pos0 < 0 || count < 0 || pos0 + count > s->max_seq) return -1;
  memcpy(s->k_cache[layer] + (size_t)pos0 * KV, k, (size_t)count * KV * sizeof(float));
  memcpy(s->v_cache[layer] + (size_t)pos0 * KV, v, (size_t)count * KV * sizeof(float));
  return 0;
}
const float* qo_session_final_hidden(const qo_session* s) { return s->final_out; }
const float* qo_session_hidden(const qo_session* s) { return s->h; }

static void proj(const qo_layer* l, int which, const qo_model* m, const float* x, float* y) {
  uint32_t out_size, in_size;
  const uint32_t QS = (uint32_t)(m->heads * m->head_dim), KV = (uint32_t)(m->kv_heads * m->head_dim);
  switch (which) {
    case QO_Q: out_size = QS; in_size = (uint32_t)m->hidden; break;
    case QO_K: case QO_V: out_size = KV; in_size = (uint32_t)m->hidden; break;
    case QO_O: out_size = (uint32_t)m->hidden; in_size = QS; break;
    case QO_GATE: case QO_UP: out_size = (uint32_t)m->inter; in_size = (uint32_t)m->hidden; break;
    default: out_size = (uint32_t)m->hidden; in_size = (uint32_t)m->inter; break;
  }
  qo_q4_matvec(x, l->w[which], l->s[which], y, in_size, out_size, in_size / 32u, 32u);
}

/* enqueueAutoregressiveToken + dispatchAutoregressiveToken (webgpu-runtime.js:471-496)
 * and dispatchAutoregressiveLayerPass (:498-562). Hidden buffers ping-pong as in
 * :275-277; the embedding row is gathered with halfToFloat (:606-612). */
int qo_forward(qo_session* s, int32_t token, int position) {
  const qo_model* m = s->m;
  if (token < 0 || token >= m->vocab) return -1;
  if (position < 0 || position >= s->max_seq) return -2;
  const uint64_t last = (uint64_t)position * (uint64_t)s->rope_row_stride + (uint64_t)(m->head_dim / 2);
  if (last > (uint64_t)m->rope_rows * (uint64_t)(m->head_dim / 2)) return -3;
  const uint32_t H = (uint32_t)m->hidden, I = (uint32_t)m->inter;
  const uint32_t KV = (uint32_t)(m->kv_heads * m->head_dim);
  for (uint32_t i = 0; i < H; ++i) s->h[i] = qo_half_to_float(m->embed[(uint64_t)token * H + i]);
  float* in = s->h;
  float* out = s->h2;
  for (int li = 0; li < m->layers; ++li) {
    const qo_layer* l = &m->layer[li];
    qo_rms_norm(in, l->norm_input, s->norm, H, m->eps);
    proj(l, QO_Q, m, s->norm, s->q);
    proj(l, QO_K, m, s->norm, s->k);
    proj(l, QO_V, m, s->norm, s->v);
    qo_head_rms_norm(s->q, l->norm_q, s->qn, (uint32_t)m->head_dim, (uint32_t)m->heads, m->eps);
    qo_head_rms_norm(s->k, l->norm_k, s->kn, (uint32_t)m->head_dim, (uint32_t)m->kv_heads, m->eps);
    qo_rope(s->qn, m->cos_tab, m->sin_tab, s->qr, (uint32_t)m->heads, (uint32_t)m->head_dim,
            (uint32_t)position, (uint32_t)s->rope_row_stride);
    qo_rope(s->kn, m->cos_tab, m->sin_tab, s->kr, (uint32_t)m->kv_heads, (uint32_t)m->head_dim,
            (uint32_t)position, (uint32_t)s->rope_row_stride);
    qo_cache_write(s->kr, s->k_cache[li], KV, (uint32_t)position, s->kv_f16);
    qo_cache_write(s->v, s->v_cache[li], KV, (uint32_t)position, s->kv_f16);
    qo_gqa_decode(s->qr, s->k_cache[li], s->v_cache[li], s->attn, (uint32_t)position + 1u,
                  (uint32_t)m->heads, (uint32_t)m->kv_heads, (uint32_t)m->head_dim);
    proj(l, QO_O, m, s->attn, s->o);
    qo_residual_add(in, s->o, s->attn_res, H);
    qo_rms_norm(s->attn_res, l->norm_post, s->post, H, m->eps);
    proj(l, QO_GATE, m, s->post, s->gate);
    proj(l, QO_UP, m, s->post, s->up);
    qo_silu_mul(s->gate, s->up, s->act, I);
    proj(l, QO_DOWN, m, s->act, s->down);
    qo_residual_add(s->attn_res, s->down, out, H);
    if (s->trace) memcpy(s->trace + (size_t)li * H, out, H * sizeof(float));
    float* t = in; in = out; out = t;
  }
  qo_rms_norm(in, m->final_norm, s->final_out, H, m->eps);
  if (in != s->h) memcpy(s->h, in, H * sizeof(float));
  return 0;
}

/* Two largest distinct-index logits' gap (reported, never asserted on). */
static float top2_gap(const float* logits, uint32_t n) {
  float a = -INFINITY, b = -INFINITY;
  for (uint32_t i = 0; i < n; ++i) {
    const float v = logits[i];
    if (v > a) { b = a; a = v; } else if (v > b) { b = v; }
  }
  return a - b;
}

/* greedyNextTokenResident, webgpu-runtime.js:580-604. */
int qo_next_token(qo_session* s, float* logits_out, uint32_t result[2], float* top2_margin) {
  const qo_model* m = s->m;
  qo_lm_head_f16(s->final_out, m->embed, s->logits, (uint32_t)m->hidden, (uint32_t)m->vocab);
  qo_argmax(s->logits, (uint32_t)m->vocab, result);
  if (logits_out) memcpy(logits_out, s->logits, sizeof(float) * (size_t)m->vocab);
  if (top2_margin) *top2_margin = top2_gap(s->logits, (uint32_t)m->vocab);
  return 0;
}

/* runCustomQwenGreedyPrompt, webgpu-runtime.js:165-214: the prompt at positions
 * 0..n-1, then each step feeds the previous generated token at n+step-1. */
int qo_greedy(qo_session* s, const int32_t* ids, int n_prompt, int max_new, int32_t* out_ids,
              float* top2_margins) {
  if (n_prompt <= 0 || max_new < 0) return -4;
  if (n_prompt + max_new > s->max_seq + 1) return -2;
  for (int i = 0; i < n_prompt; ++i) {
    const int rc = qo_forward(s, ids[i], i);
    if (rc) return rc;
  }
  for (int step = 0; step < max_new; ++step) {
    if (step > 0) {
      const int rc = qo_forward(s, out_ids[step - 1], n_prompt + step - 1);
      if (rc) return rc;
    }
    uint32_t r[2];
    qo_next_token(s, NULL, r, top2_margins ? &top2_margins[step] : NULL);
    out_ids[step] = (int32_t)r[0];
  }
  return 0;
}

/* ---- sampling beyond greedy (the library's definition, not the reference's: the
 * reference decodes greedily only, README.md:172-173) ------------------------------ */

static uint64_t qo_splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

/* value order of the sampler: larger first, NaN below every number, ties to the lower index */
static int qo_better(float a, uint32_t ia, float b, uint32_t ib) {
  const int na = a != a, nb = b != b;
  if (na != nb) return nb;
  if (!na && a != b) return a > b;
  return ia < ib;
}

/* One draw from logits[vocab]: top_k candidates (1..64, else 64), p_i = exp((v_i -
 * v_0) / temperature) summed in candidate order in f32, the shortest prefix reaching
 * top_p of the sum, u = (splitmix64(seed ^ step * 0xD1B54A32D192ED03) >> 40) * 2^-24,
 * the first kept candidate whose running sum exceeds u * (kept sum).
 * temperature <= 0 or top_k == 1: the argmax. */
int32_t qo_sample(const float* logits, uint32_t vocab, float temperature, int top_k, float top_p, uint64_t seed,
                  uint32_t step) {
  if (vocab == 0) return -1;
  const int greedy = !(temperature > 0.0f) || top_k == 1;
  int K = greedy ? 1 : ((top_k >= 1 && top_k <= 64) ? top_k : 64);
  if ((uint32_t)K > vocab) K = (int)vocab;
  if (greedy) temperature = 1.0f;
  float cv[64];
  uint32_t ci[64];
  int n = 0;
  for (uint32_t i = 0; i < vocab; ++i) {  /* insertion into a sorted list of the K best */
    const float v = logits[i];
    if (n == K && !qo_better(v, i, cv[n - 1], ci[n - 1])) continue;
    int j = n < K ? n++ : K - 1;
    while (j > 0 && qo_better(v, i, cv[j - 1], ci[j - 1])) {
      cv[j] = cv[j - 1];
      ci[j] = ci[j - 1];
      --j;
    }
    cv[j] = v;
    ci[j] = i;
  }
  const float v0 = cv[0];
  float cum[64] = {0.0f};
  float s = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float v = cv[i];
    const float p = (v == v && v0 == v0) ? expf((v - v0) / temperature) : (i == 0 ? 1.0f : 0.0f);
    s += p;
    cum[i] = s;
  }
  int m = n - 1;
  if (top_p < 1.0f)
    for (int i = 0; i < n; ++i)
      if (cum[i] >= top_p * s) { m = i; break; }
  const uint64_t h = qo_splitmix64(seed ^ ((uint64_t)step * 0xD1B54A32D192ED03ull));
  const float u = (float)(h >> 40) * 5.9604644775390625e-08f;
  const float target = u * cum[m];
  int pick = m;
  for (int i = 0; i <= m; ++i)
    if (cum[i] > target) { pick = i; break; }
  return (int32_t)ci[pick];
}

/* qo_greedy's flow with each generated token drawn by qo_sample (step = its index). */
int qo_generate_sample(qo_session* s, const int32_t* ids, int n_prompt, int max_new, float temperature, int top_k,
                       float top_p, uint64_t seed, int32_t* out_ids) {
  if (n_prompt <= 0 || max_new < 0) return -4;
  if (n_prompt + max_new > s->max_seq + 1) return -2;
  for (int i = 0; i < n_prompt; ++i) {
    const int rc = qo_forward(s, ids[i], i);
    if (rc) return rc;
  }
  for (int step = 0; step < max_new; ++step) {
    if (step > 0) {
      const int rc = qo_forward(s, out_ids[step - 1], n_prompt + step - 1);
      if (rc) return rc;
    }
    const qo_model* m = s->m;
    qo_lm_head_f16(s->final_out, m->embed, s->logits, (uint32_t)m->hidden, (uint32_t)m->vocab);
    out_ids[step] = qo_sample(s->logits, (uint32_t)m->vocab, temperature, top_k, top_p, seed, (uint32_t)step);
  }
  return 0;
}
