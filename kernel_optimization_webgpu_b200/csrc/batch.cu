// Batched decode and prefill: B independent sequences on one engine's weights.
// The host flow per step is the reference's decode token
// (webgpu-runtime.js:471-604: embedding row, 28 layers, final norm, LM head,
// argmax fed back) applied to B rows at once; see batch.cuh for the kernels.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/qdecode.h"
#include "batch.cuh"
#include "gemm_tc.cuh"
#include "internal.cuh"

using namespace qd;

struct qd_batch {
  qd_engine* e = nullptr;
  std::string err;
  int B = 0, max_seq = 0;
  int splits = 1, split_len = 512;  // decode attention split-KV
  int sq = 1, so = 1, sg = 1, sd = 1;  // split-K of the qkv, o, gate/up, down GEMMs
  int ktq = 0, kto = 0, ktg = 0, ktd = 0;
  int lm_tiles = 0;
  void* kv = nullptr;        // K then V caches of every layer
  size_t kv_layer = 0;       // elements of one layer's K (or V) cache
  void* dec = nullptr;       // decode step buffers
  float* h = nullptr;        // [B][H]
  __half *xh = nullptr, *xl = nullptr;  // [B][max K]
  float* parts = nullptr;    // split-K partials
  float* q = nullptr;        // [B][QS]
  float2* part_ml = nullptr;
  float* part_o = nullptr;
  float* logits = nullptr;   // [B][V] (allocated on request)
  float* lm_pv = nullptr;
  uint32_t* lm_pi = nullptr;
  uint32_t* result = nullptr;
  int *tokens = nullptr, *pos = nullptr, *out = nullptr, *step = nullptr, *errw = nullptr;
  int max_steps = 0;         // rows of `out`
  int* pinned = nullptr;     // host staging of generated ids
  size_t pinned_n = 0;
  int* pinned_io = nullptr;  // host staging: [0] status word, [16, 16 + 2B) tokens and positions
  std::vector<int> host_pos;
  bool keep_logits = false;
  cudaGraphExec_t g_step[2] = {nullptr, nullptr};  // [keep_logits]
  CUtensorMap kvmap;         // the whole KV allocation as [rows][128] f16, 64x64 boxes, 128-byte swizzle
  // wide buffers (context fill, prefill), grown on demand
  void* wide = nullptr;
  long long wide_rows = 0;
  float *w_h = nullptr, *w_y = nullptr, *w_q = nullptr;
  __half *w_xh = nullptr, *w_xl = nullptr;
  __half *w_ah = nullptr, *w_al = nullptr;  // prefill: silu(gate)*up operands of the down GEMM
  int* w_tok = nullptr;
  // vocabulary-sharded LM head (qd_batch_set_vocab_shard); gather/pair buffers are the caller's
  int shard_rank = 0, shard_world = 0, shard_v0 = 0, shard_v1 = 0, shard_tiles = 0;
  __half *gx_hi = nullptr, *gx_lo = nullptr;
  uint32_t *pairs_local = nullptr, *pairs_all = nullptr;
  void* shard_buf = nullptr;            // [world*B][tiles] (max, index) per vocabulary tile of the slice
  float* shard_pv = nullptr;
  uint32_t* shard_pi = nullptr;
  cudaGraphExec_t g_layers = nullptr;   // layers + final norm + copy into the gather buffer
  int shard_steps = 0;                  // merged steps since the last qd_batch_shard_sync
  // engine prompt pass (B = 1): split-K partials and one graph per prompt length
  float* pp = nullptr;
  long long pp_elems = 0;
  std::vector<std::pair<int, cudaGraphExec_t>> g_prompt;
};

namespace {

int bfail(qd_batch* b, const QdError& err) {
  if (b) b->err = err.msg;
  set_thread_error(err.msg);
  return err.code;
}

unsigned long long g_attn_smem_mask = 0, g_attn_smem_mask2 = 0, g_pf_smem_mask = 0, g_pf_smem_mask2 = 0;

// Dynamic shared memory of kb_prefill_attn<G>: two K/V stages + the Q tile (hi/lo) + alignment.
size_t pf_smem(int G) { return (size_t)2 * kBAttnStage + (size_t)G * 4 * kPfQBytes + 1024; }

struct Dims {
  int L, H, I, NH, NKV, QS, KVS, R, V, G;
  float eps;
};

Dims dims(const qd_engine* e) {
  const qd_profile& p = e->p;
  Dims d;
  d.L = p.layers; d.H = p.hidden; d.I = p.intermediate; d.NH = p.heads; d.NKV = p.kv_heads;
  d.QS = p.heads * kHeadDim; d.KVS = p.kv_heads * kHeadDim; d.R = d.QS + 2 * d.KVS; d.V = p.vocab;
  d.G = p.heads / p.kv_heads; d.eps = p.eps;
  return d;
}

__half* kc_of(qd_batch* b, int l) { return static_cast<__half*>(b->kv) + (size_t)l * b->kv_layer; }
__half* vc_of(qd_batch* b, int l) {
  return static_cast<__half*>(b->kv) + (size_t)(b->e->p.layers + l) * b->kv_layer;
}

// q4 record matrix as GEMM weights: row r at base + r * rec (gate/up pairs are
// [gate j | up j] records, i.e. flat rows 2j and 2j + 1).
TcArgs q4_args(const char* base, int K, int n_rows) {
  TcArgs a{};
  const long long rec = rec_bytes(K), nb = K / kBlockCols;
  a.w = base;
  a.s = base + nb * 16;
  a.w_stride = a.s_stride = rec;
  a.n_rows = n_rows;
  a.K = K;
  return a;
}

void gemm_q4(const char* base, int K, int n_rows, const __half* xh, const __half* xl, int rows, int splits,
             int kt_split, float* y, cudaStream_t s, int* err) {
  TcArgs a = q4_args(base, K, n_rows);
  a.x_hi = xh;
  a.x_lo = xl;
  a.B = rows;
  a.kt_split = kt_split;
  a.y = y;
  a.ldy = n_rows;
  a.y_split = (long long)rows * n_rows;
  a.err = err;
  a.stall = err ? err + 1 : nullptr;
  launch_gemm(a, splits, kGemmQ4Store, s);
}

// gate/up GEMM with silu(gate) * up fused into the epilogue (one split): writes
// the down GEMM's hi/lo operands [rows][I] directly.
void gemm_q4_silu(const char* base, int K, int I, const __half* xh, const __half* xl, int rows, __half* out_hi,
                  __half* out_lo, cudaStream_t s, int* err) {
  TcArgs a = q4_args(base, K, 2 * I);
  a.x_hi = xh;
  a.x_lo = xl;
  a.B = rows;
  a.kt_split = K / kTcK;
  a.ldy = I;
  a.y_hi = out_hi;
  a.y_lo = out_lo;
  a.err = err;
  a.stall = err ? err + 1 : nullptr;
  launch_gemm(a, 1, kGemmQ4Silu, s);
}

void lm_head(qd_batch* b, const __half* xh, const __half* xl, long long ldx, int rows, float* logits, cudaStream_t s) {
  const Dims d = dims(b->e);
  TcArgs a{};
  a.a16 = b->e->embed;
  a.a16_stride = d.H;
  a.n_rows = d.V;
  a.K = d.H;
  a.kt_split = d.H / kTcK;
  a.x_hi = xh;
  a.x_lo = xl;
  a.ldx = ldx;
  a.B = rows;
  a.y = logits;
  a.ldy = d.V;
  a.part_v = b->lm_pv;
  a.part_i = b->lm_pi;
  a.err = b->errw;
  a.stall = b->errw + 1;
  launch_gemm(a, 1, kGemmF16Argmax, s);
}

void launch_attn(qd_batch* b, int l, cudaStream_t s) {
  const Dims d = dims(b->e);
  const dim3 grid(d.NKV, b->splits, b->B);
  const float scale = 1.0f / std::sqrt((float)kHeadDim);
  const long long layer_rows = (long long)b->B * d.NKV * b->max_seq;
  const long long k_row0 = (long long)l * layer_rows, v_row0 = (long long)(d.L + l) * layer_rows;
  if (d.G == 1) {
    allow_smem(kb_attn<1>, kBAttnSmem, g_attn_smem_mask);
    launch_ex(kb_attn<1>, grid, dim3(kBAttnThreads), kBAttnSmem, s, b->kvmap, k_row0, v_row0, (const float*)b->q,
              (const int*)b->pos, d.NH, d.NKV, b->max_seq, b->split_len, b->splits, scale, b->part_ml, b->part_o,
              b->errw);
  } else {
    allow_smem(kb_attn<2>, kBAttnSmem, g_attn_smem_mask2);
    launch_ex(kb_attn<2>, grid, dim3(kBAttnThreads), kBAttnSmem, s, b->kvmap, k_row0, v_row0, (const float*)b->q,
              (const int*)b->pos, d.NH, d.NKV, b->max_seq, b->split_len, b->splits, scale, b->part_ml, b->part_o,
              b->errw);
  }
  launch_ex(kb_attn_combine, dim3(d.NH, b->B), dim3(kHeadDim), 0, s, (const float2*)b->part_ml,
            (const float*)b->part_o, b->splits, d.NH, b->xh, b->xl);
}

// Every layer of one decode step, then the final norm into x_hi / x_lo (launch
// order: see batch.cuh).
void enqueue_layers(qd_batch* b, cudaStream_t s) {
  qd_engine* e = b->e;
  const Dims d = dims(e);
  const int B = b->B;
  const long long sB = B;
  const int rope_grid = rope_grid_for(sB * (d.NH + 2 * d.NKV), 4096);
  for (int l = 0; l < d.L; ++l) {
    const LayerDev& L = e->layers[l];
    if (l == 0)
      launch_ex(kb_resid_norm, dim3(B), dim3(kNormThreads), 0, s, b->h, (const float*)nullptr, 0, 0LL, (const __half*)e->embed,
             (const int*)b->tokens, d.V, L.n_in, d.H, d.eps, b->xh, b->xl, b->errw);
    else
      launch_ex(kb_resid_norm, dim3(B), dim3(kNormThreads), 0, s, b->h, (const float*)b->parts, b->sd, sB * d.H, (const __half*)nullptr,
             (const int*)nullptr, d.V, L.n_in, d.H, d.eps, b->xh, b->xl, b->errw);
    gemm_q4(L.qkv, d.H, d.R, b->xh, b->xl, B, b->sq, b->ktq, b->parts, s, b->errw);
    launch(kb_rope_cache<true>, dim3(rope_grid), s, (const float*)b->parts, b->sq, sB * d.R, B, d.NH, d.NKV, L.n_q, L.n_k,
           d.eps, (const float*)e->cos_t, (const float*)e->sin_t, e->opt.rope_row_stride, (const int*)b->pos, 1, 0LL,
           b->max_seq, kc_of(b, l), vc_of(b, l), b->q, b->errw);
    launch_attn(b, l, s);  // attention + split combine
    gemm_q4(L.o, d.QS, d.H, b->xh, b->xl, B, b->so, b->kto, b->parts, s, b->errw);
    launch_ex(kb_resid_norm, dim3(B), dim3(kNormThreads), 0, s, b->h, (const float*)b->parts, b->so, sB * d.H, (const __half*)nullptr,
           (const int*)nullptr, d.V, L.n_post, d.H, d.eps, b->xh, b->xl, b->errw);
    gemm_q4(L.gu, d.H, 2 * d.I, b->xh, b->xl, B, b->sg, b->ktg, b->parts, s, b->errw);
    const int silu_grid = (int)std::min<long long>((sB * d.I + 255) / 256, 4096);
    launch(kb_silu_split, dim3(silu_grid), s, (const float*)b->parts, b->sg, sB * 2 * d.I, B, d.I, b->xh, b->xl);
    gemm_q4(L.d, d.I, d.H, b->xh, b->xl, B, b->sd, b->ktd, b->parts, s, b->errw);
  }
  launch_ex(kb_resid_norm, dim3(B), dim3(kNormThreads), 0, s, b->h, (const float*)b->parts, b->sd, sB * d.H, (const __half*)nullptr,
         (const int*)nullptr, d.V, (const float*)e->final_norm, d.H, d.eps, b->xh, b->xl, b->errw);
}

// One decode step of every sequence: the layers, the LM head + argmax, the ids fed back.
void enqueue_step(qd_batch* b, bool keep_logits, cudaStream_t s) {
  const Dims d = dims(b->e);
  const int B = b->B;
  enqueue_layers(b, s);
  lm_head(b, b->xh, b->xl, d.H, B, keep_logits ? b->logits : nullptr, s);
  BatchState st{b->tokens, b->pos, b->out, b->step, b->max_steps};
  launch(kb_argmax_merge, dim3((B + 7) / 8), s, (const float*)b->lm_pv, (const uint32_t*)b->lm_pi, b->lm_tiles, B, st,
         b->result);
  launch(kb_step_done, dim3(1), s, b->step);
}

int step_kernel_count(const qd_batch* b) { return b->e->p.layers * 10 + 4; }  // incl. the split combine

void check_err(qd_batch* b) {
  qd_engine* e = b->e;
  QD_CK(cudaMemcpyAsync(b->pinned_io, b->errw, 4, cudaMemcpyDeviceToHost, e->stream));
  QD_CK(cudaStreamSynchronize(e->stream));
  const int w = b->pinned_io[0];
  if (!w) return;
  QD_CK(cudaMemsetAsync(b->errw, 0, 4, e->stream));
  QD_CK(cudaStreamSynchronize(e->stream));
  if (w & (kTcErrTimeout | kBErrTimeout)) throw QdError{QD_E_TIMEOUT, "device: a bounded wait expired in a batched kernel"};
  if (w & kErrToken) throw QdError{QD_E_DEVICE, "device: token id outside the vocabulary"};
  if (w & kErrPosition) throw QdError{QD_E_DEVICE, "device: position beyond max_seq"};
  throw QdError{QD_E_DEVICE, "device: status word " + std::to_string(w)};
}

void ensure_pinned(qd_batch* b, size_t n) {
  if (b->pinned_n >= n) return;
  if (b->pinned) cudaFreeHost(b->pinned);
  b->pinned = nullptr;
  b->pinned_n = 0;
  if (cudaHostAlloc(reinterpret_cast<void**>(&b->pinned), n * 4, cudaHostAllocDefault) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate pinned host memory"};
  b->pinned_n = n;
}

// Wide buffers for `rows` rows at once (context fill chunks, prefill).
void ensure_wide(qd_batch* b, long long rows) {
  if (b->wide_rows >= rows) return;
  const Dims d = dims(b->e);
  if (b->wide) {
    QD_CK(cudaStreamSynchronize(b->e->stream));
    cudaFree(b->wide);
    b->wide = nullptr;
    b->wide_rows = 0;
  }
  const long long maxk = std::max(std::max(d.H, d.QS), d.I);
  const long long maxn = std::max(d.R, 2 * d.I);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_h = take(rows * d.H * 4), o_y = take(rows * maxn * 4), o_q = take(rows * d.QS * 4);
  const size_t o_xh = take(rows * maxk * 2), o_xl = take(rows * maxk * 2), o_tok = take(rows * 4);
  const size_t o_ah = take(rows * d.I * 2), o_al = take(rows * d.I * 2);
  if (cudaMalloc(&b->wide, off) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate prefill buffers"};
  char* base = static_cast<char*>(b->wide);
  b->w_h = reinterpret_cast<float*>(base + o_h);
  b->w_y = reinterpret_cast<float*>(base + o_y);
  b->w_q = reinterpret_cast<float*>(base + o_q);
  b->w_xh = reinterpret_cast<__half*>(base + o_xh);
  b->w_xl = reinterpret_cast<__half*>(base + o_xl);
  b->w_tok = reinterpret_cast<int*>(base + o_tok);
  b->w_ah = reinterpret_cast<__half*>(base + o_ah);
  b->w_al = reinterpret_cast<__half*>(base + o_al);
  b->wide_rows = rows;
}

void drop_graphs(qd_batch* b) {
  for (auto& g : b->g_step)
    if (g) {
      cudaGraphExecDestroy(g);
      g = nullptr;
    }
  for (auto& g : b->g_prompt) cudaGraphExecDestroy(g.second);
  b->g_prompt.clear();
  if (b->g_layers) {
    cudaGraphExecDestroy(b->g_layers);
    b->g_layers = nullptr;
  }
}

cudaGraphExec_t capture_step(qd_batch* b, bool keep_logits) {
  qd_engine* e = b->e;
  cudaGraph_t g = nullptr;
  QD_CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  try {
    enqueue_step(b, keep_logits, e->stream);
  } catch (...) {
    cudaStreamEndCapture(e->stream, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  QD_CK(cudaStreamEndCapture(e->stream, &g));
  cudaGraphExec_t x = nullptr;
  const cudaError_t rc = cudaGraphInstantiate(&x, g, 0);
  cudaGraphDestroy(g);
  QD_CK(rc);
  return x;
}

void free_batch(qd_batch* b) {
  if (!b) return;
  if (b->e) {
    cudaSetDevice(b->e->dev);
    cudaStreamSynchronize(b->e->stream);
  }
  drop_graphs(b);
  if (b->kv) cudaFree(b->kv);
  if (b->pp) cudaFree(b->pp);
  if (b->dec) cudaFree(b->dec);
  if (b->logits) cudaFree(b->logits);
  if (b->wide) cudaFree(b->wide);
  if (b->shard_buf) cudaFree(b->shard_buf);
  if (b->pinned) cudaFreeHost(b->pinned);
  if (b->pinned_io) cudaFreeHost(b->pinned_io);
  delete b;
}

void create_batch(qd_engine* e, int B, int max_seq, qd_batch* b) {
  const Dims d = dims(e);
  if (B < 1 || B > 65535) throw QdError{QD_E_INVALID, "batch must be 1..65535"};
  if (max_seq < 1) throw QdError{QD_E_INVALID, "max_seq must be positive"};
  if (d.G != 1 && d.G != 2) throw QdError{QD_E_INVALID, "batched attention supports q_heads / kv_heads of 1 or 2"};
  if (d.H % kTcK || d.QS % kTcK || d.I % kTcK) throw QdError{QD_E_INVALID, "batched path: hidden, q and intermediate sizes must be multiples of 64"};
  if (d.H > 4096) throw QdError{QD_E_INVALID, "batched path: hidden size above 4096"};
  const long long last = (long long)(max_seq - 1) * e->opt.rope_row_stride + kHeadDim / 2;
  if (last > (long long)e->p.rope_rows * (kHeadDim / 2))
    throw QdError{QD_E_RANGE, "max_seq beyond the RoPE table for this row stride"};
  b->e = e;
  b->B = B;
  b->max_seq = max_seq;
  // Decode attention: 512-position splits (fewer for short contexts).
  b->split_len = std::min(512, (max_seq + kBAttnTile - 1) / kBAttnTile * kBAttnTile);
  b->splits = (max_seq + b->split_len - 1) / b->split_len;
  // Split-K so that each GEMM launches about one CTA per SM (at most kMaxParts
  // partials for the consumer to add; measured at 64 x 2048: 15.8k tok/s against
  // 15.6k for two CTAs per SM and 15.2k for three).
  auto plan = [&](int n_rows, int K, int* kt) {
    const int tiles = (n_rows + kTcM - 1) / kTcM * ((B + 255) / 256);
    return gemm_plan_splits(K, std::max(1, std::min(kMaxParts, e->sms / std::max(1, tiles))), kt);
  };
  b->sq = plan(d.R, d.H, &b->ktq);
  b->so = plan(d.H, d.QS, &b->kto);
  b->sg = plan(2 * d.I, d.H, &b->ktg);
  b->sd = plan(d.H, d.I, &b->ktd);
  b->lm_tiles = (d.V + kTcM - 1) / kTcM;

  b->kv_layer = (size_t)B * d.NKV * max_seq * kHeadDim;
  const size_t kv_bytes = b->kv_layer * 2 * 2 * d.L;
  const unsigned long long kv_rows = (unsigned long long)2 * d.L * B * d.NKV * max_seq;
  if (kv_rows + kBAttnTile >= (1ull << 31)) throw QdError{QD_E_RANGE, "batch KV cache beyond 2^31 rows"};
  if (cudaMalloc(&b->kv, kv_bytes) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate the batch KV cache (" + std::to_string(kv_bytes >> 20) + " MiB)"};
  QD_CK(cudaMemsetAsync(b->kv, 0, kv_bytes, e->stream));
  std::string terr;
  if (!make_tmap_2d(&b->kvmap, b->kv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kHeadDim, kv_rows, kHeadDim * 2, 64,
                    kBAttnTile, CU_TENSOR_MAP_SWIZZLE_128B, &terr))
    throw QdError{QD_E_CUDA, "KV tensor map: " + terr};

  const long long maxk = std::max(std::max(d.H, d.QS), d.I);
  const long long parts = std::max(std::max((long long)b->sq * d.R, (long long)b->so * d.H),
                                   std::max((long long)b->sg * 2 * d.I, (long long)b->sd * d.H)) *
                          B;
  b->max_steps = 256;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_h = take((size_t)B * d.H * 4), o_xh = take((size_t)B * maxk * 2), o_xl = take((size_t)B * maxk * 2);
  const size_t o_p = take((size_t)parts * 4), o_q = take((size_t)B * d.QS * 4);
  const size_t o_ml = take((size_t)B * b->splits * d.NH * 8), o_po = take((size_t)B * b->splits * d.QS * 4);
  const size_t o_pv = take((size_t)B * b->lm_tiles * 4), o_pi = take((size_t)B * b->lm_tiles * 4);
  const size_t o_res = take((size_t)B * 8), o_tok = take((size_t)B * 4), o_pos = take((size_t)B * 4);
  const size_t o_out = take((size_t)b->max_steps * B * 4), o_step = take(4), o_err = take(8);  // [0] status word, [1] stall hook
  if (cudaMalloc(&b->dec, off) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate batch step buffers"};
  QD_CK(cudaMemsetAsync(b->dec, 0, off, e->stream));
  char* base = static_cast<char*>(b->dec);
  b->h = reinterpret_cast<float*>(base + o_h);
  b->xh = reinterpret_cast<__half*>(base + o_xh);
  b->xl = reinterpret_cast<__half*>(base + o_xl);
  b->parts = reinterpret_cast<float*>(base + o_p);
  b->q = reinterpret_cast<float*>(base + o_q);
  b->part_ml = reinterpret_cast<float2*>(base + o_ml);
  b->part_o = reinterpret_cast<float*>(base + o_po);
  b->lm_pv = reinterpret_cast<float*>(base + o_pv);
  b->lm_pi = reinterpret_cast<uint32_t*>(base + o_pi);
  b->result = reinterpret_cast<uint32_t*>(base + o_res);
  b->tokens = reinterpret_cast<int*>(base + o_tok);
  b->pos = reinterpret_cast<int*>(base + o_pos);
  b->out = reinterpret_cast<int*>(base + o_out);
  b->step = reinterpret_cast<int*>(base + o_step);
  b->errw = reinterpret_cast<int*>(base + o_err);
  b->host_pos.assign(B, 0);
  ensure_pinned(b, (size_t)b->max_steps * B);
  if (cudaHostAlloc(reinterpret_cast<void**>(&b->pinned_io), (2 * (size_t)B + 16) * 4, cudaHostAllocDefault) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate pinned host memory"};
  QD_CK(cudaStreamSynchronize(e->stream));
}

void upload_tokens_positions(qd_batch* b, const int32_t* tokens, const int32_t* positions) {
  qd_engine* e = b->e;
  const int B = b->B;
  QD_CK(cudaStreamSynchronize(e->stream));
  int* stage = b->pinned_io + 16;
  if (tokens) {
    std::memcpy(stage, tokens, (size_t)B * 4);
    QD_CK(cudaMemcpyAsync(b->tokens, stage, (size_t)B * 4, cudaMemcpyHostToDevice, e->stream));
  }
  if (positions) {
    std::memcpy(stage + B, positions, (size_t)B * 4);
    QD_CK(cudaMemcpyAsync(b->pos, stage + B, (size_t)B * 4, cudaMemcpyHostToDevice, e->stream));
  }
  QD_CK(cudaStreamSynchronize(e->stream));
  if (positions) b->host_pos.assign(positions, positions + B);
}

// ---- context fill -------------------------------------------------------------
void fill_context(qd_batch* b, int ctx, uint32_t seed) {
  qd_engine* e = b->e;
  const Dims d = dims(e);
  cudaStream_t s = e->stream;
  const long long rows = (long long)b->B * ctx;
  const long long chunk = std::min<long long>(rows, 16384);
  ensure_wide(b, chunk);
  for (int l = 0; l < d.L; ++l) {
    const LayerDev& L = e->layers[l];
    for (long long r0 = 0; r0 < rows; r0 += chunk) {
      const int R = (int)std::min(chunk, rows - r0);
      launch(kb_ctx_hidden, dim3(R), s, seed, (uint32_t)l, r0, d.H, L.n_in, d.eps, b->w_xh, b->w_xl);
      // k and v rows of the fused qkv matrix
      gemm_q4(L.qkv + (size_t)d.QS * rec_bytes(d.H), d.H, 2 * d.KVS, b->w_xh, b->w_xl, R, 1, d.H / kTcK, b->w_y, s,
              b->errw);
      const int grid = rope_grid_for((long long)R * 2 * d.NKV, 8192);
      launch(kb_rope_cache<false>, dim3(grid), s, (const float*)b->w_y, 1, 0LL, R, 0, d.NKV, L.n_q, L.n_k, d.eps,
             (const float*)e->cos_t, (const float*)e->sin_t, e->opt.rope_row_stride, (const int*)nullptr, ctx, r0,
             b->max_seq, kc_of(b, l), vc_of(b, l), (float*)nullptr, b->errw);
    }
  }
  std::vector<int32_t> p(b->B, ctx);
  QD_CK(cudaStreamSynchronize(s));
  check_err(b);
  upload_tokens_positions(b, nullptr, p.data());
}

// ---- decode loop ----------------------------------------------------------------
void decode(qd_batch* b, int steps, int32_t* out_ids) {
  qd_engine* e = b->e;
  cudaStream_t s = e->stream;
  const int B = b->B;
  for (int i = 0; i < B; ++i)
    if (b->host_pos[i] < 0 || (long long)b->host_pos[i] + steps > b->max_seq)
      throw QdError{QD_E_RANGE, "sequence " + std::to_string(i) + ": position + steps beyond max_seq"};
  const int k = b->keep_logits ? 1 : 0;
  if (!b->g_step[k]) b->g_step[k] = capture_step(b, b->keep_logits);
  for (int done = 0; done < steps;) {
    const int n = std::min(steps - done, b->max_steps);
    QD_CK(cudaMemsetAsync(b->step, 0, 4, s));
    for (int i = 0; i < n; ++i) QD_CK(cudaGraphLaunch(b->g_step[k], s));
    if (out_ids) QD_CK(cudaMemcpyAsync(b->pinned, b->out, (size_t)n * B * 4, cudaMemcpyDeviceToHost, s));
    QD_CK(cudaStreamSynchronize(s));
    check_err(b);
    if (out_ids) std::memcpy(out_ids + (size_t)done * B, b->pinned, (size_t)n * B * 4);
    done += n;
  }
  for (int i = 0; i < B; ++i) b->host_pos[i] += steps;
}

// ---- prefill ------------------------------------------------------------------------
// Residual (+ one partial) + RMSNorm of `rows` rows into the GEMM operands: one warp
// per row where the hidden size allows (128 NV columns, NV = 4 or 8), else one CTA
// per row.
// `np` split-K partials `stride` floats apart (np = 1 when parts is set and np is 0).
// Fewer rows than 4 per SM (a short prompt) take one CTA per row instead: a warp
// alone would add up to 16 partials of its row one round trip after another
// (measured 15 us per launch at 7 rows and 16 partials).
void rows_norm(qd_batch* b, float* h, const float* parts, const __half* embed, const int* tokens, const float* w,
               long long rows, cudaStream_t s, int np = 0, long long stride = 0) {
  const Dims d = dims(b->e);
  const unsigned grid = (unsigned)((rows + kNormThreads / 32 - 1) / (kNormThreads / 32));
  if (!parts) np = 0;
  else if (np < 1) np = 1;
  if (rows < 4LL * b->e->sms)
    launch_ex(kb_resid_norm, dim3((unsigned)rows), dim3(kNormThreads), 0, s, h, parts, np, stride, embed, tokens, d.V,
              w, d.H, d.eps, b->w_xh, b->w_xl, b->errw);
  else if (d.H == 1024)
    launch_ex(kb_resid_norm_rows<8>, dim3(grid), dim3(kNormThreads), 0, s, h, parts, np, stride, embed, tokens, d.V, w,
              (int)rows, d.eps, b->w_xh, b->w_xl, b->errw);
  else if (d.H == 512)
    launch_ex(kb_resid_norm_rows<4>, dim3(grid), dim3(kNormThreads), 0, s, h, parts, np, stride, embed, tokens, d.V, w,
              (int)rows, d.eps, b->w_xh, b->w_xl, b->errw);
  else
    launch_ex(kb_resid_norm, dim3((unsigned)rows), dim3(kNormThreads), 0, s, h, parts, np, stride, embed, tokens, d.V,
              w, d.H, d.eps, b->w_xh, b->w_xl, b->errw);
}

// All prompts at once: B * n rows through every layer (GEMMs over the rows,
// causal attention inside each prompt), then the LM head on each prompt's last
// row; each sequence's first generated id becomes its next input at position n.
void prefill(qd_batch* b, const int32_t* ids, int n, int32_t* first_ids) {
  qd_engine* e = b->e;
  const Dims d = dims(e);
  cudaStream_t s = e->stream;
  const int B = b->B;
  const long long T = (long long)B * n;
  if (T > (1ll << 31) / std::max(d.R, 2 * d.I)) throw QdError{QD_E_RANGE, "prefill: batch * n_prompt too large"};
  ensure_wide(b, T);
  QD_CK(cudaMemcpyAsync(b->w_tok, ids, (size_t)T * 4, cudaMemcpyHostToDevice, s));
  const float scale = 1.0f / std::sqrt((float)kHeadDim);
  const long long layer_rows = (long long)B * d.NKV * b->max_seq;
  const int qtiles = (n + kPfTile - 1) / kPfTile;
  const int rope_grid = rope_grid_for(T * (d.NH + 2 * d.NKV), 1 << 20);
  for (int l = 0; l < d.L; ++l) {
    const LayerDev& L = e->layers[l];
    if (l == 0)
      rows_norm(b, b->w_h, nullptr, e->embed, b->w_tok, L.n_in, T, s);
    else
      rows_norm(b, b->w_h, b->w_y, nullptr, nullptr, L.n_in, T, s);
    gemm_q4(L.qkv, d.H, d.R, b->w_xh, b->w_xl, (int)T, 1, d.H / kTcK, b->w_y, s, b->errw);
    launch(kb_rope_cache<false>, dim3(rope_grid), s, (const float*)b->w_y, 1, 0LL, (int)T, d.NH, d.NKV, L.n_q, L.n_k, d.eps,
           (const float*)e->cos_t, (const float*)e->sin_t, e->opt.rope_row_stride, (const int*)nullptr, n, 0LL,
           b->max_seq, kc_of(b, l), vc_of(b, l), b->w_q, b->errw);
    const long long k_row0 = (long long)l * layer_rows, v_row0 = (long long)(d.L + l) * layer_rows;
    const dim3 agrid(d.NKV, qtiles, B);
    if (d.G == 1) {
      allow_smem(kb_prefill_attn<1>, pf_smem(1), g_pf_smem_mask);
      launch_ex(kb_prefill_attn<1>, agrid, dim3(128), pf_smem(1), s, b->kvmap, k_row0, v_row0, (const float*)b->w_q, n,
                d.NH, d.NKV, b->max_seq, scale, b->w_xh, b->w_xl, b->errw);
    } else {
      allow_smem(kb_prefill_attn<2>, pf_smem(2), g_pf_smem_mask2);
      launch_ex(kb_prefill_attn<2>, agrid, dim3(256), pf_smem(2), s, b->kvmap, k_row0, v_row0, (const float*)b->w_q, n,
                d.NH, d.NKV, b->max_seq, scale, b->w_xh, b->w_xl, b->errw);
    }
    gemm_q4(L.o, d.QS, d.H, b->w_xh, b->w_xl, (int)T, 1, d.QS / kTcK, b->w_y, s, b->errw);
    rows_norm(b, b->w_h, b->w_y, nullptr, nullptr, L.n_post, T, s);
    // gate/up: silu(gate) * up goes straight into the down GEMM's operands
    gemm_q4_silu(L.gu, d.H, d.I, b->w_xh, b->w_xl, (int)T, b->w_ah, b->w_al, s, b->errw);
    gemm_q4(L.d, d.I, d.H, b->w_ah, b->w_al, (int)T, 1, d.I / kTcK, b->w_y, s, b->errw);
  }
  rows_norm(b, b->w_h, b->w_y, nullptr, nullptr, e->final_norm, T, s);
  // LM head on each prompt's last row; the merge feeds the id back and moves the position to n.
  lm_head(b, b->w_xh + (size_t)(n - 1) * d.H, b->w_xl + (size_t)(n - 1) * d.H, (long long)n * d.H, B,
          b->keep_logits ? b->logits : nullptr, s);
  std::vector<int32_t> p(B, n - 1);
  std::memcpy(b->pinned_io + 16 + B, p.data(), (size_t)B * 4);
  QD_CK(cudaMemcpyAsync(b->pos, b->pinned_io + 16 + B, (size_t)B * 4, cudaMemcpyHostToDevice, s));
  QD_CK(cudaMemsetAsync(b->step, 0, 4, s));
  BatchState st{b->tokens, b->pos, b->out, b->step, b->max_steps};
  launch(kb_argmax_merge, dim3((B + 7) / 8), s, (const float*)b->lm_pv, (const uint32_t*)b->lm_pi, b->lm_tiles, B, st,
         b->result);
  if (first_ids) QD_CK(cudaMemcpyAsync(b->pinned, b->out, (size_t)B * 4, cudaMemcpyDeviceToHost, s));
  QD_CK(cudaStreamSynchronize(s));
  check_err(b);
  if (first_ids) std::memcpy(first_ids, b->pinned, (size_t)B * 4);
  b->host_pos.assign(B, n);
}

// ---- engine prompt pass ------------------------------------------------------------
// The engine's prompt tokens 0..T-1 as T rows of one sequence: per layer the input
// norm, the QKV GEMM, head norm + RoPE + K/V append, causal prompt attention, the O
// GEMM, the post-attention norm, gate/up, silu(gate) * up and the down GEMM, with
// split-K planned for about two CTAs per SM (T is small: few row tiles per GEMM; at 7
// rows two per SM measured 1.587 against 1.610 ms from prompt to first id). The
// last layer stops after its K/V append (nothing after it feeds the cache), and the
// K/V rows are then copied into the engine's cache layout.
struct PromptPlan {
  int sq, so, sg, sd, ktq, kto, ktg, ktd;
  long long parts;  // floats of the largest GEMM's partials
};

PromptPlan prompt_plan(qd_batch* b, int T) {
  const Dims d = dims(b->e);
  const int col_tiles = T <= 128 ? 1 : (T + 255) / 256;
  auto plan = [&](int n_rows, int K, int* kt) {
    const int tiles = (n_rows + kTcM - 1) / kTcM * col_tiles;
    return gemm_plan_splits(K, std::max(1, std::min(kMaxParts, 2 * b->e->sms / std::max(1, tiles))), kt);
  };
  PromptPlan p{};
  p.sq = plan(d.R, d.H, &p.ktq);
  p.so = plan(d.H, d.QS, &p.kto);
  p.sg = plan(2 * d.I, d.H, &p.ktg);
  p.sd = plan(d.H, d.I, &p.ktd);
  p.parts = std::max(std::max((long long)p.sq * d.R, (long long)p.so * d.H),
                     std::max((long long)p.sg * 2 * d.I, (long long)p.sd * d.H)) *
            T;
  return p;
}

// With first_id set, every layer runs to its end, and the final norm, the LM head on
// the last row and the argmax merge follow: the id goes to first_id[0] (the engine's
// token slot after the prompt) and out0[0] (its first output slot).
void enqueue_prompt(qd_batch* b, const int* ids, int T, const PromptPlan& pl, cudaStream_t s, int* first_id = nullptr,
                    int* out0 = nullptr) {
  qd_engine* e = b->e;
  const Dims d = dims(e);
  const long long sT = T;
  const float scale = 1.0f / std::sqrt((float)kHeadDim);
  const long long layer_rows = (long long)d.NKV * b->max_seq;  // one sequence
  const int qtiles = (T + kPfTile - 1) / kPfTile;
  const int rope_grid = rope_grid_for(sT * (d.NH + 2 * d.NKV), 4096);
  const int silu_grid = (int)std::min<long long>((sT * d.I + 255) / 256, 4096);
  for (int l = 0; l < d.L; ++l) {
    const LayerDev& L = e->layers[l];
    if (l == 0)
      rows_norm(b, b->w_h, nullptr, e->embed, ids, L.n_in, T, s);
    else
      rows_norm(b, b->w_h, b->pp, nullptr, nullptr, L.n_in, T, s, pl.sd, sT * d.H);
    gemm_q4(L.qkv, d.H, d.R, b->w_xh, b->w_xl, T, pl.sq, pl.ktq, b->pp, s, b->errw);
    launch(kb_rope_cache<true>, dim3(rope_grid), s, (const float*)b->pp, pl.sq, sT * d.R, T, d.NH, d.NKV, L.n_q, L.n_k,
           d.eps, (const float*)e->cos_t, (const float*)e->sin_t, e->opt.rope_row_stride, (const int*)nullptr, T,
           0LL, b->max_seq, kc_of(b, l), vc_of(b, l), b->w_q, b->errw);
    if (l == d.L - 1 && !first_id) break;
    const long long k_row0 = (long long)l * layer_rows, v_row0 = (long long)(d.L + l) * layer_rows;
    const dim3 agrid(d.NKV, qtiles, 1);
    if (d.G == 1) {
      allow_smem(kb_prefill_attn<1>, pf_smem(1), g_pf_smem_mask);
      launch_ex(kb_prefill_attn<1>, agrid, dim3(128), pf_smem(1), s, b->kvmap, k_row0, v_row0, (const float*)b->w_q, T,
                d.NH, d.NKV, b->max_seq, scale, b->w_xh, b->w_xl, b->errw);
    } else {
      allow_smem(kb_prefill_attn<2>, pf_smem(2), g_pf_smem_mask2);
      launch_ex(kb_prefill_attn<2>, agrid, dim3(256), pf_smem(2), s, b->kvmap, k_row0, v_row0, (const float*)b->w_q, T,
                d.NH, d.NKV, b->max_seq, scale, b->w_xh, b->w_xl, b->errw);
    }
    gemm_q4(L.o, d.QS, d.H, b->w_xh, b->w_xl, T, pl.so, pl.kto, b->pp, s, b->errw);
    rows_norm(b, b->w_h, b->pp, nullptr, nullptr, L.n_post, T, s, pl.so, sT * d.H);
    gemm_q4(L.gu, d.H, 2 * d.I, b->w_xh, b->w_xl, T, pl.sg, pl.ktg, b->pp, s, b->errw);
    launch(kb_silu_split, dim3(silu_grid), s, (const float*)b->pp, pl.sg, sT * 2 * d.I, T, d.I, b->w_ah, b->w_al);
    gemm_q4(L.d, d.I, d.H, b->w_ah, b->w_al, T, pl.sd, pl.ktd, b->pp, s, b->errw);
  }
  if (first_id) {
    rows_norm(b, b->w_h, b->pp, nullptr, nullptr, e->final_norm, T, s, pl.sd, sT * d.H);
    lm_head(b, b->w_xh + (size_t)(T - 1) * d.H, b->w_xl + (size_t)(T - 1) * d.H, d.H, 1, nullptr, s);
    QD_CK(cudaMemsetAsync(b->step, 0, 4, s));
    BatchState st{first_id, b->pos, out0, b->step, 1};
    launch(kb_argmax_merge, dim3(1), s, (const float*)b->lm_pv, (const uint32_t*)b->lm_pi, b->lm_tiles, 1, st,
           (uint32_t*)nullptr);
  }
  const long long ekv_layer = (long long)e->opt.max_seq * d.KVS * 2;  // bytes of one layer's K (f16)
  const long long copies = (long long)d.L * 2 * T * d.NKV * 16;
  launch(kb_kv_to_engine, dim3((unsigned)std::min<long long>((copies + 255) / 256, 4 * e->sms)), s,
         (const __half*)b->kv, (long long)b->kv_layer, d.L, d.NKV, b->max_seq, T, static_cast<char*>(e->kv), ekv_layer);
}

// ---- vocabulary-sharded LM head ------------------------------------------------------
cudaGraphExec_t capture_layers_to_gather(qd_batch* b) {
  cudaStream_t s = b->e->stream;
  const Dims d = dims(b->e);
  const size_t rows_bytes = (size_t)b->B * d.H * 2;
  const size_t off = (size_t)b->shard_rank * b->B * d.H;
  cudaGraph_t g = nullptr;
  QD_CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  try {
    enqueue_layers(b, s);
    QD_CK(cudaMemcpyAsync(b->gx_hi + off, b->xh, rows_bytes, cudaMemcpyDeviceToDevice, s));
    QD_CK(cudaMemcpyAsync(b->gx_lo + off, b->xl, rows_bytes, cudaMemcpyDeviceToDevice, s));
  } catch (...) {
    cudaStreamEndCapture(s, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  QD_CK(cudaStreamEndCapture(s, &g));
  cudaGraphExec_t x = nullptr;
  const cudaError_t rc = cudaGraphInstantiate(&x, g, 0);
  cudaGraphDestroy(g);
  QD_CK(rc);
  return x;
}

void require_shard(const qd_batch* b) {
  if (!b->shard_world) throw QdError{QD_E_INVALID, "no vocabulary shard set (qd_batch_set_vocab_shard)"};
}

}  // namespace

namespace qd {

bool prompt_pass_fits(qd_engine* e, int n) {
  if (!e->opt.prompt_pass || e->opt.kv_dtype != QD_KV_F16 || e->pbatch_unfit) return false;
  if (n < kPromptPassMin || n > kPromptPassMax || n > e->opt.max_seq) return false;
  if (e->pbatch) return true;
  qd_batch* b = new qd_batch();
  try {
    create_batch(e, 1, std::min(kPromptPassMax, e->opt.max_seq), b);
  } catch (const QdError&) {  // a shape or size the batched path does not take: token by token
    free_batch(b);
    e->pbatch_unfit = true;
    return false;
  }
  e->pbatch = b;
  return true;
}

void prompt_pass(qd_engine* e, int n, bool with_head) {
  qd_batch* b = e->pbatch;
  if (!b || n > b->max_seq) throw QdError{QD_E_INVALID, "prompt pass: no batch for this length"};
  const PromptPlan pl = prompt_plan(b, n);
  const int key = 2 * n + (with_head ? 1 : 0);
  cudaGraphExec_t x = nullptr;
  for (auto& g : b->g_prompt)
    if (g.first == key) x = g.second;
  if (!x) {
    // Buffers first (a graph holds their addresses): wide rows for the longest prompt,
    // partials for this plan.
    ensure_wide(b, b->max_seq);
    if (b->pp_elems < pl.parts) {
      QD_CK(cudaStreamSynchronize(e->stream));
      for (auto& g : b->g_prompt) cudaGraphExecDestroy(g.second);
      b->g_prompt.clear();
      if (b->pp) cudaFree(b->pp);
      b->pp = nullptr;
      b->pp_elems = 0;
      if (cudaMalloc(&b->pp, (size_t)pl.parts * 4) != cudaSuccess)
        throw QdError{QD_E_NOMEM, "cannot allocate the prompt pass partials"};
      b->pp_elems = pl.parts;
    }
    cudaGraph_t g = nullptr;
    QD_CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    try {
      if (with_head) enqueue_prompt(b, e->tokens, n, pl, e->stream, e->tokens + n, e->out_host_dev);
      else enqueue_prompt(b, e->tokens, n, pl, e->stream);
    } catch (...) {
      cudaStreamEndCapture(e->stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    QD_CK(cudaStreamEndCapture(e->stream, &g));
    const cudaError_t rc = cudaGraphInstantiate(&x, g, 0);
    cudaGraphDestroy(g);
    QD_CK(rc);
    if (b->g_prompt.size() >= 8) {
      cudaGraphExecDestroy(b->g_prompt.front().second);
      b->g_prompt.erase(b->g_prompt.begin());
    }
    b->g_prompt.emplace_back(key, x);
  }
  QD_CK(cudaGraphLaunch(x, e->stream));
}

void prompt_pass_check(qd_engine* e) {
  if (e->pbatch) check_err(e->pbatch);
}

void prompt_pass_free(qd_engine* e) {
  if (e->pbatch) free_batch(e->pbatch);
  e->pbatch = nullptr;
}

}  // namespace qd

extern "C" {

int qd_batch_set_vocab_shard(qd_batch* b, int rank, int world, void* gather_hi, void* gather_lo, void* pairs_local,
                             void* pairs_all) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    if (world < 1 || rank < 0 || rank >= world) throw QdError{QD_E_INVALID, "rank must be 0..world-1"};
    if (!gather_hi || !gather_lo || !pairs_local || !pairs_all) throw QdError{QD_E_INVALID, "NULL buffer"};
    if ((reinterpret_cast<uintptr_t>(gather_hi) | reinterpret_cast<uintptr_t>(gather_lo)) & 15)
      throw QdError{QD_E_INVALID, "gather buffers must be 16-byte aligned"};
    const Dims d = dims(b->e);
    if ((long long)world * b->B > 65535) throw QdError{QD_E_RANGE, "world * batch above 65535 rows"};
    QD_CK(cudaSetDevice(b->e->dev));
    QD_CK(cudaStreamSynchronize(b->e->stream));
    drop_graphs(b);
    if (b->shard_buf) {
      cudaFree(b->shard_buf);
      b->shard_buf = nullptr;
    }
    b->shard_rank = rank;
    b->shard_world = world;
    b->shard_v0 = (int)((long long)d.V * rank / world);
    b->shard_v1 = (int)((long long)d.V * (rank + 1) / world);
    b->shard_tiles = (b->shard_v1 - b->shard_v0 + kTcM - 1) / kTcM;
    const size_t n = (size_t)world * b->B * b->shard_tiles;
    if (cudaMalloc(&b->shard_buf, n * 8) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate LM-slice partials"};
    b->shard_pv = static_cast<float*>(b->shard_buf);
    b->shard_pi = reinterpret_cast<uint32_t*>(b->shard_pv + n);
    b->gx_hi = static_cast<__half*>(gather_hi);
    b->gx_lo = static_cast<__half*>(gather_lo);
    b->pairs_local = static_cast<uint32_t*>(pairs_local);
    b->pairs_all = static_cast<uint32_t*>(pairs_all);
    b->shard_steps = 0;
    QD_CK(cudaMemsetAsync(b->step, 0, 4, b->e->stream));
    QD_CK(cudaStreamSynchronize(b->e->stream));
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_step_layers(qd_batch* b) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    require_shard(b);
    if (b->shard_steps >= b->max_steps) throw QdError{QD_E_RANGE, "too many steps since the last qd_batch_shard_sync"};
    for (int i = 0; i < b->B; ++i)
      if (b->host_pos[i] < 0 || (long long)b->host_pos[i] + b->shard_steps + 1 > b->max_seq)
        throw QdError{QD_E_RANGE, "sequence " + std::to_string(i) + ": position beyond max_seq"};
    QD_CK(cudaSetDevice(b->e->dev));
    if (!b->g_layers) b->g_layers = capture_layers_to_gather(b);
    QD_CK(cudaGraphLaunch(b->g_layers, b->e->stream));
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_step_lm_slice(qd_batch* b) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    require_shard(b);
    QD_CK(cudaSetDevice(b->e->dev));
    const Dims d = dims(b->e);
    cudaStream_t s = b->e->stream;
    const int rows = b->shard_world * b->B;
    TcArgs a{};
    a.a16 = b->e->embed + (size_t)b->shard_v0 * d.H;
    a.a16_stride = d.H;
    a.n_rows = b->shard_v1 - b->shard_v0;
    a.row0 = b->shard_v0;
    a.K = d.H;
    a.kt_split = d.H / kTcK;
    a.x_hi = b->gx_hi;
    a.x_lo = b->gx_lo;
    a.ldx = d.H;
    a.B = rows;
    a.part_v = b->shard_pv;
    a.part_i = b->shard_pi;
    a.err = b->errw;
    launch_gemm(a, 1, kGemmF16Argmax, s);
    BatchState none{nullptr, nullptr, nullptr, nullptr, 0};
    launch(kb_argmax_merge, dim3((rows + 7) / 8), s, (const float*)b->shard_pv, (const uint32_t*)b->shard_pi,
           b->shard_tiles, rows, none, b->pairs_local);
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_step_merge(qd_batch* b) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    require_shard(b);
    QD_CK(cudaSetDevice(b->e->dev));
    cudaStream_t s = b->e->stream;
    BatchState st{b->tokens, b->pos, b->out, b->step, b->max_steps};
    launch(kb_shard_merge, dim3((b->B + 255) / 256), s, (const uint32_t*)b->pairs_all, b->shard_world, b->shard_rank,
           b->B, st);
    launch(kb_step_done, dim3(1), s, b->step);
    b->shard_steps += 1;
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_shard_sync(qd_batch* b, int steps, int32_t* out_ids) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    require_shard(b);
    if (steps != b->shard_steps) throw QdError{QD_E_INVALID, "steps must equal the merged steps since the last sync"};
    QD_CK(cudaSetDevice(b->e->dev));
    cudaStream_t s = b->e->stream;
    if (out_ids && steps) {
      ensure_pinned(b, (size_t)steps * b->B);
      QD_CK(cudaMemcpyAsync(b->pinned, b->out, (size_t)steps * b->B * 4, cudaMemcpyDeviceToHost, s));
    }
    QD_CK(cudaMemsetAsync(b->step, 0, 4, s));
    QD_CK(cudaStreamSynchronize(s));
    check_err(b);
    if (out_ids && steps) std::memcpy(out_ids, b->pinned, (size_t)steps * b->B * 4);
    for (int i = 0; i < b->B; ++i) b->host_pos[i] += steps;
    b->shard_steps = 0;
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_create(qd_engine* e, int batch, int max_seq, qd_batch** out) {
  if (!out) return bfail(nullptr, QdError{QD_E_INVALID, "NULL out"});
  *out = nullptr;
  if (!e) return bfail(nullptr, QdError{QD_E_INVALID, "NULL engine"});
  qd_batch* b = new qd_batch();
  try {
    QD_CK(cudaSetDevice(e->dev));
    create_batch(e, batch, max_seq, b);
  } catch (const QdError& err) {
    const int rc = bfail(nullptr, err);
    free_batch(b);
    return rc;
  }
  *out = b;
  return QD_OK;
}

void qd_batch_destroy(qd_batch* b) { free_batch(b); }

int qd_batch_size(const qd_batch* b, int* batch, int* max_seq) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  if (batch) *batch = b->B;
  if (max_seq) *max_seq = b->max_seq;
  return QD_OK;
}

int qd_batch_fill_context(qd_batch* b, int ctx, uint32_t seed) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    if (ctx < 0 || ctx > b->max_seq) throw QdError{QD_E_RANGE, "ctx must be 0..max_seq"};
    if ((long long)b->B * ctx >= (1ll << 31) / std::max(1, b->e->p.hidden) * 1ll)
      throw QdError{QD_E_RANGE, "batch * ctx * hidden beyond the context generator's 32-bit row index"};
    QD_CK(cudaSetDevice(b->e->dev));
    if (ctx == 0) {
      std::vector<int32_t> p(b->B, 0);
      upload_tokens_positions(b, nullptr, p.data());
      return QD_OK;
    }
    fill_context(b, ctx, seed);
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_set_tokens(qd_batch* b, const int32_t* tokens, const int32_t* positions) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    const int V = b->e->p.vocab;
    for (int i = 0; tokens && i < b->B; ++i)
      if (tokens[i] < 0 || tokens[i] >= V) throw QdError{QD_E_RANGE, "token id outside the vocabulary"};
    for (int i = 0; positions && i < b->B; ++i)
      if (positions[i] < 0 || positions[i] >= b->max_seq) throw QdError{QD_E_RANGE, "position outside 0..max_seq-1"};
    QD_CK(cudaSetDevice(b->e->dev));
    upload_tokens_positions(b, tokens, positions);
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_positions(qd_batch* b, int32_t* positions) {
  if (!b || !positions) return bfail(b, QdError{QD_E_INVALID, "NULL argument"});
  std::copy(b->host_pos.begin(), b->host_pos.end(), positions);
  return QD_OK;
}

int qd_batch_decode(qd_batch* b, int steps, int32_t* out_ids) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    if (steps < 0) throw QdError{QD_E_INVALID, "steps must be >= 0"};
    QD_CK(cudaSetDevice(b->e->dev));
    decode(b, steps, out_ids);
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_keep_logits(qd_batch* b, int keep) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "NULL batch"});
  try {
    QD_CK(cudaSetDevice(b->e->dev));
    if (keep && !b->logits) {
      const size_t n = (size_t)b->B * b->e->p.vocab * 4;
      if (cudaMalloc(&b->logits, n) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate batch logits"};
      QD_CK(cudaMemset(b->logits, 0, n));
    }
    b->keep_logits = keep != 0;
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_logits(qd_batch* b, float* host_logits) {
  if (!b || !host_logits) return bfail(b, QdError{QD_E_INVALID, "NULL argument"});
  try {
    if (!b->logits) throw QdError{QD_E_INVALID, "logits are not kept (qd_batch_keep_logits)"};
    QD_CK(cudaSetDevice(b->e->dev));
    QD_CK(cudaStreamSynchronize(b->e->stream));
    QD_CK(cudaMemcpy(host_logits, b->logits, (size_t)b->B * b->e->p.vocab * 4, cudaMemcpyDeviceToHost));
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

static void kv_range_check(qd_batch* b, int layer, int seq, int pos0, int count) {
  if (layer < 0 || layer >= b->e->p.layers || seq < 0 || seq >= b->B || pos0 < 0 || count < 0 ||
      (long long)pos0 + count > b->max_seq)
    throw QdError{QD_E_RANGE, "KV rows outside the batch cache"};
}

int qd_batch_read_kv(qd_batch* b, int layer, int seq, int pos0, int count, float* k, float* v) {
  if (!b || !k || !v) return bfail(b, QdError{QD_E_INVALID, "NULL argument"});
  try {
    kv_range_check(b, layer, seq, pos0, count);
    QD_CK(cudaSetDevice(b->e->dev));
    QD_CK(cudaStreamSynchronize(b->e->stream));
    const int NKV = b->e->p.kv_heads;
    std::vector<__half> tmp((size_t)count * kHeadDim);
    for (int which = 0; which < 2; ++which) {
      const __half* cache = which ? vc_of(b, layer) : kc_of(b, layer);
      float* dst = which ? v : k;
      for (int g = 0; g < NKV; ++g) {
        const __half* src = cache + (((size_t)seq * NKV + g) * b->max_seq + pos0) * kHeadDim;
        QD_CK(cudaMemcpy(tmp.data(), src, tmp.size() * 2, cudaMemcpyDeviceToHost));
        for (int r = 0; r < count; ++r)
          for (int c = 0; c < kHeadDim; ++c)
            dst[((size_t)r * NKV + g) * kHeadDim + c] = __half2float(tmp[(size_t)r * kHeadDim + c]);
      }
    }
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_write_kv(qd_batch* b, int layer, int seq, int pos0, int count, const float* k, const float* v) {
  if (!b || !k || !v) return bfail(b, QdError{QD_E_INVALID, "NULL argument"});
  try {
    kv_range_check(b, layer, seq, pos0, count);
    QD_CK(cudaSetDevice(b->e->dev));
    QD_CK(cudaStreamSynchronize(b->e->stream));
    const int NKV = b->e->p.kv_heads;
    std::vector<__half> tmp((size_t)count * kHeadDim);
    for (int which = 0; which < 2; ++which) {
      __half* cache = which ? vc_of(b, layer) : kc_of(b, layer);
      const float* src = which ? v : k;
      for (int g = 0; g < NKV; ++g) {
        for (int r = 0; r < count; ++r)
          for (int c = 0; c < kHeadDim; ++c)
            tmp[(size_t)r * kHeadDim + c] = __float2half_rn(src[((size_t)r * NKV + g) * kHeadDim + c]);
        __half* dst = cache + (((size_t)seq * NKV + g) * b->max_seq + pos0) * kHeadDim;
        QD_CK(cudaMemcpy(dst, tmp.data(), tmp.size() * 2, cudaMemcpyHostToDevice));
      }
    }
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_inject_stall(qd_batch* b) {
  if (!b) return bfail(nullptr, QdError{QD_E_INVALID, "batch is NULL"});
  try {
    qd_engine* e = b->e;
    QD_CK(cudaSetDevice(e->dev));
    static const int one = 1;
    QD_CK(cudaMemcpyAsync(b->errw + 1, &one, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    QD_CK(cudaStreamSynchronize(e->stream));
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_batch_step_kernels(const qd_batch* b) { return b ? step_kernel_count(b) : 0; }

int qd_batch_prefill(qd_batch* b, const int32_t* ids, int n_prompt, int32_t* first_ids) {
  if (!b || !ids) return bfail(b, QdError{QD_E_INVALID, "NULL argument"});
  try {
    if (n_prompt < 1 || n_prompt > b->max_seq) throw QdError{QD_E_RANGE, "n_prompt must be 1..max_seq"};
    const long long T = (long long)b->B * n_prompt;
    for (long long i = 0; i < T; ++i)
      if (ids[i] < 0 || ids[i] >= b->e->p.vocab) throw QdError{QD_E_RANGE, "token id outside the vocabulary"};
    QD_CK(cudaSetDevice(b->e->dev));
    prefill(b, ids, n_prompt, first_ids);
  } catch (const QdError& err) {
    return bfail(b, err);
  }
  return QD_OK;
}

int qd_generate_batch(qd_engine* e, int batch, const int32_t* ids, int n_prompt, int max_new_tokens,
                      int32_t* out_ids) {
  if (!e || !ids || !out_ids) return bfail(nullptr, QdError{QD_E_INVALID, "NULL argument"});
  if (max_new_tokens < 1 || n_prompt < 1) return bfail(nullptr, QdError{QD_E_INVALID, "n_prompt and max_new_tokens must be >= 1"});
  qd_batch* b = nullptr;
  int rc = qd_batch_create(e, batch, n_prompt + max_new_tokens, &b);
  if (rc) return rc;
  std::vector<int32_t> first(batch), rest((size_t)batch * (max_new_tokens - 1));
  rc = qd_batch_prefill(b, ids, n_prompt, first.data());
  if (!rc && max_new_tokens > 1) rc = qd_batch_decode(b, max_new_tokens - 1, rest.data());
  if (!rc)
    for (int i = 0; i < batch; ++i) {
      out_ids[(size_t)i * max_new_tokens] = first[i];
      for (int t = 1; t < max_new_tokens; ++t)
        out_ids[(size_t)i * max_new_tokens + t] = rest[(size_t)(t - 1) * batch + i];
    }
  qd_batch_destroy(b);
  return rc;
}

}  // extern "C"
