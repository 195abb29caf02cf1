// qdecode engine: loads the reference's runtime directory, keeps every weight
// resident in HBM, captures one token (all layers, plus LM head + argmax) as a
// CUDA graph and runs the reference's greedy flow (webgpu-runtime.js:165-214).
#include <algorithm>
#include <chrono>
#include <cstddef>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/qdecode.h"
#include "json.hpp"
#include "gemm_tc.cuh"
#include "internal.cuh"
#include "kernels.cuh"
#include "persist.cuh"

using namespace qd;

namespace {

thread_local std::string t_last_error;

// ---- matvec stage planning and dispatch -------------------------------------
struct StagePlan {
  int kc, nr, grid;
};

// Register budget at 2 CTAs per SM (128 per thread): a lane holds KC * 32
// activations and KC * NR * NW uint4 of weights plus their scales. Combos over
// the budget are not instantiated (except the single-row one, which every
// shape needs); rows beyond one wave of warps go to more CTAs instead. Rows per
// warp grow only while the grid still gives every SM two CTAs (the small
// instances use 50-60 registers, so four fit per SM): the 1024 -> 3072 gate matvec
// took 3.56 us per isolated launch at 4 rows per warp on 96 CTAs, 2.69 us at 2 rows
// on 192 CTAs and 2.47 us at 1 row on 384 CTAs.
constexpr bool stage_ok(int kc, int nr, int nw) {
  return kc * 32 + kc * nr * nw * 5 < 112 || (nr == 1 && nw == 1);
}

StagePlan plan_stage(int rows, int nb, int sms, int nw = 1) {
  if (nb <= 0 || nb > 128) throw QdError{QD_E_INVALID, "q4 matvec: in_size must be 1..4096"};
  StagePlan p;
  p.kc = (nb + 31) / 32;
  const int want = (rows + sms * kWarps - 1) / (sms * kWarps);
  p.nr = 1;
  for (int nr : {2, 4, 8})
    if (p.nr < want && stage_ok(p.kc, nr, nw) && (rows + kWarps * nr - 1) / (kWarps * nr) >= 2 * sms) p.nr = nr;
  p.grid = (rows + kWarps * p.nr - 1) / (kWarps * p.nr);
  return p;
}

template <int PRO, int EPI>
void launch_stage(const StageArgs& a, const StagePlan& p, cudaStream_t s) {
  constexpr int NW = (EPI == kEpiSilu) ? 2 : 1;
#define QD_STAGE_CASE(KC, NR)                                               \
  if constexpr (stage_ok(KC, NR, NW)) {                                     \
    if (p.kc == KC && p.nr == NR) {                                         \
      launch(k_stage<KC, NR, PRO, EPI>, dim3(p.grid), s, a);                \
      return;                                                               \
    }                                                                       \
  }
#define QD_STAGE_KC(KC) QD_STAGE_CASE(KC, 1) QD_STAGE_CASE(KC, 2) QD_STAGE_CASE(KC, 4) QD_STAGE_CASE(KC, 8)
  QD_STAGE_KC(1) QD_STAGE_KC(2) QD_STAGE_KC(3) QD_STAGE_KC(4)
#undef QD_STAGE_KC
#undef QD_STAGE_CASE
  throw QdError{QD_E_INVALID, "q4 matvec: unsupported shape"};
}

void launch_lmhead(const LmArgs& a, int grid, cudaStream_t s) {
  switch (a.H / 256) {
    case 1: launch(k_lmhead<1>, dim3(grid), s, a); return;
    case 2: launch(k_lmhead<2>, dim3(grid), s, a); return;
    case 3: launch(k_lmhead<3>, dim3(grid), s, a); return;
    case 4: launch(k_lmhead<4>, dim3(grid), s, a); return;
  }
  throw QdError{QD_E_INVALID, "LM head: hidden size must be 256, 512, 768 or 1024"};
}

template <typename KVT>
void launch_attn_t(const AttnArgs& a, int group, int splits, cudaStream_t s) {
  const dim3 grid(a.kv_heads, splits);
  switch (group) {
    case 1: launch(k_attn<1, KVT>, grid, s, a); return;
    case 2: launch(k_attn<2, KVT>, grid, s, a); return;
    case 4: launch(k_attn<4, KVT>, grid, s, a); return;
    case 8: launch(k_attn<8, KVT>, grid, s, a); return;
  }
  throw QdError{QD_E_INVALID, "attention: q_heads / kv_heads must be 1, 2, 4 or 8"};
}

void launch_attn(const AttnArgs& a, int kv_dtype, int splits, cudaStream_t s) {
  const int group = a.q_heads / a.kv_heads;
  if (kv_dtype == QD_KV_F32) launch_attn_t<float>(a, group, splits, s);
  else launch_attn_t<__half>(a, group, splits, s);
}

// ---- files ----------------------------------------------------------------
std::vector<char> read_file(const std::string& path, size_t expect) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) throw QdError{QD_E_IO, "cannot open " + path};
  const size_t n = (size_t)f.tellg();
  if (expect && n != expect)
    throw QdError{QD_E_IO, path + ": expected " + std::to_string(expect) + " bytes, found " + std::to_string(n)};
  std::vector<char> buf(n);
  f.seekg(0);
  if (n && !f.read(buf.data(), (std::streamsize)n)) throw QdError{QD_E_IO, "cannot read " + path};
  return buf;
}

float h2f(uint16_t h) {
  __half_raw r;
  r.x = h;
  return __half2float(__half(r));
}

uint16_t f2h(float f) {
  const __half h = __float2half_rn(f);
  return __half_raw(h).x;
}

}  // namespace

namespace qd {
// Lets other translation units of the library report through qd_last_error(NULL).
void set_thread_error(const std::string& msg) { t_last_error = msg; }
}  // namespace qd


namespace {

struct Arena {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  }
};

void set_rows(StageArgs& a, const char* base, int k, bool pairs) {
  const long long rec = rec_bytes(k), nb = k / kBlockCols;
  a.w = base;
  a.s = base + nb * 16;
  a.w_stride = a.s_stride = pairs ? 2 * rec : rec;
  a.w_sub = a.s_sub = pairs ? rec : 0;
}

void enqueue_layer(qd_engine* e, int l, cudaStream_t s, bool embed_at_layer0 = true) {
  const qd_profile& p = e->p;
  const LayerDev& L = e->layers[l];
  const int qsize = p.heads * kHeadDim, kvsize = p.kv_heads * kHeadDim;
  // 1. RMSNorm + fused QKV projection (layer 0 gathers the embedding row on device).
  {
    StageArgs a{};
    set_rows(a, L.qkv, p.hidden, false);
    a.rows = e->rows_qkv; a.nb = p.hidden / kBlockCols; a.k_valid = p.hidden;
    a.src = e->h; a.norm_w = L.n_in; a.eps = p.eps; a.out = e->qkv;
    const StagePlan sp = plan_stage(a.rows, a.nb, e->sms);
    if (l == 0 && embed_at_layer0) {
      a.embed = e->embed; a.tokens = e->tokens; a.st = e->st; a.vocab = p.vocab; a.h_out = e->h;
      a.max_seq = e->opt.max_seq;
      launch_stage<kProEmbed, kEpiStore>(a, sp, s);
    } else {
      launch_stage<kProRms, kEpiStore>(a, sp, s);
    }
  }
  // 2. Head RMSNorm + RoPE + KV append + split-KV attention.
  {
    AttnArgs a{};
    a.q_in = e->qkv; a.k_in = e->qkv + qsize; a.v_in = e->qkv + qsize + kvsize;
    a.norm_q = L.n_q; a.norm_k = L.n_k; a.eps = p.eps;
    a.cos_t = e->cos_t; a.sin_t = e->sin_t; a.row_stride = e->opt.rope_row_stride;
    a.k_cache = L.kc; a.v_cache = L.vc; a.st = e->st; a.seq_len = 0; a.max_seq = e->opt.max_seq;
    a.q_heads = p.heads; a.kv_heads = p.kv_heads; a.scale = 1.0f / std::sqrt((float)kHeadDim);
    a.raw_q = 0; a.part_ml = e->part_ml; a.part_o = e->part_o;
    launch_attn(a, e->opt.kv_dtype, e->splits, s);
  }
  // 3. Split combine + O projection + residual.
  {
    StageArgs a{};
    set_rows(a, L.o, qsize, false);
    a.rows = p.hidden; a.nb = qsize / kBlockCols; a.k_valid = qsize;
    a.res = e->h; a.out = e->h_attn;
    a.part_ml = e->part_ml; a.part_o = e->part_o; a.splits = e->splits; a.q_heads = p.heads;
    launch_stage<kProCombine, kEpiResidual>(a, plan_stage(a.rows, a.nb, e->sms), s);
  }
  // 4. Post-attention RMSNorm + gate/up + silu_mul.
  {
    StageArgs a{};
    set_rows(a, L.gu, p.hidden, true);
    a.rows = p.intermediate; a.nb = p.hidden / kBlockCols; a.k_valid = p.hidden;
    a.src = e->h_attn; a.norm_w = L.n_post; a.eps = p.eps; a.out = e->act;
    launch_stage<kProRms, kEpiSilu>(a, plan_stage(a.rows, a.nb, e->sms, 2), s);
  }
  // 5. Down projection + residual into the stream state.
  {
    StageArgs a{};
    set_rows(a, L.d, p.intermediate, false);
    a.rows = p.hidden; a.nb = p.intermediate / kBlockCols; a.k_valid = p.intermediate;
    a.src = e->act; a.res = e->h_attn; a.out = e->h;
    launch_stage<kProPlain, kEpiResidual>(a, plan_stage(a.rows, a.nb, e->sms), s);
  }
}

void enqueue_lmhead(qd_engine* e, cudaStream_t s) {
  LmArgs a{};
  a.h = e->h; a.norm_w = e->final_norm; a.eps = e->p.eps;
  a.table = reinterpret_cast<const uint4*>(e->embed); a.vocab = e->p.vocab; a.H = e->p.hidden;
  a.logits = e->logits; a.part_v = e->lm_pv; a.part_i = e->lm_pi; a.counter = e->lm_counter;
  a.result = e->result; a.st = e->st; a.tokens = e->tokens; a.out_dev = e->out_dev;
  a.out_host = e->out_host_dev; a.max_seq = e->opt.max_seq;
  launch_lmhead(a, e->lm_grid, s);
}

template <int G, typename KVT>
void launch_persist_t(qd_engine* e, const PArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(e->sms);
  cfg.blockDim = dim3(kPT);
  cfg.dynamicSmemBytes = e->persist_smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they exchange data
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QD_CK(cudaLaunchKernelEx(&cfg, k_decode_persistent<G, KVT>, a));
}

PArgs persist_args(qd_engine* e, int head) {
  const bool with_head = head != kHeadNone;
  const qd_profile& p = e->p;
  PArgs a{};
  a.layers = e->d_players;
  a.L = p.layers; a.H = p.hidden; a.I = p.intermediate; a.NH = p.heads; a.NKV = p.kv_heads;
  a.vocab = p.vocab; a.max_seq = e->opt.max_seq; a.row_stride = e->opt.rope_row_stride;
  a.eps = p.eps; a.scale = 1.0f / std::sqrt((float)kHeadDim);
  a.embed = e->embed; a.cos_t = e->cos_t; a.sin_t = e->sin_t; a.final_norm = e->final_norm;
  a.xb = e->xbuf; a.xstride = e->xstride; a.st = e->st;
  a.tokens = e->tokens; a.out_dev = e->out_dev; a.out_host = e->out_host_dev;
  a.logits = e->logits; a.part_v = e->lm_pv; a.part_i = e->lm_pi; a.counter = e->lm_counter;
  a.with_head = with_head ? 1 : 0; a.lm_rows = e->lm_rows; a.timeline = e->timeline;
  a.rec_h = rec_bytes(p.hidden); a.rec_q = rec_bytes(p.heads * kHeadDim); a.rec_i = rec_bytes(p.intermediate);
  a.OS = e->os; a.rec_og = e->rec_og; a.oslice_rows = e->oslice_rows; a.oacc = e->oacc; a.n_mlp = e->n_mlp;
  a.pruned = head == kHeadArgmax && e->lm_q8 ? 1 : 0;
  a.lm_q8 = reinterpret_cast<const uint2*>(e->lm_q8); a.lm_scale = e->lm_scale; a.lm_bound = e->lm_bound;
  return a;
}

void launch_persist(qd_engine* e, int head, cudaStream_t s) {
  const PArgs a = persist_args(e, head);
  const int group = e->p.heads / e->p.kv_heads;
  if (e->opt.kv_dtype == QD_KV_F32) {
    if (group == 1) launch_persist_t<1, float>(e, a, s); else launch_persist_t<2, float>(e, a, s);
  } else {
    if (group == 1) launch_persist_t<1, __half>(e, a, s); else launch_persist_t<2, __half>(e, a, s);
  }
}

template <int G, typename KVT>
cudaError_t prepare_persist_t(size_t smem, int* blocks) {
  cudaError_t rc = cudaFuncSetAttribute(k_decode_persistent<G, KVT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (rc != cudaSuccess) return rc;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, k_decode_persistent<G, KVT>, kPT, smem);
}

// Packs, for one layer, the O-projection slices of the fused attention stage: slice
// (g, s) holds rows [H s / OS, H (s+1) / OS) restricted to KV head g's G * 128 input
// columns, as row records (G * 4 q4 blocks, their f16 scales, padding to 16 bytes).
__global__ void k_pack_oslices(const char* o, char* dst, int H, int NKV, int OS, int G, long long rec_q, int nbq,
                               long long rec_og, long long rows_max) {
  const int nbg = G * 4;  // 32-column blocks of one KV head's columns
  const long long n = (long long)NKV * OS * rows_max;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int slice = (int)(i / rows_max), rl = (int)(i % rows_max);
    const int g = slice / OS, s = slice % OS;
    const int lo = (int)((long long)H * s / OS), hi = (int)((long long)H * (s + 1) / OS);
    char* out = dst + i * rec_og;
    for (long long b = 0; b < rec_og; ++b) out[b] = 0;
    if (lo + rl >= hi) continue;
    const char* row = o + (long long)(lo + rl) * rec_q;
    for (int b = 0; b < nbg * 16; ++b) out[b] = row[(long long)g * nbg * 16 + b];
    for (int b = 0; b < nbg * 2; ++b) out[nbg * 16 + b] = row[(long long)nbq * 16 + (long long)g * nbg * 2 + b];
  }
}

// Packs, for one layer, the down-projection slices of the fused MLP stage: CTA c of g
// owns intermediate columns [I c / g, I (c+1) / g) (at most kDMaxCols, so within two
// q4 blocks); its slice holds, per hidden row, those columns' nibbles from nibble 0
// (unused ones 8) and the f16 scales of the first block and the next one.
__global__ void k_pack_dslices(const char* d, char* dst, int H, int I, int g, long long rec_i) {
  const int nb = I / kBlockCols;
  const long long n = (long long)g * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i / H), r = (int)(i % H);
    const int lo = (int)((unsigned)I * (unsigned)c / (unsigned)g), hi = (int)((unsigned)I * (unsigned)(c + 1) / (unsigned)g);
    const unsigned char* row = reinterpret_cast<const unsigned char*>(d + (long long)r * rec_i);
    const unsigned short* scl = reinterpret_cast<const unsigned short*>(row + (long long)nb * 16);
    uint32_t w[3] = {0x88888888u, 0x88888888u, 0x88888888u};
    for (int j = 0; j < hi - lo && j < kDMaxCols; ++j) {
      const int col = lo + j, blk = col / kBlockCols, cc = col % kBlockCols;
      const uint32_t nib = (row[blk * 16 + cc / 2] >> (4 * (cc & 1))) & 15u;
      w[j >> 3] = (w[j >> 3] & ~(15u << (4 * (j & 7)))) | (nib << (4 * (j & 7)));
    }
    const int b0 = lo / kBlockCols;
    const uint32_t sa = hi > lo ? scl[b0] : 0u, sb = hi > lo && b0 + 1 < nb ? scl[b0 + 1] : 0u;
    reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[0], w[1], w[2], sa | (sb << 16));
  }
}

// The LM head table as int8 for the argmax-only head: row r holds q = rint(E / s_r),
// s_r = max|E_r| / 127, stored biased (q + 128), and a bound coefficient b_r such that
// every fp32 evaluation of the f16 logit E_r . x and of the int8 logit s_r (q . x)
// (dots of depth <= H) differ by at most b_r ||x||_1: the largest elementwise
// |E - s q| (measured), the rounding of both dots ((H + 2) 2^-24 each, relative to
// max|E_r| ||x||_1) and of this arithmetic. Rows with a non-finite entry get b_r = inf
// (always recomputed exactly).
__global__ void k_prep_lm_q8(const __half* E, int V, int H, uint8_t* q8, float* scale, float* bound) {
  const int lane = threadIdx.x & 31, wpb = blockDim.x / 32;
  const float gamma = (float)(H + 2) * 5.9604645e-08f * 1.01f;
  for (long long r = (long long)blockIdx.x * wpb + (threadIdx.x >> 5); r < V; r += (long long)gridDim.x * wpb) {
    const __half* row = E + r * H;
    float m = 0.0f;
    bool fin = true;
    for (int j = lane; j < H; j += 32) {
      const float v = __half2float(row[j]);
      fin = fin && isfinite(v);
      m = fmaxf(m, fabsf(v));
    }
    m = warp_max(m);
    fin = __all_sync(0xffffffffu, fin);
    const float sc = (fin && m > 0.0f) ? m / 127.0f : 0.0f;
    const float inv = sc > 0.0f ? 127.0f / m : 0.0f;
    float err = 0.0f;
    for (int j = lane; j < H; j += 32) {
      const float v = __half2float(row[j]);
      const float q = fminf(fmaxf(rintf(v * inv), -127.0f), 127.0f);
      q8[r * H + j] = (uint8_t)(int)(q + 128.0f);
      if (fin) err = fmaxf(err, fabsf(v - sc * q));
    }
    err = warp_max(err);
    if (lane == 0) {
      scale[r] = sc;
      bound[r] = fin ? (err + m * (2.1f * gamma + 4.8e-7f)) * (1.0f + 3.0f * gamma) : INFINITY;
    }
  }
}

// The final hidden state from the persistent kernel's exchange words (value bits in the low half).
__global__ void k_words_to_f32(const unsigned long long* w, float* h, int n) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) h[i] = __uint_as_float((uint32_t)w[i]);
  pdl_trigger();
}

// Decide whether the persistent kernel fits this shape and device; set it up if so.
void setup_persist(qd_engine* e) {
  const qd_profile& p = e->p;
  const int G = p.heads / p.kv_heads, H = p.hidden, I = p.intermediate, QS = p.heads * kHeadDim;
  const int R = QS + 2 * p.kv_heads * kHeadDim, g = e->sms;
  auto per_cta = [g](long long n, long long bytes) { return (n + g - 1) / g * bytes; };
  int coop = 0, optin = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, e->dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, e->dev);
  const long long rec_h = rec_bytes(H), rec_q = rec_bytes(QS), rec_i = rec_bytes(I);
  // attention CTAs per KV head: each owns H / OS rows of the O projection
  const int OS = std::min(16, g / std::max(1, p.kv_heads));
  const long long rec_og = rec_bytes(G * kHeadDim), oslice_rows = OS > 0 ? (H + OS - 1) / OS : 0;
  // intermediate columns per CTA (gate/up pairs, then their down partial)
  const long long cols_i = (I + g - 1) / g;
  bool ok = e->opt.persistent && coop && G <= 2 && H <= 1024 && QS <= 2048 && I <= 3072 && p.kv_heads <= g &&
            cols_i <= kDMaxCols && 2 * cols_i <= kMaxRes / 2 && (long long)H * kDRec <= kSlotBytes &&
            OS >= 1 && oslice_rows <= kMaxRes && oslice_rows * rec_og <= kSlotBytes &&
            per_cta(R, rec_h) <= kSlotBytes && per_cta(I, 2 * rec_h) <= kSlotBytes &&
            2LL * H <= kSlotBytes;
  if (!ok) return;
  const int maxk = std::max(std::max(H, QS), I);
  const long long xs_floats = std::max<long long>(maxk, (long long)kPW * G * kHeadDim);
  const long long misc_floats =
      std::max<long long>((G + 2) * kHeadDim + G * kHeadDim + 2 * kHeadDim + 2 * kPW * G + G * 64, 2 * kPW);
  const size_t smem = (size_t)kSlots * kSlotBytes + (size_t)(xs_floats + 2 * H) * 4 + kSlots * 8 + kPW * 4 + 16 +
                      (size_t)(kMaxRes + misc_floats) * 4;
  // per-CTA row counts must fit the stage result buffer
  if (per_cta(R, 1) > kMaxRes || 2 * per_cta(I, 1) > kMaxRes || 3 * per_cta(H, 1) > kMaxRes) return;
  if ((long long)smem > optin) return;
  int blocks = 0;
  const cudaError_t rc = e->opt.kv_dtype == QD_KV_F32
                             ? (G == 1 ? prepare_persist_t<1, float>(smem, &blocks) : prepare_persist_t<2, float>(smem, &blocks))
                             : (G == 1 ? prepare_persist_t<1, __half>(smem, &blocks) : prepare_persist_t<2, __half>(smem, &blocks));
  if (rc != cudaSuccess || blocks < 1) {
    cudaGetLastError();
    return;
  }
  e->persist_smem = smem;
  e->lm_rows = kSlotBytes / (2 * H);
  e->xstride = (long long)H + R + QS + H + I;
  const size_t xbytes = (size_t)(p.layers + 1) * e->xstride * 8;
  if (cudaMalloc(&e->xbuf, xbytes) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate exchange buffers"};
  QD_CK(cudaMemset(e->xbuf, 0, xbytes));
  // O slices of the fused attention stage, and their double-buffered sums
  e->os = OS;
  e->rec_og = rec_og;
  e->oslice_rows = oslice_rows;
  const long long slices_per_layer = (long long)p.kv_heads * OS * oslice_rows * rec_og;
  if (cudaMalloc(&e->oslices, (size_t)slices_per_layer * p.layers) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate the packed O slices"};
  for (int l = 0; l < p.layers; ++l)
    k_pack_oslices<<<64, 256, 0, e->stream>>>(e->layers[l].o, e->oslices + (size_t)slices_per_layer * l, H,
                                              p.kv_heads, OS, G, rec_q, QS / kBlockCols, rec_og, oslice_rows);
  QD_CK(cudaGetLastError());
  QD_CK(cudaStreamSynchronize(e->stream));
  // down slices of the fused MLP stage (one per CTA of the launch)
  e->n_mlp = std::min(g, I);
  const long long dslice_per_layer = (long long)g * H * kDRec;
  if (cudaMalloc(&e->dslices, (size_t)dslice_per_layer * p.layers) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate the packed down slices"};
  for (int l = 0; l < p.layers; ++l)
    k_pack_dslices<<<148, 256, 0, e->stream>>>(e->layers[l].d, e->dslices + (size_t)dslice_per_layer * l, H, I, g,
                                               rec_i);
  QD_CK(cudaGetLastError());
  QD_CK(cudaStreamSynchronize(e->stream));
  const size_t acc_bytes = (size_t)2 * p.layers * 2 * H * 8;
  if (cudaMalloc(&e->oacc, acc_bytes) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate the O / down sums"};
  QD_CK(cudaMemset(e->oacc, 0, acc_bytes));
  std::vector<PLayer> pl(p.layers);
  for (int l = 0; l < p.layers; ++l) {
    const LayerDev& L = e->layers[l];
    pl[l] = PLayer{L.qkv, L.o, L.gu, L.d, L.n_in, L.n_q, L.n_k, L.n_post, L.kc, L.vc,
                   e->oslices + (size_t)slices_per_layer * l, e->dslices + (size_t)dslice_per_layer * l};
  }
  if (cudaMalloc(&e->d_players, sizeof(PLayer) * p.layers) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate the layer table"};
  QD_CK(cudaMemcpy(e->d_players, pl.data(), sizeof(PLayer) * p.layers, cudaMemcpyHostToDevice));
  // the int8 LM head table of the argmax-only head
  {
    const size_t tb = (size_t)p.vocab * H;
    if (cudaMalloc(&e->lm_q8, tb) != cudaSuccess || cudaMalloc(&e->lm_scale, (size_t)p.vocab * 4) != cudaSuccess ||
        cudaMalloc(&e->lm_bound, (size_t)p.vocab * 4) != cudaSuccess)
      throw QdError{QD_E_NOMEM, "cannot allocate the int8 LM head table"};
    k_prep_lm_q8<<<4 * e->sms, 256, 0, e->stream>>>(e->embed, p.vocab, H, e->lm_q8, e->lm_scale, e->lm_bound);
    QD_CK(cudaGetLastError());
    QD_CK(cudaStreamSynchronize(e->stream));
  }
  if (e->opt.timeline) {
    const size_t tb = (size_t)e->sms * timeline_events(p.layers) * 8;
    if (cudaMalloc(&e->timeline, tb) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate the timeline"};
    QD_CK(cudaMemset(e->timeline, 0, tb));
  }
  e->persist = true;
}

void enqueue_token(qd_engine* e, int head, cudaStream_t s) {
  if (e->persist) {
    launch_persist(e, head, s);
    return;
  }
  for (int l = 0; l < e->p.layers; ++l) enqueue_layer(e, l, s);
  if (head != kHeadNone) enqueue_lmhead(e, s);
  else launch(k_advance, dim3(1), s, e->st);
}

cudaGraphExec_t capture(qd_engine* e, int head) {
  cudaGraph_t g = nullptr;
  QD_CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  try {
    enqueue_token(e, head, e->stream);
  } catch (...) {
    cudaStreamEndCapture(e->stream, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  QD_CK(cudaStreamEndCapture(e->stream, &g));
  cudaGraphExec_t ex = nullptr;
  const cudaError_t rc = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  QD_CK(rc);
  return ex;
}

// One token: kHeadNone (layers only), kHeadFull (logits + argmax) or kHeadArgmax
// (the argmax only, where the persistent kernel prunes the LM head; the logits are
// then recomputed from the final hidden state if asked for).
void run_token(qd_engine* e, int head) {
  if (e->opt.use_graph) {
    cudaGraphExec_t g = head == kHeadNone ? e->g_layers : head == kHeadFull ? e->g_full : e->g_argmax;
    QD_CK(cudaGraphLaunch(g, e->stream));
  } else {
    enqueue_token(e, head, e->stream);
  }
  if (head != kHeadNone) e->logits_stale = head == kHeadArgmax && e->persist && e->lm_q8;
}

int dims_of(const Json& entry, size_t i) { return (int)entry.at("dims").at(i).as_int(); }

// Host-only half of engine creation: parse and validate the manifest against
// the shapes the kernels support (no CUDA call, so it is testable without a GPU).
Json parse_manifest(qd_engine* e, const std::string& dir) {
  std::string text;
  {
    auto buf = read_file(dir + "/manifest.json", 0);
    text.assign(buf.begin(), buf.end());
  }
  Json m;
  try {
    m = parse_json(text);
  } catch (const std::exception& ex) {
    throw QdError{QD_E_IO, ex.what()};
  }
  qd_profile& p = e->p;
  try {
    p.hidden = (int)m.at("hiddenSize").as_int();
    p.intermediate = (int)m.at("intermediateSize").as_int();
    p.heads = (int)m.at("attentionHeads").as_int();
    p.kv_heads = (int)m.at("kvHeads").as_int();
    p.head_dim = (int)m.at("headDim").as_int();
    p.layers = (int)m.at("layers").size();
    const Json& emb = m.at("shared").at("embedTokens");
    p.vocab = dims_of(emb, 0);
    if (dims_of(emb, 1) != p.hidden) throw QdError{QD_E_IO, "embed_tokens dims do not match hiddenSize"};
    const Json& cs = m.at("shared").at("cosCache");
    p.rope_rows = dims_of(cs, 0);
    if (dims_of(cs, 1) != p.head_dim / 2) throw QdError{QD_E_IO, "cos_cache width must be headDim/2"};
    const Json* eps = m.find("normEpsilon");
    p.eps = eps ? (float)eps->as_num() : 1e-6f;  // qwenProfile.normEpsilon (src/model/qwen3-0.6b.js:13)
  } catch (const std::runtime_error& ex) {
    throw QdError{QD_E_IO, ex.what()};
  }
  if (p.head_dim != kHeadDim) throw QdError{QD_E_INVALID, "head_dim must be 128"};
  if (p.hidden % 256 || p.hidden > 1024) throw QdError{QD_E_INVALID, "hidden size must be a multiple of 256, at most 1024"};
  if (p.intermediate % 32 || p.intermediate > 4096) throw QdError{QD_E_INVALID, "intermediate size must be a multiple of 32, at most 4096"};
  if (p.kv_heads <= 0 || p.heads % p.kv_heads) throw QdError{QD_E_INVALID, "heads must be a multiple of kv_heads"};
  const int group = p.heads / p.kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8) throw QdError{QD_E_INVALID, "heads / kv_heads must be 1, 2, 4 or 8"};
  if (p.heads * kHeadDim > 4096) throw QdError{QD_E_INVALID, "heads * head_dim must be at most 4096"};
  if (p.layers <= 0 || p.vocab <= 0) throw QdError{QD_E_IO, "manifest has no layers or no vocabulary"};

  qd_options& o = e->opt;
  if (o.rope_row_stride <= 0) o.rope_row_stride = p.head_dim;  // rope.wgsl:27 with headDim
  if (o.rope_row_stride % 4) throw QdError{QD_E_INVALID, "rope_row_stride must be a multiple of 4"};
  if (o.max_seq <= 0) throw QdError{QD_E_INVALID, "max_seq must be positive"};
  const long long last = (long long)(o.max_seq - 1) * o.rope_row_stride + p.head_dim / 2;
  if (last > (long long)p.rope_rows * (p.head_dim / 2))
    throw QdError{QD_E_RANGE, "max_seq exceeds the RoPE table (positions * row_stride must stay inside cos_cache)"};

  // Every projection must match the model shape (extract-qwen-runtime-assets.mjs:94-100).
  static const char* kProjNames[7] = {"q", "k", "v", "o", "gate", "up", "down"};
  const int QS0 = p.heads * kHeadDim, KV0 = p.kv_heads * kHeadDim;
  const int out_sz[7] = {QS0, KV0, KV0, p.hidden, p.intermediate, p.intermediate, p.hidden};
  const int in_sz[7] = {p.hidden, p.hidden, p.hidden, QS0, p.hidden, p.hidden, p.intermediate};
  try {
    for (int l = 0; l < p.layers; ++l)
      for (int j = 0; j < 7; ++j) {
        const Json& d = m.at("layers").at(l).at("projections").at(kProjNames[j]).at("matmulNBits");
        const int outS = (int)d.at("outSize").as_int(), inS = (int)d.at("inSize").as_int();
        const int bpr = (int)d.at("blocksPerRow").as_int(), bs = (int)d.at("blockSize").as_int();
        if (outS != out_sz[j] || inS != in_sz[j] || bs != kBlockCols || bpr * bs != inS)
          throw QdError{QD_E_IO, "layer " + std::to_string(l) + " " + kProjNames[j] +
                                     ": matmulNBits dims do not match the model shape (block size must be 32)"};
      }
  } catch (const std::runtime_error& ex) {
    throw QdError{QD_E_IO, ex.what()};
  }
  return m;
}

void load_engine(qd_engine* e, const std::string& dir, const Json& m) {
  const qd_profile& p = e->p;
  const qd_options& o = e->opt;
  const int H = p.hidden, I = p.intermediate, QS = p.heads * kHeadDim, KV = p.kv_heads * kHeadDim;
  e->rows_qkv = QS + 2 * KV;
  const int half = p.head_dim / 2;

  // Offsets in one weight arena.
  Arena ar;
  const size_t o_embed = ar.take((size_t)p.vocab * H * 2);
  const size_t o_cos = ar.take((size_t)p.rope_rows * half * 4);
  const size_t o_sin = ar.take((size_t)p.rope_rows * half * 4);
  const size_t o_fn = ar.take((size_t)H * 4);
  struct LOff { size_t qkv, o, gu, d, n_in, n_q, n_k, n_post; };
  const long long rec_h = rec_bytes(H), rec_q = rec_bytes(QS), rec_i = rec_bytes(I);
  std::vector<LOff> lo(p.layers);
  for (int l = 0; l < p.layers; ++l) {
    lo[l].qkv = ar.take((size_t)e->rows_qkv * rec_h);
    lo[l].o = ar.take((size_t)H * rec_q);
    lo[l].gu = ar.take((size_t)2 * I * rec_h);
    lo[l].d = ar.take((size_t)H * rec_i);
    lo[l].n_in = ar.take((size_t)H * 4);
    lo[l].n_q = ar.take(kHeadDim * 4);
    lo[l].n_k = ar.take(kHeadDim * 4);
    lo[l].n_post = ar.take((size_t)H * 4);
  }
  if (cudaMalloc(&e->blob, ar.off) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate " + std::to_string(ar.off) + " bytes of weights"};
  char* base = static_cast<char*>(e->blob);
  auto up = [&](size_t off, const void* src, size_t bytes) {
    QD_CK(cudaMemcpy(base + off, src, bytes, cudaMemcpyHostToDevice));
  };
  auto f16_to_f32 = [&](const std::vector<char>& b) {
    std::vector<float> out(b.size() / 2);
    const uint16_t* s = reinterpret_cast<const uint16_t*>(b.data());
    for (size_t i = 0; i < out.size(); ++i) out[i] = h2f(s[i]);
    return out;
  };
  auto file = [&](const Json& entry) { return dir + "/" + entry.at("file").as_str(); };

  try {
    {
      auto b = read_file(file(m.at("shared").at("embedTokens")), (size_t)p.vocab * H * 2);
      up(o_embed, b.data(), b.size());
    }
    for (int which = 0; which < 2; ++which) {
      const Json& entry = m.at("shared").at(which ? "sinCache" : "cosCache");
      auto v = f16_to_f32(read_file(file(entry), (size_t)p.rope_rows * half * 2));
      up(which ? o_sin : o_cos, v.data(), v.size() * 4);
    }
    {
      auto v = f16_to_f32(read_file(file(m.at("finalNorm")), (size_t)H * 2));
      up(o_fn, v.data(), v.size() * 4);
    }
    static const char* kProj[7] = {"q", "k", "v", "o", "gate", "up", "down"};
    for (int l = 0; l < p.layers; ++l) {
      const Json& le = m.at("layers").at(l);
      const Json& norms = le.at("norms");
      auto nv = [&](const char* k, size_t n, size_t off) {
        auto v = f16_to_f32(read_file(file(norms.at(k)), n * 2));
        up(off, v.data(), v.size() * 4);
      };
      nv("input", H, lo[l].n_in);
      nv("q", kHeadDim, lo[l].n_q);
      nv("k", kHeadDim, lo[l].n_k);
      nv("postAttention", H, lo[l].n_post);
      // Row offsets of each projection inside the fused device matrices.
      const int out_sz[7] = {QS, KV, KV, H, I, I, H};
      const int in_sz[7] = {H, H, H, QS, H, H, I};
      // Record placement: (first record, record stride, offset inside the record).
      const long long rec[7] = {rec_h, rec_h, rec_h, rec_q, rec_h, rec_h, rec_i};
      const long long stride[7] = {rec_h, rec_h, rec_h, rec_q, 2 * rec_h, 2 * rec_h, rec_i};
      const long long first[7] = {0, (long long)QS * rec_h, (long long)(QS + KV) * rec_h, 0, 0, rec_h, 0};
      // Host staging of the four record matrices of this layer.
      const size_t m_bytes[4] = {(size_t)e->rows_qkv * rec_h, (size_t)H * rec_q, (size_t)2 * I * rec_h,
                                 (size_t)H * rec_i};
      const int m_of[7] = {0, 0, 0, 1, 2, 2, 3};
      std::vector<char> mats[4];
      for (int k = 0; k < 4; ++k) mats[k].assign(m_bytes[k], 0);
      for (int j = 0; j < 7; ++j) {
        const Json& pj = le.at("projections").at(kProj[j]);
        const int outS = out_sz[j], bpr = in_sz[j] / kBlockCols;  // validated by parse_manifest
        auto wb = read_file(file(pj.at("weight")), (size_t)outS * bpr * 16);
        auto sb = read_file(file(pj.at("scales")), (size_t)outS * bpr * 4);
        const float* sf = reinterpret_cast<const float*>(sb.data());
        char* dst0 = mats[m_of[j]].data() + first[j];
        for (int r = 0; r < outS; ++r) {
          char* dst = dst0 + (size_t)r * stride[j];
          std::memcpy(dst, wb.data() + (size_t)r * bpr * 16, (size_t)bpr * 16);
          uint16_t* sc = reinterpret_cast<uint16_t*>(dst + (size_t)bpr * 16);
          for (int b = 0; b < bpr; ++b) {
            const float v = sf[(size_t)r * bpr + b];
            sc[b] = f2h(v);
            const float back = h2f(sc[b]);
            if (!(back == v) && !(std::isnan(back) && std::isnan(v)))
              throw QdError{QD_E_IO, std::string("layer ") + std::to_string(l) + " " + kProj[j] +
                                         ": a block scale is not an f16 value (the q4f16 format stores f16 scales)"};
          }
        }
        (void)rec;
      }
      const size_t m_off[4] = {lo[l].qkv, lo[l].o, lo[l].gu, lo[l].d};
      for (int k = 0; k < 4; ++k) up(m_off[k], mats[k].data(), m_bytes[k]);
    }
  } catch (const std::runtime_error& ex) {
    throw QdError{QD_E_IO, ex.what()};
  }

  e->embed = reinterpret_cast<__half*>(base + o_embed);
  e->cos_t = reinterpret_cast<float*>(base + o_cos);
  e->sin_t = reinterpret_cast<float*>(base + o_sin);
  e->final_norm = reinterpret_cast<float*>(base + o_fn);
  e->layers.resize(p.layers);

  // KV cache [layer][pos][kv_head][128] for K and V.
  const size_t kv_elem = o.kv_dtype == QD_KV_F32 ? 4 : 2;
  const size_t kv_layer = (size_t)o.max_seq * KV * kv_elem;
  if (cudaMalloc(&e->kv, kv_layer * 2 * p.layers) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate the KV cache"};
  QD_CK(cudaMemset(e->kv, 0, kv_layer * 2 * p.layers));
  for (int l = 0; l < p.layers; ++l) {
    LayerDev& L = e->layers[l];
    L.qkv = base + lo[l].qkv;
    L.o = base + lo[l].o;
    L.gu = base + lo[l].gu;
    L.d = base + lo[l].d;
    L.n_in = reinterpret_cast<const float*>(base + lo[l].n_in);
    L.n_q = reinterpret_cast<const float*>(base + lo[l].n_q);
    L.n_k = reinterpret_cast<const float*>(base + lo[l].n_k);
    L.n_post = reinterpret_cast<const float*>(base + lo[l].n_post);
    L.kc = static_cast<char*>(e->kv) + (size_t)(2 * l) * kv_layer;
    L.vc = static_cast<char*>(e->kv) + (size_t)(2 * l + 1) * kv_layer;
  }

  // Activations, partials and per-engine state.
  e->splits = (o.max_seq + kAttnChunk - 1) / kAttnChunk;
  e->lm_grid = e->sms;
  Arena sa;
  const size_t s_h = sa.take(H * 4), s_ha = sa.take(H * 4), s_qkv = sa.take((size_t)e->rows_qkv * 4);
  const size_t s_act = sa.take((size_t)I * 4), s_log = sa.take((size_t)p.vocab * 4);
  const size_t s_pml = sa.take((size_t)e->splits * p.heads * 8);
  const size_t s_po = sa.take((size_t)e->splits * p.heads * kHeadDim * 4);
  const size_t s_st = sa.take(sizeof(DevState));
  const size_t s_tok = sa.take((size_t)(o.max_seq + 1) * 4), s_out = sa.take((size_t)(o.max_seq + 1) * 4);
  const size_t s_res = sa.take(8), s_pv = sa.take((size_t)e->lm_grid * 4), s_pi = sa.take((size_t)e->lm_grid * 4);
  const size_t s_ctr = sa.take(4);
  if (cudaMalloc(&e->scratch, sa.off) != cudaSuccess) throw QdError{QD_E_NOMEM, "cannot allocate activations"};
  QD_CK(cudaMemset(e->scratch, 0, sa.off));
  char* sb = static_cast<char*>(e->scratch);
  e->h = reinterpret_cast<float*>(sb + s_h);
  e->h_attn = reinterpret_cast<float*>(sb + s_ha);
  e->qkv = reinterpret_cast<float*>(sb + s_qkv);
  e->act = reinterpret_cast<float*>(sb + s_act);
  e->logits = reinterpret_cast<float*>(sb + s_log);
  e->part_ml = reinterpret_cast<float2*>(sb + s_pml);
  e->part_o = reinterpret_cast<float*>(sb + s_po);
  e->st = reinterpret_cast<DevState*>(sb + s_st);
  e->tokens = reinterpret_cast<int*>(sb + s_tok);
  e->out_dev = reinterpret_cast<int*>(sb + s_out);
  e->result = reinterpret_cast<uint32_t*>(sb + s_res);
  e->lm_pv = reinterpret_cast<float*>(sb + s_pv);
  e->lm_pi = reinterpret_cast<uint32_t*>(sb + s_pi);
  e->lm_counter = reinterpret_cast<unsigned*>(sb + s_ctr);

  if (cudaHostAlloc(reinterpret_cast<void**>(&e->out_host), (size_t)(o.max_seq + 1) * 4, cudaHostAllocMapped) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate mapped host memory"};
  QD_CK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->out_host_dev), e->out_host, 0));
  if (cudaHostAlloc(reinterpret_cast<void**>(&e->pinned_ids), (size_t)(o.max_seq + 1) * 4, cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void**>(&e->pinned_state), sizeof(DevState), cudaHostAllocDefault) != cudaSuccess)
    throw QdError{QD_E_NOMEM, "cannot allocate pinned host memory"};
  setup_persist(e);
  QD_CK(cudaEventCreateWithFlags(&e->ev[0], cudaEventDisableTiming));
  QD_CK(cudaEventCreateWithFlags(&e->ev[1], cudaEventDisableTiming));
  if (o.use_graph) {
    e->g_layers = capture(e, kHeadNone);
    e->g_full = capture(e, kHeadFull);
    e->g_argmax = capture(e, kHeadArgmax);
  }
  QD_CK(cudaStreamSynchronize(e->stream));
}

void free_engine(qd_engine* e) {
  if (!e) return;
  if (!e->own_stream) {  // failed before any CUDA resource was created
    delete e;
    return;
  }
  cudaSetDevice(e->dev);
  if (e->stream) cudaStreamSynchronize(e->stream);
  prompt_pass_free(e);
  if (e->g_layers) cudaGraphExecDestroy(e->g_layers);
  if (e->g_full) cudaGraphExecDestroy(e->g_full);
  if (e->g_argmax) cudaGraphExecDestroy(e->g_argmax);
  if (e->lm_q8) cudaFree(e->lm_q8);
  if (e->lm_scale) cudaFree(e->lm_scale);
  if (e->lm_bound) cudaFree(e->lm_bound);
  for (auto& ev : e->ev)
    if (ev) cudaEventDestroy(ev);
  if (e->blob) cudaFree(e->blob);
  if (e->kv) cudaFree(e->kv);
  if (e->scratch) cudaFree(e->scratch);
  if (e->xbuf) cudaFree(e->xbuf);
  if (e->d_players) cudaFree(e->d_players);
  if (e->oslices) cudaFree(e->oslices);
  if (e->dslices) cudaFree(e->dslices);
  if (e->sample_ws) cudaFree(e->sample_ws);
  if (e->oacc) cudaFree(e->oacc);
  if (e->timeline) cudaFree(e->timeline);
  if (e->out_host) cudaFreeHost(e->out_host);
  if (e->pinned_ids) cudaFreeHost(e->pinned_ids);
  if (e->pinned_state) cudaFreeHost(e->pinned_state);
  if (e->stream != e->own_stream) cudaStreamSynchronize(e->stream);
  cudaStreamDestroy(e->own_stream);
  delete e;
}

int fail(qd_engine* e, const QdError& err) {
  if (e) e->err = err.msg;
  t_last_error = err.msg;
  return err.code;
}

void set_state(qd_engine* e, int pos, int max_new, int step = 0) {
  e->pinned_state->pos = pos;
  e->pinned_state->step = step;
  e->pinned_state->max_new = max_new;
  e->pinned_state->err = 0;
  // pos, step, max_new, err only: epoch and abort belong to the device
  QD_CK(cudaMemcpyAsync(e->st, e->pinned_state, offsetof(DevState, epoch), cudaMemcpyHostToDevice, e->stream));
}

void check_state(qd_engine* e) {
  if (e->pbatch_used) {  // the prompt pass's own status word first
    e->pbatch_used = false;
    prompt_pass_check(e);
  }
  QD_CK(cudaMemcpyAsync(e->pinned_state, e->st, sizeof(DevState), cudaMemcpyDeviceToHost, e->stream));
  QD_CK(cudaStreamSynchronize(e->stream));
  const int err = e->pinned_state->err;
  if (err || e->pinned_state->abort) {
    // Repair for the next launch: skip past any epoch a failed launch may have
    // tagged words with, clear the abort flag and the merge counter.
    e->pinned_state->epoch += 2;
    e->pinned_state->abort = 0;
    e->pinned_state->err = 0;
    e->pinned_state->stall_epoch = 0;
    QD_CK(cudaMemcpyAsync(e->st, e->pinned_state, sizeof(DevState), cudaMemcpyHostToDevice, e->stream));
    QD_CK(cudaMemsetAsync(e->lm_counter, 0, 4, e->stream));
    if (e->oacc)  // a failed launch may leave partial O / down sums in its parity
      QD_CK(cudaMemsetAsync(e->oacc, 0, (size_t)2 * e->p.layers * 2 * e->p.hidden * 8, e->stream));
    QD_CK(cudaStreamSynchronize(e->stream));
  }
  if (err & kErrTimeout) throw QdError{QD_E_TIMEOUT, "device: a persistent-kernel wait expired; the launch was abandoned"};
  if (err & kErrToken) throw QdError{QD_E_DEVICE, "device: token id outside the vocabulary"};
  if (err & kErrPosition) throw QdError{QD_E_DEVICE, "device: position beyond max_seq"};
  if (err & kErrOverflow)
    throw QdError{QD_E_DEVICE, "device: an attention output projection partial beyond the fixed-point range (2^22)"};
}

// The first n prompt tokens' K/V in one batched pass where the engine takes it
// (returns n), else nothing (returns 0: the tokens go through the decode kernel).
int run_prompt(qd_engine* e, int n) {
  if (!prompt_pass_fits(e, n)) return 0;
  prompt_pass(e, n);
  e->pbatch_used = true;
  return n;
}

double ms_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

namespace qd {

void bench_layer_from_hidden(qd_engine* e, int l, cudaStream_t s) { enqueue_layer(e, l, s, false); }

void bench_set_position(qd_engine* e, int pos) { set_state(e, pos, 0); }

void bench_check_state(qd_engine* e) { check_state(e); }

void bench_rows_matvec(qd_engine* e, const char* base, long long row_stride, int rows, int k, const float* x,
                       float* y, cudaStream_t s) {
  StageArgs a{};
  const long long nb = k / kBlockCols;
  a.w = base;
  a.s = base + nb * 16;
  a.w_stride = a.s_stride = row_stride;
  a.rows = rows;
  a.nb = (int)nb;
  a.k_valid = k;
  a.src = x;
  a.out = y;
  launch_stage<kProPlain, kEpiStore>(a, plan_stage(rows, a.nb, e->sms), s);
}

}  // namespace qd

// ---------------------------------------------------------------------------
// ---- tcgen05 GEMM ---------------------------------------------------------------

namespace {

template <int BN, bool AF16, int EPI>
void launch_gemm_t(TcArgs a, int splits, cudaStream_t s) {
  const size_t smem = tc_smem_total<BN, AF16>();
  static unsigned long long configured = 0;  // one bit per device ordinal: the attribute is per context
  allow_smem(k_gemm_tc<BN, AF16, EPI>, smem, configured);
  std::string err;
  bool ok;
  if (AF16)
    ok = make_tmap_2d(&a.tm_w, a.a16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.K, a.n_rows, a.a16_stride * 2, kTcK, kTcM,
                      CU_TENSOR_MAP_SWIZZLE_128B, &err);
  else
    ok = make_tmap_2d(&a.tm_w, a.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.K / 2, a.n_rows, a.w_stride, 32, kTcM,
                      CU_TENSOR_MAP_SWIZZLE_NONE, &err);
  ok = ok && make_tmap_2d(&a.tm_xh, a.x_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.K, a.B, a.ldx * 2, kTcK, BN,
                          CU_TENSOR_MAP_SWIZZLE_128B, &err);
  ok = ok && make_tmap_2d(&a.tm_xl, a.x_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.K, a.B, a.ldx * 2, kTcK, BN,
                          CU_TENSOR_MAP_SWIZZLE_128B, &err);
  if (!ok) throw QdError{QD_E_CUDA, "GEMM tensor maps: " + err};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.n_rows + kTcM - 1) / kTcM, (a.B + BN - 1) / BN, splits);
  cfg.blockDim = dim3(tc_block_threads<BN, AF16>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QD_CK(cudaLaunchKernelEx(&cfg, k_gemm_tc<BN, AF16, EPI>, a));
}

}  // namespace

namespace qd {

int gemm_plan_splits(int K, int want, int* kt_split) {
  const int kt_total = K / kTcK;
  want = std::max(1, std::min(want, kt_total));
  *kt_split = (kt_total + want - 1) / want;
  return (kt_total + *kt_split - 1) / *kt_split;
}

void launch_gemm(TcArgs a, int splits, int mode, cudaStream_t s) {
  if (a.K % kTcK || a.K <= 0 || a.B <= 0 || a.n_rows <= 0) throw QdError{QD_E_INVALID, "GEMM: bad dimensions"};
  if (mode == kGemmQ4Store && ((reinterpret_cast<uintptr_t>(a.w) & 15) || (a.w_stride & 15) ||
                               (reinterpret_cast<uintptr_t>(a.s) & 3) || (a.s_stride & 3)))
    throw QdError{QD_E_INVALID, "GEMM: q4 rows must be 16-byte aligned, scales 4-byte aligned"};
  if ((reinterpret_cast<uintptr_t>(a.x_hi) & 15) || (reinterpret_cast<uintptr_t>(a.x_lo) & 15))
    throw QdError{QD_E_INVALID, "GEMM: activations must be 16-byte aligned"};
  if (a.kt_split <= 0) a.kt_split = (a.K / kTcK + splits - 1) / splits;
  if (a.ldx == 0) a.ldx = a.K;
  if (mode == kGemmQ4Store) {
    if (a.B <= 64) launch_gemm_t<64, false, kTcStore>(a, splits, s);
    else if (a.B <= 128) launch_gemm_t<128, false, kTcStore>(a, splits, s);
    else launch_gemm_t<256, false, kTcStore>(a, splits, s);
  } else if (mode == kGemmQ4Silu) {
    if (splits != 1 || (a.n_rows & 1) || !a.y_hi || !a.y_lo)
      throw QdError{QD_E_INVALID, "GEMM: the silu epilogue needs one split, paired rows and hi/lo outputs"};
    if (a.B <= 128) launch_gemm_t<128, false, kTcSilu>(a, splits, s);
    else launch_gemm_t<256, false, kTcSilu>(a, splits, s);
  } else {
    if (a.B <= 64) launch_gemm_t<64, true, kTcArgmax>(a, splits, s);
    else launch_gemm_t<128, true, kTcArgmax>(a, splits, s);
  }
}

}  // namespace qd


extern "C" {

void qd_options_default(qd_options* opt) {
  if (!opt) return;
  opt->device = 0;
  opt->max_seq = 256;
  opt->kv_dtype = QD_KV_F16;
  opt->rope_row_stride = 0;
  opt->variant = "optimized";
  opt->use_graph = 1;
  opt->persistent = 1;
  opt->timeline = 0;
  opt->prompt_pass = 1;
}

int qd_engine_create(const char* runtime_dir, const qd_options* opt, qd_engine** out) {
  if (!out) return fail(nullptr, QdError{QD_E_INVALID, "out is NULL"});
  *out = nullptr;
  if (!runtime_dir) return fail(nullptr, QdError{QD_E_INVALID, "runtime_dir is NULL"});
  qd_engine* e = new qd_engine();
  qd_options_default(&e->opt);
  if (opt) e->opt = *opt;
  e->variant = e->opt.variant ? e->opt.variant : "optimized";
  e->opt.variant = nullptr;
  if (e->opt.kv_dtype != QD_KV_F16 && e->opt.kv_dtype != QD_KV_F32) {
    delete e;
    return fail(nullptr, QdError{QD_E_INVALID, "kv_dtype must be QD_KV_F16 or QD_KV_F32"});
  }
  try {
    e->dev = e->opt.device;
    const Json m = parse_manifest(e, runtime_dir);
    QD_CK(cudaSetDevice(e->dev));
    e->sms = sm_count(e->dev);
    QD_CK(cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking));
    e->stream = e->own_stream;
    load_engine(e, runtime_dir, m);
  } catch (const QdError& err) {
    const int code = fail(nullptr, err);
    free_engine(e);
    return code;
  } catch (const std::exception& ex) {
    const int code = fail(nullptr, QdError{QD_E_IO, ex.what()});
    free_engine(e);
    return code;
  }
  *out = e;
  return QD_OK;
}

void qd_engine_destroy(qd_engine* e) { free_engine(e); }

const char* qd_last_error(const qd_engine* e) { return e ? e->err.c_str() : t_last_error.c_str(); }

int qd_engine_profile(const qd_engine* e, qd_profile* out) {
  if (!e || !out) return QD_E_INVALID;
  *out = e->p;
  return QD_OK;
}

namespace {

int generate(qd_engine* e, const int32_t* input_ids, int n_prompt, int max_new_tokens, const qd_sampling* sampling,
             int32_t* out_ids, qd_token_cb on_token, void* user, qd_stats* stats) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    if (sampling) check_sampling(*sampling);
    const bool sample = sampling && !sampling_is_greedy(*sampling);
    if (!input_ids || n_prompt < 1) throw QdError{QD_E_INVALID, "the prompt needs at least one token"};
    if (max_new_tokens < 0 || (max_new_tokens > 0 && !out_ids)) throw QdError{QD_E_INVALID, "bad max_new_tokens or out_ids"};
    // Positions written: 0 .. n_prompt + max_new - 2 (the last token is never fed back).
    if ((long long)n_prompt + max_new_tokens - 1 > e->opt.max_seq)
      throw QdError{QD_E_RANGE, "prompt + generation length exceeds max_seq (" + std::to_string(e->opt.max_seq) + ")"};
    for (int i = 0; i < n_prompt; ++i)
      if (input_ids[i] < 0 || input_ids[i] >= e->p.vocab) throw QdError{QD_E_RANGE, "prompt token id outside the vocabulary"};
    QD_CK(cudaSetDevice(e->dev));
    const auto t0 = std::chrono::steady_clock::now();
    std::memcpy(e->pinned_ids, input_ids, (size_t)n_prompt * 4);
    QD_CK(cudaMemcpyAsync(e->tokens, e->pinned_ids, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, e->stream));
    const int n_layers_only = max_new_tokens > 0 ? n_prompt - 1 : n_prompt;
    // A greedy generation of two or more ids whose whole prompt fits the batched pass
    // takes its first id from the pass as well (final norm + LM head on the last
    // prompt row); the decode kernel then starts at the first generated token. With
    // one id the decode kernel computes it, so that qd_engine_logits has the final
    // hidden state it recomputes logits from.
    int first = 0, step0 = 0;
    if (!sample && max_new_tokens >= 2 && prompt_pass_fits(e, n_prompt)) {
      prompt_pass(e, n_prompt, true);
      e->pbatch_used = true;
      first = n_prompt;
      step0 = 1;
      QD_CK(cudaEventRecord(e->ev[0], e->stream));  // out_host[0] is written
    } else {
      first = run_prompt(e, n_layers_only);
    }
    set_state(e, first, max_new_tokens, step0);
    for (int i = first; i < n_layers_only; ++i) run_token(e, kHeadNone);
    double first_ms = 0.0;
    int produced = 0;
    bool stop = false;
    for (int step = step0; step < max_new_tokens && !stop; ++step) {
      run_token(e, sample ? kHeadFull : kHeadArgmax);  // the sampler reads the logits
      if (sample) enqueue_engine_sample(e, *sampling);
      QD_CK(cudaEventRecord(e->ev[step & 1], e->stream));
      if (step > 0) {  // deliver the previous token while this one runs
        QD_CK(cudaEventSynchronize(e->ev[(step - 1) & 1]));
        const int tok = *reinterpret_cast<volatile int*>(e->out_host + step - 1);
        out_ids[step - 1] = tok;
        ++produced;
        if (step == 1) first_ms = ms_since(t0);
        if (on_token && on_token(tok, user)) stop = true;
      }
    }
    QD_CK(cudaStreamSynchronize(e->stream));
    if (max_new_tokens > 0 && !stop) {
      const int last = max_new_tokens - 1;
      const int tok = *reinterpret_cast<volatile int*>(e->out_host + last);
      out_ids[last] = tok;
      ++produced;
      if (last == 0) first_ms = ms_since(t0);
      if (on_token) on_token(tok, user);
    }
    const double gen_ms = ms_since(t0);
    check_state(e);
    if (stats) {
      stats->generate_ms = gen_ms;
      stats->first_token_ms = first_ms;
      stats->generated_tokens = produced;
      stats->prompt_tokens = n_prompt;
      stats->steady_ms_per_token = produced > 1 ? (gen_ms - first_ms) / (produced - 1) : NAN;
    }
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

}  // namespace

int qd_generate_greedy(qd_engine* e, const int32_t* input_ids, int n_prompt, int max_new_tokens,
                       int32_t* out_ids, qd_token_cb on_token, void* user, qd_stats* stats) {
  return generate(e, input_ids, n_prompt, max_new_tokens, nullptr, out_ids, on_token, user, stats);
}

int qd_generate_sample(qd_engine* e, const int32_t* input_ids, int n_prompt, int max_new_tokens,
                       const qd_sampling* sampling, int32_t* out_ids, qd_token_cb on_token, void* user,
                       qd_stats* stats) {
  if (!sampling) return fail(e, QdError{QD_E_INVALID, "sampling parameters are NULL"});
  return generate(e, input_ids, n_prompt, max_new_tokens, sampling, out_ids, on_token, user, stats);
}

int qd_engine_logits(qd_engine* e, float* host_logits) {
  if (!e || !host_logits) return fail(e, QdError{QD_E_INVALID, "NULL argument"});
  try {
    QD_CK(cudaSetDevice(e->dev));
    if (e->logits_stale) {  // the last token computed the argmax only: logits from its final hidden state
      launch(k_words_to_f32, dim3((e->p.hidden + kThreads - 1) / kThreads), e->stream,
             (const unsigned long long*)(e->xbuf + (long long)e->p.layers * e->xstride), e->h, e->p.hidden);
      LmArgs a{};
      a.h = e->h; a.norm_w = e->final_norm; a.eps = e->p.eps;
      a.table = reinterpret_cast<const uint4*>(e->embed); a.vocab = e->p.vocab; a.H = e->p.hidden;
      a.logits = e->logits; a.part_v = e->lm_pv; a.part_i = e->lm_pi; a.counter = e->lm_counter;
      a.result = e->result;  // no token state: st stays null
      launch_lmhead(a, e->lm_grid, e->stream);
      e->logits_stale = false;
    }
    QD_CK(cudaMemcpyAsync(host_logits, e->logits, (size_t)e->p.vocab * 4, cudaMemcpyDeviceToHost, e->stream));
    QD_CK(cudaStreamSynchronize(e->stream));
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_engine_hidden(qd_engine* e, float* host_hidden) {
  if (!e || !host_hidden) return fail(e, QdError{QD_E_INVALID, "NULL argument"});
  try {
    QD_CK(cudaSetDevice(e->dev));
    if (e->persist) {  // the persistent kernel leaves it in the exchange words after the last layer
      std::vector<unsigned long long> w(e->p.hidden);
      QD_CK(cudaMemcpyAsync(w.data(), e->xbuf + (long long)e->p.layers * e->xstride, w.size() * 8,
                            cudaMemcpyDeviceToHost, e->stream));
      QD_CK(cudaStreamSynchronize(e->stream));
      for (int i = 0; i < e->p.hidden; ++i) {
        const uint32_t bits = (uint32_t)w[i];
        std::memcpy(host_hidden + i, &bits, 4);
      }
    } else {
      QD_CK(cudaMemcpyAsync(host_hidden, e->h, (size_t)e->p.hidden * 4, cudaMemcpyDeviceToHost, e->stream));
      QD_CK(cudaStreamSynchronize(e->stream));
    }
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_engine_forward_trace(qd_engine* e, int32_t token, int position, float* host_trace) {
  if (!e || !host_trace) return fail(e, QdError{QD_E_INVALID, "NULL argument"});
  try {
    if (token < 0 || token >= e->p.vocab) throw QdError{QD_E_RANGE, "token id outside the vocabulary"};
    if (position < 0 || position >= e->opt.max_seq) throw QdError{QD_E_RANGE, "position beyond max_seq"};
    QD_CK(cudaSetDevice(e->dev));
    e->pinned_ids[0] = token;
    QD_CK(cudaMemcpyAsync(e->tokens + position, e->pinned_ids, 4, cudaMemcpyHostToDevice, e->stream));
    set_state(e, position, 0);
    for (int l = 0; l < e->p.layers; ++l) {
      enqueue_layer(e, l, e->stream);
      QD_CK(cudaMemcpyAsync(host_trace + (size_t)l * e->p.hidden, e->h, (size_t)e->p.hidden * 4,
                            cudaMemcpyDeviceToHost, e->stream));
    }
    QD_CK(cudaStreamSynchronize(e->stream));
    check_state(e);
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_engine_set_stream(qd_engine* e, void* stream) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    QD_CK(cudaSetDevice(e->dev));
    QD_CK(cudaStreamSynchronize(e->stream));
    e->stream = stream ? static_cast<cudaStream_t>(stream) : e->own_stream;
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_decode_begin(qd_engine* e, const int32_t* input_ids, int n_prompt, int max_new_tokens) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    if (!input_ids || n_prompt < 1 || n_prompt > e->opt.max_seq) throw QdError{QD_E_INVALID, "bad prompt length"};
    if (max_new_tokens < 0 || max_new_tokens > e->opt.max_seq) throw QdError{QD_E_INVALID, "bad max_new_tokens"};
    for (int i = 0; i < n_prompt; ++i)
      if (input_ids[i] < 0 || input_ids[i] >= e->p.vocab) throw QdError{QD_E_RANGE, "prompt token id outside the vocabulary"};
    QD_CK(cudaSetDevice(e->dev));
    QD_CK(cudaStreamSynchronize(e->stream));  // pinned staging buffers are reused below
    std::memcpy(e->pinned_ids, input_ids, (size_t)n_prompt * 4);
    QD_CK(cudaMemcpyAsync(e->tokens, e->pinned_ids, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, e->stream));
    const int first = run_prompt(e, n_prompt - 1);
    set_state(e, first, max_new_tokens);
    e->stepping_max_new = max_new_tokens;
    for (int i = first; i < n_prompt - 1; ++i) run_token(e, kHeadNone);
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_decode_step(qd_engine* e) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    run_token(e, kHeadArgmax);
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_decode_seek(qd_engine* e, int position) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    if (position < 0 || position >= e->opt.max_seq) throw QdError{QD_E_RANGE, "position beyond max_seq"};
    launch(k_seek, dim3(1), e->stream, e->st, position);
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_decode_sync(qd_engine* e, int32_t* out_ids, int n) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    QD_CK(cudaSetDevice(e->dev));
    check_state(e);
    const int k = std::min(n, e->stepping_max_new);
    for (int i = 0; out_ids && i < k; ++i) out_ids[i] = *reinterpret_cast<volatile int*>(e->out_host + i);
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_engine_inject_stall(qd_engine* e) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    if (!e->persist) throw QdError{QD_E_INVALID, "the stall hook needs the persistent decode kernel"};
    QD_CK(cudaSetDevice(e->dev));
    // The next launch tags its words with the device's epoch + 1.
    QD_CK(cudaMemcpyAsync(e->pinned_state, e->st, sizeof(DevState), cudaMemcpyDeviceToHost, e->stream));
    QD_CK(cudaStreamSynchronize(e->stream));
    e->pinned_state->stall_epoch = e->pinned_state->epoch + 1;
    QD_CK(cudaMemcpyAsync(&e->st->stall_epoch, &e->pinned_state->stall_epoch, sizeof(int), cudaMemcpyHostToDevice,
                          e->stream));
    QD_CK(cudaStreamSynchronize(e->stream));
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}

int qd_engine_uses_persistent(const qd_engine* e) { return e ? (e->persist ? 1 : 0) : 0; }

int qd_engine_timeline(qd_engine* e, uint64_t* host_out, int* ctas, int* events_per_cta) {
  if (!e) return fail(nullptr, QdError{QD_E_INVALID, "engine is NULL"});
  try {
    if (!e->timeline) throw QdError{QD_E_INVALID, "timeline not enabled (qd_options.timeline) or no persistent kernel"};
    const int ev = timeline_events(e->p.layers);
    const int nctas = e->sms;
    if (ctas) *ctas = nctas;
    if (events_per_cta) *events_per_cta = ev;
    if (host_out) {
      QD_CK(cudaSetDevice(e->dev));
      QD_CK(cudaMemcpyAsync(host_out, e->timeline, (size_t)nctas * ev * 8, cudaMemcpyDeviceToHost, e->stream));
      QD_CK(cudaStreamSynchronize(e->stream));
    }
  } catch (const QdError& err) {
    return fail(e, err);
  }
  return QD_OK;
}


int qd_decode_step_kernels(const qd_engine* e) { return e ? (e->persist ? 1 : e->p.layers * 5 + 1) : 0; }

// ---- kernel level -------------------------------------------------------------

int qd_q4_matvec(const float* x, const uint32_t* weights, const uint16_t* scales_f16, float* y,
                 uint32_t in_size, uint32_t out_size, uint32_t blocks_per_row, uint32_t block_size,
                 void* stream) {
  try {
    if (!x || !weights || !scales_f16 || !y) throw QdError{QD_E_INVALID, "NULL pointer"};
    if (block_size != (uint32_t)kBlockCols) throw QdError{QD_E_INVALID, "only block_size 32 is supported"};
    if (out_size == 0 || blocks_per_row == 0 || blocks_per_row > 128 || in_size == 0 ||
        in_size > blocks_per_row * block_size)
      throw QdError{QD_E_INVALID, "bad matvec dimensions (in_size <= blocks_per_row * 32 <= 4096)"};
    if ((reinterpret_cast<uintptr_t>(weights) & 15) != 0) throw QdError{QD_E_INVALID, "weights must be 16-byte aligned"};
    StageArgs a{};
    a.w = reinterpret_cast<const char*>(weights);
    a.s = reinterpret_cast<const char*>(scales_f16);
    a.w_stride = (long long)blocks_per_row * 16;
    a.s_stride = (long long)blocks_per_row * 2;
    a.rows = (int)out_size; a.nb = (int)blocks_per_row; a.k_valid = (int)in_size; a.src = x; a.out = y;
    launch_stage<kProPlain, kEpiStore>(a, plan_stage(a.rows, a.nb, current_sms()), static_cast<cudaStream_t>(stream));
  } catch (const QdError& err) {
    return fail(nullptr, err);
  }
  return QD_OK;
}

size_t qd_q4_gemm_workspace_bytes(uint32_t M, uint32_t in_size) { return 256 + (size_t)M * in_size * 4; }

int qd_q4_gemm(const float* x, const uint32_t* weights, const uint16_t* scales_f16, float* y, uint32_t M,
               uint32_t in_size, uint32_t out_size, uint32_t block_size, void* workspace, void* stream) {
  try {
    if (!x || !weights || !scales_f16 || !y || !workspace) throw QdError{QD_E_INVALID, "NULL pointer"};
    if (block_size != (uint32_t)kBlockCols) throw QdError{QD_E_INVALID, "only block_size 32 is supported"};
    if (M == 0 || out_size == 0 || in_size == 0 || in_size % kTcK || in_size > 4096)
      throw QdError{QD_E_INVALID, "qd_q4_gemm: in_size must be a positive multiple of 64, at most 4096"};
    if ((reinterpret_cast<uintptr_t>(weights) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15))
      throw QdError{QD_E_INVALID, "weights and workspace must be 16-byte aligned"};
    if (reinterpret_cast<uintptr_t>(scales_f16) & 3) throw QdError{QD_E_INVALID, "scales_f16 must be 4-byte aligned"};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    __half* xh = reinterpret_cast<__half*>(static_cast<char*>(workspace) + 256);
    __half* xl = xh + (size_t)M * in_size;
    const int n = (int)(M * in_size);
    launch(k_split_hilo, dim3(std::min((n + kThreads - 1) / kThreads, 4096)), s, x, n, xh, xl);
    TcArgs a{};
    a.w = reinterpret_cast<const char*>(weights);
    a.s = reinterpret_cast<const char*>(scales_f16);
    a.w_stride = (long long)in_size / 2;
    a.s_stride = (long long)in_size / kBlockCols * 2;
    a.n_rows = (int)out_size;
    a.K = (int)in_size;
    a.kt_split = (int)in_size / kTcK;
    a.x_hi = xh;
    a.x_lo = xl;
    a.B = (int)M;
    a.y = y;
    a.ldy = (int)out_size;
    launch_gemm(a, 1, kGemmQ4Store, s);
  } catch (const QdError& err) {
    return fail(nullptr, err);
  }
  return QD_OK;
}

static constexpr int kLmMaxGrid = 1024;

size_t qd_lm_head_argmax_workspace_bytes(uint32_t) { return 256 + (size_t)kLmMaxGrid * 8; }

int qd_lm_head_argmax(const float* hidden, const float* norm_weight, float eps, const uint16_t* embed_f16,
                      float* logits, uint32_t* result, uint32_t hidden_size, uint32_t vocab, void* workspace,
                      void* stream) {
  try {
    if (!hidden || !embed_f16 || !result || !workspace) throw QdError{QD_E_INVALID, "NULL pointer"};
    if (hidden_size % 256 || hidden_size == 0 || hidden_size > 1024)
      throw QdError{QD_E_INVALID, "hidden_size must be 256, 512, 768 or 1024"};
    if (vocab == 0) throw QdError{QD_E_INVALID, "vocab must be positive"};
    if ((reinterpret_cast<uintptr_t>(embed_f16) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15))
      throw QdError{QD_E_INVALID, "embed_f16 and workspace must be 16-byte aligned"};
    char* ws = static_cast<char*>(workspace);
    LmArgs a{};
    a.h = hidden; a.norm_w = norm_weight; a.eps = eps; a.table = reinterpret_cast<const uint4*>(embed_f16);
    a.vocab = (int)vocab; a.H = (int)hidden_size; a.logits = logits;
    a.counter = reinterpret_cast<unsigned*>(ws);
    a.part_v = reinterpret_cast<float*>(ws + 256);
    a.part_i = reinterpret_cast<uint32_t*>(ws + 256 + kLmMaxGrid * 4);
    a.result = result;
    const int grid = std::min(current_sms(), kLmMaxGrid);
    launch_lmhead(a, grid, static_cast<cudaStream_t>(stream));
  } catch (const QdError& err) {
    return fail(nullptr, err);
  }
  return QD_OK;
}

size_t qd_gqa_decode_workspace_bytes(uint32_t seq_len, uint32_t q_heads) {
  const size_t splits = (seq_len + kAttnChunk - 1) / kAttnChunk;
  return 256 + splits * q_heads * 8 + splits * q_heads * kHeadDim * 4;
}

int qd_gqa_decode(const float* q, const void* k_cache, const void* v_cache, int kv_dtype, float* y,
                  uint32_t seq_len, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, void* workspace,
                  void* stream) {
  try {
    if (!q || !k_cache || !v_cache || !y || !workspace) throw QdError{QD_E_INVALID, "NULL pointer"};
    if (head_dim != (uint32_t)kHeadDim) throw QdError{QD_E_INVALID, "head_dim must be 128"};
    if (seq_len == 0 || kv_heads == 0 || q_heads % kv_heads) throw QdError{QD_E_INVALID, "bad attention dimensions"};
    if (kv_dtype != QD_KV_F16 && kv_dtype != QD_KV_F32) throw QdError{QD_E_INVALID, "bad kv_dtype"};
    const int splits = (int)((seq_len + kAttnChunk - 1) / kAttnChunk);
    char* ws = static_cast<char*>(workspace);
    AttnArgs a{};
    a.q_in = q; a.k_cache = const_cast<void*>(k_cache); a.v_cache = const_cast<void*>(v_cache);
    a.st = nullptr; a.seq_len = (int)seq_len; a.max_seq = (int)seq_len;
    a.q_heads = (int)q_heads; a.kv_heads = (int)kv_heads; a.scale = 1.0f / std::sqrt((float)kHeadDim);
    a.raw_q = 1;
    a.part_ml = reinterpret_cast<float2*>(ws + 256);
    a.part_o = reinterpret_cast<float*>(ws + 256 + (size_t)splits * q_heads * 8);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    launch_attn(a, kv_dtype, splits, s);
    const int n = (int)q_heads * kHeadDim;
    launch(k_attn_combine, dim3((n + kThreads - 1) / kThreads), s, (const float2*)a.part_ml, (const float*)a.part_o,
           splits, (int)q_heads, y);
  } catch (const QdError& err) {
    return fail(nullptr, err);
  }
  return QD_OK;
}

}  // extern "C"
