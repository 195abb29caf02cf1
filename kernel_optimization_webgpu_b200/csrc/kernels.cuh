// Batch-1 decode kernels for sm_100a.
//
// Every kernel is launched with programmatic dependent launch (PDL): it issues
// the loads that do not depend on the previous kernel (the q4 weights and
// scales, or the first LM-head rows) before `griddepcontrol.wait`, so the
// weight stream of one stage overlaps the tail of the stage before it.
#pragma once

#include "common.cuh"

namespace qd {

// ---------------------------------------------------------------------------
// q4 MatMulNBits matvec stage (matmul_nbits_q4.wgsl:43-92) with fused
// prologue (activation source) and epilogue (what to do with each row).
// Device layout of a q4 matrix: [rows][nb] uint4 (one uint4 = one 32-column
// block = the ONNX [N][K/32][16 B] layout unchanged) and [rows][nb] f16 scales.
// ---------------------------------------------------------------------------
enum Pro : int {
  kProPlain = 0,    // x = src[0..k_valid), zero beyond
  kProRms = 1,      // x = rms_norm(src) * norm_w              (rms_norm.wgsl:15-44)
  kProEmbed = 2,    // x = rms_norm(f16 embed[tokens[pos]]) * norm_w; CTA 0 writes the f32 row
  kProCombine = 3,  // x = split-KV attention combine of the partials
};
enum Epi : int {
  kEpiStore = 0,    // out[r] = y
  kEpiResidual = 1, // out[r] = res[r] + y                     (residual_add.wgsl:13-19)
  kEpiSilu = 2,     // out[r] = silu(y_gate[r]) * y_up[r]       (silu_mul.wgsl:13-23)
};

// Row r (sub-row j: 0, or 1 for the up row of a gate/up pair) keeps its nb
// 16-byte blocks at w + r*w_stride + j*w_sub and its nb f16 scales at
// s + r*s_stride + j*s_sub. The engine interleaves them into one row record
// ([q4 blocks | scales], 16-byte aligned); the standalone entry passes two arrays.
struct StageArgs {
  const char* w;
  const char* s;
  long long w_stride, w_sub, s_stride, s_sub;
  int rows;                // output rows
  int nb;                  // blocks per row (= in_size / 32, rounded up)
  int k_valid;             // in_size: activations at or beyond it count as zero
  const float* src;
  const float* norm_w;
  float eps;
  const float* res;
  float* out;
  const __half* embed;     // kProEmbed
  const int* tokens;
  DevState* st;
  int vocab;
  int max_seq;             // tokens[] holds max_seq + 1 ids
  float* h_out;
  const float2* part_ml;   // kProCombine: [splits][q_heads] (max, sum)
  const float* part_o;     //              [splits][q_heads][128]
  int splits;
  int q_heads;
};

template <int KC, int NR, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) k_stage(const StageArgs a) {
  constexpr int NW = (EPI == kEpiSilu) ? 2 : 1;
  __shared__ __align__(16) float xs[KC * 1024];
  __shared__ float red[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * kWarps + warp, W = gridDim.x * kWarps;

  // 1. Weights and scales do not depend on the previous kernel: load them first.
  uint4 wr[NR][NW][KC];
  __half sr[NR][NW][KC];
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    const int r = gw + i * W;
#pragma unroll
    for (int j = 0; j < NW; ++j)
#pragma unroll
      for (int c = 0; c < KC; ++c) {
        const int b = c * 32 + lane;
        if (r < a.rows && b < a.nb) {
          wr[i][j][c] = ld_stream(reinterpret_cast<const uint4*>(a.w + r * a.w_stride + j * a.w_sub) + b);
          sr[i][j][c] = reinterpret_cast<const __half*>(a.s + r * a.s_stride + j * a.s_sub)[b];
        } else {
          wr[i][j][c] = make_uint4(0u, 0u, 0u, 0u);
          sr[i][j][c] = __float2half_rn(0.0f);
        }
      }
  }
  pdl_trigger();
  pdl_wait();

  // 2. Prologue: the activation vector into shared memory.
  const int ncols = a.nb * kBlockCols;
  if constexpr (PRO == kProPlain) {
    for (int e = threadIdx.x; e < ncols; e += kThreads) xs_store(xs, e, e < a.k_valid ? a.src[e] : 0.0f);
  } else if constexpr (PRO == kProRms || PRO == kProEmbed) {
    const float* src = a.src;
    const __half* erow = nullptr;
    if constexpr (PRO == kProEmbed) {
      const int pos = a.st->pos;
      int tok = (pos >= 0 && pos <= a.max_seq) ? a.tokens[pos] : -1;
      if (tok < 0 || tok >= a.vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&a.st->err, kErrToken);
        tok = 0;
      }
      erow = a.embed + (size_t)tok * a.k_valid;
    }
    float ss = 0.0f;
    for (int e = threadIdx.x; e < a.k_valid; e += kThreads) {
      const float v = (PRO == kProEmbed) ? __half2float(erow[e]) : src[e];
      ss += v * v;
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)a.k_valid + a.eps);
    for (int e = threadIdx.x; e < ncols; e += kThreads) {
      float v = 0.0f;
      if (e < a.k_valid) {
        const float raw = (PRO == kProEmbed) ? __half2float(erow[e]) : src[e];
        if (PRO == kProEmbed && blockIdx.x == 0) a.h_out[e] = raw;
        v = raw * inv * a.norm_w[e];
      }
      xs_store(xs, e, v);
    }
  } else {  // kProCombine
    for (int e = threadIdx.x; e < ncols; e += kThreads) {
      float v = 0.0f;
      if (e < a.k_valid) {
        const int h = e / kHeadDim;
        float m = -INFINITY;
        for (int sp = 0; sp < a.splits; ++sp) m = fmaxf(m, a.part_ml[sp * a.q_heads + h].x);
        float l = 0.0f, o = 0.0f;
        for (int sp = 0; sp < a.splits; ++sp) {
          const float2 ml = a.part_ml[sp * a.q_heads + h];
          const float f = (ml.y > 0.0f) ? expf(ml.x - m) : 0.0f;
          l += ml.y * f;
          o += a.part_o[(size_t)sp * a.q_heads * kHeadDim + e] * f;
        }
        v = o / l;
      }
      xs_store(xs, e, v);
    }
  }
  __syncthreads();

  // 3. Activations into registers: lane l holds the 32 columns of block c*32 + l.
  float2 xr[KC][16];
#pragma unroll
  for (int c = 0; c < KC; ++c) {
    const int b = c * 32 + lane;
    const int f0 = b * 8;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (b < a.nb) v = reinterpret_cast<const float4*>(xs)[xs_slot(f0 + q)];
      xr[c][2 * q] = make_float2(v.x, v.y);
      xr[c][2 * q + 1] = make_float2(v.z, v.w);
    }
  }

  // 4. Row dots, warp reduction, epilogue.
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    const int r = gw + i * W;
    float y[NW];
#pragma unroll
    for (int j = 0; j < NW; ++j) {
      float acc = 0.0f;
#pragma unroll
      for (int c = 0; c < KC; ++c)
        if (c * 32 + lane < a.nb) acc += __half2float(sr[i][j][c]) * q4_block_dot(wr[i][j][c], xr[c]);
      y[j] = warp_sum(acc);
    }
    if (r < a.rows && lane == 0) {
      if constexpr (EPI == kEpiStore) a.out[r] = y[0];
      else if constexpr (EPI == kEpiResidual) a.out[r] = a.res[r] + y[0];
      else a.out[r] = (y[0] / (1.0f + expf(-y[0]))) * y[NW - 1];
    }
  }
}

// ---------------------------------------------------------------------------
// Decode attention: head RMSNorm + RoPE + KV-cache append fused with a
// split-KV GQA pass (head_rms_norm.wgsl, rope.wgsl, cache_write.wgsl,
// gqa_decode.wgsl). Grid (kv_heads, splits); the G = q_heads / kv_heads query
// heads of one KV head share each K/V row read. Writes per-split partials
// (running max, exp-sum, unnormalised output) combined by the O projection.
// ---------------------------------------------------------------------------
struct AttnArgs {
  const float* q_in;       // raw q (projection output) or, with raw_q, the final q
  const float* k_in;       // raw k projection for the new row
  const float* v_in;       // raw v projection for the new row
  const float* norm_q;
  const float* norm_k;
  float eps;
  const float* cos_t;      // [rope_rows * 64] f32
  const float* sin_t;
  int row_stride;          // table offset = position * row_stride + pair (rope.wgsl:27)
  void* k_cache;           // [max_seq][kv_heads][128] (f16 or f32)
  void* v_cache;
  DevState* st;            // position source (engine); null: use seq_len
  int seq_len;             // standalone: attend over [0, seq_len)
  int max_seq;
  int q_heads, kv_heads;
  float scale;             // 1/sqrt(128), computed on the host
  int raw_q;               // 1: q_in is final (no norm/rope) and no cache append
  float2* part_ml;         // [splits][q_heads]
  float* part_o;           // [splits][q_heads][128]
};

template <typename T> __device__ __forceinline__ float4 ld4(const T* p);
template <> __device__ __forceinline__ float4 ld4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <> __device__ __forceinline__ float4 ld4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
// Stores 4 values; returns what a later read of the cache gives back.
template <typename T> __device__ __forceinline__ float4 st4(T* p, float4 v);
template <> __device__ __forceinline__ float4 st4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
  return v;
}
template <> __device__ __forceinline__ float4 st4<__half>(__half* p, float4 v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
  const float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

template <int G, typename KVT>
__global__ void __launch_bounds__(kThreads, 2) k_attn(const AttnArgs a) {
  __shared__ __align__(16) float qs[G][kHeadDim];
  __shared__ __align__(16) float kn[kHeadDim];
  __shared__ __align__(16) float vn[kHeadDim];
  __shared__ float sc[G][kAttnChunk];
  __shared__ float2 mls[G];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = blockIdx.x, sp = blockIdx.y;
  KVT* kc = reinterpret_cast<KVT*>(a.k_cache);
  KVT* vc = reinterpret_cast<KVT*>(a.v_cache);
  const size_t row_elems = (size_t)a.kv_heads * kHeadDim;

  pdl_trigger();
  pdl_wait();
  int pos, seq;
  if (a.st) {
    pos = a.st->pos;
    if (pos < 0 || pos >= a.max_seq) {
      if (g == 0 && sp == 0 && threadIdx.x == 0) atomicOr(&a.st->err, kErrPosition);
      pos = 0;  // keep every access in bounds; the host reports the error
    }
    seq = pos + 1;
  } else {
    seq = a.seq_len;
    pos = seq - 1;
  }
  const int lo = sp * kAttnChunk;
  const int hi = min(seq, lo + kAttnChunk);
  const bool append = !a.raw_q && pos >= lo && pos < lo + kAttnChunk;

  // Phase A: query heads (and the new K/V row in the split that holds it).
  for (int t = warp; t < G + 2; t += kWarps) {
    if (t >= G && !append) continue;
    const float* src = (t < G) ? a.q_in + (size_t)(g * G + t) * kHeadDim
                               : (t == G ? a.k_in + (size_t)g * kHeadDim : a.v_in + (size_t)g * kHeadDim);
    const float4 x = reinterpret_cast<const float4*>(src)[lane];
    if (t == G + 1) {  // V is cached as projected (webgpu-runtime.js:523-527)
      const float4 r = st4<KVT>(vc + (size_t)pos * row_elems + (size_t)g * kHeadDim + 4 * lane, x);
      reinterpret_cast<float4*>(vn)[lane] = r;
      continue;
    }
    if (t < G && a.raw_q) {
      reinterpret_cast<float4*>(qs[t])[lane] = x;
      continue;
    }
    const float* nw = (t < G) ? a.norm_q : a.norm_k;
    float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)kHeadDim + a.eps);
    const float4 w4 = reinterpret_cast<const float4*>(nw)[lane];
    const float4 y = make_float4(x.x * inv * w4.x, x.y * inv * w4.y, x.z * inv * w4.z, x.w * inv * w4.w);
    // rotate-half RoPE: dims d and d +- 64 live in lanes l and l ^ 16 (rope.wgsl:22-30)
    float4 p;
    p.x = __shfl_xor_sync(0xffffffffu, y.x, 16);
    p.y = __shfl_xor_sync(0xffffffffu, y.y, 16);
    p.z = __shfl_xor_sync(0xffffffffu, y.z, 16);
    p.w = __shfl_xor_sync(0xffffffffu, y.w, 16);
    const int pair0 = (4 * lane) & (kHeadDim / 2 - 1);
    const size_t toff = (size_t)pos * a.row_stride + pair0;
    const float4 c = *reinterpret_cast<const float4*>(a.cos_t + toff);
    const float4 s = *reinterpret_cast<const float4*>(a.sin_t + toff);
    const float sign = (lane >= 16) ? 1.0f : -1.0f;
    const float4 r = make_float4(y.x * c.x + sign * p.x * s.x, y.y * c.y + sign * p.y * s.y,
                                 y.z * c.z + sign * p.z * s.z, y.w * c.w + sign * p.w * s.w);
    if (t < G) {
      reinterpret_cast<float4*>(qs[t])[lane] = r;
    } else {
      const float4 rr = st4<KVT>(kc + (size_t)pos * row_elems + (size_t)g * kHeadDim + 4 * lane, r);
      reinterpret_cast<float4*>(kn)[lane] = rr;
    }
  }
  __syncthreads();

  const int nh = a.q_heads;
  if (lo >= seq) {  // empty split: neutral partial
    if (threadIdx.x < G) a.part_ml[sp * nh + g * G + threadIdx.x] = make_float2(-INFINITY, 0.0f);
    for (int e = threadIdx.x; e < G * kHeadDim; e += kThreads)
      a.part_o[((size_t)sp * nh + g * G) * kHeadDim + e] = 0.0f;
    return;
  }

  // Phase B: scores, one warp per position; lane l holds dims 4l..4l+3.
  float4 qv[G];
#pragma unroll
  for (int h = 0; h < G; ++h) qv[h] = reinterpret_cast<const float4*>(qs[h])[lane];
  for (int p = lo + warp; p < hi; p += kWarps) {
    const float4 k4 = (append && p == pos) ? reinterpret_cast<const float4*>(kn)[lane]
                                           : ld4<KVT>(kc + (size_t)p * row_elems + (size_t)g * kHeadDim + 4 * lane);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float d = qv[h].x * k4.x + qv[h].y * k4.y + qv[h].z * k4.z + qv[h].w * k4.w;
      d = warp_sum(d);
      if (lane == 0) sc[h][p - lo] = d * a.scale;
    }
  }
  __syncthreads();
  const int n = hi - lo;
  if (warp < G) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[warp][i]);
    m = warp_max(m);
    float l = 0.0f;
    for (int i = lane; i < n; i += 32) {
      const float e = expf(sc[warp][i] - m);
      sc[warp][i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) mls[warp] = make_float2(m, l);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * kHeadDim; e += kThreads) {
    const int h = e / kHeadDim, d = e % kHeadDim;
    float acc = 0.0f;
    for (int p = lo; p < hi; ++p) {
      const float v = (append && p == pos) ? vn[d]
                                           : static_cast<float>(vc[(size_t)p * row_elems + (size_t)g * kHeadDim + d]);
      acc += sc[h][p - lo] * v;
    }
    a.part_o[((size_t)sp * nh + g * G + h) * kHeadDim + d] = acc;
  }
  if (threadIdx.x < G) a.part_ml[sp * nh + g * G + threadIdx.x] = mls[threadIdx.x];
}

// Standalone split combine (the engine fuses this into the O projection).
static __global__ void __launch_bounds__(kThreads) k_attn_combine(const float2* part_ml, const float* part_o,
                                                            int splits, int q_heads, float* y) {
  pdl_trigger();
  pdl_wait();
  const int n = q_heads * kHeadDim;
  for (int e = blockIdx.x * kThreads + threadIdx.x; e < n; e += gridDim.x * kThreads) {
    const int h = e / kHeadDim;
    float m = -INFINITY;
    for (int sp = 0; sp < splits; ++sp) m = fmaxf(m, part_ml[sp * q_heads + h].x);
    float l = 0.0f, o = 0.0f;
    for (int sp = 0; sp < splits; ++sp) {
      const float2 ml = part_ml[sp * q_heads + h];
      const float f = (ml.y > 0.0f) ? expf(ml.x - m) : 0.0f;
      l += ml.y * f;
      o += part_o[(size_t)sp * n + e] * f;
    }
    y[e] = o / l;
  }
}

// ---------------------------------------------------------------------------
// LM head + argmax (lm_head_f16.wgsl:19-58, argmax_stage1/2.wgsl) in one
// kernel: optional final RMSNorm prologue, each warp streams whole f16 rows of
// the tied table (128-bit loads), keeps a running (max, lowest index), and the
// last CTA to finish merges the per-CTA partials. With an engine state it also
// appends the token and advances the position, so only the 4-byte token id
// leaves the device.
// ---------------------------------------------------------------------------
struct LmArgs {
  const float* h;          // [H] hidden (pre-norm when norm_w is set)
  const float* norm_w;     // final norm weight or null
  float eps;
  const uint4* table;      // [vocab][H/8]
  int vocab;
  int H;
  float* logits;           // [vocab] or null
  float* part_v;           // [gridDim.x]
  uint32_t* part_i;        // [gridDim.x]
  unsigned* counter;       // zero before the first launch; the last CTA re-zeroes it
  uint32_t* result;        // [2] = {index, f32 bits of the max}
  DevState* st;            // engine epilogue (null for the standalone entry)
  int* tokens;
  int* out_dev;
  int* out_host;
  int max_seq;
};

template <int KC>  // KC = H / 256: uint4 chunks per lane per row
__global__ void __launch_bounds__(kThreads, 1) k_lmhead(const LmArgs a) {
  constexpr int U = 4;  // rows in flight per warp
  __shared__ __align__(16) float xs[KC * 256];
  __shared__ float red[kWarps];
  __shared__ float bv_s[kWarps];
  __shared__ uint32_t bi_s[kWarps];
  __shared__ int am_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * kWarps + warp, W = gridDim.x * kWarps;
  const int rpr = a.H / 8;  // uint4 per row

  uint4 cur[U][KC];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int r = gw + u * W;
#pragma unroll
    for (int c = 0; c < KC; ++c)
      cur[u][c] = (r < a.vocab) ? ld_stream(a.table + (size_t)r * rpr + c * 32 + lane) : make_uint4(0, 0, 0, 0);
  }
  pdl_trigger();
  pdl_wait();

  // Final RMSNorm (rms_norm.wgsl) into shared memory, then into registers.
  if (a.norm_w) {
    float ss = 0.0f;
    for (int e = threadIdx.x; e < a.H; e += kThreads) ss += a.h[e] * a.h[e];
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)a.H + a.eps);
    for (int e = threadIdx.x; e < a.H; e += kThreads) xs[e] = a.h[e] * inv * a.norm_w[e];
  } else {
    for (int e = threadIdx.x; e < a.H; e += kThreads) xs[e] = a.h[e];
  }
  __syncthreads();
  float2 xr[KC][4];
#pragma unroll
  for (int c = 0; c < KC; ++c) {
    const float4* p = reinterpret_cast<const float4*>(xs + (c * 32 + lane) * 8);
    const float4 v0 = p[0], v1 = p[1];
    xr[c][0] = make_float2(v0.x, v0.y);
    xr[c][1] = make_float2(v0.z, v0.w);
    xr[c][2] = make_float2(v1.x, v1.y);
    xr[c][3] = make_float2(v1.z, v1.w);
  }

  float bv = kNegMax;
  uint32_t bi = 0;
  for (int base = 0; gw + base * W < a.vocab; base += U) {
    uint4 nxt[U][KC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r = gw + (base + U + u) * W;
#pragma unroll
      for (int c = 0; c < KC; ++c)
        nxt[u][c] = (r < a.vocab) ? ld_stream(a.table + (size_t)r * rpr + c * 32 + lane) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r = gw + (base + u) * W;
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < KC; ++c) acc = f16x8_dot(cur[u][c], xr[c], acc);
      const float v = warp_sum(acc.x + acc.y);
      if (r < a.vocab) {
        if (lane == 0 && a.logits) a.logits[r] = v;
        if (am_better(v, (uint32_t)r, bv, bi)) { bv = v; bi = (uint32_t)r; }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int c = 0; c < KC; ++c) cur[u][c] = nxt[u][c];
  }

  if (lane == 0) { bv_s[warp] = bv; bi_s[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = bv_s[0];
    uint32_t i = bi_s[0];
    for (int w = 1; w < kWarps; ++w)
      if (am_better(bv_s[w], bi_s[w], v, i)) { v = bv_s[w]; i = bi_s[w]; }
    a.part_v[blockIdx.x] = v;
    a.part_i[blockIdx.x] = i;
    __threadfence();
    const unsigned prev = atomicAdd(a.counter, 1u);
    am_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!am_last) return;
  __threadfence();
  float v = kNegMax;
  uint32_t i = 0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += kThreads) {
    const float pv = __ldcg(a.part_v + b);
    const uint32_t pi = __ldcg(a.part_i + b);
    if (am_better(pv, pi, v, i)) { v = pv; i = pi; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (am_better(ov, oi, v, i)) { v = ov; i = oi; }
  }
  if (lane == 0) { bv_s[warp] = v; bi_s[warp] = i; }
  __syncthreads();
  if (threadIdx.x == 0) {
    v = bv_s[0];
    i = bi_s[0];
    for (int w = 1; w < kWarps; ++w)
      if (am_better(bv_s[w], bi_s[w], v, i)) { v = bv_s[w]; i = bi_s[w]; }
    a.result[0] = i;
    a.result[1] = __float_as_uint(v);
    *a.counter = 0u;
    if (a.st) {
      const int pos = a.st->pos, step = a.st->step;
      if (pos + 1 <= a.max_seq) a.tokens[pos + 1] = (int)i;
      if (step < a.st->max_new) {
        a.out_dev[step] = (int)i;
        if (a.out_host) *reinterpret_cast<volatile int*>(a.out_host + step) = (int)i;
      }
      a.st->step = step + 1;
      a.st->pos = pos + 1;
    }
  }
}

// Move the decode position (stepping interface); keeps the step counter.
static __global__ void k_seek(DevState* st, int pos) {
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) st->pos = pos;
}

// Advance the position after a prompt token that needs no LM head.
static __global__ void k_advance(DevState* st) {
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) st->pos += 1;
}

}  // namespace qd
