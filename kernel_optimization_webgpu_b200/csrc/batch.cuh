// Batched decode and prefill kernels: many independent sequences advance
// together, so the q4 projections and the LM head are dense contractions on the
// tensor cores (gemm_tc.cuh) and everything between two GEMMs is one fused
// kernel that also sums the GEMM's split-K partials in a fixed order.
//
// Layer order per step (the reference's decode layer, webgpu-runtime.js:498-562,
// with B rows instead of one):
//   kb_resid_norm   h += sum(partials of the previous down GEMM); x = rms(h)*w_in -> hi/lo
//   GEMM qkv        [B][q|k|v] partials
//   kb_rope_cache   head RMSNorm + RoPE on q and k, K/V rows appended to the cache
//   kb_attn         split-KV attention, K/V tiles bulk-copied into shared memory
//   kb_attn_combine splits merged -> hi/lo operand of the o GEMM
//   GEMM o          partials
//   kb_resid_norm   h += sum(o partials); x = rms(h)*w_post -> hi/lo
//   GEMM gate/up    interleaved partials
//   kb_silu_split   silu(gate)*up -> hi/lo
//   GEMM down       partials (consumed by the next layer's kb_resid_norm)
// and after the last layer kb_resid_norm with the final norm, the LM head GEMM
// with its (max, index) epilogue and kb_argmax_merge.
//
// KV cache of the batched path: [layer][seq][kv_head][pos][128] f16, so the 64
// cached rows of one (sequence, KV head) tile are one contiguous 16 KB range
// that a single cp.async.bulk moves into shared memory.
#pragma once

#include "common.cuh"
#include "gemm_tc.cuh"
#include "tma.cuh"

namespace qd {

constexpr int kBAttnTile = 64;  // positions per staged K/V tile
constexpr int kBAttnThreads = 256;
constexpr int kBErrTimeout = 16;
constexpr int kMaxParts = 16;   // split-K partials a consumer kernel sums (GEMM split plans stay within)
// One stage of kb_attn: K and V tiles, each as two 64-position x 64-dim boxes
// (128-byte rows, 128-byte swizzle), 8 KB per box.
constexpr int kBAttnBox = kBAttnTile * 64 * 2;
constexpr int kBAttnStage = 4 * kBAttnBox;
// K/V stages of kb_attn's ring and its dynamic shared memory (plus alignment slack
// for the swizzle atoms). Two stages (65 KB, three CTAs per SM) measured best at
// 64 sequences x 2048 positions: three stages (two CTAs per SM) ran 7% slower and
// four (one CTA per SM) 30% slower; the attention warps' latency, not the bytes in
// flight, sets the pace.
constexpr int kBAttnStages = 2;
constexpr int kBAttnSmem = kBAttnStages * kBAttnStage + 1024;

struct BatchState {
  int* tokens;    // [B] input token of the step (the previous step's output)
  int* pos;       // [B] position the step writes and attends up to
  int* out;       // [max_steps][B] generated ids
  int* step;      // [1] steps taken since the last reset
  int max_steps;
};

// Sum of the split-K partials of element i: parts[s * stride + i], s ascending
// (nparts <= kMaxParts). The loads are unconditional (indices clamped to the
// last split) so that all of them are in flight before the first add.
template <int MAXP>
__device__ __forceinline__ float sum_parts_n(const float* parts, int nparts, long long stride, long long i) {
  float v[MAXP];
#pragma unroll
  for (int s = 0; s < MAXP; ++s) v[s] = parts[(long long)min(s, nparts - 1) * stride + i];
  float acc = v[0];
#pragma unroll
  for (int s = 1; s < MAXP; ++s)
    if (s < nparts) acc += v[s];
  return acc;
}

__device__ __forceinline__ float sum_parts(const float* parts, int nparts, long long stride, long long i) {
  if (nparts <= 4) return sum_parts_n<4>(parts, nparts, stride, i);
  if (nparts <= 8) return sum_parts_n<8>(parts, nparts, stride, i);
  return sum_parts_n<kMaxParts>(parts, nparts, stride, i);
}

// ---- residual + RMSNorm into the GEMM's hi/lo operands ----------------------------
// Row b (one CTA of 256 threads, 4 consecutive elements per thread and pass):
// h[b] = embed row of tokens[b] (embedding mode), or h[b] + sum(parts) (residual
// mode; parts == nullptr leaves h as is); then x = rms_norm(h[b]) * w ->
// x_hi[b], x_lo[b]. h is written back in place. K is a multiple of 4, <= 4096.
constexpr int kNormThreads = 256;
static __global__ void __launch_bounds__(kNormThreads) kb_resid_norm(float* h, const float* parts, int nparts,
                                                                     long long part_stride, const __half* embed,
                                                                     const int* tokens, int vocab, const float* w,
                                                                     int K, float eps, __half* x_hi, __half* x_lo,
                                                                     int* err) {
  constexpr int kMaxPer = 4;  // float4 items per thread (K <= 4096)
  __shared__ float red[kNormThreads / 32];
  pdl_wait();
  const int b = blockIdx.x;
  float4* hr = reinterpret_cast<float4*>(h + (long long)b * K);
  const __half* er = nullptr;
  if (embed) {
    int tok = tokens[b];
    if (tok < 0 || tok >= vocab) {
      if (threadIdx.x == 0) atomicOr(err, kErrToken);
      tok = 0;
    }
    er = embed + (long long)tok * K;
  }
  const int K4 = K >> 2;
  float4 v[kMaxPer];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int e4 = threadIdx.x + k * kNormThreads;
    if (e4 >= K4) break;
    float4 x;
    if (er) {
      const uint2 u = *reinterpret_cast<const uint2*>(er + 4 * e4);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      x = make_float4(a.x, a.y, c.x, c.y);
    } else {
      x = hr[e4];
      if (parts) {
        const long long i4 = (long long)b * K4 + e4;
        const float4* p4 = reinterpret_cast<const float4*>(parts);
        const long long s4 = part_stride >> 2;
        float4 acc = p4[i4];
        if (nparts > 1) {
          float4 pv[kMaxParts - 1];
#pragma unroll
          for (int s = 1; s < kMaxParts; ++s) pv[s - 1] = p4[(long long)min(s, nparts - 1) * s4 + i4];
#pragma unroll
          for (int s = 1; s < kMaxParts; ++s)
            if (s < nparts) {
              acc.x += pv[s - 1].x;
              acc.y += pv[s - 1].y;
              acc.z += pv[s - 1].z;
              acc.w += pv[s - 1].w;
            }
        }
        x.x += acc.x;
        x.y += acc.y;
        x.z += acc.z;
        x.w += acc.w;
      }
    }
    if (er || parts) hr[e4] = x;
    v[k] = x;
    ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  pdl_trigger();
  float t = 0.0f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) t += red[k];
  const float inv = rsqrtf(t / (float)K + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int e4 = threadIdx.x + k * kNormThreads;
    if (e4 >= K4) break;
    const float4 ww = w4[e4];
    __half h0, l0, h1, l1, h2, l2, h3, l3;
    split_f16(v[k].x * inv * ww.x, h0, l0);
    split_f16(v[k].y * inv * ww.y, h1, l1);
    split_f16(v[k].z * inv * ww.z, h2, l2);
    split_f16(v[k].w * inv * ww.w, h3, l3);
    __half2 hh[2] = {__halves2half2(h0, h1), __halves2half2(h2, h3)};
    __half2 ll[2] = {__halves2half2(l0, l1), __halves2half2(l2, l3)};
    *reinterpret_cast<uint2*>(x_hi + (long long)b * K + 4 * e4) = *reinterpret_cast<const uint2*>(hh);
    *reinterpret_cast<uint2*>(x_lo + (long long)b * K + 4 * e4) = *reinterpret_cast<const uint2*>(ll);
  }
}

// The same with one warp per row, for many rows of K = 128 NV columns (prefill):
// lane l holds float4s l, l + 32, ... of the row, so each lane has all its h and
// partial loads in flight at once and the sum of squares needs no CTA barrier.
// Partials: parts[s * part_stride + row * K + e], s < nparts, added in order.
template <int NV>
static __global__ void __launch_bounds__(kNormThreads) kb_resid_norm_rows(float* h, const float* parts, int nparts,
                                                                          long long part_stride, const __half* embed,
                                                                          const int* tokens, int vocab, const float* w,
                                                                          int rows, float eps, __half* x_hi,
                                                                          __half* x_lo, int* err) {
  constexpr int K = 128 * NV;
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long b = (long long)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (b >= rows) {
    pdl_trigger();
    return;
  }
  float4 v[NV];
  float4* hr = reinterpret_cast<float4*>(h + b * K);
  if (embed) {
    int tok = tokens[b];
    if (tok < 0 || tok >= vocab) {
      if (lane == 0) atomicOr(err, kErrToken);
      tok = 0;
    }
    const uint2* er = reinterpret_cast<const uint2*>(embed + (long long)tok * K);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint2 u = er[lane + 32 * i];
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[i] = make_float4(a.x, a.y, c.x, c.y);
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = hr[lane + 32 * i];
    if (parts) {
      const float4* p4 = reinterpret_cast<const float4*>(parts) + b * (K / 4);
      float4 acc[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) acc[i] = p4[lane + 32 * i];
      for (int s = 1; s < nparts; ++s) {
        const float4* ps = p4 + (long long)s * (part_stride >> 2);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const float4 y = ps[lane + 32 * i];
          acc[i].x += y.x;
          acc[i].y += y.y;
          acc[i].z += y.z;
          acc[i].w += y.w;
        }
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        v[i].x += acc[i].x;
        v[i].y += acc[i].y;
        v[i].z += acc[i].z;
        v[i].w += acc[i].w;
      }
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  ss = warp_sum(ss);
  pdl_trigger();
  const float inv = rsqrtf(ss / (float)K + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int e4 = lane + 32 * i;
    if (embed || parts) hr[e4] = v[i];
    const float4 ww = w4[e4];
    __half h0, l0, h1, l1, h2, l2, h3, l3;
    split_f16(v[i].x * inv * ww.x, h0, l0);
    split_f16(v[i].y * inv * ww.y, h1, l1);
    split_f16(v[i].z * inv * ww.z, h2, l2);
    split_f16(v[i].w * inv * ww.w, h3, l3);
    __half2 hh[2] = {__halves2half2(h0, h1), __halves2half2(h2, h3)};
    __half2 ll[2] = {__halves2half2(l0, l1), __halves2half2(l2, l3)};
    *reinterpret_cast<uint2*>(x_hi + b * K + 4 * e4) = *reinterpret_cast<const uint2*>(hh);
    *reinterpret_cast<uint2*>(x_lo + b * K + 4 * e4) = *reinterpret_cast<const uint2*>(ll);
  }
}

// ---- head RMSNorm + RoPE + KV append --------------------------------------------
// Row r of a GEMM output laid out [q_heads*128 | NKV*128 (k) | NKV*128 (v)]
// (split-K partials, summed here). Row r belongs to sequence
// seq = (row0 + r) / rows_per_seq at position
// (pos ? pos[seq] : 0) + (row0 + r) % rows_per_seq.
// One warp per kRopeTasks consecutive head tasks: q heads are normalised,
// rotated and stored to q_out [r][q_heads*128]; k heads normalised, rotated
// (rope.wgsl:14-31, table offset position * row_stride + pair) and appended to
// the cache; v heads appended as projected. Cache row (seq, g, p) sits at
// ((seq*NKV + g)*max_seq + p)*128. The warp issues the partial loads of all
// its tasks before the first reduction, so that kRopeTasks * 512 bytes of
// partials per warp are in flight at once.
constexpr int kRopeTasks = 4;
template <bool kSplit>
static __global__ void __launch_bounds__(256, kSplit ? 2 : 3) kb_rope_cache(const float* parts, int nparts, long long part_stride, int R,
                                                     int q_heads, int NKV, const float* norm_q, const float* norm_k,
                                                     float eps, const float* cos_t, const float* sin_t, int row_stride,
                                                     const int* pos, int rows_per_seq, long long row0, int max_seq,
                                                     __half* kc, __half* vc, float* q_out, int* err) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tasks = q_heads + 2 * NKV;
  const int ld = tasks * kHeadDim;
  const int nt = R * tasks;  // the host keeps R * tasks and row0 + R below 2^31
  const int r0 = (int)row0;
  const int pair0 = (4 * lane) & (kHeadDim / 2 - 1);
  for (int t0 = (blockIdx.x * 8 + warp) * kRopeTasks; t0 < nt; t0 += gridDim.x * 8 * kRopeTasks) {
    // the partials of every task first (several loads in flight), in split order
    float4 x[kRopeTasks];
#pragma unroll
    for (int i = 0; i < kRopeTasks; ++i) {
      const int task = min(t0 + i, nt - 1);
      const int r = task / tasks, t = task - r * tasks;
      x[i] = __ldg(reinterpret_cast<const float4*>(parts + (long long)r * ld + (long long)t * kHeadDim) + lane);
    }
    // split-K partials, added in split order. kSplit (decode, short prompts: up to 16
    // splits): four splits' loads in flight at once (split indices clamped, the extra
    // loads unused; 126 registers, two CTAs per SM). Otherwise (one split, the
    // prefill's wide launches: three CTAs per SM) one split after another.
    if constexpr (!kSplit) {
      for (int s = 1; s < nparts; ++s) {
#pragma unroll
        for (int i = 0; i < kRopeTasks; ++i) {
          const int task = min(t0 + i, nt - 1);
          const int r = task / tasks, t = task - r * tasks;
          const float4 y = __ldg(reinterpret_cast<const float4*>(parts + (long long)s * part_stride +
                                                                 (long long)r * ld + (long long)t * kHeadDim) + lane);
          x[i].x += y.x;
          x[i].y += y.y;
          x[i].z += y.z;
          x[i].w += y.w;
        }
      }
    } else {
     for (int s0 = 1; s0 < nparts; s0 += 4) {
      float4 y[4][kRopeTasks];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long so = (long long)min(s0 + u, nparts - 1) * part_stride;
#pragma unroll
        for (int i = 0; i < kRopeTasks; ++i) {
          const int task = min(t0 + i, nt - 1);
          const int r = task / tasks, t = task - r * tasks;
          y[u][i] = __ldg(reinterpret_cast<const float4*>(parts + so + (long long)r * ld + (long long)t * kHeadDim) + lane);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (s0 + u < nparts) {
#pragma unroll
          for (int i = 0; i < kRopeTasks; ++i) {
            x[i].x += y[u][i].x;
            x[i].y += y[u][i].y;
            x[i].z += y[u][i].z;
            x[i].w += y[u][i].w;
          }
        }
     }
    }
#pragma unroll
    for (int i = 0; i < kRopeTasks; ++i) {
      const int task = t0 + i;
      if (task >= nt) break;
      const int r = task / tasks, t = task - r * tasks;
      const int grow = r0 + r;
      const int seq = grow / rows_per_seq;
      const int p = (pos ? pos[seq] : 0) + (grow - seq * rows_per_seq);
      if (p < 0 || p >= max_seq) {
        if (lane == 0) atomicOr(err, kErrPosition);
        continue;
      }
      if (t >= q_heads + NKV) {  // v: cached as projected
        const int g = t - q_heads - NKV;
        __half* dst = vc + (((long long)seq * NKV + g) * max_seq + p) * kHeadDim + 4 * lane;
        reinterpret_cast<__half2*>(dst)[0] = __floats2half2_rn(x[i].x, x[i].y);
        reinterpret_cast<__half2*>(dst)[1] = __floats2half2_rn(x[i].z, x[i].w);
        continue;
      }
      const long long toff = (long long)p * row_stride + pair0;
      const float4 c = __ldg(reinterpret_cast<const float4*>(cos_t + toff));
      const float4 sn = __ldg(reinterpret_cast<const float4*>(sin_t + toff));
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(t < q_heads ? norm_q : norm_k) + lane);
      float ss = x[i].x * x[i].x + x[i].y * x[i].y + x[i].z * x[i].z + x[i].w * x[i].w;
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)kHeadDim + eps);
      const float4 y = make_float4(x[i].x * inv * w4.x, x[i].y * inv * w4.y, x[i].z * inv * w4.z, x[i].w * inv * w4.w);
      // rotate-half: dims d and d +- 64 sit 16 lanes apart
      float4 pr;
      pr.x = __shfl_xor_sync(0xffffffffu, y.x, 16);
      pr.y = __shfl_xor_sync(0xffffffffu, y.y, 16);
      pr.z = __shfl_xor_sync(0xffffffffu, y.z, 16);
      pr.w = __shfl_xor_sync(0xffffffffu, y.w, 16);
      const float sg = lane < 16 ? -1.0f : 1.0f;  // first half: x*cos - x[d+64]*sin
      const float4 o = make_float4(y.x * c.x + sg * pr.x * sn.x, y.y * c.y + sg * pr.y * sn.y,
                                   y.z * c.z + sg * pr.z * sn.z, y.w * c.w + sg * pr.w * sn.w);
      if (t < q_heads) {
        reinterpret_cast<float4*>(q_out + (long long)r * q_heads * kHeadDim + (long long)t * kHeadDim)[lane] = o;
      } else {
        const int g = t - q_heads;
        __half* dst = kc + (((long long)seq * NKV + g) * max_seq + p) * kHeadDim + 4 * lane;
        reinterpret_cast<__half2*>(dst)[0] = __floats2half2_rn(o.x, o.y);
        reinterpret_cast<__half2*>(dst)[1] = __floats2half2_rn(o.z, o.w);
      }
    }
  }
  pdl_trigger();
}

// Grid of kb_rope_cache for nt head tasks: one warp per kRopeTasks tasks, capped
// (the kernel strides over the rest).
inline int rope_grid_for(long long nt, long long cap) {
  const long long per_cta = 8LL * kRopeTasks;
  return (int)std::max<long long>(1, std::min<long long>((nt + per_cta - 1) / per_cta, cap));
}

// ---- split-KV decode attention with TMA staging ------------------------------------
// Grid (NKV, splits, B); 256 threads (8 warps) serve the G query heads of KV head g.
// The CTA covers positions [sp*split_len, min(len, (sp+1)*split_len)) of
// sequence b, len = pos[b] + 1, in 64-position tiles double-buffered through
// shared memory by TMA: K and V as two 64x64 boxes each with the 128-byte
// swizzle (16-byte chunk c of row r sits at chunk c ^ (r & 7)). Thread 0
// refills a stage once all 8 warps have arrived on its "empty" barrier.
//
// Warp w owns positions 8w..8w+7 of every tile and keeps its own online softmax
// (running max, sum, P*V accumulator): scores with 4 lanes per position (lane =
// position + 8 * chunk group; the swizzle makes the 8 rows of a load phase hit
// distinct banks), two shuffles to finish each dot, three for the warp's tile
// max and sum; P*V with lane = 4 dims. No CTA barrier inside the tile loop; the
// 8 warps' states are merged once at the end.
// Partials: ml[b][sp][h] = (max, sum of exp), o[b][sp][h][128] unnormalised.
template <int G>
__global__ void __launch_bounds__(kBAttnThreads) kb_attn(const __grid_constant__ CUtensorMap kvmap, long long k_row0,
                                                          long long v_row0, const float* q, const int* pos, int NH,
                                                          int NKV, int max_seq, int split_len, int splits, float scale,
                                                          float2* part_ml, float* part_o, int* err) {
  extern __shared__ unsigned char attn_raw[];
  unsigned char* stages =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(attn_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kWarps = kBAttnThreads / 32;
  __shared__ __align__(16) float qsm[G][kHeadDim];
  __shared__ float wm[kWarps][G], wl[kWarps][G];
  constexpr int kS = kBAttnStages;
  __shared__ unsigned long long full[kS], empty[kS];
  __shared__ int failed;
  const int g = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < kS; ++i) {
      tc_mbar_init(&full[i]);
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc_smem(&empty[i])), "r"(kWarps) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_map(&kvmap);
    failed = 0;
  }
  pdl_wait();
  const int len = min(pos[b], max_seq - 1) + 1;
  const int lo = sp * split_len, hi = min(len, lo + split_len);
  const long long slot = ((long long)b * splits + sp) * NH + (long long)g * G;
  if (lo >= hi) {
    if (tid < G) part_ml[slot + tid] = make_float2(-INFINITY, 0.0f);
    for (int e = tid; e < G * kHeadDim; e += kBAttnThreads) part_o[slot * kHeadDim + e] = 0.0f;
    pdl_trigger();
    return;
  }
  const long long seq_row = ((long long)b * NKV + g) * max_seq;
  const int nt = (hi - lo + kBAttnTile - 1) / kBAttnTile;
  auto issue = [&](int t) {  // one thread: tile t into stage t % kS
    const long long row = seq_row + lo + (long long)t * kBAttnTile;
    unsigned long long* mb = &full[t % kS];
    unsigned char* st = stages + (t % kS) * kBAttnStage;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(mb)), "r"(kBAttnStage)
                 : "memory");
    // KV rows are read once per step: evict-first keeps the step's small tensors in L2
    const unsigned long long pol = l2_evict_first();
    tma_load_2d_hint(st, &kvmap, 0, (int)(k_row0 + row), mb, pol);
    tma_load_2d_hint(st + kBAttnBox, &kvmap, 64, (int)(k_row0 + row), mb, pol);
    tma_load_2d_hint(st + 2 * kBAttnBox, &kvmap, 0, (int)(v_row0 + row), mb, pol);
    tma_load_2d_hint(st + 3 * kBAttnBox, &kvmap, 64, (int)(v_row0 + row), mb, pol);
  };
  __syncthreads();  // barrier init visible
  int issued = 0;   // thread 0 only
  if (tid == 0)
    for (; issued < min(kS, nt); ++issued) issue(issued);
  for (int e = tid; e < G * kHeadDim; e += kBAttnThreads)
    qsm[e / kHeadDim][e % kHeadDim] = q[((long long)b * NH + (long long)g * G) * kHeadDim + e];
  __syncthreads();

  const int pl = lane & 7, l4 = lane >> 3;  // scores: position 8w + pl, chunk group l4
  float m_run[G], l_run[G], acc[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.0f;
    acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.0f;
  }
  // P*V: lane holds dims 4*lane .. 4*lane + 3 (half lane >> 4 of the row)
  const int vcol = (4 * lane) & 63, vcc = vcol >> 3, vhalf = lane >> 4;
  int consumed = 0;  // tiles this warp has waited for
  bool ok = true;
  for (int t = 0; t < nt && ok; ++t) {
    const int buf = t % kS;
    if (tid == 0 && t >= 1 && t - 1 + kS < nt) {  // refill the stage tile t-1 used with tile t-1+kS
      ok = tc_mbar_wait(&empty[(t - 1) % kS], (unsigned)((t - 1) / kS) & 1u);
      if (ok) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(t - 1 + kS);
        issued = t + kS;
      }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (ok) ok = tc_mbar_wait(&full[buf], (unsigned)(t / kS) & 1u);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    consumed = t + 1;
    const int n = min(kBAttnTile, hi - (lo + t * kBAttnTile));
    const unsigned char* st = stages + buf * kBAttnStage;
    const int j = 8 * warp + pl;
    // scores
    float s[G];
#pragma unroll
    for (int h = 0; h < G; ++h) s[h] = 0.0f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int c = l4 + 4 * m;  // 16-byte chunk of the row (dims 8c .. 8c+7)
      const uint4 u = *reinterpret_cast<const uint4*>(st + (c >> 3) * kBAttnBox + j * 128 + (((c & 7) ^ pl) << 4));
      const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
      const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float4 qa = reinterpret_cast<const float4*>(qsm[h])[2 * c];
        const float4 qb = reinterpret_cast<const float4*>(qsm[h])[2 * c + 1];
        s[h] += qa.x * k0.x + qa.y * k0.y + qa.z * k1.x + qa.w * k1.y + qb.x * k2.x + qb.y * k2.y + qb.z * k3.x +
                qb.w * k3.y;
      }
    }
    float p[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      s[h] += __shfl_xor_sync(0xffffffffu, s[h], 8);
      s[h] += __shfl_xor_sync(0xffffffffu, s[h], 16);
      const float sv = j < n ? s[h] * scale : -INFINITY;
      float tm = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, 1));
      tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 2));
      tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 4));
      const float mn = fmaxf(m_run[h], tm);  // finite: the warp holds at least one valid position or mn = m_run
      p[h] = (j < n) ? expf(sv - mn) : 0.0f;
      float ps = p[h] + __shfl_xor_sync(0xffffffffu, p[h], 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      const float f = (m_run[h] == -INFINITY) ? 0.0f : expf(m_run[h] - mn);
      if (mn != -INFINITY) {
        l_run[h] = l_run[h] * f + ps;
        m_run[h] = mn;
        acc[h][0] *= f;
        acc[h][1] *= f;
        acc[h][2] *= f;
        acc[h][3] *= f;
      }
    }
    // P*V over the warp's 8 positions
    const unsigned char* vrow = st + (2 + vhalf) * kBAttnBox + (vcol & 7) * 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int jj = 8 * warp + k;
      float pk[G];
#pragma unroll
      for (int h = 0; h < G; ++h) pk[h] = __shfl_sync(0xffffffffu, p[h], k);
      if (jj < n) {
        const uint2 u = *reinterpret_cast<const uint2*>(vrow + jj * 128 + ((vcc ^ k) << 4));
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
#pragma unroll
        for (int h = 0; h < G; ++h) {
          acc[h][0] += pk[h] * v01.x;
          acc[h][1] += pk[h] * v01.y;
          acc[h][2] += pk[h] * v23.x;
          acc[h][3] += pk[h] * v23.y;
        }
      }
    }
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc_smem(&empty[buf])) : "memory");
  }
  if (!ok && lane == 0) atomicOr(&failed, 1);
  __syncthreads();
  if (failed) {
    // Copies still in flight land in this CTA's shared memory: give each a
    // bounded chance to finish before exiting.
    if (tid == 0) {
      for (int t = consumed; t < issued; ++t) (void)tc_mbar_wait(&full[t % kS], (unsigned)(t / kS) & 1u);
      atomicOr(err, kBErrTimeout);
    }
    pdl_trigger();
    return;
  }
  pdl_trigger();
  // Merge the 8 warps' softmax states (the stages are free now: every tile was consumed).
  float* wo = reinterpret_cast<float*>(stages);  // [kWarps][G][128]
#pragma unroll
  for (int h = 0; h < G; ++h) {
    *reinterpret_cast<float4*>(&wo[(warp * G + h) * kHeadDim + 4 * lane]) =
        make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    if (lane == 0) {
      wm[warp][h] = m_run[h];
      wl[warp][h] = l_run[h];
    }
  }
  __syncthreads();
  if (tid < G * kHeadDim) {
    const int h = tid / kHeadDim, d = tid % kHeadDim;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w][h]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = wm[w][h] == -INFINITY ? 0.0f : expf(wm[w][h] - M);
      L += wl[w][h] * f;
      O += wo[(w * G + h) * kHeadDim + d] * f;
    }
    part_o[(slot + h) * kHeadDim + d] = O;
    if (d == 0) part_ml[slot + h] = make_float2(M, L);
  }
}

// Merge the splits of head h (blockIdx.x) of row b (blockIdx.y) into the o GEMM's
// operands x_hi/x_lo [B][NH*128]; one thread per dim.
static __global__ void __launch_bounds__(kHeadDim) kb_attn_combine(const float2* part_ml, const float* part_o,
                                                                   int splits, int NH, __half* x_hi, __half* x_lo) {
  pdl_wait();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x, QS = NH * kHeadDim;
  const float2* ml = part_ml + (long long)b * splits * NH + h;
  const float* po = part_o + (long long)b * splits * QS + (long long)h * kHeadDim + d;
  float M = -INFINITY, L = 0.0f, O = 0.0f;
  // Up to 8 splits at a time: all of their loads in flight before the first use.
  for (int s0 = 0; s0 < splits; s0 += 8) {
    float2 m[8];
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int s = min(s0 + k, splits - 1);
      m[k] = ml[(long long)s * NH];
      o[k] = po[(long long)s * QS];
    }
    float Mc = M;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (s0 + k < splits) Mc = fmaxf(Mc, m[k].x);
    // rescale what the earlier groups summed (online softmax over split groups)
    const float r = (M == -INFINITY) ? 0.0f : expf(M - Mc);
    L *= r;
    O *= r;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (s0 + k < splits) {
        const float f = m[k].y > 0.0f ? expf(m[k].x - Mc) : 0.0f;
        L += m[k].y * f;
        O += o[k] * f;
      }
    M = Mc;
  }
  pdl_trigger();
  __half hh, ll;
  split_f16(O / L, hh, ll);
  x_hi[(long long)b * QS + h * kHeadDim + d] = hh;
  x_lo[(long long)b * QS + h * kHeadDim + d] = ll;
}

// silu(gate) * up from the gate/up GEMM's interleaved partials (column 2j = gate
// row j, 2j+1 = up row j) -> the down GEMM's operands x_hi/x_lo [B][I].
static __global__ void __launch_bounds__(256) kb_silu_split(const float* parts, int nparts, long long part_stride, int B,
                                                     int I, __half* x_hi, __half* x_lo) {
  pdl_wait();
  const long long n = (long long)B * I;
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
    const long long b = i / I, j = i % I;
    const long long gi = b * 2 * I + 2 * j;
    const float gv = sum_parts(parts, nparts, part_stride, gi);
    const float uv = sum_parts(parts, nparts, part_stride, gi + 1);
    const float act = gv / (1.0f + expf(-gv)) * uv;
    __half hh, ll;
    split_f16(act, hh, ll);
    x_hi[i] = hh;
    x_lo[i] = ll;
  }
  pdl_trigger();
}

// Per-row merge of the LM head's per-CTA (max, index) pairs (ties: lowest
// index; NaN never wins), then the token is fed back and recorded and the
// position advanced. One warp per row.
static __global__ void __launch_bounds__(256) kb_argmax_merge(const float* part_v, const uint32_t* part_i, int nparts, int B,
                                                       BatchState st, uint32_t* result) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + warp;
  if (b < B) {
    float bv = kNegMax;
    uint32_t bi = 0;
    for (int k = lane; k < nparts; k += 32) {
      const float v = part_v[(long long)b * nparts + k];
      const uint32_t i = part_i[(long long)b * nparts + k];
      if (am_better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (am_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      if (result) {
        result[2 * b] = bi;
        result[2 * b + 1] = __float_as_uint(bv);
      }
      if (st.tokens) {
        const int s = *st.step;
        st.tokens[b] = (int)bi;
        st.pos[b] += 1;
        if (s < st.max_steps) st.out[(long long)s * B + b] = (int)bi;
      }
    }
  }
  pdl_trigger();
}

// Vocabulary-sharded LM head, last step: ranks r < world each hold (index, value
// bits) pairs of every rank's rows over their vocabulary slice, all[w][row][2]
// with row = rank * B + b. Row b of this rank takes the best of the world
// candidates (larger value, then lower index: slices are in vocabulary order)
// and feeds it back like kb_argmax_merge.
static __global__ void __launch_bounds__(256) kb_shard_merge(const uint32_t* all, int world, int rank, int B,
                                                             BatchState st) {
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    float bv = kNegMax;
    uint32_t bi = 0;
    for (int w = 0; w < world; ++w) {
      const long long o = ((long long)w * world * B + (long long)rank * B + b) * 2;
      const uint32_t i = all[o];
      const float v = __uint_as_float(all[o + 1]);
      if (am_better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
    const int s = *st.step;
    st.tokens[b] = (int)bi;
    st.pos[b] += 1;
    if (s < st.max_steps) st.out[(long long)s * B + b] = (int)bi;
  }
  pdl_trigger();
}

static __global__ void kb_step_done(int* step) {
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) *step += 1;
  pdl_trigger();
}

// ---- seeded synthetic context ---------------------------------------------------
// Integer hash (a 32-bit finaliser of the xorshift-multiply family).
__host__ __device__ __forceinline__ uint32_t ctx_hash(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// Hidden-state value d of context row `row` (= seq * ctx + position) of
// `layer`: the sum of four 24-bit uniforms from the hash, centred and scaled to
// unit variance (an Irwin-Hall approximation of N(0, 1)). Integer work and two
// f32 multiplies (the first by a power of two), so any IEEE host reproduces it.
__host__ __device__ __forceinline__ float ctx_normal(uint32_t seed, uint32_t layer, uint32_t row, uint32_t d,
                                                    uint32_t H) {
  const uint32_t key = ctx_hash(seed * 0x9E3779B9u + layer * 0x85EBCA6Bu + 0x632BE5ABu);
  const uint32_t base = (row * H + d) * 4u;
  int s = 0;
  for (uint32_t j = 0; j < 4; ++j) s += (int)(ctx_hash(key ^ (base + j)) >> 8);
  s -= 2 << 24;
  return ((float)s * 5.9604644775390625e-08f) * 1.7320508f;
}

// Rows [row0, row0 + R) of the synthetic hidden states of `layer`, RMS-normed
// with the layer's input norm into the k/v GEMM's operands x_hi/x_lo [R][H].
static __global__ void __launch_bounds__(256) kb_ctx_hidden(uint32_t seed, uint32_t layer, long long row0, int H,
                                                     const float* w, float eps, __half* x_hi, __half* x_lo) {
  __shared__ float red[8];
  __shared__ float row[4096];
  pdl_wait();
  const long long r = blockIdx.x;
  const uint32_t grow = (uint32_t)(row0 + r);
  float ss = 0.0f;
  for (int e = threadIdx.x; e < H; e += 256) {
    const float v = ctx_normal(seed, layer, grow, (uint32_t)e, (uint32_t)H);
    row[e] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  pdl_trigger();
  float t = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) t += red[k];
  const float inv = rsqrtf(t / (float)H + eps);
  for (int e = threadIdx.x; e < H; e += 256) {
    __half hi, lo;
    split_f16(row[e] * inv * w[e], hi, lo);
    x_hi[r * H + e] = hi;
    x_lo[r * H + e] = lo;
  }
}

// ---- causal prefill attention (tensor cores) ------------------------------------------
// Grid (NKV, ceil(n / 64), B); 128 * G threads. CTA = one 64-position query tile
// of prompt b and the G query heads of KV head g; warp w takes head w / 4 and
// positions 16 (w % 4) .. + 15 of the tile. Key/value tiles (64 positions) come
// from the cache by TMA (same tensor map and 128-byte swizzle as decode),
// double-buffered; tiles 0 .. qt are visited, the diagonal one masked.
//
// Math on mma.sync m16n8k16 (f16 in, f32 accumulate): S = Q K^T with Q split
// into f16 hi + lo parts (K is exact in f16), online softmax per row in
// registers, O += P V with P split the same way (V exact). ldmatrix reads the
// swizzled tiles conflict-free. The output rows (O / l) are written as the hi/lo
// operands of the o GEMM: x_hi/x_lo [T][NH*128], T = B * n.
constexpr int kPfTile = 64;
constexpr int kPfQBytes = kPfTile * 64 * 2;  // one 64-position x 64-dim f16 half of a head's Q tile

__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0,
                                         unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ unsigned pack_h2(float lo_elem, float hi_elem) {
  const __half2 h = __floats2half2_rn(lo_elem, hi_elem);
  return *reinterpret_cast<const unsigned*>(&h);
}
// f16 hi/lo split of a pair: hi = f16(x), lo = f16(x - hi) (unscaled).
__device__ __forceinline__ void split_pair(float x0, float x1, unsigned& hi, unsigned& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const unsigned*>(&h);
  lo = pack_h2(x0 - hf.x, x1 - hf.y);
}
// Byte offset of (row r, 16-byte chunk c of the 64-dim half) in a 128-byte-swizzled box.
__device__ __forceinline__ unsigned swz(int r, int c) { return (unsigned)(r * 128 + (((c ^ r) & 7) << 4)); }

template <int G>
__global__ void __launch_bounds__(128 * G) kb_prefill_attn(const __grid_constant__ CUtensorMap kvmap, long long k_row0,
                                                           long long v_row0, const float* q, int n, int NH, int NKV,
                                                           int max_seq, float scale, __half* x_hi, __half* x_lo,
                                                           int* err) {
  extern __shared__ unsigned char pf_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* kv = base;                          // [2 stages][K0 K1 V0 V1] boxes of 8 KB
  unsigned char* qs = base + 2 * kBAttnStage;        // [G][hi|lo][2 halves] boxes of 8 KB
  __shared__ unsigned long long full[2];
  const int g = blockIdx.x, b = blockIdx.z;
  const int qt = (int)gridDim.y - 1 - (int)blockIdx.y;  // longest tiles first
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = warp >> 2, wq = warp & 3;  // head within the group, 16-row slice of the tile
  const int QS = NH * kHeadDim;
  if (tid == 0) {
    tc_mbar_init(&full[0]);
    tc_mbar_init(&full[1]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_map(&kvmap);
  }
  pdl_wait();
  const long long seq_row = ((long long)b * NKV + g) * max_seq;
  const int nkt = qt + 1;
  auto issue = [&](int t) {
    const long long row = seq_row + (long long)t * kPfTile;
    unsigned char* st = kv + (t & 1) * kBAttnStage;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(&full[t & 1])),
                 "r"(kBAttnStage)
                 : "memory");
    tma_load_2d(st, &kvmap, 0, (int)(k_row0 + row), &full[t & 1]);
    tma_load_2d(st + kBAttnBox, &kvmap, 64, (int)(k_row0 + row), &full[t & 1]);
    tma_load_2d(st + 2 * kBAttnBox, &kvmap, 0, (int)(v_row0 + row), &full[t & 1]);
    tma_load_2d(st + 3 * kBAttnBox, &kvmap, 64, (int)(v_row0 + row), &full[t & 1]);
  };
  __syncthreads();
  if (tid == 0) {
    issue(0);
    if (nkt > 1) issue(1);
  }
  // Q tile -> f16 hi/lo, swizzled like the K boxes. Rows beyond n are zero. Each
  // thread's 16 float4 loads are all issued before the first split (one round trip).
  constexpr int kQPer = kPfTile * 32 / 128;  // items (4 dims each) per thread: G * 64 * 32 over 128 * G threads
  float4 qv[kQPer];
#pragma unroll
  for (int i = 0; i < kQPer; ++i) {
    const int e = tid + i * 128 * G;
    const int hh = e / (kPfTile * 32), r = (e / 32) % kPfTile, d4 = e % 32;
    const int p = qt * kPfTile + r;
    qv[i] = p < n ? *reinterpret_cast<const float4*>(q + ((long long)b * n + p) * QS +
                                                      ((long long)g * G + hh) * kHeadDim + 4 * d4)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < kQPer; ++i) {
    const int e = tid + i * 128 * G;
    const int hh = e / (kPfTile * 32), r = (e / 32) % kPfTile, d4 = e % 32;
    const float4 v = qv[i];
    unsigned h01, l01, h23, l23;
    split_pair(v.x, v.y, h01, l01);
    split_pair(v.z, v.w, h23, l23);
    const int dim = 4 * d4, half = dim >> 6, c = (dim & 63) >> 3;
    const unsigned off = swz(r, c) + (dim & 7) * 2;
    unsigned char* qh = qs + ((hh * 2 + 0) * 2 + half) * kPfQBytes;
    unsigned char* ql = qs + ((hh * 2 + 1) * 2 + half) * kPfQBytes;
    *reinterpret_cast<uint2*>(qh + off) = make_uint2(h01, h23);
    *reinterpret_cast<uint2*>(ql + off) = make_uint2(l01, l23);
  }
  __syncthreads();

  const int r0 = wq * 16;           // first tile row of this warp
  const int ra = r0 + (lane >> 2);  // accumulator rows ra and ra + 8
  const int qa = qt * kPfTile + ra, qb = qa + 8;
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
  const unsigned qh_base = tc_smem(qs + (h * 2 + 0) * 2 * kPfQBytes);
  const unsigned ql_base = tc_smem(qs + (h * 2 + 1) * 2 * kPfQBytes);
  bool ok = true;
  int consumed = 0;
  for (int t = 0; t < nkt; ++t) {
    const int buf = t & 1;
    ok = tc_mbar_wait(&full[buf], (unsigned)(t >> 1) & 1u);
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    consumed = t + 1;
    const unsigned kb = tc_smem(kv + buf * kBAttnStage);
    const unsigned vb = kb + 2 * kBAttnBox;
    // S = Q K^T for 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {  // 16 dims per step
      // A: rows r0.., matrices (rows +0/+8) x (dims +0/+8)
      const int mi = lane >> 3, rr = r0 + (lane & 7) + 8 * (mi & 1), ch = 2 * kk + (mi >> 1);
      const unsigned aoff = (unsigned)((ch >> 3) * kPfQBytes) + swz(rr, ch & 7);
      unsigned ah0, ah1, ah2, ah3, al0, al1, al2, al3;
      ldsm_x4(qh_base + aoff, ah0, ah1, ah2, ah3);
      ldsm_x4(ql_base + aoff, al0, al1, al2, al3);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {  // two n-tiles of 8 keys per ldmatrix.x4
        const int key = 8 * (j + (mi >> 1)) + (lane & 7), kc = 2 * kk + (mi & 1);
        unsigned b0, b1, b2, b3;
        ldsm_x4(kb + (unsigned)((kc >> 3) * kBAttnBox) + swz(key, kc & 7), b0, b1, b2, b3);
        mma16816(s[j], ah0, ah1, ah2, ah3, b0, b1);
        mma16816(s[j], al0, al1, al2, al3, b0, b1);
        mma16816(s[j + 1], ah0, ah1, ah2, ah3, b2, b3);
        mma16816(s[j + 1], al0, al1, al2, al3, b2, b3);
      }
    }
    // scale, causal mask, online softmax (rows qa, qb; each quad holds one row pair)
    float mt_a = -INFINITY, mt_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = t * kPfTile + 8 * j + 2 * (lane & 3) + e;
        s[j][e] = (key <= qa && key < n) ? s[j][e] * scale : -INFINITY;
        s[j][2 + e] = (key <= qb && key < n) ? s[j][2 + e] * scale : -INFINITY;
        mt_a = fmaxf(mt_a, s[j][e]);
        mt_b = fmaxf(mt_b, s[j][2 + e]);
      }
    }
    mt_a = fmaxf(mt_a, __shfl_xor_sync(0xffffffffu, mt_a, 1));
    mt_a = fmaxf(mt_a, __shfl_xor_sync(0xffffffffu, mt_a, 2));
    mt_b = fmaxf(mt_b, __shfl_xor_sync(0xffffffffu, mt_b, 1));
    mt_b = fmaxf(mt_b, __shfl_xor_sync(0xffffffffu, mt_b, 2));
    const float mn_a = fmaxf(m_a, mt_a), mn_b = fmaxf(m_b, mt_b);
    const float fa = (m_a == -INFINITY || mn_a == -INFINITY) ? (mn_a == -INFINITY ? 1.0f : 0.0f) : expf(m_a - mn_a);
    const float fb = (m_b == -INFINITY || mn_b == -INFINITY) ? (mn_b == -INFINITY ? 1.0f : 0.0f) : expf(m_b - mn_b);
    float ps_a = 0.0f, ps_b = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[j][e] = s[j][e] == -INFINITY ? 0.0f : expf(s[j][e] - mn_a);
        s[j][2 + e] = s[j][2 + e] == -INFINITY ? 0.0f : expf(s[j][2 + e] - mn_b);
        ps_a += s[j][e];
        ps_b += s[j][2 + e];
      }
    }
    ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 1);
    ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 2);
    ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 1);
    ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 2);
    l_a = l_a * fa + ps_a;
    l_b = l_b * fb + ps_b;
    m_a = mn_a;
    m_b = mn_b;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= fa;
      o[i][1] *= fa;
      o[i][2] *= fb;
      o[i][3] *= fb;
    }
    // O += P V: P from the S accumulators (hi + lo f16), V by transposed ldmatrix
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {  // 16 keys per step
      unsigned ph[4], plo[4];
      split_pair(s[2 * ks][0], s[2 * ks][1], ph[0], plo[0]);
      split_pair(s[2 * ks][2], s[2 * ks][3], ph[1], plo[1]);
      split_pair(s[2 * ks + 1][0], s[2 * ks + 1][1], ph[2], plo[2]);
      split_pair(s[2 * ks + 1][2], s[2 * ks + 1][3], ph[3], plo[3]);
      const int mi = lane >> 3;
      const int key = 16 * ks + (lane & 7) + 8 * (mi & 1);
#pragma unroll
      for (int dn = 0; dn < 16; dn += 2) {  // two 8-dim n-tiles per ldmatrix.x4
        const int vc = dn + (mi >> 1);       // 8-dim chunk of the row (0..15)
        unsigned b0, b1, b2, b3;
        ldsm_x4_t(vb + (unsigned)((vc >> 3) * kBAttnBox) + swz(key, vc & 7), b0, b1, b2, b3);
        mma16816(o[dn], ph[0], ph[1], ph[2], ph[3], b0, b1);
        mma16816(o[dn], plo[0], plo[1], plo[2], plo[3], b0, b1);
        mma16816(o[dn + 1], ph[0], ph[1], ph[2], ph[3], b2, b3);
        mma16816(o[dn + 1], plo[0], plo[1], plo[2], plo[3], b2, b3);
      }
    }
    __syncthreads();  // stage consumed
    if (tid == 0 && t + 2 < nkt) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(t + 2);
    }
  }
  if (!ok) {
    if (tid == 0) {
      for (int t = consumed; t < min(nkt, consumed + 2); ++t) (void)tc_mbar_wait(&full[t & 1], (unsigned)(t >> 1) & 1u);
      atomicOr(err, kBErrTimeout);
    }
    pdl_trigger();
    return;
  }
  pdl_trigger();
  const float ia = 1.0f / l_a, ib = 1.0f / l_b;
  const int col0 = (g * G + h) * kHeadDim + 2 * (lane & 3);
#pragma unroll
  for (int dn = 0; dn < 16; ++dn) {
    const int col = col0 + 8 * dn;
    if (qa < n) {
      unsigned hi, lo;
      const float x0 = o[dn][0] * ia, x1 = o[dn][1] * ia;
      const __half2 hh = __floats2half2_rn(x0, x1);
      const float2 hf = __half22float2(hh);
      hi = *reinterpret_cast<const unsigned*>(&hh);
      lo = pack_h2((x0 - hf.x) * kLoScale, (x1 - hf.y) * kLoScale);
      *reinterpret_cast<unsigned*>(x_hi + ((long long)b * n + qa) * QS + col) = hi;
      *reinterpret_cast<unsigned*>(x_lo + ((long long)b * n + qa) * QS + col) = lo;
    }
    if (qb < n) {
      unsigned hi, lo;
      const float x0 = o[dn][2] * ib, x1 = o[dn][3] * ib;
      const __half2 hh = __floats2half2_rn(x0, x1);
      const float2 hf = __half22float2(hh);
      hi = *reinterpret_cast<const unsigned*>(&hh);
      lo = pack_h2((x0 - hf.x) * kLoScale, (x1 - hf.y) * kLoScale);
      *reinterpret_cast<unsigned*>(x_hi + ((long long)b * n + qb) * QS + col) = hi;
      *reinterpret_cast<unsigned*>(x_lo + ((long long)b * n + qb) * QS + col) = lo;
    }
  }
}

// ---- engine prompt pass: K/V rows into the engine's cache ----------------------------
// Positions 0..n-1 of sequence 0 of a batch cache (K of every layer, then V; row
// (g, p) of a layer at (g * max_seq + p) * 128) into an engine cache of f16 rows:
// layer l's K at ekv + 2l * ekv_layer bytes, its V at (2l + 1) * ekv_layer, row
// (p, g) at (p * NKV + g) * 256 bytes. One thread per 16 bytes.
static __global__ void __launch_bounds__(256) kb_kv_to_engine(const __half* kv, long long kv_layer, int L, int NKV,
                                                            int max_seq, int n, char* ekv, long long ekv_layer) {
  pdl_wait();
  const long long total = (long long)L * 2 * n * NKV * 16;
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    const int q = (int)(i & 15);
    long long r = i >> 4;
    const int g = (int)(r % NKV);
    r /= NKV;
    const int p = (int)(r % n);
    const int lk = (int)(r / n);  // layer * 2 + (0: K, 1: V)
    const int l = lk >> 1, kind = lk & 1;
    const uint4* src = reinterpret_cast<const uint4*>(kv + (long long)(kind * L + l) * kv_layer +
                                                      ((long long)g * max_seq + p) * kHeadDim) + q;
    uint4* dst = reinterpret_cast<uint4*>(ekv + (long long)lk * ekv_layer + ((long long)p * NKV + g) * kHeadDim * 2) + q;
    *dst = *src;
  }
  pdl_trigger();
}

}  // namespace qd
