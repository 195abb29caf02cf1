// Batch-1 decode of one token as ONE persistent kernel (one CTA per SM,
// cooperative launch so every CTA is resident).
//
// Weights: every stage's rows are split into one contiguous slice per CTA; each
// CTA streams its layer slices, in consumption order, into an 8-slot shared-
// memory ring with cp.async.bulk (completion on one mbarrier per slot). A slot
// is refilled as soon as the stage that used it is done, so the weight stream
// runs up to 8 stages (two layers) ahead of the dependency chain. The LM head
// (one pass over the 311 MB table) streams with direct 128-bit loads.
//
// Activations: a stage's outputs go to global memory as 64-bit words
// {f32 value, epoch}; consumers poll the words they need until each carries
// this launch's epoch. Value and "ready" travel in one store, so a stage
// boundary costs one store-to-load trip through L2 instead of a grid barrier.
//
// Attention and the O projection are one stage: OS CTAs per KV head each run
// the head's attention (the same math, redundantly) and multiply it by their
// slice of O rows x the head's columns; the KV-head partials are summed in
// 64-bit counted fixed-point words (2^56 + round(v * 2^28) per contribution:
// the top byte counts contributions, the rest is their exact sum, so the sum
// does not depend on arrival order), and consumers poll those words until the
// count reaches the number of KV heads. The MLP is one stage the same way:
// every CTA owns a run of <= 24 intermediate columns, computes their gate/up
// rows and silu(gate) * up, multiplies them by its slice of the down columns
// (packed per CTA, 16 bytes per down row) and adds the partial down sums to
// counted words that the next layer polls. The accumulators are double-buffered
// by launch parity; each launch zeroes the other parity for the next one.
// Every wait has a deadline (globaltimer) and an abort flag: on expiry the
// kernel sets an error bit, waits for its own copies in flight and returns.
#pragma once

#include "kernels.cuh"

namespace qd {

constexpr int kPT = 512;                   // threads per CTA
constexpr int kPW = kPT / 32;              // warps per CTA
constexpr int kSlots = 8;                  // ring slots
constexpr int kSlotBytes = 24576;          // per slot (the largest per-CTA slice at Qwen3-0.6B shapes)
constexpr unsigned long long kWaitNs = 200ull * 1000 * 1000;  // deadline of any single wait
constexpr int kErrTimeout = 4;             // DevErr bit: a wait expired (kernel aborted)
constexpr int kErrOverflow = 16;           // DevErr bit: an O partial beyond the fixed-point range (clamped)
constexpr int kMaxRes = 256;               // per-CTA row results of one stage (floats)
constexpr unsigned kPollBackoffNs = 0;     // pause between re-polls of exchange words (none: measured fastest)
constexpr int kAttnPf = 2;                 // cached K/V rows each attention warp loads ahead

// Stage timeline (opt-in): per CTA, event 0 = start, then per layer
// 19 events (QKV input ready, QKV weights ready, QKV stored, attention + O slice
// done, h_attn ready, (unused: = h_attn ready), gate/up input ready, gate/up stored,
// down input ready, down stored, QKV norm done, (unused: = h_attn ready), gate/up
// norm done, down weights ready; attention CTAs only: q/k/v arrived, head norm +
// RoPE done, attention done, O slice weights ready, O slice dots done), then
// LM-head input ready, LM-head done, merged.
constexpr int kTimelinePerLayer = 19;
__host__ __device__ constexpr int timeline_events(int layers) { return 1 + kTimelinePerLayer * layers + 3; }

struct PLayer {
  const char *qkv, *o, *gu, *d;            // row records (gate/up: pair records)
  const float *n_in, *n_q, *n_k, *n_post;
  void *kc, *vc;
  // O rows x one KV head's columns, packed per attention CTA: slice (g, s) at
  // oslice + (g * OS + s) * oslice_rows * rec_og, rows of s's range as row records
  const char* oslice;
  // down rows x one CTA's intermediate columns, packed per CTA: CTA c's slice at
  // dslice + c * H * kDRec; row record = 3 words of 8 nibbles (its <= 24 columns
  // from nibble 0, unused ones 8) and the f16 scales of the two blocks they span
  const char* dslice;
};
constexpr int kDRec = 16;      // bytes of one packed down row
constexpr int kDMaxCols = 24;  // intermediate columns per CTA at most

struct PArgs {
  const PLayer* layers;
  int L, H, I, NH, NKV, vocab, max_seq, row_stride;
  float eps, scale;
  const __half* embed;
  const float *cos_t, *sin_t, *final_norm;
  unsigned long long* xb;                  // exchange words
  long long xstride;                       // words per layer: h | qkv | attn | h_attn | act
  DevState* st;
  int *tokens, *out_dev, *out_host;
  float* logits;
  float* part_v;
  uint32_t* part_i;
  unsigned* counter;
  int with_head;
  int lm_rows;                             // unused (kept for the host's slot-size check)
  unsigned long long* timeline;            // optional [gridDim.x][timeline_events(L)] stage stamps (ns)
  long long rec_h, rec_q, rec_i;           // row record bytes for K = H, NH*128, I
  int OS;                                  // attention CTAs per KV head (each owns a slice of O rows)
  long long rec_og, oslice_rows;           // O slice row record bytes (K = G*128), rows per slice (max)
  unsigned long long* oacc;                // [2 parities][L][O | down][H] counted fixed-point sums
  int n_mlp;                               // CTAs that own intermediate columns (contributors to the down sums)
  // argmax-only LM head (pruned = 1): the table as int8 (q + 128, per-row scale) and a
  // per-row bound coefficient: |f16 logit - int8 logit| <= lm_bound[r] * ||x||_1
  int pruned;
  const uint2* lm_q8;                      // [vocab][H / 8]
  const float *lm_scale, *lm_bound;        // [vocab]
};
constexpr int kLmCand = 64;                // candidate rows per warp of the pruned head
constexpr int kLmRows = 16;                // int8 rows per ring chunk of the pruned head (4 warps x 4)

// ---- small PTX helpers --------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_word(unsigned long long* p, float v, unsigned epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void mbar_init(unsigned long long* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(unsigned long long* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(unsigned long long* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, unsigned long long* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(b))
               : "memory");
}
// L2 policy of the layer-weight stream: every byte is read once per token, so
// it is marked evict-first and leaves L2 to the exchange words and KV rows
// (measured: +5% tokens/s at the Qwen3-0.6B shape).
__device__ __forceinline__ unsigned long long policy_evict_first() {
  unsigned long long p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, unsigned bytes, unsigned long long* b,
                                               unsigned long long policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(b)), "l"(policy)
      : "memory");
}

// All of warp 0 stores the same word: a store by one lane leaves the warp diverged,
// and its next warp-collective step then pays ~800 cycles to reconverge (measured),
// which the stamps would report as that step's own time.
__device__ __forceinline__ void stamp(unsigned long long* tl, int ev) {
  if (tl && threadIdx.x < 32) tl[ev] = gtimer();
}

// Contiguous split of n rows over g CTAs (n * g < 2^31 for every shape served).
__device__ __forceinline__ void range_of(int n, int c, int g, int& lo, int& hi) {
  lo = (int)((unsigned)n * (unsigned)c / (unsigned)g);
  hi = (int)((unsigned)n * (unsigned)(c + 1) / (unsigned)g);
}

struct PShared {
  char* ring;
  float* xs;            // activation staging (swizzled; also the attention merge area)
  float* hs;            // layer input h (kept for the O residual)
  float* has;           // h_attn (kept for the down residual)
  unsigned long long* mbar;
  float* red;           // [kPW]
  int* flag;            // [0]: this CTA is the last to finish
  float* res;           // [kMaxRes] stage row results
  float* misc;          // attention: raw q/k/v, normed q, new k/v, warp (m, l); merge partials
};

// Row ranges of this CTA, computed once per launch.
struct Ranges {
  int qkv_lo, qkv_hi, h_lo, h_hi, i_lo, i_hi, v_lo, v_hi;
  int att, ag, as, o_lo, o_hi;             // attention role: KV head ag, O rows [o_lo, o_hi) (att = 0: none)
};

// The layer-weight chunk i of this CTA: chunks 4l..4l+3 are layer l's QKV, O,
// gate/up and down slices.
__device__ __forceinline__ void chunk_src(const PArgs& a, const Ranges& rg, int i, const char*& src, unsigned& bytes) {
  const PLayer& P = a.layers[i >> 2];
  switch (i & 3) {
    case 0: src = P.qkv + rg.qkv_lo * a.rec_h; bytes = (unsigned)((rg.qkv_hi - rg.qkv_lo) * a.rec_h); break;
    case 1:  // this attention CTA's O slice (nothing for the others)
      src = P.oslice + (long long)(rg.ag * a.OS + rg.as) * a.oslice_rows * a.rec_og;
      bytes = rg.att ? (unsigned)((rg.o_hi - rg.o_lo) * a.rec_og) : 0u;
      break;
    case 2: src = P.gu + rg.i_lo * 2 * a.rec_h; bytes = (unsigned)((rg.i_hi - rg.i_lo) * 2 * a.rec_h); break;
    default:  // this CTA's packed down columns
      src = P.dslice + (long long)blockIdx.x * a.H * kDRec;
      bytes = rg.i_hi > rg.i_lo ? (unsigned)(a.H * kDRec) : 0u;
      break;
  }
}

// One thread: put chunk i in flight into its slot (after a barrier that ends the
// slot's last reads).
__device__ __forceinline__ void issue_chunk(const PArgs& a, const PShared& S, const Ranges& rg, int i, int n) {
  if (i >= n) return;
  const char* src;
  unsigned bytes;
  chunk_src(a, rg, i, src, bytes);
  const int slot = i % kSlots;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_arrive_tx(&S.mbar[slot], bytes);
  if (bytes) bulk_load_hint(S.ring + slot * kSlotBytes, src, bytes, &S.mbar[slot], policy_evict_first());
}

__device__ __forceinline__ bool aborted(const PArgs& a) { return *reinterpret_cast<volatile int*>(&a.st->abort) != 0; }

// Every thread: wait for chunk i to land. False on timeout/abort.
__device__ __forceinline__ bool wait_chunk(const PArgs& a, const PShared& S, int i) {
  const int slot = i % kSlots;
  const unsigned parity = (unsigned)(i / kSlots) & 1u;
  if (mbar_test(&S.mbar[slot], parity)) return true;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_test(&S.mbar[slot], parity)) return true;
    if ((it & 63) == 0 && (aborted(a) || gtimer() - t0 > kWaitNs)) return false;
  }
}

// Every thread: wait until word p carries this launch's epoch. False on timeout/abort.
__device__ __forceinline__ bool poll_word(const PArgs& a, const unsigned long long* p, unsigned epoch, float& out) {
  unsigned long long v = ld_word(p);
  unsigned long long t0 = 0;
  for (unsigned it = 0; (unsigned)(v >> 32) != epoch; ++it) {
    if (it == 0) t0 = gtimer();
    else if ((it & 15) == 0 && (aborted(a) || gtimer() - t0 > kWaitNs)) return false;
    if (kPollBackoffNs) __nanosleep(kPollBackoffNs);
    v = ld_word(p);
  }
  out = __uint_as_float((unsigned)v);
  return true;
}

// On failure: wait (bounded, ignoring the abort flag) for this CTA's chunks
// still in flight, so no bulk copy targets shared memory after the CTA exits.
__device__ __forceinline__ void drain(const PShared& S, int next, int n_chunks) {
  const int end = min(next + kSlots, n_chunks);
  for (int i = next; i < end; ++i) {
    const int slot = i % kSlots;
    const unsigned parity = (unsigned)(i / kSlots) & 1u;
    const unsigned long long t0 = gtimer();
    while (!mbar_test(&S.mbar[slot], parity))
      if (gtimer() - t0 > kWaitNs) break;
  }
}

// Raise the abort flag (any thread).
__device__ __forceinline__ void raise_abort(const PArgs& a) {
  atomicOr(&a.st->err, kErrTimeout);
  atomicExch(&a.st->abort, 1);
}

// All threads agree whether to continue (also a block barrier).
__device__ __forceinline__ bool stage_ok(const PArgs& a, bool mine) {
  if (!mine) raise_abort(a);
  return __syncthreads_and(mine ? 1 : 0) != 0;
}

// ---- counted fixed-point sums ------------------------------------------------------
constexpr float kFxScale = 268435456.0f;              // 2^28
constexpr float kFxInv = 3.7252902984619140625e-9f;   // 2^-28
constexpr float kFxMax = 524288.0f;                   // 2^19: 148 such partials still fit 55 bits

__device__ __forceinline__ void red_fx(const PArgs& a, unsigned long long* p, float v) {
  if (!(fabsf(v) < kFxMax)) {  // also catches NaN
    atomicOr(&a.st->err, kErrOverflow);
    v = v != v ? 0.0f : copysignf(kFxMax, v);
  }
  const long long q = __float2ll_rn(v * kFxScale);
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"((1ull << 56) + (unsigned long long)q)
               : "memory");
}
__device__ __forceinline__ unsigned fx_count(unsigned long long w) { return (unsigned)((w + (1ull << 55)) >> 56); }
__device__ __forceinline__ float fx_value(unsigned long long w) {
  const unsigned long long c = (w + (1ull << 55)) >> 56;
  return __ll2float_rn((long long)(w - (c << 56))) * kFxInv;
}

// Every thread: poll counted words src[e], e = threadIdx.x + k*kPT < n (n <= 4 kPT),
// until each holds `need` contributions; dst[e] = base[e] + sum. False on timeout/abort.
static __device__ __noinline__ bool poll_fx(const PArgs& a, const unsigned long long* src, int n, unsigned need,
                                        const float* base, float* dst) {
  constexpr int K = 4;
  unsigned long long v[K];
  unsigned pend = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int e = threadIdx.x + k * kPT;
    v[k] = 0ull;
    if (e < n) {
      v[k] = ld_word(src + e);
      pend |= 1u << k;
    }
  }
  unsigned long long t0 = 0;
  for (unsigned it = 0;; ++it) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (((pend >> k) & 1u) && fx_count(v[k]) == need) {
        pend &= ~(1u << k);
        const int e = threadIdx.x + k * kPT;
        dst[e] = base[e] + fx_value(v[k]);
      }
    }
    if (!pend) return true;
    if (it == 0) t0 = gtimer();
    else if ((it & 15) == 0 && (aborted(a) || gtimer() - t0 > kWaitNs)) return false;
    if (kPollBackoffNs) __nanosleep(kPollBackoffNs);
#pragma unroll
    for (int k = 0; k < K; ++k)
      if ((pend >> k) & 1u) v[k] = ld_word(src + threadIdx.x + k * kPT);
  }
}

// f16 rounding of a float4 as the f16 KV cache stores it (identity for an f32 cache).
template <typename KVT> __device__ __forceinline__ float4 rnd4(float4 v);
template <> __device__ __forceinline__ float4 rnd4<float>(float4 v) { return v; }
template <> __device__ __forceinline__ float4 rnd4<__half>(float4 v) {
  const float2 a = __half22float2(__floats2half2_rn(v.x, v.y)), b = __half22float2(__floats2half2_rn(v.z, v.w));
  return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Sum over the warp of 4 per-lane values at once (transposing butterfly, 6
// shuffles): on return lane l holds the total of value l >> 3.
__device__ __forceinline__ float reduce4(float p0, float p1, float p2, float p3) {
  const int lane = threadIdx.x & 31;
  const bool hi16 = lane & 16, hi8 = lane & 8;
  float a0 = (hi16 ? p2 : p0) + __shfl_xor_sync(0xffffffffu, hi16 ? p0 : p2, 16);
  float a1 = (hi16 ? p3 : p1) + __shfl_xor_sync(0xffffffffu, hi16 ? p1 : p3, 16);
  float r = (hi8 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, hi8 ? a0 : a1, 8);
  r += __shfl_xor_sync(0xffffffffu, r, 4);
  r += __shfl_xor_sync(0xffffffffu, r, 2);
  r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

// Block dots of one stage from the ring slot into res[c * n_items + item].
// Items are (row, sub-row) pairs: item = row * nw + j; a row record holds nw
// sub-rows of `rec` bytes. Warps are grouped by 32-block column chunk c
// (kPW / kc warps per chunk, each holding only that chunk's activations) and
// process 4 items at a time, so four independent dot chains overlap and share
// one 6-shuffle reduction.
template <int NW>
__device__ __forceinline__ void stage_dots(const char* slot, int n_rows, int rec, int nb, int kc, const float* xs,
                                           float* res) {
  constexpr int nw = NW;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wpc = kPW / kc;
  const int c = warp / wpc, u = warp - c * wpc;
  const int n_items = n_rows * nw;
  if (c >= kc || u * 4 >= n_items) return;  // idle warps skip the activation loads
  const int b = c * 32 + lane;
  const bool live = b < nb;
  float2 xr[16];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = reinterpret_cast<const float4*>(xs)[xs_slot(b * 8 + q)];
    xr[2 * q] = make_float2(v.x, v.y);
    xr[2 * q + 1] = make_float2(v.z, v.w);
  }
  // A warp takes 4 consecutive items at a time: the activation chunk each warp
  // loads from shared memory (4 KB) is the dominant cost, so few warps with more
  // items each beat many warps with one item each.
  for (int i0 = u * 4; i0 < n_items; i0 += wpc * 4) {
    uint4 w[4];
    float s[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int it = i0 + k;
      w[k] = make_uint4(0u, 0u, 0u, 0u);
      s[k] = 0.0f;
      if (live && it < n_items) {
        const int row = nw == 1 ? it : (it >> 1), j = nw == 1 ? 0 : (it & 1);
        const char* r = slot + row * nw * rec + j * rec;
        w[k] = reinterpret_cast<const uint4*>(r)[b];
        s[k] = __half2float(reinterpret_cast<const __half*>(r + nb * 16)[b]);
      }
    }
    float p[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = s[k] * q4_block_dot(w[k], xr);
    const float t = reduce4(p[0], p[1], p[2], p[3]);
    const int it = i0 + (lane >> 3);
    if ((lane & 7) == 0 && it < n_items) res[c * n_items + it] = t;
  }
}

// Block dots of n row records of NB (<= 32) blocks each: lane l owns block l % NB
// of item (row) warp * (32 / NB) + l / NB + k * kPW * (32 / NB), so every lane does
// one block dot per step and NB-lane groups reduce with log2(NB) shuffles.
template <int NB>
__device__ __forceinline__ void slice_dots(const char* slot, int n_rows, int rec, const float* xs, float* res) {
  static_assert(NB == 4 || NB == 8 || NB == 16 || NB == 32, "power-of-two blocks per row");
  constexpr int IPS = 32 / NB;  // items per warp step
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = lane % NB, sub = lane / NB;
  float2 xr[16];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 v = reinterpret_cast<const float4*>(xs)[xs_slot(b * 8 + q)];
    xr[2 * q] = make_float2(v.x, v.y);
    xr[2 * q + 1] = make_float2(v.z, v.w);
  }
  for (int i0 = warp * IPS; i0 < n_rows; i0 += kPW * IPS) {
    const int it = i0 + sub;
    float p = 0.0f;
    if (it < n_rows) {
      const char* r = slot + it * rec;
      p = __half2float(reinterpret_cast<const __half*>(r + NB * 16)[b]) *
          q4_block_dot(reinterpret_cast<const uint4*>(r)[b], xr);
    }
#pragma unroll
    for (int o = NB / 2; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    if (b == 0 && it < n_rows) res[it] = p;
  }
}

// Every thread: poll words src[e], e = threadIdx.x + k*kPT < n, into shared
// memory (swizzled staging when swz, else dst[e]). A thread's words are
// re-polled together, so it pays one round trip after its last word lands.
// Misses back off briefly so that pollers do not flood L2. False on timeout/abort.
__device__ __forceinline__ bool poll_to_smem(const PArgs& a, const unsigned long long* src, int n, unsigned epoch,
                                          float* dst, bool swz) {
  constexpr int K = 8;
  unsigned long long v[K];
  unsigned need = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int e = threadIdx.x + k * kPT;
    v[k] = 0ull;
    if (e < n) {
      v[k] = ld_word(src + e);
      need |= 1u << k;
    }
  }
  unsigned long long t0 = 0;
  for (unsigned it = 0;; ++it) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if ((need >> k) & 1u) {
        if ((unsigned)(v[k] >> 32) == epoch) {
          need &= ~(1u << k);
          const int e = threadIdx.x + k * kPT;
          const float f = __uint_as_float((unsigned)v[k]);
          if (swz) xs_store(dst, e, f);
          else dst[e] = f;
        }
      }
    }
    if (!need) return true;
    if (it == 0) t0 = gtimer();
    else if ((it & 15) == 0 && (aborted(a) || gtimer() - t0 > kWaitNs)) return false;
    if (kPollBackoffNs) __nanosleep(kPollBackoffNs);
#pragma unroll
    for (int k = 0; k < K; ++k)
      if ((need >> k) & 1u) v[k] = ld_word(src + threadIdx.x + k * kPT);
  }
}

// ---- attention for one KV head (G query heads) + this CTA's O-projection slice ----
// Every CTA of the head's group runs the same attention (bitwise identically) and
// multiplies its result by O rows [o_lo, o_hi) x the head's G*128 columns; the
// partial goes to the counted fixed-point sums `acc`. Up to `cap` cached positions
// (the K/V rows fit the activation staging area), the rows are copied into shared
// memory while the q/k/v words are awaited and the scores, the softmax and the
// weighted sum run position-parallel; longer contexts use a per-warp online softmax.
template <int G, typename KVT>
__device__ __forceinline__ bool attn_o_stage(const PArgs& a, const PShared& S, const Ranges& rg, int l, int pos,
                                             unsigned epoch, const unsigned long long* xq, unsigned long long* acc,
                                             int chunk, int xs_floats, unsigned long long* tl, int ev) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = rg.ag;
  const PLayer& P = a.layers[l];
  KVT* kc = reinterpret_cast<KVT*>(P.kc);
  KVT* vc = reinterpret_cast<KVT*>(P.vc);
  const long long row_el = (long long)a.NKV * kHeadDim;
  const int QS = a.NH * kHeadDim, KVS = a.NKV * kHeadDim;
  float* raw = S.misc;                                      // [(G + 2) * 128]
  float* qs = raw + (G + 2) * kHeadDim;                     // [G * 128]
  float* kn = qs + G * kHeadDim;                            // [128]
  float* vn = kn + kHeadDim;                                // [128]
  float2* wml = reinterpret_cast<float2*>(vn + kHeadDim);   // [kPW * G]
  float* scs = reinterpret_cast<float*>(wml + kPW * G);     // [G][64] scores / probabilities
  float* ostage = S.has;                                    // the O dots' input (G * 128), swizzled
  const int cap = min(63, (xs_floats * 4) / (2 * kHeadDim * (int)sizeof(KVT)));
  const bool compact = pos <= cap;
  KVT* Ks = reinterpret_cast<KVT*>(S.xs);                   // [cap][128] cached K rows (compact)
  KVT* Vs = Ks + cap * kHeadDim;                            // [cap][128]

  // Everything that does not depend on this token's q/k/v, started before the wait:
  // the norm weights, this position's RoPE row, and the cached K/V rows.
  const float4 wq4 = reinterpret_cast<const float4*>(P.n_q)[lane];
  const float4 wk4 = reinterpret_cast<const float4*>(P.n_k)[lane];
  const int pair0 = (4 * lane) & (kHeadDim / 2 - 1);
  const long long toff = (long long)pos * a.row_stride + pair0;
  const float4 cr = *reinterpret_cast<const float4*>(a.cos_t + toff);
  const float4 sr = *reinterpret_cast<const float4*>(a.sin_t + toff);
  constexpr int kChunks = kHeadDim * (int)sizeof(KVT) / 16;  // 16-byte pieces of one row
  float4 kpf[kAttnPf], vpf[kAttnPf];
#pragma unroll
  for (int j = 0; j < kAttnPf; ++j) kpf[j] = vpf[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (compact) {
    for (int i = threadIdx.x; i < 2 * pos * kChunks; i += kPT) {
      const int which = i / (pos * kChunks), r = i - which * pos * kChunks;
      const int p = r / kChunks, c = r - p * kChunks;
      const KVT* src = (which ? vc : kc) + p * row_el + g * kHeadDim;
      KVT* dst = (which ? Vs : Ks) + p * kHeadDim;
      cp_async16(reinterpret_cast<char*>(dst) + 16 * c, reinterpret_cast<const char*>(src) + 16 * c);
    }
    cp_async_commit();
  } else {
#pragma unroll
    for (int j = 0; j < kAttnPf; ++j) {
      const int pp = warp + j * kPW;
      if (pp < pos) {
        kpf[j] = ld4<KVT>(kc + pp * row_el + g * kHeadDim + 4 * lane);
        vpf[j] = ld4<KVT>(vc + pp * row_el + g * kHeadDim + 4 * lane);
      }
    }
  }
  // q heads g*G.., k head g, v head g from the QKV exchange words (one word per thread for G <= 2).
  bool ok = true;
  for (int e0 = 0; e0 < (G + 2) * kHeadDim; e0 += kPT) {
    const int e = e0 + threadIdx.x;
    if (e < (G + 2) * kHeadDim) {
      const int t = e / kHeadDim, d = e % kHeadDim;
      const int src = t < G ? (g * G + t) * kHeadDim + d : (t == G ? QS + g * kHeadDim + d : QS + KVS + g * kHeadDim + d);
      ok = ok && poll_word(a, xq + src, epoch, raw[e]);
    }
  }
  if (compact) cp_async_wait_all();
  if (!stage_ok(a, ok)) return false;
  stamp(tl, ev + 14);

  // head RMSNorm + RoPE (q heads, k); the group's first CTA appends k, v to the cache
  const bool owner = rg.as == 0;
  for (int t = warp; t < G + 2; t += kPW) {
    const float4 x = reinterpret_cast<const float4*>(raw + t * kHeadDim)[lane];
    KVT* krow = kc + (long long)pos * row_el + g * kHeadDim + 4 * lane;
    KVT* vrow = vc + (long long)pos * row_el + g * kHeadDim + 4 * lane;
    if (t == G + 1) {
      reinterpret_cast<float4*>(vn)[lane] = owner ? st4<KVT>(vrow, x) : rnd4<KVT>(x);
      continue;
    }
    const float4 w4 = t < G ? wq4 : wk4;
    float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)kHeadDim + a.eps);
    const float4 y = make_float4(x.x * inv * w4.x, x.y * inv * w4.y, x.z * inv * w4.z, x.w * inv * w4.w);
    float4 p;
    p.x = __shfl_xor_sync(0xffffffffu, y.x, 16);
    p.y = __shfl_xor_sync(0xffffffffu, y.y, 16);
    p.z = __shfl_xor_sync(0xffffffffu, y.z, 16);
    p.w = __shfl_xor_sync(0xffffffffu, y.w, 16);
    const float sign = (lane >= 16) ? 1.0f : -1.0f;
    const float4 r = make_float4(y.x * cr.x + sign * p.x * sr.x, y.y * cr.y + sign * p.y * sr.y,
                                 y.z * cr.z + sign * p.z * sr.z, y.w * cr.w + sign * p.w * sr.w);
    if (t < G) reinterpret_cast<float4*>(qs + t * kHeadDim)[lane] = r;
    else reinterpret_cast<float4*>(kn)[lane] = owner ? st4<KVT>(krow, r) : rnd4<KVT>(r);
  }
  __syncthreads();
  stamp(tl, ev + 15);

  if (compact) {
    // scores: warp w takes positions w, w + kPW, ... <= pos
    float4 q[G];
#pragma unroll
    for (int h = 0; h < G; ++h) q[h] = reinterpret_cast<const float4*>(qs + h * kHeadDim)[lane];
    for (int p = warp; p <= pos; p += kPW) {
      const float4 k4 = p == pos ? reinterpret_cast<const float4*>(kn)[lane] : ld4<KVT>(Ks + p * kHeadDim + 4 * lane);
      float d[G];
#pragma unroll
      for (int h = 0; h < G; ++h) d[h] = q[h].x * k4.x + q[h].y * k4.y + q[h].z * k4.z + q[h].w * k4.w;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int h = 0; h < G; ++h) d[h] += __shfl_xor_sync(0xffffffffu, d[h], o);
      if (lane == 0)
#pragma unroll
        for (int h = 0; h < G; ++h) scs[h * 64 + p] = d[h] * a.scale;
    }
    __syncthreads();
    stamp(tl, ev + 11);
    // softmax of each head (warp h): probabilities in place
    if (warp < G) {
      const float s0 = lane <= pos ? scs[warp * 64 + lane] : -INFINITY;
      const float s1 = lane + 32 <= pos ? scs[warp * 64 + lane + 32] : -INFINITY;
      const float m = warp_max(fmaxf(s0, s1));
      const float e0 = lane <= pos ? expf(s0 - m) : 0.0f, e1 = lane + 32 <= pos ? expf(s1 - m) : 0.0f;
      const float inv = 1.0f / warp_sum(e0 + e1);
      if (lane <= pos) scs[warp * 64 + lane] = e0 * inv;
      if (lane + 32 <= pos) scs[warp * 64 + lane + 32] = e1 * inv;
    }
    __syncthreads();
    stamp(tl, ev + 5);
    // weighted sum of the V rows: thread e -> (head e / 128, dim e % 128)
    for (int e = threadIdx.x; e < G * kHeadDim; e += kPT) {
      const int h = e / kHeadDim, d = e % kHeadDim;
      const float* pr = scs + h * 64;
      float o[4] = {pr[pos] * vn[d], 0.0f, 0.0f, 0.0f};
      int p = 0;
      for (; p + 4 <= pos; p += 4) {  // four independent chains: the loads go out together
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float v;
          if constexpr (sizeof(KVT) == 2) v = __half2float(reinterpret_cast<const __half*>(Vs)[(p + j) * kHeadDim + d]);
          else v = reinterpret_cast<const float*>(Vs)[(p + j) * kHeadDim + d];
          o[j] = fmaf(pr[p + j], v, o[j]);
        }
      }
      for (; p < pos; ++p) {
        float v;
        if constexpr (sizeof(KVT) == 2) v = __half2float(reinterpret_cast<const __half*>(Vs)[p * kHeadDim + d]);
        else v = reinterpret_cast<const float*>(Vs)[p * kHeadDim + d];
        o[0] = fmaf(pr[p], v, o[0]);
      }
      xs_store(ostage, e, (o[0] + o[1]) + (o[2] + o[3]));
    }
  } else {
    // Online softmax per warp over positions warp, warp + kPW, ... <= pos.
    float4 q[G];
#pragma unroll
    for (int h = 0; h < G; ++h) q[h] = reinterpret_cast<const float4*>(qs + h * kHeadDim)[lane];
    float m[G], lsum[G];
    float4 accv[G];
#pragma unroll
    for (int h = 0; h < G; ++h) { m[h] = -INFINITY; lsum[h] = 0.0f; accv[h] = make_float4(0.f, 0.f, 0.f, 0.f); }
    for (int p = warp; p <= pos; p += kPW) {
      float4 k4 = kpf[0], v4 = vpf[0];
      if (p == pos) {
        k4 = reinterpret_cast<const float4*>(kn)[lane];
        v4 = reinterpret_cast<const float4*>(vn)[lane];
      }
#pragma unroll
      for (int j = 0; j + 1 < kAttnPf; ++j) {
        kpf[j] = kpf[j + 1];
        vpf[j] = vpf[j + 1];
      }
      const int pn = p + kAttnPf * kPW;
      if (pn < pos) {  // refill the pipeline kAttnPf rows ahead
        kpf[kAttnPf - 1] = ld4<KVT>(kc + pn * row_el + g * kHeadDim + 4 * lane);
        vpf[kAttnPf - 1] = ld4<KVT>(vc + pn * row_el + g * kHeadDim + 4 * lane);
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float d = q[h].x * k4.x + q[h].y * k4.y + q[h].z * k4.z + q[h].w * k4.w;
        const float sc = warp_sum(d) * a.scale;
        const float mn = fmaxf(m[h], sc);
        const float co = expf(m[h] - mn), cn = expf(sc - mn);
        lsum[h] = lsum[h] * co + cn;
        accv[h] = make_float4(accv[h].x * co + cn * v4.x, accv[h].y * co + cn * v4.y, accv[h].z * co + cn * v4.z,
                              accv[h].w * co + cn * v4.w);
        m[h] = mn;
      }
    }
    // Merge the warps in a fixed order (deterministic).
    float* wacc = S.xs;  // [kPW][G][128]
#pragma unroll
    for (int h = 0; h < G; ++h) {
      reinterpret_cast<float4*>(wacc + (warp * G + h) * kHeadDim)[lane] = accv[h];
      if (lane == 0) wml[warp * G + h] = make_float2(m[h], lsum[h]);
    }
    __syncthreads();
    static_assert(kPW == 16, "the merge pairs two heads per warp");
    float* fw = raw;  // [G][kPW] (raw is no longer needed)
    if (threadIdx.x < ((G * kPW + 31) / 32) * 32) {
      const int h = threadIdx.x / kPW, w = threadIdx.x % kPW;
      const bool on = h < G;
      const float2 mw = on ? wml[w * G + h] : make_float2(-INFINITY, 0.0f);
      float M = mw.x;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      const float e = mw.y > 0.0f ? expf(mw.x - M) : 0.0f;
      float Ls = mw.y * e;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o);
      if (on) fw[h * kPW + w] = e / Ls;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < G * kHeadDim; e += kPT) {
      const int h = e / kHeadDim, d = e % kHeadDim;
      float o = 0.0f;
#pragma unroll
      for (int w = 0; w < kPW; ++w) o += wacc[(w * G + h) * kHeadDim + d] * fw[h * kPW + w];
      xs_store(ostage, e, o);
    }
  }
  __syncthreads();

  stamp(tl, ev + 16);
  // O rows [o_lo, o_hi) over the head's columns -> counted fixed-point sums
  if (!stage_ok(a, wait_chunk(a, S, chunk))) return false;
  stamp(tl, ev + 17);
  const int n = rg.o_hi - rg.o_lo;
  slice_dots<G * kHeadDim / kBlockCols>(S.ring + (chunk % kSlots) * kSlotBytes, n, (int)a.rec_og, ostage, S.res);
  __syncthreads();
  stamp(tl, ev + 18);
  if (threadIdx.x < n) red_fx(a, acc + rg.o_lo + threadIdx.x, S.res[threadIdx.x]);
  return true;
}

// This CTA's partial of the down projection: rows r = tid, tid + kPT (< H) over its
// intermediate columns, added to the counted sums acc[r]. act[0, kDMaxCols) holds the
// activations of the columns in the record's first q4 block (zero elsewhere) and
// act[kDMaxCols, 2 kDMaxCols) those in its second (shared memory, 16-byte aligned),
// so both scale segments accumulate without per-column selects. The nibbles become
// floats two at a time through the 2^23 + n bit pattern (one packed subtract).
__device__ __forceinline__ void down_partial(const PArgs& a, const char* slot, const float* act,
                                             unsigned long long* acc, int H) {
  static_assert(kDMaxCols == 24, "three words of eight nibbles per record");
  const float4* xa4 = reinterpret_cast<const float4*>(act);
  const float4* xb4 = reinterpret_cast<const float4*>(act + kDMaxCols);
  const float2 bias = make_float2(-8388616.0f, -8388616.0f);
#pragma unroll 1
  for (int k = 0; k < 2; ++k) {
    const int r = threadIdx.x + k * kPT;
    if (r >= H) break;
    const uint4 rec = reinterpret_cast<const uint4*>(slot)[r];
    const uint32_t w[3] = {rec.x, rec.y, rec.z};
    float2 pa = make_float2(0.0f, 0.0f), pb = pa;
#pragma unroll
    for (int q = 0; q < 3; ++q) {  // word q: columns 8q .. 8q + 7 (nibble i = column 8q + i)
      const uint32_t lo = w[q] & 0x0F0F0F0Fu, hi = (w[q] >> 4) & 0x0F0F0F0Fu;  // even / odd columns
      const float4 a0 = xa4[2 * q], a1 = xa4[2 * q + 1], b0 = xb4[2 * q], b1 = xb4[2 * q + 1];  // broadcast
      const float2 xa[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w), make_float2(a1.x, a1.y),
                            make_float2(a1.z, a1.w)};
      const float2 xb[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                            make_float2(b1.z, b1.w)};
#pragma unroll
      for (int m = 0; m < 4; ++m) {  // columns 8q + 2m, 8q + 2m + 1
        const float2 v = __fadd2_rn(make_float2(__int_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + m)),
                                                __int_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + m))),
                                    bias);
        pa = __ffma2_rn(v, xa[m], pa);
        pb = __ffma2_rn(v, xb[m], pb);
      }
    }
    const float sa = __half2float(__ushort_as_half((unsigned short)(rec.w & 0xFFFFu)));
    const float sb = __half2float(__ushort_as_half((unsigned short)(rec.w >> 16)));
    red_fx(a, acc + r, sa * (pa.x + pa.y) + sb * (pb.x + pb.y));
  }
}

// RMSNorm folded into the dots that follow it: xs holds v[e] * w[e] (e = tid,
// tid + kPT), red[warp] the warps' sums of squares; the dots over xs times
// rms_inv(red) are the dots over the normalised vector, so no barrier sits between
// the input and the dots. The caller's next barrier publishes both.
__device__ __forceinline__ void weigh_own(const float* v, const float (&w)[2], int n, float* xs, float* red) {
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int e = threadIdx.x + k * kPT;
    if (e < n) {
      const float x = v[e];
      ss += x * x;
      xs_store(xs, e, x * w[k]);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
}
__device__ __forceinline__ float rms_inv(const float* red, int n, float eps) {
  float t = 0.0f;
#pragma unroll
  for (int k = 0; k < kPW; ++k) t += red[k];
  return rsqrtf(t / (float)n + eps);
}

// Every thread: the final hidden state = h_attn of the last layer + its down sums
// into S.hs, and this CTA's rows of it out as words (read back by the host). H <= 2 kPT.
__device__ __forceinline__ bool final_hidden(const PArgs& a, const Ranges& rg, unsigned epoch, int H,
                                             const PShared& S) {
  const unsigned long long* acc_d = a.oacc + ((long long)(epoch & 1u) * a.L + (a.L - 1)) * 2 * H + H;
  if (!poll_fx(a, acc_d, H, (unsigned)a.n_mlp, S.has, S.hs)) return false;
  unsigned long long* xf = a.xb + (long long)a.L * a.xstride;
#pragma unroll
  for (int k = 0; k < 2; ++k) {  // the elements this thread polled itself (no barrier needed)
    const int e = threadIdx.x + k * kPT;
    if (e >= rg.h_lo && e < rg.h_hi) st_word(xf + e, S.hs[e], epoch);
  }
  return true;
}

// ---- the kernel -------------------------------------------------------------------
template <int G, typename KVT>
__global__ void __launch_bounds__(kPT, 1) k_decode_persistent(const __grid_constant__ PArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int cta = blockIdx.x, ng = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = a.H, I = a.I, QS = a.NH * kHeadDim, R = QS + 2 * a.NKV * kHeadDim;
  const int maxk = max(max(H, QS), I);

  PShared S;
  S.ring = reinterpret_cast<char*>(smem);
  S.xs = reinterpret_cast<float*>(smem + kSlots * kSlotBytes);
  const int xs_floats = max(maxk, kPW * G * kHeadDim);
  S.hs = S.xs + xs_floats;
  S.has = S.hs + H;
  S.mbar = reinterpret_cast<unsigned long long*>(S.has + H);
  S.red = reinterpret_cast<float*>(S.mbar + kSlots);
  S.flag = reinterpret_cast<int*>(S.red + kPW);
  S.res = reinterpret_cast<float*>(S.flag + 4);
  S.misc = S.res + kMaxRes;

  const int pos = a.st->pos;
  const unsigned epoch = (unsigned)a.st->epoch + 1u;
  const bool stall = a.st->stall_epoch != 0 && (unsigned)a.st->stall_epoch == epoch;
  if (pos < 0 || pos >= a.max_seq) {  // the host keeps positions in range; never index out of bounds
    if (threadIdx.x == 0) atomicOr(&a.st->err, kErrPosition);
    return;
  }
  unsigned long long* tl = a.timeline ? a.timeline + (long long)cta * timeline_events(a.L) : nullptr;
  stamp(tl, 0);
  Ranges rg;
  range_of(R, cta, ng, rg.qkv_lo, rg.qkv_hi);
  range_of(H, cta, ng, rg.h_lo, rg.h_hi);
  range_of(I, cta, ng, rg.i_lo, rg.i_hi);
  range_of(a.vocab, cta, ng, rg.v_lo, rg.v_hi);
  rg.att = cta < a.NKV * a.OS;
  rg.ag = rg.att ? cta / a.OS : 0;
  rg.as = rg.att ? cta % a.OS : 0;
  range_of(H, rg.as, a.OS, rg.o_lo, rg.o_hi);
  if (!rg.att) rg.o_hi = rg.o_lo;
  const int n_chunks = 4 * a.L;
  // The next launch's O sums start at zero: clear the other parity's words.
  {
    const long long words = (long long)a.L * 2 * H;
    unsigned long long* other = a.oacc + (long long)((epoch + 1u) & 1u) * words;
    const long long lo = words * cta / ng, hi = words * (cta + 1) / ng;
    for (long long i = lo + threadIdx.x; i < hi; i += kPT) other[i] = 0ull;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) mbar_init(&S.mbar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 0; i < kSlots; ++i) issue_chunk(a, S, rg, i, n_chunks);

  // Layer-0 input: the embedding row of tokens[pos], computed by every CTA.
  {
    int tok = a.tokens[pos];
    if (tok < 0 || tok >= a.vocab) {
      if (cta == 0 && threadIdx.x == 0) atomicOr(&a.st->err, kErrToken);
      tok = 0;
    }
    const __half* er = a.embed + (long long)tok * H;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int e = threadIdx.x + k * kPT;
      if (e < H) S.hs[e] = __half2float(er[e]);
    }
  }

  int chunk = 0;
#define QD_FAIL_IF(cond)              \
  if (cond) {                         \
    drain(S, chunk, n_chunks);        \
    return;                           \
  }
  for (int l = 0; l < a.L; ++l) {
    const PLayer& P = a.layers[l];
    unsigned long long* xq = a.xb + (long long)l * a.xstride + H;
    unsigned long long* acc_o = a.oacc + ((long long)(epoch & 1u) * a.L + l) * 2 * H;  // O sums
    unsigned long long* acc_d = acc_o + H;                                              // down sums
    const int ev = 1 + l * kTimelinePerLayer;

    // 1. layer input (the embedding row, or h_attn + the down sums of the previous
    //    layer), RMSNorm, QKV rows
    {
      float nw[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) nw[k] = threadIdx.x + k * kPT < H ? P.n_in[threadIdx.x + k * kPT] : 0.0f;
      if (l > 0) QD_FAIL_IF(!stage_ok(a, poll_fx(a, acc_o - H, H, (unsigned)a.n_mlp, S.has, S.hs)));
      stamp(tl, ev + 0);
      weigh_own(S.hs, nw, H, S.xs, S.red);
      stamp(tl, ev + 10);
      QD_FAIL_IF(!stage_ok(a, wait_chunk(a, S, chunk)));
      stamp(tl, ev + 1);
      const int n = rg.qkv_hi - rg.qkv_lo;
      stage_dots<1>(S.ring + (chunk % kSlots) * kSlotBytes, n, (int)a.rec_h, H / kBlockCols, 1, S.xs, S.res);
      __syncthreads();
      if (threadIdx.x < n && !(stall && l == 0))
        st_word(xq + rg.qkv_lo + threadIdx.x, S.res[threadIdx.x] * rms_inv(S.red, H, a.eps), epoch);
      // The slot's weights are consumed; the last thread (never a result row: n <= kMaxRes)
      // refills it, so the refill does not hold back the stores and needs no barrier.
      if (threadIdx.x == kPT - 1) issue_chunk(a, S, rg, chunk + kSlots, n_chunks);
      stamp(tl, ev + 2);
      ++chunk;
    }

    // 2. attention + O slice (the attention CTAs; every CTA passes chunk 4l+1, empty for
    //    the others), then 3. h_attn = h + the O sums (every CTA)
    {
      if (rg.att) {
        QD_FAIL_IF((!attn_o_stage<G, KVT>(a, S, rg, l, pos, epoch, xq, acc_o, chunk, xs_floats, tl, ev)));
      } else {
        QD_FAIL_IF(!stage_ok(a, wait_chunk(a, S, chunk)));
      }
      __syncthreads();
      stamp(tl, ev + 3);
      if (threadIdx.x == 0) issue_chunk(a, S, rg, chunk + kSlots, n_chunks);
      ++chunk;
      QD_FAIL_IF(!stage_ok(a, poll_fx(a, acc_o, H, (unsigned)a.NKV, S.hs, S.has)));
      stamp(tl, ev + 4);
    }

    // 4. post-attention RMSNorm, gate/up rows of this CTA's intermediate columns,
    //    silu(gate) * up, and their partial of the down projection into the down sums
    {
      float nw[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) nw[k] = threadIdx.x + k * kPT < H ? P.n_post[threadIdx.x + k * kPT] : 0.0f;
      stamp(tl, ev + 6);
      weigh_own(S.has, nw, H, S.xs, S.red);
      stamp(tl, ev + 12);
      QD_FAIL_IF(!stage_ok(a, wait_chunk(a, S, chunk)));
      const int n = rg.i_hi - rg.i_lo;
      stage_dots<2>(S.ring + (chunk % kSlots) * kSlotBytes, n, (int)a.rec_h, H / kBlockCols, 1, S.xs, S.res);
      __syncthreads();
      // The gate/up weights are consumed: the last thread (no activation to write) refills the slot.
      if (threadIdx.x == kPT - 1) issue_chunk(a, S, rg, chunk + kSlots, n_chunks);
      ++chunk;
      // this CTA's activations, split by the q4 block of the down record they fall in:
      // act[j] for the first block's columns, act[kDMaxCols + j] for the second's (zero past n)
      float* act = S.res + kMaxRes / 2;
      static_assert(kMaxRes / 2 + 2 * kDMaxCols <= kMaxRes, "both halves fit the result buffer");
      if (threadIdx.x < kDMaxCols) {
        float v = 0.0f;
        if (threadIdx.x < n) {
          const float inv = rms_inv(S.red, H, a.eps);
          const float gt = S.res[2 * threadIdx.x] * inv, upv = S.res[2 * threadIdx.x + 1] * inv;
          v = (gt / (1.0f + expf(-gt))) * upv;
        }
        const bool first = (int)threadIdx.x < kBlockCols - rg.i_lo % kBlockCols;
        act[threadIdx.x] = first ? v : 0.0f;
        act[kDMaxCols + threadIdx.x] = first ? 0.0f : v;
      }
      stamp(tl, ev + 7);
      // the down slice's wait ends in a barrier, which also publishes the activations
      QD_FAIL_IF(!stage_ok(a, wait_chunk(a, S, chunk)));
      stamp(tl, ev + 8);
      stamp(tl, ev + 13);
      if (n > 0) down_partial(a, S.ring + (chunk % kSlots) * kSlotBytes, act, acc_d, H);
      __syncthreads();
      stamp(tl, ev + 9);
      if (threadIdx.x == 0) issue_chunk(a, S, rg, chunk + kSlots, n_chunks);
      ++chunk;
    }
  }
#undef QD_FAIL_IF

  // ---- LM head + argmax (or, for a prompt token, just finish) ----
  // Every ring chunk has been consumed here: nothing is in flight, so a failure
  // below may return directly.
  float bv = kNegMax;
  uint32_t bi = 0;
  if (a.with_head) {
    // This warp streams rows v_lo + (i*kPW + warp)*4 + k (k < 4): 4 rows at once,
    // lane holding chunk c*32 + lane (columns 8 (c*32 + lane) .. +7) of each row. The
    // first batch is loaded before waiting for the final hidden state.
    const int kc8 = H / 256;
    const int n_rows = rg.v_hi - rg.v_lo;
    const uint4* tab = reinterpret_cast<const uint4*>(a.embed);
    const int rpr = H / 8;
    int i0 = warp * 4;
    auto load_batch = [&](uint4 (&dst)[4][4], int first) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int rr = first + k;
          dst[k][c] = (c < kc8 && rr < n_rows) ? ld_stream(tab + (long long)(rg.v_lo + rr) * rpr + c * 32 + lane)
                                               : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    // The final hidden state, its RMSNorm into plain staging and this lane's columns
    // (c*32+lane)*8 .. +7 of it; false on timeout/abort.
    auto normed_x = [&](float2 (&xr)[4][4]) -> bool {
      float fw[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) fw[k] = threadIdx.x + k * kPT < H ? a.final_norm[threadIdx.x + k * kPT] : 0.0f;
      if (!stage_ok(a, final_hidden(a, rg, epoch, H, S))) return false;
      float fv[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) fv[k] = threadIdx.x + k * kPT < H ? S.hs[threadIdx.x + k * kPT] : 0.0f;
      stamp(tl, 1 + kTimelinePerLayer * a.L);
      float ss = 0.0f;
#pragma unroll
      for (int k = 0; k < 2; ++k)
        if (threadIdx.x + k * kPT < H) ss += fv[k] * fv[k];
      ss = warp_sum(ss);
      if (lane == 0) S.red[warp] = ss;
      __syncthreads();
      float t = 0.0f;
#pragma unroll
      for (int k = 0; k < kPW; ++k) t += S.red[k];
      const float inv = rsqrtf(t / (float)H + a.eps);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        if (threadIdx.x + k * kPT < H) S.xs[threadIdx.x + k * kPT] = fv[k] * inv * fw[k];
      __syncthreads();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c < kc8) {
          const float4* p = reinterpret_cast<const float4*>(S.xs + (c * 32 + lane) * 8);
          const float4 v0 = p[0], v1 = p[1];
          xr[c][0] = make_float2(v0.x, v0.y);
          xr[c][1] = make_float2(v0.z, v0.w);
          xr[c][2] = make_float2(v1.x, v1.y);
          xr[c][3] = make_float2(v1.z, v1.w);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) xr[c][k] = make_float2(0.f, 0.f);
        }
      }
      return true;
    };
    // Exact f16 logits of 4 rows (row offsets rk[k] in this CTA's range, < 0: none);
    // the same arithmetic for every row wherever it is computed.
    auto exact4 = [&](const float2 (&xr)[4][4], const int (&rk)[4]) {
      uint4 w[4][4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          w[k][c] = (c < kc8 && rk[k] >= 0) ? ld_stream(tab + (long long)(rg.v_lo + rk[k]) * rpr + c * 32 + lane)
                                            : make_uint4(0u, 0u, 0u, 0u);
      float p[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) acc = f16x8_dot(w[k][c], xr[c], acc);
        p[k] = acc.x + acc.y;
      }
      const float v = reduce4(p[0], p[1], p[2], p[3]);
      const int m = lane >> 3, rr = m == 0 ? rk[0] : m == 1 ? rk[1] : m == 2 ? rk[2] : rk[3];
      if ((lane & 7) == 0 && rr >= 0) {
        const int r = rg.v_lo + rr;
        if (am_better(v, (uint32_t)r, bv, bi)) { bv = v; bi = (uint32_t)r; }
      }
    };
    if (!a.pruned) {
      uint4 cur[4][4];
      load_batch(cur, i0);
      float2 xr[4][4];
      if (!normed_x(xr)) return;
      for (; i0 < n_rows; i0 += kPW * 4) {
        float p[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < 4; ++c) acc = f16x8_dot(cur[k][c], xr[c], acc);
          p[k] = acc.x + acc.y;
        }
        if (i0 + kPW * 4 < n_rows) load_batch(cur, i0 + kPW * 4);
        const float v = reduce4(p[0], p[1], p[2], p[3]);
        const int rr = i0 + (lane >> 3);
        if ((lane & 7) == 0 && rr < n_rows) {
          const int r = rg.v_lo + rr;
          a.logits[r] = v;
          if (am_better(v, (uint32_t)r, bv, bi)) { bv = v; bi = (uint32_t)r; }
        }
      }
    } else {
      // The int8 rows stream through the (now idle) weight ring by bulk copies: chunk j
      // = rows [16 j, 16 j + 16) goes to ring index n_chunks + j; warp group g (warps
      // 4g .. 4g+3) takes chunks g, g + 4, ... (its two slots) and refills each slot
      // with the chunk 8 ahead once its four warps are done with it.
      const int n_lc = (n_rows + kLmRows - 1) / kLmRows;
      auto lc_issue = [&](int j) {
        const int gi = n_chunks + j, slot = gi % kSlots;
        const int rows = min(kLmRows, n_rows - j * kLmRows);
        const unsigned bytes = (unsigned)(rows * H);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_tx(&S.mbar[slot], bytes);
        bulk_load_hint(S.ring + slot * kSlotBytes, reinterpret_cast<const char*>(a.lm_q8) + (long long)(rg.v_lo + j * kLmRows) * H,
                       bytes, &S.mbar[slot], policy_evict_first());
      };
      // bounded wait for chunk j (ignoring the abort flag: these are this CTA's own copies)
      auto lc_wait = [&](int j) -> bool {
        const int gi = n_chunks + j;
        const unsigned parity = (unsigned)(gi / kSlots) & 1u;
        const unsigned long long t0 = gtimer();
        while (!mbar_test(&S.mbar[gi % kSlots], parity))
          if (gtimer() - t0 > kWaitNs) return false;
        return true;
      };
      if (threadIdx.x == 0)
        for (int j = 0; j < min(kSlots, n_lc); ++j) lc_issue(j);
      float2 xr[4][4];
      if (!normed_x(xr)) {
        for (int j = 0; j < min(kSlots, n_lc); ++j) (void)lc_wait(j);
        return;
      }
      // Argmax only. (1) Coarse logits from the int8 table, each within
      // lm_bound[r] * ||x||_1 (+ a rounding margin) of the row's f16 logit; the
      // warps keep the rows whose upper bound reaches the best lower bound seen so
      // far. (2) The rows whose upper bound reaches the CTA's best lower bound get
      // their exact f16 logits; no other row of the CTA can be its argmax (its
      // logit is below that of the row holding the best lower bound), so the
      // result is the full head's, ties and NaN rules included. A warp whose list
      // overflows, or a non-finite ||x||_1, takes the exact path for all its rows.
      // per-warp scalars in the misc area; the candidate lists in the activation
      // staging, which is free once ||x||_1 is summed (the ring carries the int8 rows)
      int* cnt = reinterpret_cast<int*>(S.misc);                  // [kPW]
      float* wlb = S.misc + kPW;                                  // [kPW]
      float* l1s = S.misc + 2 * kPW;                              // [kPW]
      int2* cand = reinterpret_cast<int2*>(S.xs);                 // [kPW][kLmCand] (row offset, ub bits)
      static_assert(kPW * kLmCand * 2 <= kPW * kHeadDim, "the lists fit the staging area (at least kPW * 128 floats)");
      float l1 = 0.0f;
#pragma unroll
      for (int k = 0; k < 2; ++k)
        if (threadIdx.x + k * kPT < H) l1 += fabsf(S.xs[threadIdx.x + k * kPT]);
      l1 = warp_sum(l1);
      if (lane == 0) {
        l1s[warp] = l1;
        cnt[warp] = 0;
      }
      __syncthreads();
      float L1 = 0.0f;
#pragma unroll
      for (int k = 0; k < kPW; ++k) L1 += l1s[k];
      const bool bounded = isfinite(L1);  // the same in every CTA
      float lane_lb = -INFINITY;
      // 4 rows of a landed chunk (rows `first` .. +3 of the CTA's range, chunk row
      // offset `local`): coarse logits, bounds, candidates
      auto coarse4 = [&](const char* chunk, int local, int first) {
          float p[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const char* row = chunk + (local + k) * H;
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint2 w = (c < kc8 && first + k < n_rows) ? reinterpret_cast<const uint2*>(row)[c * 32 + lane]
                                                              : make_uint2(0x80808080u, 0x80808080u);
              acc = q8x8_dot(w, xr[c], acc);
            }
            p[k] = acc.x + acc.y;
          }
          const float t = reduce4(p[0], p[1], p[2], p[3]);
          const int rr = first + (lane >> 3);
          if ((lane & 7) == 0 && rr < n_rows) {
            const int r = rg.v_lo + rr;
            const float coarse = a.lm_scale[r] * t;
            const float bnd = fmaf(fabsf(coarse), 1e-6f, a.lm_bound[r] * L1);
            const float lb = coarse - bnd, ub = coarse + bnd;
            if (lb > lane_lb) lane_lb = lb;
            if (!(ub < lane_lb)) {  // NaN bounds stay candidates
              const int slot = atomicAdd(&cnt[warp], 1);
              if (slot < kLmCand) cand[warp * kLmCand + slot] = make_int2(rr, __float_as_int(ub));
            }
          }
      };
      {
        const int g = warp >> 2, wq = warp & 3;
        bool lc_ok = true;
        for (int j = g; j < n_lc; j += 4) {
          lc_ok = lc_wait(j) && lc_ok;
          if (bounded) coarse4(S.ring + ((n_chunks + j) % kSlots) * kSlotBytes, wq * 4, j * kLmRows + wq * 4);
          asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(128) : "memory");  // the group is done with the slot
          if ((threadIdx.x & 127) == 0 && j + kSlots < n_lc) lc_issue(j + kSlots);
        }
        if (!lc_ok) {  // a copy never landed: the token is void (QD_E_TIMEOUT)
          raise_abort(a);
          // wait once more for the group's last chunk in each of its two slots (only
          // those can still be in flight; older phases of a slot are not waited on again)
          const int last = g + (n_lc - 1 - g) / 4 * 4;
          if (last >= g) (void)lc_wait(last);
          if (last - 4 >= g) (void)lc_wait(last - 4);
        }
      }
      const float wmax = warp_max(lane_lb);
      if (lane == 0) wlb[warp] = wmax;
      __syncthreads();
      float LB = -INFINITY;
#pragma unroll
      for (int k = 0; k < kPW; ++k) LB = fmaxf(LB, wlb[k]);
      const int nc = cnt[warp];
      if (!bounded || nc > kLmCand) {
        for (int j0 = warp * 4; j0 < n_rows; j0 += kPW * 4) {
          int rk[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) rk[k] = j0 + k < n_rows ? j0 + k : -1;
          exact4(xr, rk);
        }
      } else {
        // this warp's candidates that reach the CTA's best lower bound, 4 at a time
        int j = 0;
        while (true) {
          int rk[4];
          int got = 0;
          for (; j < nc && got < 4; ++j) {
            const int2 e = cand[warp * kLmCand + j];
            if (!(__int_as_float(e.y) < LB)) rk[got++] = e.x;
          }
          if (got == 0) break;
          for (int k = got; k < 4; ++k) rk[k] = -1;
          exact4(xr, rk);
        }
      }
    }
    // warp argmax (total order: larger value, then lower index)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
  }
  if (!a.with_head && !stage_ok(a, final_hidden(a, rg, epoch, H, S))) return;
  stamp(tl, 2 + kTimelinePerLayer * a.L);

  // CTA partial -> last CTA merges, emits the token and advances the state.
  float* bvs = S.misc;
  uint32_t* bis = reinterpret_cast<uint32_t*>(S.misc + kPW);
  __syncthreads();
  if (lane == 0) { bvs[warp] = bv; bis[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = bvs[0];
    uint32_t i = bis[0];
    for (int w = 1; w < kPW; ++w)
      if (am_better(bvs[w], bis[w], v, i)) { v = bvs[w]; i = bis[w]; }
    a.part_v[cta] = v;
    a.part_i[cta] = i;
    __threadfence();
    const unsigned prev = atomicAdd(a.counter, 1u);
    S.flag[0] = (prev == (unsigned)ng - 1);
  }
  __syncthreads();
  if (!S.flag[0]) return;
  __threadfence();
  float v = kNegMax;
  uint32_t i = 0;
  if (a.with_head) {
    for (int b = threadIdx.x; b < ng; b += kPT) {
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
    if (lane == 0) { bvs[warp] = v; bis[warp] = i; }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (a.with_head) {
      v = bvs[0];
      i = bis[0];
      for (int w = 1; w < kPW; ++w)
        if (am_better(bvs[w], bis[w], v, i)) { v = bvs[w]; i = bis[w]; }
      const int step = a.st->step;
      if (pos + 1 <= a.max_seq) a.tokens[pos + 1] = (int)i;
      if (step < a.st->max_new) {
        a.out_dev[step] = (int)i;
        if (a.out_host) *reinterpret_cast<volatile int*>(a.out_host + step) = (int)i;
      }
      a.st->step = step + 1;
    }
    a.st->pos = pos + 1;
    a.st->epoch = (int)epoch;
    *a.counter = 0u;
    stamp(tl, 3 + kTimelinePerLayer * a.L);
  }
}

}  // namespace qd
