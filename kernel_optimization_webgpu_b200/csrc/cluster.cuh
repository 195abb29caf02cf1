// Batch-1 decode of one token as ONE persistent kernel on thread-block clusters
// of kCC CTAs (one CTA per SM, 512 threads).
//
// Work split of a layer (the reference's per-layer dispatch order,
// webgpu-runtime.js:498-562, fused):
//  * attention clusters (cluster g < kv_heads) own KV head g: each CTA computes
//    1/kCC of the group's q/k/v rows; the cluster exchanges them through
//    distributed shared memory, every CTA applies head RMSNorm + RoPE, the CTA
//    whose position range holds `pos` appends K/V to the cache, each CTA runs
//    the softmax over 1/kCC of the positions, and the partials are combined
//    in-cluster. Each CTA then computes the O-projection rows [o_lo, o_hi) over
//    the group's input columns: a split-K partial of the attention output.
//  * every cluster owns a range of whole 32-column intermediate blocks: its
//    CTAs compute gate/up rows and silu(gate) * up for 1/kCC of them, exchange
//    the activations in-cluster, and compute the down-projection rows
//    [o_lo, o_hi) over the cluster's columns: a split-K partial.
// The two split-K sums (O and down) are the only grid-wide exchanges: every CTA
// adds its partials as 64-bit fixed-point integers (value * 2^32, so the sum is
// exact and independent of arrival order) with red.add, then bumps a counter
// with release semantics; consumers wait on the counter (one thread, acquire)
// and read the sums. Accumulators and counters are double-buffered by launch
// parity; a launch zeroes the other parity's buffers for the next one.
//
// Weights: each CTA's slices of every layer (q/k/v rows, O rows x group columns,
// gate/up pair rows, down rows x cluster columns) are packed contiguously as
// row records (nb q4 blocks of 16 bytes, then nb f16 scales, padded to 16) and
// streamed, with the LM-head rows after them, through a shared-memory ring with
// cp.async.bulk, running ahead of the dependency chain.
//
// Every wait is bounded: counter polls and ring waits have a deadline and an
// abort flag. On expiry the kernel records kErrTimeout and continues in abort
// mode (no further waits on other clusters, every cluster barrier still taken,
// so no cluster-mate is left waiting), drains its own copies and returns.
#pragma once

#include <algorithm>

#include "persist.cuh"

namespace qd {

constexpr int kCC = 8;                     // CTAs per cluster
constexpr int kCT = 512;                   // threads per CTA
constexpr int kCW = kCT / 32;              // warps per CTA
constexpr int kCMaxSlots = 8;              // ring slots at most
constexpr int kCTimelinePerLayer = 11;     // timeline events per layer
constexpr int kCAttnPf = 2;                // cached K/V rows each attention warp loads ahead
__host__ __device__ constexpr int ctimeline_events(int layers) { return 1 + kCTimelinePerLayer * layers + 3; }

// Bytes of a row record of k columns (nb q4 blocks, nb f16 scales, padded to 16).
__host__ __device__ constexpr int crec(int k) { return ((k / 32) * 18 + 15) / 16 * 16; }

// One CTA's share of a layer (identical arithmetic on host and device).
struct CGeo {
  int cl, r, attn;
  int qkv_rows;        // rows of the KV group's [q heads | k | v] row space, from r * qkv_rows
  int o_lo, o_hi;      // output rows of the O and down partials
  int cb_lo, cb_hi;    // the cluster's intermediate blocks
  int p_lo, p_hi;      // this CTA's gate/up pairs (intermediate indices)
  int off[4], sz[4];   // byte offset inside the CTA's layer slice and size: qkv, o, gate/up, down
  int bytes;           // the CTA's layer slice
};

__host__ __device__ inline void cgeo(int cta, int ncl, int H, int I, int NH, int NKV, CGeo& g) {
  g.cl = cta / kCC;
  g.r = cta % kCC;
  g.attn = g.cl < NKV;
  const int G = NH / NKV;
  g.qkv_rows = (G + 2) * 128 / kCC;
  g.o_lo = H * g.r / kCC;
  g.o_hi = H * (g.r + 1) / kCC;
  const int nbI = I / 32;
  g.cb_lo = nbI * g.cl / ncl;
  g.cb_hi = nbI * (g.cl + 1) / ncl;
  const int cp = (g.cb_hi - g.cb_lo) * 32;
  g.p_lo = g.cb_lo * 32 + cp * g.r / kCC;
  g.p_hi = g.cb_lo * 32 + cp * (g.r + 1) / kCC;
  g.sz[0] = g.attn ? g.qkv_rows * crec(H) : 0;
  g.sz[1] = g.attn ? (g.o_hi - g.o_lo) * crec(G * 128) : 0;
  g.sz[2] = 2 * (g.p_hi - g.p_lo) * crec(H);
  g.sz[3] = (g.o_hi - g.o_lo) * crec(cp);
  int o = 0;
  for (int k = 0; k < 4; ++k) {
    g.off[k] = o;
    o += g.sz[k];
  }
  g.bytes = o;
}

// Per-layer norm weights of the cluster kernel, one contiguous f32 table:
// layer l at norms + l * cnorm_stride(H): input (H), post-attention (H), q head (128), k head (128).
__host__ __device__ constexpr int cnorm_stride(int H) { return 2 * H + 2 * kHeadDim; }

struct CArgs {
  const float* norms;           // [L][cnorm_stride(H)]
  char* kv;                     // KV cache: layer l's K at kv + 2l * kv_layer_bytes, V after it
  long long kv_layer_bytes;
  const char* wblob;            // packed slices: layer l at wblob + l * layer_bytes
  long long layer_bytes;
  const long long* cta_off;     // [grid] offset of each CTA's slice inside a layer
  int L, H, I, NH, NKV, vocab, max_seq, row_stride, ncl;
  float eps, scale;
  const __half* embed;
  const float *cos_t, *sin_t, *final_norm;
  long long* acc;               // [2][L][2][H] fixed-point sums (O, down) per launch parity
  unsigned* cnt;                // [2][L][2][32] counters (one 128-byte line each)
  DevState* st;
  int *tokens, *out_dev, *out_host;
  float* logits;
  float* hidden;                // [H] residual stream after the last layer
  float* part_v;
  uint32_t* part_i;
  unsigned* counter;
  int with_head;
  int slot_bytes, n_slots, lm_rows;
  unsigned long long* timeline;  // optional [grid][ctimeline_events(L)]
  unsigned long long* fine;      // optional [grid][L][kCFine] SM clock stamps inside each layer
};
constexpr int kCFine = 28;

// ---- cluster and memory-order helpers -----------------------------------------------
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ unsigned cl_addr(const void* p, int rank) {
  unsigned o;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(o) : "r"(smem_u32(p)), "r"(rank));
  return o;
}
__device__ __forceinline__ float ld_cl(unsigned a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ float2 ld_cl2(unsigned a) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_s64(long long* p, long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ long long ld_relaxed_s64(const long long* p) {
  long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Fixed point with 32 fraction bits: exact for |v| >= 2^-8, error <= 2^-33 below.
__device__ __forceinline__ long long to_fx(float v) { return __float2ll_rn(v * 4294967296.0f); }
__device__ __forceinline__ float from_fx(long long s) { return (float)((double)s * 2.3283064365386963e-10); }

struct CShared {
  char* ring;
  unsigned long long* mbar;  // [kCMaxSlots]
  float *rv, *rv2;           // residual stream r_l and r_l' (after attention), [H]
  float* xs;                 // stage-dot activations (swizzled); attention warp partials
  float* res;                // [kCT] stage-dot row results
  float* grp;                // [(G+2)*128] the group's q/k/v rows
  float* exq;                // [kCT] this CTA's q/k/v rows (read by the cluster)
  float* exa;                // [kCT] this CTA's activations (read by the cluster)
  float *qs, *kn, *vn;       // [G*128], [128], [128]
  float* apo;                // [G*128] this CTA's attention partial (read by the cluster)
  float2* apm;               // [G] its (max, sum)
  float* fw;                 // [G*kCC] combine weights of the cluster's partials
  float* wf;                 // [G*kCW] per-warp rescale factors of this CTA's partial
  float2* wml;               // [kCW*G] per-warp (max, sum)
  float* red;                // [kCW]
  int* flag;                 // [4]
};

// Ring state of one CTA (thread 0 issues; every thread waits).
struct CRing {
  int n_chunks, n_layer_chunks, kpl, issued;
  long long base;            // this CTA's slice offset inside a layer
  int v_lo, v_hi;            // LM-head rows of this CTA
};

__device__ __forceinline__ bool c_aborted(const CArgs& a) {
  return *reinterpret_cast<volatile int*>(&a.st->abort) != 0;
}
__device__ __forceinline__ void c_raise(const CArgs& a) {
  atomicOr(&a.st->err, kErrTimeout);
  atomicExch(&a.st->abort, 1);
}

// Thread 0: put chunk i of this CTA's stream in flight into its slot (none once
// the CTA runs in abort mode).
__device__ __forceinline__ void c_issue(const CArgs& a, const CShared& S, const CGeo& g, CRing& R, int i, bool live) {
  if (i >= R.n_chunks || !live) return;
  const char* src;
  unsigned bytes;
  if (i < R.n_layer_chunks) {
    const int l = i / R.kpl, kind = g.attn ? i % R.kpl : 2 + i % R.kpl;
    src = a.wblob + (long long)l * a.layer_bytes + R.base + g.off[kind];
    bytes = (unsigned)g.sz[kind];
  } else {
    const int j = i - R.n_layer_chunks;
    const int r0 = R.v_lo + j * a.lm_rows, r1 = min(R.v_hi, r0 + a.lm_rows);
    src = reinterpret_cast<const char*>(a.embed + (long long)r0 * a.H);
    bytes = (unsigned)((r1 - r0) * a.H * 2);
  }
  // The slot's previous contents were only read (generic proxy) before the CTA
  // barrier that precedes this call, so no proxy fence is needed.
  const int slot = i % a.n_slots;
  mbar_arrive_tx(&S.mbar[slot], bytes);
  if (bytes) bulk_load_hint(S.ring + (size_t)slot * a.slot_bytes, src, bytes, &S.mbar[slot], policy_evict_first());
  R.issued = i + 1;
}

// Every thread: wait for chunk i (bounded; a chunk never issued is not waited for).
__device__ __forceinline__ const char* c_wait(const CArgs& a, const CShared& S, const CRing& R, int i, bool& ok) {
  const int slot = i % a.n_slots;
  const char* p = S.ring + (size_t)slot * a.slot_bytes;
  if (i >= R.issued) {  // only after an abort: R.issued is thread 0's view, broadcast below
    ok = false;
    return p;
  }
  const unsigned parity = (unsigned)(i / a.n_slots) & 1u;
  if (mbar_test(&S.mbar[slot], parity)) return p;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_test(&S.mbar[slot], parity)) return p;
    if ((it & 63) == 0 && gtimer() - t0 > kWaitNs) {
      ok = false;
      return p;
    }
  }
}

// Thread 0: wait until counter p reaches `target` (bounded). False on timeout or abort.
__device__ __forceinline__ bool c_wait_count(const CArgs& a, const unsigned* p, unsigned target) {
  if (ld_acquire(p) >= target) return true;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 1;; ++it) {
    __nanosleep(32);
    if (ld_acquire(p) >= target) return true;
    if ((it & 31) == 0 && (c_aborted(a) || gtimer() - t0 > kWaitNs)) return false;
  }
}

__device__ __forceinline__ void cstamp(unsigned long long* tl, int ev) {
  if (tl && threadIdx.x == 0) tl[ev] = gtimer();
}
__device__ __forceinline__ void cfine(unsigned long long* fl, int ev) {
  if (fl && threadIdx.x == 0) fl[ev] = clock64();
}

// Dot products of n row records (nb <= LB blocks each, row i at chunk + i*rec)
// against the staged activations: res[i] = sum_b scale(i,b) * dot(block(i,b), x_b).
// Lane b of each group of LB lanes owns block b and holds its 32 activations in
// registers for the whole stage; a warp takes NB row-steps (32/LB rows each) at
// a time so that NB independent dot chains overlap.
template <int LB, int NB>
__device__ __forceinline__ void cdots(const char* chunk, int n, int nb, int rec, const float* xs, float* res) {
  constexpr int RPW = 32 / LB;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / LB, b = lane % LB;
  const bool live = b < nb;
  float2 xr[16];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = reinterpret_cast<const float4*>(xs)[xs_slot(b * 8 + q)];
    xr[2 * q] = make_float2(v.x, v.y);
    xr[2 * q + 1] = make_float2(v.z, v.w);
  }
  const int steps = (n + RPW - 1) / RPW;
  for (int s0 = warp * NB; s0 < steps; s0 += kCW * NB) {
    uint4 w[NB];
    float sc[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int row = (s0 + k) * RPW + sub;
      w[k] = make_uint4(0u, 0u, 0u, 0u);
      sc[k] = 0.0f;
      if (live && s0 + k < steps && row < n) {
        const char* rp = chunk + (size_t)row * rec;
        w[k] = *reinterpret_cast<const uint4*>(rp + b * 16);
        sc[k] = __half2float(*reinterpret_cast<const __half*>(rp + nb * 16 + b * 2));
      }
    }
    float p[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k) p[k] = sc[k] * q4_block_dot(w[k], xr);
    if constexpr (LB == 32 && NB == 4) {
      const float t = reduce4(p[0], p[1], p[2], p[3]);
      const int row = s0 + (lane >> 3);
      if ((lane & 7) == 0 && row < n) res[row] = t;
    } else {
#pragma unroll
      for (int k = 0; k < NB; ++k) {
#pragma unroll
        for (int o = LB / 2; o > 0; o >>= 1) p[k] += __shfl_xor_sync(0xffffffffu, p[k], o);
        const int row = (s0 + k) * RPW + sub;
        if (b == 0 && s0 + k < steps && row < n) res[row] = p[k];
      }
    }
  }
}

__device__ __forceinline__ void cdots_any(const char* chunk, int n, int nb, int rec, const float* xs, float* res) {
  if (nb > 16) cdots<32, 4>(chunk, n, nb, rec, xs, res);
  else if (nb > 8) cdots<16, 2>(chunk, n, nb, rec, xs, res);
  else cdots<8, 2>(chunk, n, nb, rec, xs, res);
}

// Sum of squares of v[0..n) over the CTA (every thread gets the total); ends with a barrier.
__device__ __forceinline__ float c_sumsq(const float* v, int n, float* red) {
  float ss = 0.0f;
  for (int e = threadIdx.x; e < n; e += kCT) ss += v[e] * v[e];
  ss = warp_sum(ss);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t += red[w];
  return t;
}

// ---- the kernel -------------------------------------------------------------------
template <int G, typename KVT>
__global__ void __launch_bounds__(kCT, 1) k_decode_cluster(const __grid_constant__ CArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int cta = blockIdx.x, ng = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = a.H, KVS = a.NKV * kHeadDim;
  constexpr int GR = (G + 2) * kHeadDim;   // rows of a KV group's [q heads | k | v]

  CGeo g;
  cgeo(cta, a.ncl, H, a.I, a.NH, a.NKV, g);
  const int cp = (g.cb_hi - g.cb_lo) * 32;     // this cluster's intermediate columns
  const int np = g.p_hi - g.p_lo;
  const int no = g.o_hi - g.o_lo;

  CShared S;
  S.ring = reinterpret_cast<char*>(smem);
  char* q = reinterpret_cast<char*>(smem) + (size_t)a.n_slots * a.slot_bytes;
  S.mbar = reinterpret_cast<unsigned long long*>(q);
  q += kCMaxSlots * 8;
  float* f = reinterpret_cast<float*>(q);
  const int xs_n = max((max(H, cp) + 31) / 32 * 32, kCW * G * kHeadDim);
  S.rv = f; f += H;
  S.rv2 = f; f += H;
  S.xs = f; f += xs_n;
  S.res = f; f += kCT;
  S.grp = f; f += GR;
  S.exq = f; f += kCT;
  S.exa = f; f += kCT;
  S.qs = f; f += G * kHeadDim;
  S.kn = f; f += kHeadDim;
  S.vn = f; f += kHeadDim;
  S.apo = f; f += G * kHeadDim;
  S.apm = reinterpret_cast<float2*>(f); f += 2 * G;
  S.fw = f; f += G * kCC;
  S.wf = f; f += G * kCW;
  S.wml = reinterpret_cast<float2*>(f); f += 2 * kCW * G;
  S.red = f; f += kCW;
  S.flag = reinterpret_cast<int*>(f);

  const int pos = a.st->pos;
  const unsigned epoch = (unsigned)a.st->epoch + 1u;
  const int par = (int)(epoch & 1u);
  if (pos < 0 || pos >= a.max_seq) {  // the host keeps positions in range; never index out of bounds
    if (cta == 0 && threadIdx.x == 0) atomicOr(&a.st->err, kErrPosition);
    return;  // uniform over the grid: no cluster barrier has been taken
  }
  unsigned long long* tl = a.timeline ? a.timeline + (long long)cta * ctimeline_events(a.L) : nullptr;
  cstamp(tl, 0);

  // Zero the other parity's accumulators and counters for the next launch.
  {
    const int op = par ^ 1;
    long long* acc_o = a.acc + (long long)op * a.L * 2 * H;
    const long long n_acc = (long long)a.L * 2 * H;
    for (long long i = (long long)cta * kCT + threadIdx.x; i < n_acc; i += (long long)ng * kCT) acc_o[i] = 0;
    unsigned* cn = a.cnt + (long long)op * a.L * 2 * 32;
    for (int i = cta * kCT + threadIdx.x; i < a.L * 2 * 32; i += ng * kCT) cn[i] = 0u;
  }
  long long* acc = a.acc + (long long)par * a.L * 2 * H;
  unsigned* cnt = a.cnt + (long long)par * a.L * 2 * 32;

  // Ring set-up.
  CRing R;
  R.kpl = g.attn ? 4 : 2;
  R.n_layer_chunks = R.kpl * a.L;
  range_of(a.vocab, cta, ng, R.v_lo, R.v_hi);
  R.n_chunks = R.n_layer_chunks + (a.with_head ? (R.v_hi - R.v_lo + a.lm_rows - 1) / a.lm_rows : 0);
  R.base = a.cta_off[cta];
  R.issued = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.n_slots; ++s) mbar_init(&S.mbar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < a.n_slots; ++i) c_issue(a, S, g, R, i, true);
  }
  R.issued = min(R.n_chunks, a.n_slots);
  __syncthreads();
  int chunk = 0;
  bool live = true;  // false once this CTA has seen a wait expire or the abort flag (abort mode)

  // Consume chunk `chunk` (all threads), returning its slot.
  // Each thread waits on the slot's mbarrier itself (no CTA barrier). A wait that
  // expires raises the abort flag and puts this thread in abort mode; the next
  // grid-wide exchange makes that uniform over the CTA.
  auto take = [&]() -> const char* {
    bool ok = true;
    const char* p = c_wait(a, S, R, chunk, ok);
    if (!ok) {
      if (live) c_raise(a);
      live = false;
    }
    return p;
  };
  // After the CTA is done reading the chunk: thread 0 refills its slot, every
  // thread advances its copy of the ring state.
  auto release = [&]() {
    __syncthreads();
    if (threadIdx.x == 0) c_issue(a, S, g, R, chunk + a.n_slots, live);
    if (live) R.issued = min(R.n_chunks, max(R.issued, chunk + a.n_slots + 1));
    ++chunk;
  };
  // Grid-wide exchange: thread 0 waits for `target` producers, then everybody reads.
  // Once any CTA has given up (abort flag), every CTA stops waiting on others.
  auto wait_count = [&](const unsigned* p, unsigned target) {
    int bad = live ? 0 : 1;
    if (threadIdx.x == 0) {
      if (live) bad = c_wait_count(a, p, target) ? 0 : 1;
      if (!bad && c_aborted(a)) bad = 2;
    }
    bad = __syncthreads_or(bad);
    if (bad) {
      if (live && threadIdx.x == 0) c_raise(a);
      live = false;
    }
  };

  // Layer-0 input: the embedding row of tokens[pos], read by every CTA.
  {
    int tok = a.tokens[pos];
    if (tok < 0 || tok >= a.vocab) {
      if (cta == 0 && threadIdx.x == 0) atomicOr(&a.st->err, kErrToken);
      tok = 0;
    }
    const __half* er = a.embed + (long long)tok * H;
    for (int e = threadIdx.x; e < H; e += kCT) S.rv[e] = __half2float(er[e]);
  }
  __syncthreads();

  // Attention position range of this CTA (positions 0..pos split over the cluster).
  const int n_pos = pos + 1, chp = (n_pos + kCC - 1) / kCC;
  const int pa_lo = min(n_pos, g.r * chp), pa_hi = min(n_pos, pa_lo + chp);
  const bool owner = pa_lo <= pos && pos < pa_hi;

  for (int l = 0; l < a.L; ++l) {
    const float* nrm = a.norms + (long long)l * cnorm_stride(H);
    // this thread's input-norm and post-attention-norm weights, loaded before any wait
    float w_in[2], w_post[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int e = threadIdx.x + k * kCT;
      w_in[k] = e < H ? nrm[e] : 0.0f;
      w_post[k] = e < H ? nrm[H + e] : 0.0f;
    }
    long long* acc_ol = acc + (long long)(2 * l) * H;
    long long* acc_dl = acc + (long long)(2 * l + 1) * H;
    unsigned* cnt_ol = cnt + (2 * l) * 32;
    unsigned* cnt_dl = cnt + (2 * l + 1) * 32;
    const int ev = 1 + l * kCTimelinePerLayer;
    unsigned long long* fl = a.fine ? a.fine + ((long long)cta * a.L + l) * kCFine : nullptr;

    // Attention inputs that do not depend on this token (head-norm weights, this
    // position's RoPE row, the first cached K/V rows), loaded before the wait so
    // that their latency hides behind it.
    const int kv = g.cl;
    KVT* kc = reinterpret_cast<KVT*>(a.kv + (long long)(2 * l) * a.kv_layer_bytes);
    KVT* vc = reinterpret_cast<KVT*>(a.kv + (long long)(2 * l + 1) * a.kv_layer_bytes);
    const long long row_el = (long long)KVS;
    float4 wq4 = make_float4(0.f, 0.f, 0.f, 0.f), wk4 = wq4, cr = wq4, sr = wq4;
    float4 kpf[kCAttnPf], vpf[kCAttnPf];
#pragma unroll
    for (int j = 0; j < kCAttnPf; ++j) kpf[j] = vpf[j] = wq4;
    if (g.attn) {
      wq4 = reinterpret_cast<const float4*>(nrm + 2 * H)[lane];
      wk4 = reinterpret_cast<const float4*>(nrm + 2 * H + kHeadDim)[lane];
      const int pair0 = (4 * lane) & (kHeadDim / 2 - 1);
      const long long toff = (long long)pos * a.row_stride + pair0;
      cr = *reinterpret_cast<const float4*>(a.cos_t + toff);
      sr = *reinterpret_cast<const float4*>(a.sin_t + toff);
#pragma unroll
      for (int j = 0; j < kCAttnPf; ++j) {
        const int pp = pa_lo + warp + j * kCW;
        if (pp < pa_hi && pp < pos) {
          kpf[j] = ld4<KVT>(kc + pp * row_el + kv * kHeadDim + 4 * lane);
          vpf[j] = ld4<KVT>(vc + pp * row_el + kv * kHeadDim + 4 * lane);
        }
      }
    }

    // ---- r_l: the previous layer's down sums + r'_{l-1} ----
    if (l > 0) {
      const long long* acc_dp = acc + (long long)(2 * l - 1) * H;
      wait_count(cnt + (2 * l - 1) * 32, (unsigned)(a.ncl * kCC));
      for (int e = threadIdx.x; e < H; e += kCT) S.rv[e] = S.rv2[e] + from_fx(ld_relaxed_s64(acc_dp + e));
      __syncthreads();
    }
    cstamp(tl, ev + 0);
    cfine(fl, 0);

    if (g.attn) {
      // 1. input RMSNorm + this CTA's q/k/v rows
      {
        const float inv = rsqrtf(c_sumsq(S.rv, H, S.red) / (float)H + a.eps);
        cfine(fl, 1);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int e = threadIdx.x + k * kCT;
          if (e < H) xs_store(S.xs, e, S.rv[e] * inv * w_in[k]);
        }
        cfine(fl, 2);
        const char* w = take();
        cstamp(tl, ev + 1);
        cfine(fl, 3);
        cdots_any(w, g.qkv_rows, H / 32, crec(H), S.xs, S.res);
        cfine(fl, 4);
        __syncthreads();
        if (threadIdx.x < g.qkv_rows) S.exq[threadIdx.x] = S.res[threadIdx.x];
        release();
        cstamp(tl, ev + 2);
        cfine(fl, 5);
      }
      // 2. the group's rows from the cluster
      cluster_sync_all();
      cstamp(tl, ev + 3);
      cfine(fl, 6);
      for (int e = threadIdx.x; e < GR; e += kCT) {
        const int src = e / g.qkv_rows;
        S.grp[e] = ld_cl(cl_addr(S.exq + (e - src * g.qkv_rows), src));
      }
      __syncthreads();
      cfine(fl, 7);
      // 3. head RMSNorm + RoPE (q heads, k); the owner of `pos` appends K/V to the cache
      for (int t = warp; t < G + 2; t += kCW) {
        const float4 x = reinterpret_cast<const float4*>(S.grp + t * kHeadDim)[lane];
        KVT* krow = kc + (long long)pos * row_el + kv * kHeadDim + 4 * lane;
        KVT* vrow = vc + (long long)pos * row_el + kv * kHeadDim + 4 * lane;
        if (t == G + 1) {
          if (owner) reinterpret_cast<float4*>(S.vn)[lane] = st4<KVT>(vrow, x);
          continue;
        }
        const float4 w4 = t < G ? wq4 : wk4;
        float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / (float)kHeadDim + a.eps);
        const float4 y = make_float4(x.x * inv * w4.x, x.y * inv * w4.y, x.z * inv * w4.z, x.w * inv * w4.w);
        float4 pq;
        pq.x = __shfl_xor_sync(0xffffffffu, y.x, 16);
        pq.y = __shfl_xor_sync(0xffffffffu, y.y, 16);
        pq.z = __shfl_xor_sync(0xffffffffu, y.z, 16);
        pq.w = __shfl_xor_sync(0xffffffffu, y.w, 16);
        const float sign = (lane >= 16) ? 1.0f : -1.0f;
        const float4 rr = make_float4(y.x * cr.x + sign * pq.x * sr.x, y.y * cr.y + sign * pq.y * sr.y,
                                      y.z * cr.z + sign * pq.z * sr.z, y.w * cr.w + sign * pq.w * sr.w);
        if (t < G) reinterpret_cast<float4*>(S.qs + t * kHeadDim)[lane] = rr;
        else if (owner) reinterpret_cast<float4*>(S.kn)[lane] = st4<KVT>(krow, rr);
      }
      __syncthreads();
      cfine(fl, 8);
      // 4. online softmax per warp over this CTA's positions pa_lo + warp + k*kCW < pa_hi
      {
        float4 qv[G];
#pragma unroll
        for (int h = 0; h < G; ++h) qv[h] = reinterpret_cast<const float4*>(S.qs + h * kHeadDim)[lane];
        float m[G], ls[G];
        float4 ac[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          m[h] = -INFINITY;
          ls[h] = 0.0f;
          ac[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int p = pa_lo + warp; p < pa_hi; p += kCW) {
          float4 k4 = kpf[0], v4 = vpf[0];
          if (p == pos) {
            k4 = reinterpret_cast<const float4*>(S.kn)[lane];
            v4 = reinterpret_cast<const float4*>(S.vn)[lane];
          }
#pragma unroll
          for (int j = 0; j + 1 < kCAttnPf; ++j) {
            kpf[j] = kpf[j + 1];
            vpf[j] = vpf[j + 1];
          }
          const int pn = p + kCAttnPf * kCW;
          if (pn < pa_hi && pn < pos) {
            kpf[kCAttnPf - 1] = ld4<KVT>(kc + pn * row_el + kv * kHeadDim + 4 * lane);
            vpf[kCAttnPf - 1] = ld4<KVT>(vc + pn * row_el + kv * kHeadDim + 4 * lane);
          }
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float d = qv[h].x * k4.x + qv[h].y * k4.y + qv[h].z * k4.z + qv[h].w * k4.w;
            const float sc = warp_sum(d) * a.scale;
            const float mn = fmaxf(m[h], sc);
            const float co = expf(m[h] - mn), cn = expf(sc - mn);
            ls[h] = ls[h] * co + cn;
            ac[h] = make_float4(ac[h].x * co + cn * v4.x, ac[h].y * co + cn * v4.y, ac[h].z * co + cn * v4.z,
                                ac[h].w * co + cn * v4.w);
            m[h] = mn;
          }
        }
        cfine(fl, 9);
        float* wacc = S.xs;  // [kCW][G][128]
#pragma unroll
        for (int h = 0; h < G; ++h) {
          reinterpret_cast<float4*>(wacc + (warp * G + h) * kHeadDim)[lane] = ac[h];
          if (lane == 0) S.wml[warp * G + h] = make_float2(m[h], ls[h]);
        }
        __syncthreads();
        // CTA partial: m_c = max over warps, l_c and acc_c rescaled to m_c (unnormalised).
        static_assert(kCW == 16, "the merge takes 16 warps per head in one half-warp");
        if (threadIdx.x < ((G * kCW + 31) / 32) * 32) {
          const int h = threadIdx.x / kCW, w = threadIdx.x % kCW;
          const bool on = h < G;
          const float2 mw = on ? S.wml[w * G + h] : make_float2(-INFINITY, 0.0f);
          float M = mw.x;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
          const float e = mw.y > 0.0f ? expf(mw.x - M) : 0.0f;
          float Ls = mw.y * e;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o);
          if (on) {
            S.wf[h * kCW + w] = e;
            if (w == 0) S.apm[h] = make_float2(Ls > 0.0f ? M : -INFINITY, Ls);
          }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < G * kHeadDim; e += kCT) {
          const int h = e / kHeadDim, d = e % kHeadDim;
          float o = 0.0f;
#pragma unroll
          for (int w = 0; w < kCW; ++w) o += wacc[(w * G + h) * kHeadDim + d] * S.wf[h * kCW + w];
          S.apo[e] = o;
        }
      }
      cstamp(tl, ev + 4);
      cfine(fl, 10);
      // 5. combine the cluster's partials into the O-projection input
      cluster_sync_all();
      cstamp(tl, ev + 5);
      cfine(fl, 11);
      if (threadIdx.x < ((G * kCC + 31) / 32) * 32) {
        const int h = threadIdx.x / kCC, c = threadIdx.x % kCC;
        const bool on = h < G;
        float2 mc = make_float2(-INFINITY, 0.0f);
        if (on) mc = ld_cl2(cl_addr(S.apm + h, c));
        float M = mc.x;
#pragma unroll
        for (int o = kCC / 2; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float e = mc.y > 0.0f ? expf(mc.x - M) : 0.0f;
        float Ls = mc.y * e;
#pragma unroll
        for (int o = kCC / 2; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o);
        if (on) S.fw[h * kCC + c] = Ls > 0.0f ? e / Ls : 0.0f;
      }
      __syncthreads();
      for (int e = threadIdx.x; e < G * kHeadDim; e += kCT) {
        const int h = e / kHeadDim;
        float pv[kCC];
#pragma unroll
        for (int c = 0; c < kCC; ++c) pv[c] = ld_cl(cl_addr(S.apo + e, c));  // all in flight at once
        float o = 0.0f;
#pragma unroll
        for (int c = 0; c < kCC; ++c) o += pv[c] * S.fw[h * kCC + c];
        xs_store(S.xs, e, o);
      }
      __syncthreads();
      cfine(fl, 12);
      // 6. O-projection partial over the group's columns -> fixed-point sums
      {
        const char* w = take();
        cfine(fl, 13);
        cdots_any(w, no, G * kHeadDim / 32, crec(G * kHeadDim), S.xs, S.res);
        cfine(fl, 14);
        __syncthreads();
        if (threadIdx.x < no && live) red_add_s64(acc_ol + g.o_lo + threadIdx.x, to_fx(S.res[threadIdx.x]));
        __syncthreads();
        cfine(fl, 15);
        if (threadIdx.x == 0 && live) red_release_add(cnt_ol, 1u);
        release();
        cstamp(tl, ev + 6);
        cfine(fl, 16);
      }
    }

    // ---- r_l' = r_l + O sums ----
    wait_count(cnt_ol, (unsigned)(a.NKV * kCC));
    for (int e = threadIdx.x; e < H; e += kCT) S.rv2[e] = S.rv[e] + from_fx(ld_relaxed_s64(acc_ol + e));
    __syncthreads();
    cstamp(tl, ev + 7);
    cfine(fl, 17);

    // 7. post-attention RMSNorm + gate/up + silu * up for this CTA's pairs
    {
      const float inv = rsqrtf(c_sumsq(S.rv2, H, S.red) / (float)H + a.eps);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int e = threadIdx.x + k * kCT;
        if (e < H) xs_store(S.xs, e, S.rv2[e] * inv * w_post[k]);
      }
      cfine(fl, 18);
      const char* w = take();
      cfine(fl, 19);
      cdots_any(w, 2 * np, H / 32, crec(H), S.xs, S.res);
      cfine(fl, 20);
      __syncthreads();
      if (threadIdx.x < np) {
        const float gt = S.res[threadIdx.x], upv = S.res[np + threadIdx.x];
        S.exa[threadIdx.x] = (gt / (1.0f + expf(-gt))) * upv;
      }
      release();
      cstamp(tl, ev + 8);
      cfine(fl, 21);
    }
    // 8. the cluster's activations, then the down-projection partial
    cluster_sync_all();
    cstamp(tl, ev + 9);
    cfine(fl, 22);
    for (int e = threadIdx.x; e < cp; e += kCT) {
      int src = 0;
#pragma unroll
      for (int c = 1; c < kCC; ++c)
        if (e >= cp * c / kCC) src = c;
      xs_store(S.xs, e, ld_cl(cl_addr(S.exa + (e - cp * src / kCC), src)));
    }
    __syncthreads();
    cfine(fl, 23);
    {
      const char* w = take();
      cfine(fl, 24);
      cdots_any(w, no, cp / 32, crec(cp), S.xs, S.res);
      cfine(fl, 25);
      __syncthreads();
      if (threadIdx.x < no && live) red_add_s64(acc_dl + g.o_lo + threadIdx.x, to_fx(S.res[threadIdx.x]));
      __syncthreads();
      if (threadIdx.x == 0 && live) red_release_add(cnt_dl, 1u);
      release();
      cstamp(tl, ev + 10);
      cfine(fl, 26);
    }
  }

  // ---- r_L, final norm, LM head + argmax ----
  float w_fin[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int e = threadIdx.x + k * kCT;
    w_fin[k] = e < H ? a.final_norm[e] : 0.0f;
  }
  {
    const long long* acc_dp = acc + (long long)(2 * a.L - 1) * H;
    wait_count(cnt + (2 * a.L - 1) * 32, (unsigned)(a.ncl * kCC));
    for (int e = threadIdx.x; e < H; e += kCT) {
      S.rv[e] = S.rv2[e] + from_fx(ld_relaxed_s64(acc_dp + e));
      if (cta == 0) a.hidden[e] = S.rv[e];
    }
    __syncthreads();
  }
  // No CTA reads another's shared memory after this barrier, so each may exit freely.
  cluster_sync_all();
  cstamp(tl, 1 + kCTimelinePerLayer * a.L);

  float bv = kNegMax;
  uint32_t bi = 0;
  if (a.with_head) {
    const float inv = rsqrtf(c_sumsq(S.rv, H, S.red) / (float)H + a.eps);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int e = threadIdx.x + k * kCT;
      if (e < H) S.xs[e] = S.rv[e] * inv * w_fin[k];
    }
    __syncthreads();
    // lane holds columns (c*32 + lane)*8 .. +7, c < H/256
    const int kc8 = H / 256;
    float2 xr[4][4];
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
    const int rpr = H / 8;  // uint4 per table row
    for (int j = 0; chunk < R.n_chunks; ++j) {
      const char* w = take();
      const int r0 = R.v_lo + j * a.lm_rows, nr = min(R.v_hi - r0, a.lm_rows);
      for (int rr = warp; rr < nr; rr += kCW) {
        const uint4* row = reinterpret_cast<const uint4*>(w) + (size_t)rr * rpr;
        float2 accv = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (c < kc8) accv = f16x8_dot(row[c * 32 + lane], xr[c], accv);
        const float v = warp_sum(accv.x + accv.y);
        const uint32_t idx = (uint32_t)(r0 + rr);
        if (lane == 0) a.logits[idx] = v;
        if (am_better(v, idx, bv, bi)) {
          bv = v;
          bi = idx;
        }
      }
      release();
    }
  }
  cstamp(tl, 2 + kCTimelinePerLayer * a.L);
  // Drain: any chunk still in flight (abort mode) lands before the CTA exits.
  {
    bool ok = true;
    for (int i = chunk; i < R.issued; ++i) {
      const int slot = i % a.n_slots;
      const unsigned parity = (unsigned)(i / a.n_slots) & 1u;
      const unsigned long long t0 = gtimer();
      while (!mbar_test(&S.mbar[slot], parity))
        if (gtimer() - t0 > kWaitNs) { ok = false; break; }
    }
    (void)ok;
  }

  // CTA partial -> the last CTA merges, emits the token and advances the state.
  float* bvs = S.res;
  uint32_t* bis = reinterpret_cast<uint32_t*>(S.res + kCW);
  __syncthreads();
  if (lane == 0) {
    bvs[warp] = bv;
    bis[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = bvs[0];
    uint32_t i = bis[0];
    for (int w = 1; w < kCW; ++w)
      if (am_better(bvs[w], bis[w], v, i)) {
        v = bvs[w];
        i = bis[w];
      }
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
    for (int b = threadIdx.x; b < ng; b += kCT) {
      const float pv = __ldcg(a.part_v + b);
      const uint32_t pi = __ldcg(a.part_i + b);
      if (am_better(pv, pi, v, i)) {
        v = pv;
        i = pi;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (am_better(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (lane == 0) {
      bvs[warp] = v;
      bis[warp] = i;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (a.with_head) {
      v = bvs[0];
      i = bis[0];
      for (int w = 1; w < kCW; ++w)
        if (am_better(bvs[w], bis[w], v, i)) {
          v = bvs[w];
          i = bis[w];
        }
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
    cstamp(tl, 3 + kCTimelinePerLayer * a.L);
  }
}

// Shared-memory bytes of the kernel for a given ring.
__host__ inline size_t cluster_smem_bytes(int H, int G, int cp_max, int slot_bytes, int n_slots) {
  const int xs_n = std::max((std::max(H, cp_max) + 31) / 32 * 32, kCW * G * kHeadDim);
  const size_t floats = (size_t)2 * H + xs_n + kCT + (G + 2) * kHeadDim + 2 * kCT + G * kHeadDim + 2 * kHeadDim +
                        G * kHeadDim + 2 * G + G * kCC + G * kCW + 2 * kCW * G + kCW + 4;
  return (size_t)n_slots * slot_bytes + kCMaxSlots * 8 + floats * 4;
}

}  // namespace qd
