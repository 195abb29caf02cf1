// q4 MatMulNBits GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   Y[b][n] = sum_k X[b][k] * W[n][k],   W = (nibble - 8) * scale (q4, block 32)
//
// Used where the work is a dense contraction: batched decode (b = the sequences
// of a step) and prompt prefill (b = prompt tokens). The weights are operand A
// (M = 128 weight rows per CTA), the activations operand B (N = BN rows of X),
// so the f32 accumulator D[128][BN] lives in TMEM with row n = TMEM lane n.
//
// f32-level accuracy with f16 tensor-core inputs: each weight w = (n-8)*s is an
// exact f32 of at most 15 significant bits, split exactly into
// w_hi = f16(w * 2^S) and w_lo = f16((w * 2^S - w_hi) * 2^11) (S = 10, so scales
// up to 8 stay below the f16 maximum); activations are
// split the same way (x_hi, x_lo * 2^11). Three MMAs per k-step,
//   D_main += A_hi B_hi,   D_corr += A_hi B_lo + A_lo B_hi,
// and y = (D_main + D_corr * 2^-11) * 2^-S leave an error near 2^-22 relative
// (the dropped lo*lo term), i.e. f32 rounding level.
//
// Per CTA: 128 threads. Each k-tile (64 columns = two q4 blocks) is
// dequantised by the threads straight into the 128-byte-swizzled K-major smem
// layout the MMA reads, the activation hi/lo tiles are copied in, and thread 0
// issues the MMAs and commits them to the stage's mbarrier. Two stages overlap
// the dequantisation of tile k+1 with the MMAs of tile k.
#pragma once

#include "common.cuh"

namespace qd {

constexpr int kTcThreads = 128;
constexpr int kTcM = 128;            // weight rows per CTA (UMMA M)
constexpr int kTcK = 64;             // k-tile: one 128-byte swizzle row of f16
constexpr int kWShift = 10;          // weights are scaled by 2^10 into the f16 normal range (|scale| <= 8)
constexpr float kLoScale = 2048.0f;  // lo parts are stored times 2^11
constexpr unsigned long long kTcWaitNs = 1000ull * 1000 * 1000;

enum TcEpi : int {
  kTcStore = 0,     // y[b][n] = acc
  kTcResidual = 1,  // y[b][n] = res[b][n] + acc
  kTcSiluPair = 2,  // rows 2j, 2j+1 are gate j, up j: act[b][j] = silu(g) * u (also split to hi/lo)
};

struct TcArgs {
  // weights: row n's 16-byte blocks at w + n*w_stride, its f16 scales at s + n*s_stride
  const char* w;
  const char* s;
  long long w_stride, s_stride;
  int n_rows;                 // weight rows (N of the GEMM)
  int K;                      // columns (multiple of 64)
  // activations, pre-split: x_hi/x_lo [B rows][K] f16 (row stride K)
  const __half* x_hi;
  const __half* x_lo;
  int B;                      // activation rows actually present (<= BN * gridDim.y)
  // outputs
  float* y;                   // [B][ldy]
  int ldy;
  const float* res;           // residual [B][ldy] (kTcResidual)
  __half* y_hi;               // optional hi/lo split of the output (silu pairs), [B][ldy]
  __half* y_lo;
  int* err;                   // device status word (bit kTcErrTimeout)
};

constexpr int kTcErrTimeout = 8;

// ---- tcgen05 / TMEM helpers ------------------------------------------------------
__device__ __forceinline__ unsigned tc_smem(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

// K-major, 128-byte swizzle, 8-row atoms 1024 B apart (SBO), version 1.
__device__ __forceinline__ unsigned long long umma_desc_k_sw128(unsigned smem_addr) {
  return (unsigned long long)((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) | ((unsigned long long)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ unsigned umma_idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((unsigned)(N >> 3) << 17) | ((unsigned)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(unsigned d_tmem, unsigned long long a, unsigned long long b, unsigned idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"((unsigned)accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(unsigned long long* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(tc_smem(mbar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mbar_init(unsigned long long* b) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_smem(b)) : "memory");
}

__device__ __forceinline__ bool tc_mbar_test(unsigned long long* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(tc_smem(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long tc_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for an mbarrier phase; false if the deadline passed.
__device__ __forceinline__ bool tc_mbar_wait(unsigned long long* b, unsigned parity) {
  if (tc_mbar_test(b, parity)) return true;
  const unsigned long long t0 = tc_now();
  while (!tc_mbar_test(b, parity))
    if (tc_now() - t0 > kTcWaitNs) return false;
  return true;
}

// 32 consecutive TMEM columns of this warp's 32 lanes into registers.
__device__ __forceinline__ void tmem_ld32(unsigned taddr, float (&v)[32]) {
  unsigned r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of element (row r, column k < 64) of an f16 tile in the K-major
// 128-byte-swizzle layout (atoms of 8 rows x 128 B, 1024 B apart).
__device__ __forceinline__ unsigned sw128_off(int r, int k) {
  return (unsigned)((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 3) ^ (r & 7)) & 7) << 4) + ((k & 7) << 1));
}

// Exact split of an f32 of at most 22 significant bits into hi + lo*2^-11.
__device__ __forceinline__ void split_f16(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn((v - __half2float(hi)) * kLoScale);
}

// ---- the kernel ---------------------------------------------------------------------
// Grid: (ceil(n_rows / 128), ceil(B / BN)). Shared memory: 2 stages of
// A_hi, A_lo [128][64] f16 (16 KB each) + B_hi, B_lo [BN][64] f16, 1024-aligned.
template <int BN, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) k_q4_gemm_tc(const TcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment of every tile (the swizzle atoms)
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kA = kTcM * kTcK * 2;       // 16 KB
  constexpr int kB = BN * kTcK * 2;
  constexpr int kStage = 2 * kA + 2 * kB;
  __shared__ unsigned long long mbar[2];
  __shared__ unsigned tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kTcM;
  const int b0 = blockIdx.y * BN;
  const int kt_count = a.K / kTcK;

  if (warp == 0) {  // TMEM: D_main (BN columns) + D_corr (BN columns)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_smem(&tmem_base)),
                 "r"(2 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    tc_mbar_init(&mbar[0]);
    tc_mbar_init(&mbar[1]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = tmem_base;
  const unsigned idesc = umma_idesc_f16_f32(kTcM, BN);
  bool ok = true;

  // thread -> weight row of the tile
  const int row = tid;                       // 0..127
  const int n = n0 + row;
  const bool row_live = n < a.n_rows;
  const char* wrow = a.w + (long long)(row_live ? n : 0) * a.w_stride;
  const __half* srow = reinterpret_cast<const __half*>(a.s + (long long)(row_live ? n : 0) * a.s_stride);

  for (int kt = 0; kt < kt_count; ++kt) {
    const int st = kt & 1;
    unsigned char* A_hi = smem + st * kStage;
    unsigned char* A_lo = A_hi + kA;
    unsigned char* B_hi = A_lo + kA;
    unsigned char* B_lo = B_hi + kB;
    // The MMAs that last read this stage (k-tile kt-2) must be done.
    if (kt >= 2) ok = tc_mbar_wait(&mbar[st], (unsigned)((kt - 2) >> 1) & 1u) && ok;

    // Dequantise this row's two q4 blocks (64 columns) into A_hi / A_lo.
    {
      uint4 q[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      float sc[2] = {0.f, 0.f};
      if (row_live) {
        const uint4* wb = reinterpret_cast<const uint4*>(wrow) + kt * 2;
        q[0] = wb[0];
        q[1] = wb[1];
        sc[0] = __half2float(srow[kt * 2]) * (float)(1 << kWShift);
        sc[1] = __half2float(srow[kt * 2 + 1]) * (float)(1 << kWShift);
      }
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const uint32_t ws[4] = {q[blk].x, q[blk].y, q[blk].z, q[blk].w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {  // 8 columns per word -> one 16-byte chunk of f16
          __align__(16) __half hi8[8], lo8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float v = (float)((int)((ws[wi] >> (4 * i)) & 0xFu) - 8) * sc[blk];
            split_f16(v, hi8[i], lo8[i]);
          }
          const int k = blk * 32 + wi * 8;
          const unsigned off = sw128_off(row, k);
          *reinterpret_cast<uint4*>(A_hi + off) = *reinterpret_cast<const uint4*>(hi8);
          *reinterpret_cast<uint4*>(A_lo + off) = *reinterpret_cast<const uint4*>(lo8);
        }
      }
    }
    // Activation tiles: BN rows x 64 columns of x_hi / x_lo (rows beyond B are zero).
    for (int c = tid; c < BN * 8; c += kTcThreads) {  // 16-byte chunks
      const int r = c >> 3, ch = c & 7;
      const int b = b0 + r;
      uint4 vh = make_uint4(0, 0, 0, 0), vl = make_uint4(0, 0, 0, 0);
      if (b < a.B) {
        vh = *reinterpret_cast<const uint4*>(a.x_hi + (long long)b * a.K + kt * kTcK + ch * 8);
        vl = *reinterpret_cast<const uint4*>(a.x_lo + (long long)b * a.K + kt * kTcK + ch * 8);
      }
      const unsigned off = sw128_off(r, ch * 8);
      *reinterpret_cast<uint4*>(B_hi + off) = vh;
      *reinterpret_cast<uint4*>(B_lo + off) = vl;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kTcK / 16; ++ks) {
        const unsigned long long dah = umma_desc_k_sw128(tc_smem(A_hi) + ks * 32);
        const unsigned long long dal = umma_desc_k_sw128(tc_smem(A_lo) + ks * 32);
        const unsigned long long dbh = umma_desc_k_sw128(tc_smem(B_hi) + ks * 32);
        const unsigned long long dbl = umma_desc_k_sw128(tc_smem(B_lo) + ks * 32);
        const bool acc = kt > 0 || ks > 0;
        umma_f16(tmem, dah, dbh, idesc, acc);
        umma_f16(tmem + BN, dah, dbl, idesc, acc);
        umma_f16(tmem + BN, dal, dbh, idesc, true);
      }
      umma_commit(&mbar[st]);
    }
  }
  // Wait for the last MMAs (both stages' final commits).
  if (kt_count >= 2) ok = tc_mbar_wait(&mbar[(kt_count - 2) & 1], (unsigned)((kt_count - 2) >> 1) & 1u) && ok;
  ok = tc_mbar_wait(&mbar[(kt_count - 1) & 1], (unsigned)((kt_count - 1) >> 1) & 1u) && ok;
  tc_fence_after();

  if (!ok) {
    if (tid == 0 && a.err) atomicOr(a.err, kTcErrTimeout);
  } else {
    // Epilogue: warp w reads TMEM lanes 32w..32w+31 = weight rows n0 + 32w + lane.
    const unsigned lane_base = (unsigned)(warp * 32) << 16;
    const float unscale = 1.0f / (float)(1 << kWShift);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float dm[32], dc[32];
      tmem_ld32(tmem + lane_base + c0, dm);
      tmem_ld32(tmem + lane_base + BN + c0, dc);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int b = b0 + c0 + j;
        const float v = (dm[j] + dc[j] * (1.0f / kLoScale)) * unscale;
        if constexpr (EPI == kTcSiluPair) {
          const float other = __shfl_xor_sync(0xffffffffu, v, 1);  // lane pairs: gate (even), up (odd)
          if ((lane & 1) == 0 && row_live && b < a.B) {
            const int jrow = n >> 1;
            const float act = (v / (1.0f + expf(-v))) * other;
            a.y[(long long)b * a.ldy + jrow] = act;
            if (a.y_hi) {
              __half h, l;
              split_f16(act, h, l);
              a.y_hi[(long long)b * a.ldy + jrow] = h;
              a.y_lo[(long long)b * a.ldy + jrow] = l;
            }
          }
        } else {
          if (row_live && b < a.B) {
            const long long o = (long long)b * a.ldy + n;
            a.y[o] = (EPI == kTcResidual) ? a.res[o] + v : v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
}

// Split f32 rows into the hi/lo f16 operands of the GEMM: x_hi[b][k] = f16(x),
// x_lo[b][k] = f16((x - x_hi) * 2^11). Grid-stride over B*K elements.
__global__ void k_split_hilo(const float* x, int n, __half* hi, __half* lo) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    __half h, l;
    split_f16(x[i], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

}  // namespace qd
