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
// Per CTA: 128 R consumer threads (R = 2, or 4 for the prefill tile BN = 256), a
// producer warp and an MMA-issuer warp. Each k-tile (64 columns = two q4 blocks)
// is dequantised by R threads per weight row straight into the 128-byte-swizzled
// K-major smem layout the MMA reads, the activation hi/lo tiles are copied in by
// TMA, and one lane of the issuer warp issues the MMAs once the consumers have
// arrived on the A buffer's barrier, committing them to the stage's mbarriers. A
// double-buffered A stage overlaps the dequantisation of tile k+1 with the MMAs of
// tile k. The chain dequantise -> hand-over -> MMA issue of a k-tile is what kept the
// tensor pipe waiting, so it is spread over as many threads as the block allows and
// carries no CTA barrier (prefill, 32 x 512 prompt rows: 235k prompt tok/s with one
// thread per row issuing behind a CTA barrier, 271k with two, 284k with four; 294k
// once a warp of its own issues the MMAs).
//
// Split-K: gridDim.z CTAs share a row tile, each over its own run of k-tiles,
// and store partial sums [split][B][N]; the kernel that consumes the result
// adds the splits in a fixed order (deterministic, no atomics). This keeps
// >= 128 CTAs busy on the narrow decode projections (N = 1024..6144).
//
// The LM head (f16 embedding table, exact in f16) uses the weights directly as
// A_hi with no A_lo: two MMAs per k-step. Its epilogue reduces each sequence's
// 128 logits of the CTA to one (max, lowest index) pair, so only 8 bytes per
// (sequence, CTA) leave the kernel unless the caller also asks for the logits.
#pragma once

#include "common.cuh"
#include "tma.cuh"

namespace qd {

constexpr int kTcM = 128;            // weight rows per CTA (UMMA M)
constexpr int kTcK = 64;             // k-tile: one 128-byte swizzle row of f16
constexpr int kWShift = 10;          // weights are scaled by 2^10 into the f16 normal range (|scale| <= 8)
constexpr float kLoScale = 2048.0f;  // lo parts are stored times 2^11
constexpr unsigned long long kTcWaitNs = 1000ull * 1000 * 1000;

enum TcEpi : int {
  kTcStore = 0,   // y[split][b][n] = acc (split-K partials; the consumer sums them)
  kTcArgmax = 1,  // per (b, CTA) best (value, row) over the CTA's 128 rows; logits to y if set
  kTcSilu = 2,    // rows 2j, 2j+1 = gate j, up j (no split-K): y_hi/y_lo[b][j] = split(silu(gate) * up)
};

struct TcArgs {
  // Tensor maps (filled by the host launcher from the pointers below):
  // tm_w: q4 nibble bytes [n_rows][K/2] (box 32 B x 128 rows) or the f16 table
  // [n_rows][K] (box 64 x 128, 128-byte swizzle); tm_xh / tm_xl: the
  // activations [B][K] f16 (box 64 x BN, 128-byte swizzle).
  CUtensorMap tm_w, tm_xh, tm_xl;
  // q4 weights: row n's 16-byte blocks at w + n*w_stride, its f16 scales at s + n*s_stride
  const char* w;
  const char* s;
  long long w_stride, s_stride;
  // f16 weights (the LM head): row n at a16 + n*a16_stride (elements)
  const __half* a16;
  long long a16_stride;
  int n_rows;                 // weight rows (N of the GEMM)
  int K;                      // columns (multiple of 64)
  int kt_split;               // k-tiles per split (gridDim.z splits cover K)
  // activations, pre-split: x_hi/x_lo [B rows][K] f16, row b at b * ldx
  const __half* x_hi;
  const __half* x_lo;
  long long ldx;
  int B;                      // activation rows actually present (<= BN * gridDim.y)
  // outputs
  float* y;                   // [split][B][ldy] (kTcStore); optional logits [B][ldy] (kTcArgmax)
  int ldy;
  long long y_split;          // floats between two splits' outputs
  float* part_v;              // kTcArgmax: [B][gridDim.x] best value / row
  uint32_t* part_i;
  int row0;                   // kTcArgmax: index of the matrix's first row (a vocabulary slice starts at row0)
  __half* y_hi;               // kTcSilu: the next GEMM's operands [B][ldy]
  __half* y_lo;
  int* err;                   // device status word (bit kTcErrTimeout)
  // Test hook (qd_batch_inject_stall): CTA (0, 0, 0) of the first launch that finds
  // *stall non-zero clears it and withholds its first activation tiles, so that
  // CTA's waits run out and it reports kTcErrTimeout. NULL: no hook.
  int* stall;
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
// Transposing (max, lowest row) reduction across a warp of 32 columns: lane l
// starts with 32 candidates (one per column, all of its own row) and ends with
// the best of column l over the warp's 32 rows. 31 exchanges instead of 160.
__device__ __forceinline__ void warp_argmax_columns(float (&v)[32], uint32_t (&id)[32], int lane) {
#pragma unroll
  for (int w = 32; w > 1; w >>= 1) {
    const int o = w >> 1;
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < o; ++j) {
      const float sv = upper ? v[j] : v[j + o];
      const uint32_t si = upper ? id[j] : id[j + o];
      const float rv = __shfl_xor_sync(0xffffffffu, sv, o);
      const uint32_t ri = __shfl_xor_sync(0xffffffffu, si, o);
      float kv = upper ? v[j + o] : v[j];
      uint32_t ki = upper ? id[j + o] : id[j];
      if (am_better(rv, ri, kv, ki)) {
        kv = rv;
        ki = ri;
      }
      v[j] = kv;
      id[j] = ki;
    }
  }
}

// Consumer threads per weight row: each dequantises 8 / R of the row's eight
// nibble words of a k-tile (R = 2: one q4 block each). More threads shorten the
// dequantisation of every k-tile, which otherwise leaves the tensor pipe idle
// between k-tiles; the decode tile (BN = 64) keeps R = 2 so that two CTAs fit per SM.
template <int BN, bool AF16>
__host__ __device__ constexpr int tc_row_threads() {
  return (!AF16 && BN == 256) ? 4 : 2;
}
template <int BN, bool AF16>
__host__ __device__ constexpr int tc_consumers() {
  return kTcM * tc_row_threads<BN, AF16>();
}
template <int BN, bool AF16>
__host__ __device__ constexpr int tc_block_threads() {  // consumers + the producer warp + the MMA-issuer warp
  return tc_consumers<BN, AF16>() + 64;
}
template <int BN, bool AF16>
__host__ __device__ constexpr int tc_min_blocks() {  // the decode tiles (BN = 64) run two CTAs per SM
  return BN <= 64 ? 2 : 1;
}
template <int BN, bool AF16>
__host__ __device__ constexpr int tc_stages() {
  // BN = 64 (decode): two stages (q4, ~105 KB) or three (the f16 LM-head table,
  // ~97 KB) keep the CTA small enough for two per SM (b64 LM head: 15.9k -> 16.1k
  // tok/s against four stages and one CTA per SM)
  return AF16 ? 3 : (BN <= 64 ? 2 : (BN <= 128 ? 3 : 2));
}
template <int BN, bool AF16>
__host__ __device__ constexpr int tc_stage_bytes() {
  return (AF16 ? kTcM * kTcK * 2 : kTcM * 32) + 2 * BN * kTcK * 2;
}
template <int BN, bool AF16>
__host__ __device__ constexpr int tc_smem_total() {
  return tc_stages<BN, AF16>() * tc_stage_bytes<BN, AF16>() + (AF16 ? 0 : 2 * 2 * kTcM * kTcK * 2) + 1024;
}

// Grid: (ceil(n_rows / 128), ceil(B / BN), splits); 128 R + 64 threads. Split z
// covers k-tiles [z * kt_split, min((z + 1) * kt_split, K / 64)).
// Warp 4R is the producer: one lane streams each k-tile's weights (raw q4
// nibbles, or the f16 table tile) and the x_hi / x_lo tiles into a ring of S
// stages by TMA, refilling a stage when the MMAs that read it have committed
// to its "empty" barrier. The 128 R consumer threads dequantise the nibbles
// (R threads per weight row, each 8 / R words of it) into a double-buffered
// A_hi / A_lo stage and arrive on its "afull" barrier; one lane of warp 4R + 1
// issues the MMAs of a k-tile once its A stage and activation tiles are in, so
// no CTA barrier sits between the k-tiles. The consumer warps run the epilogue
// from TMEM: warp w reads lane quarter w % 4 (the hardware's rule) and its share
// of the columns.
template <int BN, bool AF16, int EPI>
__global__ void __launch_bounds__(tc_block_threads<BN, AF16>(), tc_min_blocks<BN, AF16>()) k_gemm_tc(const __grid_constant__ TcArgs a) {
  constexpr int R = tc_row_threads<BN, AF16>();
  constexpr int kCons = tc_consumers<BN, AF16>();
  constexpr int kWords = 8 / R;  // nibble words (8 columns each) per consumer thread and k-tile
  constexpr int S = tc_stages<BN, AF16>();
  constexpr int kW = AF16 ? kTcM * kTcK * 2 : kTcM * 32;
  constexpr int kBt = BN * kTcK * 2;
  constexpr int kStage = tc_stage_bytes<BN, AF16>();
  constexpr int kA = kTcM * kTcK * 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* ring =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* abuf = ring + S * kStage;  // q4: [2][A_hi | A_lo]
  // full_w: the stage's weight tile landed; full_b: its x_hi / x_lo tiles landed
  // afull: the consumers' A tile of the buffer is written (q4); adone: the MMAs that read it are done
  __shared__ unsigned long long full_w[S], full_b[S], empty[S], adone[2], afull[2];
  __shared__ unsigned tmem_base;
  __shared__ float red_v[EPI == kTcArgmax ? 4 : 1][EPI == kTcArgmax ? BN : 1];
  __shared__ uint32_t red_i[EPI == kTcArgmax ? 4 : 1][EPI == kTcArgmax ? BN : 1];
  __shared__ int failed;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kTcM;
  const int b0 = blockIdx.y * BN;
  const int kt_total = a.K / kTcK;
  const int kt0 = blockIdx.z * a.kt_split;
  const int nk = min(a.kt_split, kt_total - kt0);

  if (warp == 0) {  // TMEM: D_main (BN columns) + D_corr (BN columns)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_smem(&tmem_base)),
                 "r"(2 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < S; ++i) {
      tc_mbar_init(&full_w[i]);
      tc_mbar_init(&full_b[i]);
      tc_mbar_init(&empty[i]);
    }
    tc_mbar_init(&adone[0]);
    tc_mbar_init(&adone[1]);
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc_smem(&afull[0])), "r"(kCons) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc_smem(&afull[1])), "r"(kCons) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    failed = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = tmem_base;

  if (warp == kCons / 32) {
    // ---- producer ----
    if (lane == 0) {
      tma_prefetch_map(&a.tm_w);
      tma_prefetch_map(&a.tm_xh);
      tma_prefetch_map(&a.tm_xl);
      bool ok = true;
      int last_w[S], last_b[S];  // newest k-tile whose weight / activation tiles each stage was given
#pragma unroll
      for (int i = 0; i < S; ++i) last_w[i] = last_b[i] = -1;
      const bool withhold = a.stall && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 &&
                            atomicExch(a.stall, 0) != 0;
      // With one column tile (decode) every weight tile is read exactly once per
      // launch: evict-first. With several (prefill) the other column tiles reread
      // it from L2, so it keeps the normal policy.
      const bool once = gridDim.y == 1;
      const unsigned long long pol = l2_evict_first();
      auto load_w = [&](unsigned char* dst, int k, unsigned long long* mb) {
        const int x = AF16 ? (kt0 + k) * kTcK : (kt0 + k) * 32;
        if (once) tma_load_2d_hint(dst, &a.tm_w, x, n0, mb, pol);
        else tma_load_2d(dst, &a.tm_w, x, n0, mb);
      };
      // The weights are constant: the first stages' weight tiles go out before
      // waiting for the kernel that produces the activations.
      const int pre = min(S, nk);
      for (int k = 0; k < pre; ++k) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(&full_w[k])), "r"(kW)
                     : "memory");
        load_w(ring + k * kStage, k, &full_w[k]);
        last_w[k] = k;
      }
      pdl_wait();
      for (int k = 0; k < nk; ++k) {
        const int slot = k % S;
        unsigned char* st = ring + slot * kStage;
        if (k >= S) {
          if (!tc_mbar_wait(&empty[slot], (unsigned)((k / S) - 1) & 1u)) {
            ok = false;
            break;
          }
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(&full_w[slot])), "r"(kW)
                       : "memory");
          load_w(st, k, &full_w[slot]);
          last_w[slot] = k;
        }
        if (withhold && k == 0) continue;  // test hook: k-tile 0's activations never arrive
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(&full_b[slot])),
                     "r"(2 * kBt)
                     : "memory");
        tma_load_2d(st + kW, &a.tm_xh, (kt0 + k) * kTcK, b0, &full_b[slot]);
        tma_load_2d(st + kW + kBt, &a.tm_xl, (kt0 + k) * kTcK, b0, &full_b[slot]);
        last_b[slot] = k;
      }
      if (!ok) atomicOr(&failed, 1);
      // Nothing may still be landing in shared memory when the CTA exits: the
      // newest tile of each stage is the only one that can be in flight.
#pragma unroll
      for (int i = 0; i < S; ++i) {
        if (last_w[i] >= 0) (void)tc_mbar_wait(&full_w[i], (unsigned)(last_w[i] / S) & 1u);
        if (last_b[i] >= 0) (void)tc_mbar_wait(&full_b[i], (unsigned)(last_b[i] / S) & 1u);
      }
    }
  } else if (warp == kCons / 32 + 1) {
    // ---- MMA issuer (one lane) ----
    if (lane == 0) {
      const unsigned idesc = umma_idesc_f16_f32(kTcM, BN);
      bool ok = true;
      int committed = -1;  // last tile whose MMAs were committed
      for (int i = 0; i < nk; ++i) {
        const int slot = i % S, st = i & 1;
        unsigned char* stg = ring + slot * kStage;
        // q4: the consumers' dequantised A tile of k-tile i (all of them arrived on afull);
        // the f16 table: its TMA tile. Then the activation tiles.
        if constexpr (!AF16) ok = tc_mbar_wait(&afull[st], (unsigned)(i >> 1) & 1u);
        else ok = tc_mbar_wait(&full_w[slot], (unsigned)(i / S) & 1u);
        ok = ok && tc_mbar_wait(&full_b[slot], (unsigned)(i / S) & 1u);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kTcK / 16; ++ks) {
          const unsigned long long dbh = umma_desc_k_sw128(tc_smem(stg + kW) + ks * 32);
          const unsigned long long dbl = umma_desc_k_sw128(tc_smem(stg + kW + kBt) + ks * 32);
          const bool acc = i > 0 || ks > 0;
          if constexpr (!AF16) {
            const unsigned char* A_hi = abuf + st * 2 * kA;
            const unsigned long long dah = umma_desc_k_sw128(tc_smem(A_hi) + ks * 32);
            const unsigned long long dal = umma_desc_k_sw128(tc_smem(A_hi + kA) + ks * 32);
            umma_f16(tmem, dah, dbh, idesc, acc);
            umma_f16(tmem + BN, dah, dbl, idesc, acc);
            umma_f16(tmem + BN, dal, dbh, idesc, true);
          } else {
            const unsigned long long da = umma_desc_k_sw128(tc_smem(stg) + ks * 32);
            umma_f16(tmem, da, dbh, idesc, acc);
            umma_f16(tmem + BN, da, dbl, idesc, acc);
          }
        }
        umma_commit(&empty[slot]);
        umma_commit(&adone[st]);
        committed = i;
      }
      // Wait for the last MMAs (they complete in order).
      if (committed >= 0) ok = tc_mbar_wait(&adone[committed & 1], (unsigned)(committed >> 1) & 1u) && ok;
      if (!ok || committed != nk - 1) atomicOr(&failed, 1);
    }
  } else if constexpr (!AF16) {
    // ---- consumers: dequantisation of every k-tile's weights into the A stage ----
    pdl_wait();
    // Thread (row, part): weight row n0 + row, words [part * kWords, (part + 1) * kWords)
    // of every k-tile (the q4 block of word j is j / 4).
    const int row = tid & (kTcM - 1), part = tid >> 7;
    const int n = n0 + row;
    const bool row_live = n < a.n_rows;
    uint32_t sc_cur = 0, sc_next = 0;
    {
      const char* srow = a.s + (long long)(row_live ? n : 0) * a.s_stride;
      if (row_live) {
        sc_cur = *reinterpret_cast<const uint32_t*>(srow + kt0 * 4);
        if (nk > 1) sc_next = *reinterpret_cast<const uint32_t*>(srow + (kt0 + 1) * 4);
      }
    }
    for (int i = 0; i < nk; ++i) {
      const int slot = i % S, st = i & 1;
      unsigned char* stg = ring + slot * kStage;
      // the weight tile landed, and the MMAs that last read this A buffer (tile i - 2) are done
      bool ok = tc_mbar_wait(&full_w[slot], (unsigned)(i / S) & 1u);
      if (ok && i >= 2) ok = tc_mbar_wait(&adone[st], (unsigned)((i - 2) >> 1) & 1u);
      if (!ok) {  // the issuer then times out on afull and records the failure as well
        atomicOr(&failed, 1);
        break;
      }
      unsigned char* A_hi = abuf + st * 2 * kA;
      unsigned char* A_lo = A_hi + kA;
      uint32_t ws[kWords];
      if constexpr (kWords == 4) {
        const uint4 q0 = reinterpret_cast<const uint4*>(stg + row * 32)[part];
        ws[0] = q0.x;
        ws[1] = q0.y;
        ws[2] = q0.z;
        ws[3] = q0.w;
      } else {
        static_assert(kWords == 2, "2 or 4 consumer threads per row");
        const uint2 q0 = reinterpret_cast<const uint2*>(stg + row * 32)[part];
        ws[0] = q0.x;
        ws[1] = q0.y;
      }
      // f16x2 arithmetic, exact: q = n - 8 from the biased pattern 0x6400 | n (1024 + n);
      // hi = q * s' (s' = scale * 2^10, exact in f16) rounded once, as f32 math then a
      // round to f16 would; lo = (q * s' - hi) * 2^11 with the residual from one fma.
      const __half2 s2 = *reinterpret_cast<const __half2*>(&sc_cur);
      const __half2 k1024 = __float2half2_rn(1024.0f), bias = __float2half2_rn(1032.0f);
      const __half2 k2048 = __float2half2_rn(kLoScale);
      const bool blk1 = part * kWords >= 4;  // this thread's words lie in the k-tile's second q4 block
      const __half2 scl = __hmul2(blk1 ? __high2half2(s2) : __low2half2(s2), k1024);
#pragma unroll
      for (int wl = 0; wl < kWords; ++wl) {  // 8 columns per word -> one 16-byte chunk of f16
        const int wi = part * kWords + wl;   // word of the row's k-tile
        const uint32_t w = ws[wl];
        uint32_t hi_p[4], lo_p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // pair i = columns (i, i + 4) of the word
          const uint32_t bits = ((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
          const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&bits), bias);
          const __half2 h = __hmul2(q, scl);
          const __half2 l = __hmul2(__hfma2(q, scl, __hneg2(h)), k2048);
          hi_p[i] = *reinterpret_cast<const uint32_t*>(&h);
          lo_p[i] = *reinterpret_cast<const uint32_t*>(&l);
        }
        // back to column order: (c0,c1) (c2,c3) (c4,c5) (c6,c7)
        const uint4 H = make_uint4(__byte_perm(hi_p[0], hi_p[1], 0x5410), __byte_perm(hi_p[2], hi_p[3], 0x5410),
                                   __byte_perm(hi_p[0], hi_p[1], 0x7632), __byte_perm(hi_p[2], hi_p[3], 0x7632));
        const uint4 Lo = make_uint4(__byte_perm(lo_p[0], lo_p[1], 0x5410), __byte_perm(lo_p[2], lo_p[3], 0x5410),
                                    __byte_perm(lo_p[0], lo_p[1], 0x7632), __byte_perm(lo_p[2], lo_p[3], 0x7632));
        const unsigned off = sw128_off(row, wi * 8);
        *reinterpret_cast<uint4*>(A_hi + off) = H;
        *reinterpret_cast<uint4*>(A_lo + off) = Lo;
      }
      sc_cur = sc_next;
      if (row_live && i + 2 < nk)
        sc_next = *reinterpret_cast<const uint32_t*>(a.s + (long long)n * a.s_stride + (kt0 + i + 2) * 4);
      // generic-proxy stores -> visible to the MMAs (async proxy), then this thread's arrival
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc_smem(&afull[st])) : "memory");
    }
  } else {
    pdl_wait();  // the f16 table's consumers only run the epilogue
  }
  __syncthreads();
  tc_fence_after();
  pdl_trigger();

  if (tid < kCons && !failed) {
    // Epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = weight rows n0 + 32 (w % 4)
    // + lane, columns [cp * kCols, (cp + 1) * kCols) with cp = w / 4 (column parts of
    // at least 32 columns; warps beyond the parts only join the barrier below).
    constexpr int kParts = (R < BN / 32) ? R : BN / 32;
    constexpr int kCols = BN / kParts;
    static_assert(kCols % 32 == 0, "column parts are whole 32-column steps");
    const int quarter = warp & 3, cp = warp >> 2;
    const int n = n0 + quarter * 32 + lane;
    const bool row_live = n < a.n_rows;
    const unsigned lane_base = (unsigned)(quarter * 32) << 16;
    const float unscale = AF16 ? 1.0f : 1.0f / (float)(1 << kWShift);
    float* y = a.y ? a.y + (long long)blockIdx.z * a.y_split : nullptr;
#pragma unroll 1
    for (int c0 = cp * kCols; c0 < (cp + 1) * kCols && cp < kParts; c0 += 32) {
      float dm[32], dc[32];
      tmem_ld32(tmem + lane_base + c0, dm);
      tmem_ld32(tmem + lane_base + BN + c0, dc);
#pragma unroll
      for (int j = 0; j < 32; ++j) dm[j] = (dm[j] + dc[j] * (1.0f / kLoScale)) * unscale;
      if constexpr (EPI == kTcSilu) {
        // Lane pairs hold the gate (even lane) and up (odd lane) rows of pair n / 2.
        // Each step finishes two activation rows: the even lane row j, the odd lane
        // row j + 1, so that every lane computes (fast exp and divide: the result is
        // within a few ulp of silu(g) * u).
        const bool odd = lane & 1;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float o0 = __shfl_xor_sync(0xffffffffu, dm[j], 1);
          const float o1 = __shfl_xor_sync(0xffffffffu, dm[j + 1], 1);
          const float g = odd ? o1 : dm[j];
          const float u = odd ? dm[j + 1] : o0;
          const int b = b0 + c0 + j + (odd ? 1 : 0);
          if (row_live && b < a.B) {
            const float act = __fdividef(g, 1.0f + __expf(-g)) * u;
            __half hh, ll;
            split_f16(act, hh, ll);
            a.y_hi[(long long)b * a.ldy + (n >> 1)] = hh;
            a.y_lo[(long long)b * a.ldy + (n >> 1)] = ll;
          }
        }
      } else if (y) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int b = b0 + c0 + j;
          if (row_live && b < a.B) y[(long long)b * a.ldy + n] = dm[j];
        }
      }
      if constexpr (EPI == kTcArgmax) {
        uint32_t id[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          id[j] = (uint32_t)(n + a.row0);
          if (!row_live) dm[j] = kNegMax;
        }
        warp_argmax_columns(dm, id, lane);
        red_v[quarter][c0 + lane] = dm[0];
        red_i[quarter][c0 + lane] = id[0];
      }
    }
    if constexpr (EPI == kTcArgmax) {
      asm volatile("bar.sync 1, %0;" ::"r"(kCons) : "memory");
      for (int j = tid; j < BN; j += kCons) {
        const int b = b0 + j;
        if (b >= a.B) continue;
        float bv = red_v[0][j];
        uint32_t bi = red_i[0][j];
#pragma unroll
        for (int w = 1; w < 4; ++w)
          if (am_better(red_v[w][j], red_i[w][j], bv, bi)) {
            bv = red_v[w][j];
            bi = red_i[w][j];
          }
        a.part_v[(long long)b * gridDim.x + blockIdx.x] = bv;
        a.part_i[(long long)b * gridDim.x + blockIdx.x] = bi;
      }
    }
  }
  if (tid == 0 && failed && a.err) atomicOr(a.err, kTcErrTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
}

// Split f32 rows into the hi/lo f16 operands of the GEMM: x_hi[b][k] = f16(x),
// x_lo[b][k] = f16((x - x_hi) * 2^11). Grid-stride over B*K elements.
static __global__ void k_split_hilo(const float* x, int n, __half* hi, __half* lo) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    __half h, l;
    split_f16(x[i], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

}  // namespace qd
