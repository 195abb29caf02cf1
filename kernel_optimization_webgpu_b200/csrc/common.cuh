// Shared device helpers for the sm_100a decode kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace qd {

// Sets the message qd_last_error(NULL) returns on this thread (defined in engine.cu).
void set_thread_error(const std::string& msg);

constexpr int kThreads = 256;                 // every decode kernel runs 8 warps
constexpr int kWarps = kThreads / 32;
constexpr int kHeadDim = 128;                 // Qwen3 head_dim (rope.wgsl half = 64)
constexpr int kBlockCols = 32;                // MatMulNBits block: 32 columns per f16 scale
constexpr float kNegMax = -3.4028234e38f;     // argmax_stage1.wgsl:16, the shaders' "-inf"
constexpr int kAttnChunk = 256;               // KV positions per split-KV CTA

// Device-side error bits (the engine's status word; kernels never trap).
enum DevErr : int {
  kErrToken = 1,      // token id outside [0, vocab): row 0 used instead
  kErrPosition = 2,   // position beyond the KV capacity: the step was skipped
};

// Per-engine device state read by the captured kernels (no host writes per token).
struct DevState {
  int pos;            // position of the token being processed
  int step;           // index of the next generated token
  int max_new;        // generated tokens requested
  int err;            // DevErr bits
  // Below: owned by the device (the host only repairs them after a failure).
  int epoch;          // launches of the persistent decode kernel so far (exchange-word tag)
  int abort;          // set by a persistent kernel whose wait expired
  // Test hook (qd_engine_inject_stall): the persistent launch whose epoch equals
  // this withholds layer 0's q/k/v stores, so its waits run out; 0 = never.
  int stall_epoch;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 128-bit load of data read exactly once (weights): skip L1.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint2 ld_stream2(const uint2* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

// (value, index) argmax order: larger value wins, ties go to the lower index,
// NaN never wins (every comparison with NaN is false). argmax_stage1.wgsl:51-52.
__device__ __forceinline__ bool am_better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// One MatMulNBits block: 32 nibbles (a uint4 = 4 words, word k holds columns
// 8k..8k+7, nibble i of a word is column 8k+i, low nibble first) against the
// matching 32 activations held as 16 float2 pairs (x[4k+j] = columns 8k+2j, 8k+2j+1).
// Dequantisation is exact: a byte permute builds the float 2^23 + n, and one
// packed subtract of 2^23 + 8 leaves n - 8 (the implicit zero point 8).
__device__ __forceinline__ float q4_block_dot(uint4 w, const float2 (&x)[16]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  const float2 bias = make_float2(-8388616.0f, -8388616.0f);
  float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = ws[k] & 0x0F0F0F0Fu;          // even columns in bytes 0..3
    const uint32_t hi = (ws[k] >> 4) & 0x0F0F0F0Fu;   // odd columns
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = __int_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + j));
      const float b = __int_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + j));
      const float2 v = __fadd2_rn(make_float2(a, b), bias);
      acc = __ffma2_rn(v, x[4 * k + j], acc);
    }
  }
  return acc.x + acc.y;
}

// Eight f16 table entries (one uint4) against eight activations (4 float2 pairs).
__device__ __forceinline__ float2 f16x8_dot(uint4 w, const float2* x, float2 acc) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ws[k]));
    acc = __ffma2_rn(f, x[k], acc);
  }
  return acc;
}

// Eight int8 table entries stored biased (q + 128, one uint2) against eight
// activations (4 float2 pairs), the same column order as f16x8_dot. A byte permute
// builds the float 2^23 + u and one packed subtract of 2^23 + 128 leaves q exactly.
__device__ __forceinline__ float2 q8x8_dot(uint2 w, const float2* x, float2 acc) {
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);
  const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float a = __int_as_float(__byte_perm(ws[h], 0x4B000000u, 0x7540u + 2 * j));
      const float b = __int_as_float(__byte_perm(ws[h], 0x4B000000u, 0x7540u + 2 * j + 1));
      acc = __ffma2_rn(__fadd2_rn(make_float2(a, b), bias), x[2 * h + j], acc);
    }
  return acc;
}

// Activation staging in shared memory. Lane l of a warp consumes float4 slots
// (c*32 + l)*8 + q (q = 0..7) of block-chunk c; storing logical float4 f at
// f ^ ((f >> 3) & 7) puts the 8 lanes of each quarter-warp on distinct bank groups.
__device__ __forceinline__ int xs_slot(int f) { return f ^ ((f >> 3) & 7); }

__device__ __forceinline__ void xs_store(float* xs, int e, float v) {
  const int f = e >> 2;
  xs[(xs_slot(f) << 2) | (e & 3)] = v;
}

// Block-wide sum over 256 threads (result valid in every thread).
__device__ __forceinline__ float block_sum(float v, float* red8) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red8[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t += red8[w];
  return t;
}

}  // namespace qd
