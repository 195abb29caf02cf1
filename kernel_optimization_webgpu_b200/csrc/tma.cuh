// TMA (cp.async.bulk.tensor) helpers: host-side tensor-map encoding through the
// driver entry point (no link against libcuda) and the device-side 2D tile load.
// Loads only; no multicast form is used anywhere in this library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <string>

namespace qd {

// 2D tile load of box (x, y) of `map` into shared memory, completing on `mbar`
// (which must expect the box's bytes). x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y,
                                            unsigned long long* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          static_cast<unsigned>(__cvta_generic_to_shared(smem_dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
      "r"(static_cast<unsigned>(__cvta_generic_to_shared(mbar)))
      : "memory");
}

// The same with an L2 cache policy (createpolicy), e.g. evict-first for data read once.
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, int x, int y,
                                                 unsigned long long* mbar, unsigned long long policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(smem_dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
      "r"(static_cast<unsigned>(__cvta_generic_to_shared(mbar))), "l"(policy)
      : "memory");
}

// L2 policy for data each launch reads exactly once (streamed weights, KV tiles).
__device__ __forceinline__ unsigned long long l2_evict_first() {
  unsigned long long p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

#ifndef __CUDACC_RTC__
// Encodes a row-major 2D tensor: `rows` rows of `inner` elements, consecutive rows
// `row_bytes` apart; boxes of box_inner x box_rows elements. Returns false (with
// a message) if the driver rejects the description.
inline bool make_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                         uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                         CUtensorMapSwizzle swizzle, std::string* err) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
        q != cudaDriverEntryPointSuccess) {
      if (err) *err = "cuTensorMapEncodeTiled is not available from the driver";
      return false;
    }
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult rc = encode(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)rc) + ")";
    return false;
  }
  return true;
}
#endif

}  // namespace qd
