// Decode attention without any device allocation.
//
// qd_gqa_decode needs scratch memory for its split-KV partials (per split and
// query head: running max, exp-sum and an unnormalised 128-wide output), which
// its caller allocates. Some callers cannot allocate device memory when they
// call in: a host that gives all device memory to its own pool at start-up and
// forbids driver allocations afterwards, or a latency-critical loop that cannot
// take the device-wide synchronisation a cudaFree may cause. This file gives
// them qd_gqa_decode_noalloc: the same kernels, with the partials kept in one
// fixed array in device global memory that belongs to the library.
#include <cmath>
#include <mutex>
#include <string>

#include "../../include/qdecode.h"
#include "kernels.cuh"

using namespace qd;

namespace {

// The partials of every call live here. The array exists once per device that
// loads the library and stays allocated until the process exits.
static __device__ __align__(256) unsigned char g_attn_scratch[QD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
// Per device: the symbol address and the unique id of the CUDA context it was
// looked up in. A device reset or another context gets a new id (ids are never
// reused within a process), which makes the next call look the address up again.
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

int fail(int code, const std::string& msg) {
  qd::set_thread_error(msg);  // read back with qd_last_error(NULL)
  return code;
}

// cuCtxGetCurrent / cuCtxGetId through the runtime's driver entry points (the
// library does not link the driver library itself).
typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);

bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool resolved = false;
  if (!resolved) {
    void* f0 = nullptr;
    void* f1 = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f0, cudaEnableDefault) == cudaSuccess &&
        cudaGetDriverEntryPoint("cuCtxGetId", &f1, cudaEnableDefault) == cudaSuccess) {
      get_current = reinterpret_cast<CtxGetCurrentFn>(f0);
      get_id = reinterpret_cast<CtxGetIdFn>(f1);
    }
    resolved = true;
  }
  void* ctx = nullptr;
  if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx) return false;
  return get_id(ctx, id) == 0;
}

// The device address of g_attn_scratch on the current device. On the host the
// name g_attn_scratch is only a stand-in, so the address has to be asked for,
// with that device current: once per device (and again when the device's
// context is a new one).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(QD_E_CUDA, "qd_gqa_decode_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lock(g_mu);
  unsigned long long ctx = 0;
  const bool have_ctx = current_context_id(&ctx);
  if (!g_scratch_ptr[dev] || !have_ctx || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (rc != cudaSuccess || !p)
      return fail(QD_E_CUDA, std::string("qd_gqa_decode_noalloc: cudaGetSymbolAddress failed: ") +
                                 cudaGetErrorString(rc));
    g_scratch_ptr[dev] = p;
    // the lookup made the context current if it was not yet
    g_scratch_ctx[dev] = current_context_id(&ctx) ? ctx : 0;
  }
  *out = g_scratch_ptr[dev];
  return QD_OK;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_plain(void (*kernel)(KArgs...), dim3 grid, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename KVT>
cudaError_t launch_attn_group(const AttnArgs& a, int group, int splits, cudaStream_t s) {
  const dim3 grid(a.kv_heads, splits);
  switch (group) {
    case 1: return launch_plain(k_attn<1, KVT>, grid, s, a);
    case 2: return launch_plain(k_attn<2, KVT>, grid, s, a);
    case 4: return launch_plain(k_attn<4, KVT>, grid, s, a);
    case 8: return launch_plain(k_attn<8, KVT>, grid, s, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

extern "C" {

int qd_gqa_decode_noalloc(const float* q, const void* k_cache, const void* v_cache, int kv_dtype, float* y,
                          uint32_t seq_len, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                          void* stream) {
  if (!q || !k_cache || !v_cache || !y) return fail(QD_E_INVALID, "qd_gqa_decode_noalloc: NULL pointer");
  if (head_dim != (uint32_t)kHeadDim) return fail(QD_E_INVALID, "qd_gqa_decode_noalloc: head_dim must be 128");
  if (seq_len == 0 || kv_heads == 0 || q_heads % kv_heads)
    return fail(QD_E_INVALID, "qd_gqa_decode_noalloc: bad attention dimensions");
  const uint32_t group = q_heads / kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return fail(QD_E_INVALID, "qd_gqa_decode_noalloc: q_heads / kv_heads must be 1, 2, 4 or 8");
  if (kv_dtype != QD_KV_F16 && kv_dtype != QD_KV_F32) return fail(QD_E_INVALID, "qd_gqa_decode_noalloc: bad kv_dtype");
  // Partials, per split and query head as in qd_gqa_decode: (max, sum) pairs
  // [splits][q_heads] at offset 0, then outputs [splits][q_heads][128] from the
  // next 256-byte boundary (qd_gqa_decode's workspace uses other offsets).
  const size_t splits = (seq_len + kAttnChunk - 1) / kAttnChunk;
  const size_t ml_bytes = (splits * q_heads * sizeof(float2) + 255) & ~size_t(255);
  const size_t need = ml_bytes + splits * q_heads * kHeadDim * sizeof(float);
  if (need > QD_NOALLOC_SCRATCH_BYTES)
    return fail(QD_E_RANGE,
                "qd_gqa_decode_noalloc: seq_len * q_heads needs more scratch than the library's fixed "
                "QD_NOALLOC_SCRATCH_BYTES; use qd_gqa_decode with a caller-allocated workspace");
  void* base = nullptr;
  const int rc = scratch_address(&base);
  if (rc != QD_OK) return rc;
  // Nothing in the scratch has to start at zero: every split CTA writes its own
  // partial (empty splits write a neutral one) before the combine reads it.
  AttnArgs a{};
  a.q_in = q;
  a.k_cache = const_cast<void*>(k_cache);
  a.v_cache = const_cast<void*>(v_cache);
  a.st = nullptr;
  a.seq_len = (int)seq_len;
  a.max_seq = (int)seq_len;
  a.q_heads = (int)q_heads;
  a.kv_heads = (int)kv_heads;
  a.scale = 1.0f / sqrtf((float)kHeadDim);
  a.raw_q = 1;
  a.part_ml = reinterpret_cast<float2*>(base);
  a.part_o = reinterpret_cast<float*>(static_cast<char*>(base) + ml_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = (kv_dtype == QD_KV_F32) ? launch_attn_group<float>(a, (int)group, (int)splits, s)
                                          : launch_attn_group<__half>(a, (int)group, (int)splits, s);
  if (e == cudaSuccess) {
    const int n = (int)q_heads * kHeadDim;
    e = launch_plain(k_attn_combine, dim3((n + kThreads - 1) / kThreads), s, (const float2*)a.part_ml,
                     (const float*)a.part_o, (int)splits, (int)q_heads, y);
  }
  if (e != cudaSuccess) return fail(QD_E_CUDA, std::string("qd_gqa_decode_noalloc: launch failed: ") + cudaGetErrorString(e));
  return QD_OK;
}

}  // extern "C"
