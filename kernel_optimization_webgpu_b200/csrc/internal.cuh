// Library-internal declarations shared by the translation units of the engine
// (error type, launch helper, the engine object and its resident layer table).
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../../include/qdecode.h"
#include "common.cuh"
#include "persist.cuh"

namespace qd {

struct QdError {
  int code;
  std::string msg;
};

#define QD_CK(call)                                                                              \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess) throw QdError{QD_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)}; \
  } while (0)

template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QD_CK(cudaLaunchKernelEx(&cfg, kernel, args...));
}

// Same, with an explicit block size and dynamic shared memory.
template <typename... KArgs, typename... Args>
inline void launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QD_CK(cudaLaunchKernelEx(&cfg, kernel, args...));
}

// Raises a kernel's dynamic shared memory limit once per device (the attribute
// belongs to the device's context).
template <typename... KArgs>
inline void allow_smem(void (*kernel)(KArgs...), size_t bytes, unsigned long long& done_mask) {
  int dev = 0;
  QD_CK(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (done_mask & bit) return;
  QD_CK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  done_mask |= bit;
}

inline int sm_count(int dev) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  return n;
}

inline int current_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  return sm_count(dev);
}

// Records the message returned by qd_last_error(NULL) on this thread.
void set_thread_error(const std::string& msg);

// tcgen05 GEMM launch (gemm_tc.cuh): q4 weights with split-K partial outputs,
// or the f16 LM head with the per-CTA (max, index) epilogue.
enum GemmMode : int { kGemmQ4Store = 0, kGemmF16Argmax = 1, kGemmQ4Silu = 2 };
// What a decode token launch computes after its layers.
enum HeadMode : int { kHeadNone = 0, kHeadFull = 1, kHeadArgmax = 2 };
struct TcArgs;
void launch_gemm(TcArgs a, int splits, int mode, cudaStream_t s);
// Splits actually used for K columns when `want` are asked for (no empty split).
int gemm_plan_splits(int K, int want, int* kt_split);

// Used by the benchmark entries (bench_api.cu), defined in engine.cu:
// one decoder layer whose input is the engine's hidden vector (layer 0 included,
// no embedding gather); the decode position the layer kernels read; the device
// status check after a run; a q4 matvec over row records (row r at base + r * row_stride).
// Sampling (sample.cu): validation, the greedy cases, and the sampling kernels after an
// engine's LM head (reads its logits, overwrites the token the head chose).
void check_sampling(const qd_sampling& s);
bool sampling_is_greedy(const qd_sampling& s);
void enqueue_engine_sample(qd_engine* e, const qd_sampling& s);
void bench_layer_from_hidden(qd_engine* e, int l, cudaStream_t s);
void bench_set_position(qd_engine* e, int pos);
void bench_check_state(qd_engine* e);
void bench_rows_matvec(qd_engine* e, const char* base, long long row_stride, int rows, int k, const float* x,
                       float* y, cudaStream_t s);

// Prompt pass (batch.cu): the first n prompt tokens (e->tokens[0..n)) of the engine's
// sequence through every layer at once with the batched path's tensor-core GEMMs,
// leaving their K/V rows at positions 0..n-1 of the engine's cache; no LM head.
// prompt_pass_fits says whether this engine and length take it (f16 KV, option
// on, kPromptPassMin <= n <= kPromptPassMax, a shape the batched path supports).
constexpr int kPromptPassMin = 5, kPromptPassMax = 256;
// With with_head, the pass also takes the last prompt token through the final norm
// and the LM head: the first generated id lands in e->tokens[n] and out_host[0].
bool prompt_pass_fits(qd_engine* e, int n);
void prompt_pass(qd_engine* e, int n, bool with_head = false);
void prompt_pass_check(qd_engine* e);  // raises the pass's device status (synchronises)
void prompt_pass_free(qd_engine* e);

}  // namespace qd

// Bytes of one q4 row record: nb 16-byte blocks then nb f16 scales, padded to 16.
inline long long rec_bytes(int k) {
  const long long nb = k / qd::kBlockCols;
  return (nb * 16 + nb * 2 + 15) / 16 * 16;
}

// Per layer, each matrix is an array of row records (gate/up: pair records
// [gate row | up row]); a run of rows is one contiguous range of bytes.
struct LayerDev {
  const char *qkv, *o, *gu, *d;
  const float *n_in, *n_q, *n_k, *n_post;
  void *kc, *vc;
};

struct qd_engine {
  std::string err;
  int dev = 0, sms = 148;
  cudaStream_t stream = nullptr;      // the stream work is enqueued on
  cudaStream_t own_stream = nullptr;  // created with the engine
  int stepping_max_new = 0;
  qd_profile p{};
  qd_options opt{};
  std::string variant;
  int splits = 1, rows_qkv = 0, lm_grid = 0;
  void* blob = nullptr;
  void* kv = nullptr;
  void* scratch = nullptr;
  __half* embed = nullptr;
  float *cos_t = nullptr, *sin_t = nullptr, *final_norm = nullptr;
  std::vector<LayerDev> layers;
  float *h = nullptr, *h_attn = nullptr, *qkv = nullptr, *act = nullptr, *logits = nullptr, *part_o = nullptr;
  float2* part_ml = nullptr;
  qd::DevState* st = nullptr;
  int *tokens = nullptr, *out_dev = nullptr;
  int* out_host = nullptr;  // mapped pinned: the kernel writes each token here
  int* out_host_dev = nullptr;
  uint32_t* result = nullptr;
  float* lm_pv = nullptr;
  uint32_t* lm_pi = nullptr;
  unsigned* lm_counter = nullptr;
  int32_t* pinned_ids = nullptr;
  qd::DevState* pinned_state = nullptr;
  cudaGraphExec_t g_layers = nullptr, g_full = nullptr, g_argmax = nullptr;
  bool logits_stale = false;               // the last token launch computed the argmax only
  // argmax-only LM head of the persistent kernel: the table as int8 + per-row scale / bound
  uint8_t* lm_q8 = nullptr;
  float *lm_scale = nullptr, *lm_bound = nullptr;
  cudaEvent_t ev[2] = {nullptr, nullptr};
  // persistent decode kernel
  bool persist = false;
  qd::PLayer* d_players = nullptr;
  unsigned long long* xbuf = nullptr;
  long long xstride = 0;
  size_t persist_smem = 0;
  int lm_rows = 0;
  unsigned long long* timeline = nullptr;  // stage stamps of the last persistent launch (opt-in)
  void* sample_ws = nullptr;               // sampling candidates (allocated on first use)
  char* oslices = nullptr;                 // O rows x KV-head columns, packed per attention CTA
  char* dslices = nullptr;                 // down rows x one CTA's intermediate columns, packed per CTA
  int n_mlp = 0;                           // CTAs that contribute to the down sums
  unsigned long long* oacc = nullptr;      // [2][L][O | down][H] counted fixed-point sums
  int os = 0;                              // attention CTAs per KV head
  long long rec_og = 0, oslice_rows = 0;
  // prompt pass: a one-sequence batch over the engine's weights (created on first use)
  qd_batch* pbatch = nullptr;
  bool pbatch_unfit = false;               // the batched path rejected this shape
  bool pbatch_used = false;                // the current prompt took the pass
};
