// Node-API addon over libqdecode.so: the native half of cuda-runtime.js.
// Built only where Node headers (node_api.h) exist. It converts JS
// values to the C ABI of include/qdecode.h and back; no logic of its own.
#include <node_api.h>

#include <string>
#include <vector>

#include "qdecode.h"

namespace {

#define NAPI_OK(call)                                           \
  do {                                                          \
    if ((call) != napi_ok) {                                    \
      napi_throw_error(env, nullptr, "N-API call failed: " #call); \
      return nullptr;                                           \
    }                                                           \
  } while (0)

napi_value throw_qd(napi_env env, qd_engine* e, int rc) {
  const std::string msg = std::string("qdecode error ") + std::to_string(rc) + ": " + qd_last_error(e);
  napi_throw_error(env, nullptr, msg.c_str());
  return nullptr;
}

int32_t get_i32(napi_env env, napi_value obj, const char* key, int32_t dflt) {
  bool has = false;
  if (napi_has_named_property(env, obj, key, &has) != napi_ok || !has) return dflt;
  napi_value v;
  int32_t out = dflt;
  if (napi_get_named_property(env, obj, key, &v) == napi_ok) napi_get_value_int32(env, v, &out);
  return out;
}

void finalize_engine(napi_env, void* data, void*) { qd_engine_destroy(static_cast<qd_engine*>(data)); }

// engineCreate(runtimeDir: string, options?: {device, maxSeq, kvDtype, ropeRowStride}) -> External
napi_value EngineCreate(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2];
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
  size_t len = 0;
  NAPI_OK(napi_get_value_string_utf8(env, argv[0], nullptr, 0, &len));
  std::string dir(len, '\0');
  NAPI_OK(napi_get_value_string_utf8(env, argv[0], dir.data(), len + 1, &len));
  qd_options opt;
  qd_options_default(&opt);
  if (argc > 1) {
    opt.device = get_i32(env, argv[1], "device", opt.device);
    opt.max_seq = get_i32(env, argv[1], "maxSeq", opt.max_seq);
    opt.kv_dtype = get_i32(env, argv[1], "kvDtype", opt.kv_dtype);
    opt.rope_row_stride = get_i32(env, argv[1], "ropeRowStride", opt.rope_row_stride);
  }
  qd_engine* e = nullptr;
  const int rc = qd_engine_create(dir.c_str(), &opt, &e);
  if (rc != QD_OK) return throw_qd(env, nullptr, rc);
  napi_value ext;
  NAPI_OK(napi_create_external(env, e, finalize_engine, nullptr, &ext));
  return ext;
}

struct CbCtx {
  napi_env env;
  napi_value fn;
};

int on_token(int32_t token, void* user) {
  CbCtx* c = static_cast<CbCtx*>(user);
  napi_value global, arg, ret;
  napi_get_global(c->env, &global);
  napi_create_int32(c->env, token, &arg);
  return napi_call_function(c->env, global, c->fn, 1, &arg, &ret) == napi_ok ? 0 : 1;
}

// generateGreedy(engine, inputIds: number[], maxNewTokens: number, onToken?: (id) => void)
//   -> {generated: number[], generateMs, firstTokenMs}
napi_value GenerateGreedy(napi_env env, napi_callback_info info) {
  size_t argc = 4;
  napi_value argv[4];
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
  void* data = nullptr;
  NAPI_OK(napi_get_value_external(env, argv[0], &data));
  qd_engine* e = static_cast<qd_engine*>(data);
  uint32_t n = 0;
  NAPI_OK(napi_get_array_length(env, argv[1], &n));
  std::vector<int32_t> ids(n);
  for (uint32_t i = 0; i < n; ++i) {
    napi_value v;
    NAPI_OK(napi_get_element(env, argv[1], i, &v));
    NAPI_OK(napi_get_value_int32(env, v, &ids[i]));
  }
  int32_t max_new = 0;
  NAPI_OK(napi_get_value_int32(env, argv[2], &max_new));
  std::vector<int32_t> out(max_new > 0 ? max_new : 1);
  CbCtx ctx{env, argc > 3 ? argv[3] : nullptr};
  napi_valuetype t = napi_undefined;
  if (ctx.fn) napi_typeof(env, ctx.fn, &t);
  qd_stats st{};
  const int rc = qd_generate_greedy(e, ids.data(), (int)n, max_new, out.data(),
                                    t == napi_function ? on_token : nullptr, &ctx, &st);
  if (rc != QD_OK) return throw_qd(env, e, rc);
  napi_value res, gen, v;
  NAPI_OK(napi_create_object(env, &res));
  NAPI_OK(napi_create_array_with_length(env, st.generated_tokens, &gen));
  for (int i = 0; i < st.generated_tokens; ++i) {
    NAPI_OK(napi_create_int32(env, out[i], &v));
    NAPI_OK(napi_set_element(env, gen, i, v));
  }
  NAPI_OK(napi_set_named_property(env, res, "generated", gen));
  NAPI_OK(napi_create_double(env, st.generate_ms, &v));
  NAPI_OK(napi_set_named_property(env, res, "generateMs", v));
  NAPI_OK(napi_create_double(env, st.first_token_ms, &v));
  NAPI_OK(napi_set_named_property(env, res, "firstTokenMs", v));
  return res;
}

bool set_num(napi_env env, napi_value obj, const char* key, double value) {
  napi_value v;
  return napi_create_double(env, value, &v) == napi_ok && napi_set_named_property(env, obj, key, v) == napi_ok;
}

// kernelBenchmarks(engine) -> the runKernelBenchmarks result object (qd_run_kernel_benchmarks)
napi_value KernelBenchmarks(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
  void* data = nullptr;
  NAPI_OK(napi_get_value_external(env, argv[0], &data));
  qd_engine* e = static_cast<qd_engine*>(data);
  qd_kernel_bench b{};
  const int rc = qd_run_kernel_benchmarks(e, &b);
  if (rc != QD_OK) return throw_qd(env, e, rc);
  napi_value r;
  NAPI_OK(napi_create_object(env, &r));
  const struct {
    const char* key;
    double value;
  } fields[] = {
      {"baselineMatvecMs", b.baseline_matvec_ms}, {"optimizedMatvecMs", b.optimized_matvec_ms},
      {"matvecSpeedup", b.matvec_speedup}, {"baselineBytes", b.baseline_bytes},
      {"optimizedBytes", b.optimized_bytes}, {"memoryReduction", b.memory_reduction},
      {"maxAbsError", b.max_abs_error}, {"meanAbsError", b.mean_abs_error},
      {"blockDefaultMs", b.block_default_ms}, {"blockOptimizedMs", b.block_optimized_ms},
      {"blockSpeedup", b.block_speedup}, {"blockMaxAbsError", b.block_max_abs_error},
      {"blockMeanAbsError", b.block_mean_abs_error}, {"realQ4Ms", b.real_q4_ms},
      {"realQ4MaxAbsError", b.real_q4_max_abs_error}, {"realQ4MeanAbsError", b.real_q4_mean_abs_error},
      {"gqaMs", b.gqa_ms}, {"gqaMaxAbsError", b.gqa_max_abs_error}, {"gqaMeanAbsError", b.gqa_mean_abs_error},
      {"gqaSeqLen", (double)b.gqa_seq_len}, {"layer0DecodeMs", b.layer0_decode_ms},
      {"layer0Finite", (double)b.layer0_finite}, {"layer0MeanAbs", b.layer0_mean_abs}, {"rmsMs", b.rms_ms},
      {"estimatedGbps", b.estimated_gbps},
  };
  for (const auto& f : fields)
    if (!set_num(env, r, f.key, f.value)) return throw_qd(env, e, QD_E_INVALID);
  return r;
}

// engineProfile(engine) -> {layers, hidden, intermediate, heads, kvHeads, headDim, vocab}
napi_value EngineProfile(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
  void* data = nullptr;
  NAPI_OK(napi_get_value_external(env, argv[0], &data));
  qd_engine* e = static_cast<qd_engine*>(data);
  qd_profile p{};
  const int rc = qd_engine_profile(e, &p);
  if (rc != QD_OK) return throw_qd(env, e, rc);
  napi_value r;
  NAPI_OK(napi_create_object(env, &r));
  if (!set_num(env, r, "layers", p.layers) || !set_num(env, r, "hidden", p.hidden) ||
      !set_num(env, r, "intermediate", p.intermediate) || !set_num(env, r, "heads", p.heads) ||
      !set_num(env, r, "kvHeads", p.kv_heads) || !set_num(env, r, "headDim", p.head_dim) ||
      !set_num(env, r, "vocab", p.vocab))
    return throw_qd(env, e, QD_E_INVALID);
  return r;
}

// fullDecoderStackBenchmark(engine) -> {ms, warmupMs, layers, finite, meanAbs}
napi_value FullDecoderStackBenchmark(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
  void* data = nullptr;
  NAPI_OK(napi_get_value_external(env, argv[0], &data));
  qd_engine* e = static_cast<qd_engine*>(data);
  qd_stack_bench b{};
  const int rc = qd_run_full_decoder_stack_benchmark(e, &b);
  if (rc != QD_OK) return throw_qd(env, e, rc);
  napi_value r;
  NAPI_OK(napi_create_object(env, &r));
  if (!set_num(env, r, "ms", b.ms) || !set_num(env, r, "warmupMs", b.warmup_ms) ||
      !set_num(env, r, "layers", b.layers) || !set_num(env, r, "finite", b.finite) ||
      !set_num(env, r, "meanAbs", b.mean_abs))
    return throw_qd(env, e, QD_E_INVALID);
  return r;
}

napi_value Init(napi_env env, napi_value exports) {
  napi_property_descriptor props[] = {
      {"engineCreate", nullptr, EngineCreate, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"generateGreedy", nullptr, GenerateGreedy, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"engineProfile", nullptr, EngineProfile, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"kernelBenchmarks", nullptr, KernelBenchmarks, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"fullDecoderStackBenchmark", nullptr, FullDecoderStackBenchmark, nullptr, nullptr, nullptr, napi_default,
       nullptr},
  };
  napi_define_properties(env, exports, sizeof(props) / sizeof(props[0]), props);
  return exports;
}

}  // namespace

NAPI_MODULE(NODE_GYP_MODULE_NAME, Init)
