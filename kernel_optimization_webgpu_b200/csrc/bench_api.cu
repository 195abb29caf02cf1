// The reference's benchmark exports on the B200 engine:
// runKernelBenchmarks and runFullDecoderStackBenchmark (webgpu-runtime.js:62-163).
//
// Each benchmark builds the reference's own fixture inputs (createVector,
// createQ8Inputs), times back-to-back launches on the engine's stream with CUDA
// events, and compares the result with a double-precision CPU evaluation of the
// same math, as the reference's cpu* checks and errorStats do. The q4 projection,
// the attention and the decode layers are the engine's own kernels; the q8 matvec
// (a microbenchmark the reference keeps beside the q4 path) gets two small kernels
// here: one thread per row (the shape of q8_matvec_scalar.wgsl) and one warp per
// row with 128-bit loads.
#include <cmath>
#include <string>
#include <vector>

#include "../../include/qdecode.h"
#include "internal.cuh"

using namespace qd;

namespace {

// ---- device kernels ------------------------------------------------------------------

// q8 matvec, one thread per output row: y[r] = sum_c int8(w[r][c]) * scale[r] * x[c].
__global__ void k_q8_rowthread(const float* x, const uint32_t* w, const float* scales, float* y, int in_size,
                               int out_size, int words_per_row) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= out_size) return;
  const uint32_t* wr = w + (size_t)row * words_per_row;
  const float s = scales[row];
  float acc = 0.0f;
  for (int k = 0; k < words_per_row; ++k) {
    const uint32_t p = wr[k];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const int c = k * 4 + l;
      if (c < in_size) acc += (float)(int8_t)(p >> (8 * l)) * s * x[c];
    }
  }
  y[row] = acc;
}

// q8 matvec, one warp per output row: lane l reads 16 weights (one uint4) per step,
// the row's dot is a warp sum, the row scale is applied once.
__global__ void k_q8_rowwarp(const float* x, const uint32_t* w, const float* scales, float* y, int in_size,
                             int out_size, int words_per_row) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= out_size) return;
  const uint32_t* wr = w + (size_t)row * words_per_row;
  float acc = 0.0f;
  if ((words_per_row & 3) == 0) {
    const uint4* w4 = reinterpret_cast<const uint4*>(wr);
    for (int q = lane; q < words_per_row / 4; q += 32) {
      const uint4 v = w4[q];
      const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int l = 0; l < 4; ++l) {
          const int c = q * 16 + k * 4 + l;
          if (c < in_size) acc = fmaf((float)(int8_t)(ws[k] >> (8 * l)), x[c], acc);
        }
    }
  } else {
    for (int k = lane; k < words_per_row; k += 32) {
      const uint32_t p = wr[k];
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const int c = k * 4 + l;
        if (c < in_size) acc = fmaf((float)(int8_t)(p >> (8 * l)), x[c], acc);
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc * scales[row];
}

// RMSNorm of one vector (n <= 4 * blockDim.x) by one CTA: y = x / sqrt(mean(x^2) + eps) * w.
__global__ void k_rms_one(const float* x, const float* w, float* y, int n, float eps) {
  __shared__ float red[32];
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.0f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
  const float inv = rsqrtf(t / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = x[i] * inv * w[i];
}

__global__ void k_silu_mul(const float* g, const float* u, float* y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

// ---- host fixtures and CPU checks (double precision) ----------------------------------

// createVector(size, step, fn) (webgpu-runtime.js:1432): f32(fn(i * step)).
std::vector<float> make_vector(int n, double step, bool use_cos) {
  std::vector<float> v(n);
  for (int i = 0; i < n; ++i) v[i] = (float)(use_cos ? std::cos(i * step) : std::sin(i * step));
  return v;
}

struct Q8 {
  int in_size, out_size, wpr;
  std::vector<float> scales;
  std::vector<uint32_t> packed;
};

// createQ8Inputs(inSize, outSize) (webgpu-runtime.js:1464-1486).
Q8 make_q8(int in_size, int out_size) {
  Q8 q;
  q.in_size = in_size;
  q.out_size = out_size;
  q.wpr = (in_size + 3) / 4;
  q.scales.resize(out_size);
  for (int i = 0; i < out_size; ++i) q.scales[i] = (float)(0.0125 + (i % 11) * 0.0002);
  q.packed.assign((size_t)q.wpr * out_size, 0u);
  for (int r = 0; r < out_size; ++r)
    for (int w = 0; w < q.wpr; ++w) {
      uint32_t word = 0;
      for (int l = 0; l < 4; ++l) {
        const int c = w * 4 + l;
        const int v = c < in_size ? ((r * 13 + c * 7) % 255) - 127 : 0;
        word |= (uint32_t)(v & 0xff) << (8 * l);
      }
      q.packed[(size_t)r * q.wpr + w] = word;
    }
  return q;
}

std::vector<float> cpu_q8(const Q8& q, const std::vector<float>& x) {
  std::vector<float> y(q.out_size);
  for (int r = 0; r < q.out_size; ++r) {
    double acc = 0.0;
    for (int c = 0; c < q.in_size; ++c) {
      const int v = (int8_t)(q.packed[(size_t)r * q.wpr + c / 4] >> (8 * (c % 4)));
      acc += (double)v * q.scales[r] * x[c];
    }
    y[r] = (float)acc;
  }
  return y;
}

std::vector<float> cpu_rms(const std::vector<float>& x, const std::vector<float>& w, double eps) {
  double ss = 0.0;
  for (float v : x) ss += (double)v * v;
  const double inv = 1.0 / std::sqrt(ss / x.size() + eps);
  std::vector<float> y(x.size());
  for (size_t i = 0; i < x.size(); ++i) y[i] = (float)(x[i] * inv * w[i]);
  return y;
}

float half_bits_to_float(uint16_t h) {
  __half_raw r;
  r.x = h;
  return __half2float(__half(r));
}

// q4 row records (nb 16-byte blocks, then nb f16 scales): y = W x in double.
std::vector<float> cpu_q4_records(const std::vector<char>& rec, long long stride, int rows, int k,
                                  const std::vector<float>& x) {
  const int nb = k / kBlockCols;
  std::vector<float> y(rows);
  for (int r = 0; r < rows; ++r) {
    const unsigned char* q = reinterpret_cast<const unsigned char*>(rec.data() + r * stride);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(q + nb * 16);
    double acc = 0.0;
    for (int b = 0; b < nb; ++b) {
      const double s = half_bits_to_float(sc[b]);
      for (int j = 0; j < 32; ++j) {
        const int byte = q[b * 16 + j / 2];
        const int nib = (j & 1) ? (byte >> 4) : (byte & 15);
        acc += (nib - 8) * s * x[b * 32 + j];
      }
    }
    y[r] = (float)acc;
  }
  return y;
}

// cpuGqaDecode (webgpu-runtime.js:943-982) in double.
std::vector<float> cpu_gqa(const std::vector<float>& q, const std::vector<float>& kc, const std::vector<float>& vc,
                           int seq, int qh, int kvh, int hd) {
  std::vector<float> y((size_t)qh * hd);
  const int group = qh / kvh;
  const double scale = 1.0 / std::sqrt((double)hd);
  std::vector<double> sc(seq);
  for (int h = 0; h < qh; ++h) {
    const int g = h / group;
    double mx = -INFINITY;
    for (int p = 0; p < seq; ++p) {
      double d = 0.0;
      for (int i = 0; i < hd; ++i) d += (double)q[h * hd + i] * kc[((size_t)p * kvh + g) * hd + i];
      sc[p] = d * scale;
      mx = std::max(mx, sc[p]);
    }
    double den = 0.0;
    for (int p = 0; p < seq; ++p) den += (sc[p] = std::exp(sc[p] - mx));
    for (int i = 0; i < hd; ++i) {
      double acc = 0.0;
      for (int p = 0; p < seq; ++p) acc += sc[p] * vc[((size_t)p * kvh + g) * hd + i];
      y[h * hd + i] = (float)(acc / den);
    }
  }
  return y;
}

// errorStats (webgpu-runtime.js:1540-1552).
void error_stats(const std::vector<float>& got, const std::vector<float>& want, double& max_abs, double& mean_abs) {
  max_abs = 0.0;
  double sum = 0.0;
  for (size_t i = 0; i < got.size(); ++i) {
    const double e = std::fabs((double)got[i] - (double)want[i]);
    max_abs = std::max(max_abs, e);
    sum += e;
  }
  mean_abs = got.empty() ? 0.0 : sum / got.size();
}

// ---- device buffers and timing -----------------------------------------------------------

// Device allocations of one benchmark run, freed together.
struct DevBufs {
  std::vector<void*> ptrs;
  ~DevBufs() {
    for (void* p : ptrs) cudaFree(p);
  }
  template <typename T>
  T* alloc(size_t n) {
    void* p = nullptr;
    if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) throw QdError{QD_E_NOMEM, "benchmark buffers"};
    ptrs.push_back(p);
    return static_cast<T*>(p);
  }
  template <typename T>
  T* upload(const std::vector<T>& v, cudaStream_t s) {
    T* p = alloc<T>(v.size());
    QD_CK(cudaMemcpyAsync(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, s));
    return p;
  }
};

template <typename T>
std::vector<T> download(const T* p, size_t n, cudaStream_t s) {
  std::vector<T> v(n);
  QD_CK(cudaMemcpyAsync(v.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost, s));
  QD_CK(cudaStreamSynchronize(s));
  return v;
}

// Milliseconds per call of `enqueue` over `iters` calls back to back (one untimed call first).
template <typename F>
double time_ms(cudaStream_t s, int iters, F enqueue) {
  enqueue();
  cudaEvent_t a, b;
  QD_CK(cudaEventCreate(&a));
  QD_CK(cudaEventCreate(&b));
  QD_CK(cudaEventRecord(a, s));
  for (int i = 0; i < iters; ++i) enqueue();
  QD_CK(cudaEventRecord(b, s));
  QD_CK(cudaEventSynchronize(b));
  float ms = 0.0f;
  QD_CK(cudaEventElapsedTime(&ms, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return (double)ms / iters;
}

void launch_q8(bool per_warp, const float* x, const uint32_t* w, const float* sc, float* y, const Q8& q,
               cudaStream_t s) {
  if (per_warp) {
    const int rows_per_cta = 8;
    k_q8_rowwarp<<<(q.out_size + rows_per_cta - 1) / rows_per_cta, 32 * rows_per_cta, 0, s>>>(
        x, w, sc, y, q.in_size, q.out_size, q.wpr);
  } else {
    k_q8_rowthread<<<(q.out_size + 63) / 64, 64, 0, s>>>(x, w, sc, y, q.in_size, q.out_size, q.wpr);
  }
  QD_CK(cudaGetLastError());
}

int bfail(qd_engine* e, const QdError& err) {
  set_thread_error(err.msg);
  if (e) e->err = err.msg;
  return err.code;
}

// Finite count and mean |v| of a vector.
void finite_stats(const std::vector<float>& v, int& finite, double& mean_abs) {
  finite = 0;
  double sum = 0.0;
  for (float x : v) {
    if (std::isfinite(x)) ++finite;
    sum += std::fabs((double)x);
  }
  mean_abs = v.empty() ? 0.0 : sum / v.size();
}

}  // namespace

extern "C" {

int qd_run_kernel_benchmarks(qd_engine* e, qd_kernel_bench* out) {
  if (!e || !out) return bfail(e, QdError{QD_E_INVALID, "NULL argument"});
  try {
    QD_CK(cudaSetDevice(e->dev));
    cudaStream_t s = e->stream;
    const qd_profile& p = e->p;
    const int H = p.hidden, I = p.intermediate;
    *out = qd_kernel_bench{};
    DevBufs d;

    // 1. q8 matvec hidden -> intermediate: one thread per row vs one warp per row.
    {
      const Q8 q = make_q8(H, I);
      std::vector<float> x(H);
      for (int i = 0; i < H; ++i) x[i] = (float)std::sin(i * 0.017);
      const float* dx = d.upload(x, s);
      const uint32_t* dw = d.upload(q.packed, s);
      const float* ds = d.upload(q.scales, s);
      float* dy = d.alloc<float>(I);
      out->baseline_matvec_ms = time_ms(s, 40, [&] { launch_q8(false, dx, dw, ds, dy, q, s); });
      out->optimized_matvec_ms = time_ms(s, 80, [&] { launch_q8(true, dx, dw, ds, dy, q, s); });
      out->matvec_speedup = out->baseline_matvec_ms / out->optimized_matvec_ms;
      out->baseline_bytes = out->optimized_bytes = (double)(x.size() * 4 + q.packed.size() * 4 + q.scales.size() * 4);
      out->memory_reduction = 1.0;
      error_stats(download(dy, I, s), cpu_q8(q, x), out->max_abs_error, out->mean_abs_error);
      out->estimated_gbps = out->optimized_bytes / (out->optimized_matvec_ms / 1000.0) / 1e9;
    }

    // 2. q8 MLP block: RMSNorm -> gate, up -> silu * up -> down.
    {
      const Q8 qg = make_q8(H, I), qd = make_q8(I, H);  // gate and up share the fixture
      std::vector<float> x(H), w(H, 1.0f);
      for (int i = 0; i < H; ++i) x[i] = (float)std::sin(i * 0.017);
      const float *dx = d.upload(x, s), *dnw = d.upload(w, s);
      const uint32_t *dgw = d.upload(qg.packed, s), *dupw = d.upload(qg.packed, s), *ddw = d.upload(qd.packed, s);
      const float *dgs = d.upload(qg.scales, s), *dus = d.upload(qg.scales, s), *dds = d.upload(qd.scales, s);
      float *dn = d.alloc<float>(H), *dg = d.alloc<float>(I), *du = d.alloc<float>(I), *da = d.alloc<float>(I);
      float* dout = d.alloc<float>(H);
      auto block = [&](bool per_warp) {
        k_rms_one<<<1, 1024, 0, s>>>(dx, dnw, dn, H, 1e-6f);
        launch_q8(per_warp, dn, dgw, dgs, dg, qg, s);
        launch_q8(per_warp, dn, dupw, dus, du, qg, s);
        k_silu_mul<<<(I + 255) / 256, 256, 0, s>>>(dg, du, da, I);
        launch_q8(per_warp, da, ddw, dds, dout, qd, s);
      };
      out->block_default_ms = time_ms(s, 16, [&] { block(false); });
      out->block_optimized_ms = time_ms(s, 32, [&] { block(true); });
      out->block_speedup = out->block_default_ms / out->block_optimized_ms;
      // cpuMlpBlock (webgpu-runtime.js:1412-1421)
      const std::vector<float> n = cpu_rms(x, w, p.eps);
      const std::vector<float> g = cpu_q8(qg, n);
      std::vector<float> act(I);
      for (int i = 0; i < I; ++i) act[i] = (float)(g[i] / (1.0 + std::exp(-(double)g[i])) * g[i]);
      error_stats(download(dout, H, s), cpu_q8(qd, act), out->block_max_abs_error, out->block_mean_abs_error);
    }

    // 3. layer 0's resident q4 gate projection (pair records [gate j | up j]: every other record).
    {
      const long long rec = rec_bytes(H);
      std::vector<float> x(H);
      for (int i = 0; i < H; ++i) x[i] = (float)std::sin(i * 0.017);
      const float* dx = d.upload(x, s);
      float* dy = d.alloc<float>(I);
      const char* base = e->layers[0].gu;
      out->real_q4_ms = time_ms(s, 80, [&] { bench_rows_matvec(e, base, 2 * rec, I, H, dx, dy, s); });
      std::vector<char> pairs = download(base, (size_t)2 * rec * I, s);
      error_stats(download(dy, I, s), cpu_q4_records(pairs, 2 * rec, I, H, x), out->real_q4_max_abs_error,
                  out->real_q4_mean_abs_error);
    }

    // 4. decode attention over 128 positions (f32 cache, createVector data).
    {
      const int seq = 128, qh = p.heads, kvh = p.kv_heads, hd = kHeadDim;
      const std::vector<float> q = make_vector(qh * hd, 0.011, false);
      std::vector<float> kc((size_t)seq * kvh * hd), vc((size_t)seq * kvh * hd);
      for (size_t i = 0; i < kc.size(); ++i) {
        kc[i] = (float)std::cos(i * 0.007);
        vc[i] = (float)std::sin(i * 0.013);
      }
      const float *dq = d.upload(q, s), *dk = d.upload(kc, s), *dv = d.upload(vc, s);
      float* dy = d.alloc<float>((size_t)qh * hd);
      char* ws = d.alloc<char>(qd_gqa_decode_workspace_bytes(seq, qh));
      int rc = QD_OK;
      out->gqa_ms = time_ms(s, 160, [&] {
        const int r = qd_gqa_decode(dq, dk, dv, QD_KV_F32, dy, seq, qh, kvh, hd, ws, s);
        if (r != QD_OK) rc = r;
      });
      if (rc != QD_OK) throw QdError{rc, "attention benchmark: qd_gqa_decode failed"};
      out->gqa_seq_len = seq;
      error_stats(download(dy, (size_t)qh * hd, s), cpu_gqa(q, kc, vc, seq, qh, kvh, hd), out->gqa_max_abs_error,
                  out->gqa_mean_abs_error);
    }

    // 5. one decode layer (layer 0 at position 0, input sin(0.013 i)).
    {
      const std::vector<float> h = make_vector(H, 0.013, false);
      const float* dh = d.upload(h, s);
      bench_set_position(e, 0);
      out->layer0_decode_ms = time_ms(s, 8, [&] {
        QD_CK(cudaMemcpyAsync(e->h, dh, (size_t)H * 4, cudaMemcpyDeviceToDevice, s));
        bench_layer_from_hidden(e, 0, s);
      });
      bench_check_state(e);
      finite_stats(download(e->h, H, s), out->layer0_finite, out->layer0_mean_abs);
    }

    // 6. RMSNorm of cos(0.013 i), unit weight.
    {
      const std::vector<float> x = make_vector(H, 0.013, true);
      const std::vector<float> w(H, 1.0f);
      const float *dx = d.upload(x, s), *dw = d.upload(w, s);
      float* dy = d.alloc<float>(H);
      out->rms_ms = time_ms(s, 120, [&] {
        k_rms_one<<<1, 1024, 0, s>>>(dx, dw, dy, H, p.eps);
      });
      QD_CK(cudaGetLastError());
    }
    QD_CK(cudaStreamSynchronize(s));
  } catch (const QdError& err) {
    return bfail(e, err);
  }
  return QD_OK;
}

int qd_run_full_decoder_stack_benchmark(qd_engine* e, qd_stack_bench* out) {
  if (!e || !out) return bfail(e, QdError{QD_E_INVALID, "NULL argument"});
  try {
    QD_CK(cudaSetDevice(e->dev));
    cudaStream_t s = e->stream;
    const qd_profile& p = e->p;
    const int H = p.hidden;
    *out = qd_stack_bench{};
    DevBufs d;
    const std::vector<float> h = make_vector(H, 0.013, false);
    const float* dh = d.upload(h, s);
    float* dy = d.alloc<float>(H);
    bench_set_position(e, 0);
    auto stack = [&] {
      QD_CK(cudaMemcpyAsync(e->h, dh, (size_t)H * 4, cudaMemcpyDeviceToDevice, s));
      for (int l = 0; l < p.layers; ++l) bench_layer_from_hidden(e, l, s);
      k_rms_one<<<1, 1024, 0, s>>>(e->h, e->final_norm, dy, H, p.eps);
      QD_CK(cudaGetLastError());
    };
    cudaEvent_t a, b, c;
    QD_CK(cudaEventCreate(&a));
    QD_CK(cudaEventCreate(&b));
    QD_CK(cudaEventCreate(&c));
    QD_CK(cudaEventRecord(a, s));
    stack();
    QD_CK(cudaEventRecord(b, s));
    stack();
    QD_CK(cudaEventRecord(c, s));
    QD_CK(cudaEventSynchronize(c));
    float w_ms = 0.0f, ms = 0.0f;
    QD_CK(cudaEventElapsedTime(&w_ms, a, b));
    QD_CK(cudaEventElapsedTime(&ms, b, c));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaEventDestroy(c);
    bench_check_state(e);
    out->warmup_ms = w_ms;
    out->ms = ms;
    out->layers = p.layers;
    finite_stats(download(dy, H, s), out->finite, out->mean_abs);
  } catch (const QdError& err) {
    return bfail(e, err);
  }
  return QD_OK;
}

}  // extern "C"
