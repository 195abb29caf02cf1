// Top-k / top-p sampling over the LM head's logits (the reference decodes greedily
// only, README.md:172-173; this widens the token choice after the same LM head).
//
// Definition (the oracle restates it, qo_sample):
//  * candidates: the K largest logits, K = top_k if 1 <= top_k <= 64, else 64
//    (top_k = 0: no top-k limit, top-p then runs over the 64 most likely tokens),
//    ordered by value, ties to the lower index; NaN ranks below every number;
//  * p_i = exp((v_i - v_0) / temperature) over the candidates (v_0 the largest);
//  * top-p: keep the shortest prefix whose sum reaches top_p of the candidates' sum;
//  * u = (splitmix64(seed ^ (step * 0xD1B54A32D192ED03)) >> 40) * 2^-24 in [0, 1);
//    the token is the first kept candidate whose running sum exceeds u times the
//    kept sum. temperature <= 0 or top_k == 1 is greedy (the argmax), unchanged.
//
// Selection: the logits are cut into chunks of kSampleChunk; one CTA per chunk finds
// the chunk's K best by a 4-pass 8-bit radix select on order-preserving keys and
// writes them; one CTA selects the K best of those the same way, sorts them, and
// samples. Sums run sequentially in candidate order on one thread (deterministic).
#include <cmath>
#include <string>

#include "../../include/qdecode.h"
#include "internal.cuh"

namespace qd {

constexpr int kSampleK = 64;        // candidates at most
constexpr int kSampleThreads = 256;
constexpr int kSampleChunk = 2048;  // logits per first-level CTA

__host__ __device__ inline unsigned long long splitmix64(unsigned long long x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Order-preserving unsigned key of a float: larger value, larger key; NaN lowest.
__device__ __forceinline__ uint32_t okey(float v) {
  if (v != v) return 0u;
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float okey_value(uint32_t k) {
  if (k == 0u) return __int_as_float(0x7fc00000);
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// The K (<= n) best of key[0..n) (larger key first, ties to the lower position) into
// out_key / out_pos, unordered. Every thread of the CTA calls it; sm: [256 + 8] words.
__device__ void cta_select(const uint32_t* key, int n, int K, uint32_t* sm, uint32_t* out_key, int* out_pos) {
  uint32_t* hist = sm;          // [256]
  uint32_t* info = sm + 256;    // [0] digit, [1] count above, [2] output slot, [3] eq prefix
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0u, mask = 0u;
  int rem = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0u;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const uint32_t k = key[i];
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (warp == 0) {  // lane l: bins 255 - 8l .. 248 - 8l, from the top
      uint32_t c[8], s = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        s += c[j];
      }
      uint32_t incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      uint32_t above = incl - s;  // bins higher than this lane's
      if (above < (uint32_t)rem && incl >= (uint32_t)rem) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (above + c[j] >= (uint32_t)rem) {
            info[0] = 255u - 8u * lane - j;
            info[1] = above;
            break;
          }
          above += c[j];
        }
      }
    }
    __syncthreads();
    const uint32_t d = info[0];
    rem -= (int)info[1];
    prefix |= d << shift;
    mask |= 255u << shift;
    __syncthreads();
  }
  // prefix: the K-th best key; take every key above it and the first `rem` equal ones.
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  int eq = 0;
  for (int i = lo; i < hi; ++i) eq += key[i] == prefix;
  // exclusive scan of eq over threads (warp scans, then warp totals)
  int incl = eq;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (tid == 0) info[2] = 0u;
  if (lane == 31) hist[warp] = (uint32_t)incl;
  __syncthreads();
  int before = incl - eq;
  for (int w = 0; w < warp; ++w) before += (int)hist[w];
  for (int i = lo; i < hi; ++i) {
    const uint32_t k = key[i];
    bool take = k > prefix;
    if (k == prefix) {
      take = before < rem;
      ++before;
    }
    if (take) {
      const uint32_t slot = atomicAdd(&info[2], 1u);
      out_key[slot] = k;
      out_pos[slot] = i;
    }
  }
  __syncthreads();
}

// First level: the K best of each chunk -> cand[chunk][K] (key, vocabulary index).
__global__ void __launch_bounds__(kSampleThreads) k_sample_partial(const float* logits, int vocab, int K,
                                                                   uint32_t* cand_key, int* cand_idx) {
  __shared__ uint32_t key[kSampleChunk];
  __shared__ uint32_t sm[264];
  __shared__ uint32_t sk[kSampleK];
  __shared__ int sp[kSampleK];
  const int base = blockIdx.x * kSampleChunk;
  const int n = min(kSampleChunk, vocab - base);
  pdl_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) key[i] = okey(logits[base + i]);
  __syncthreads();
  const int k = min(K, n);
  cta_select(key, n, k, sm, sk, sp);
  // sorted (larger key first, then lower index), so that equal keys of the second
  // level stand in vocabulary order
  if (threadIdx.x < k) {
    const uint32_t mk = sk[threadIdx.x];
    const int mi = sp[threadIdx.x];
    int r = 0;
    for (int j = 0; j < k; ++j) r += sk[j] > mk || (sk[j] == mk && sp[j] < mi);
    cand_key[blockIdx.x * K + r] = mk;
    cand_idx[blockIdx.x * K + r] = base + mi;
  }
  for (int j = k + threadIdx.x; j < K; j += blockDim.x) {
    cand_key[blockIdx.x * K + j] = 0u;
    cand_idx[blockIdx.x * K + j] = 0x7fffffff;
  }
}

struct SampleOut {
  DevState* st;          // engine decode: token for position st->pos, output slot st->step - 1
  int* tokens;
  int* out_dev;
  int* out_host;
  int max_seq;
  int32_t* token;        // kernel-level entry: the sampled id
  int step;              // kernel-level entry: the RNG step
};

// Second level: the K best candidates, sorted; the sampled id. n_real = min(K, vocab)
// of them are tokens: a chunk shorter than K pads its candidates with (key 0, index
// 0x7fffffff) entries, which sort after every token and are never drawn.
__global__ void __launch_bounds__(kSampleThreads) k_sample_final(const uint32_t* cand_key, const int* cand_idx,
                                                                 int n_cand, int K, int n_real, float temperature,
                                                                 float top_p, unsigned long long seed, SampleOut o) {
  extern __shared__ uint32_t dyn[];
  uint32_t* key = dyn;                                   // [n_cand]
  __shared__ uint32_t sm[264];
  __shared__ uint32_t sk[kSampleK];
  __shared__ int sp[kSampleK];
  __shared__ uint32_t rk[kSampleK];
  __shared__ int ri[kSampleK];
  pdl_wait();
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) key[i] = cand_key[i];
  __syncthreads();
  int k = min(K, n_cand);
  cta_select(key, n_cand, k, sm, sk, sp);
  // rank sort: larger key first, ties to the lower vocabulary index, then to the lower
  // candidate position (padding entries repeat one key and index): a permutation of 0..k-1
  if (threadIdx.x < k) {
    const uint32_t mk = sk[threadIdx.x];
    const int mp = sp[threadIdx.x], mi = cand_idx[mp];
    int r = 0;
    for (int j = 0; j < k; ++j) {
      const uint32_t ok = sk[j];
      const int op = sp[j], oi = cand_idx[op];
      r += ok > mk || (ok == mk && (oi < mi || (oi == mi && op < mp)));
    }
    rk[r] = mk;
    ri[r] = mi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int step = o.step;
    if (o.st) step = o.st->step - 1;
    const float v0 = okey_value(rk[0]);
    float cum[kSampleK];
    float s = 0.0f;
    k = min(k, n_real);  // the tokens among the candidates
    for (int i = 0; i < k; ++i) {
      const float v = okey_value(rk[i]);
      const float p = (v == v && v0 == v0) ? expf((v - v0) / temperature) : (i == 0 ? 1.0f : 0.0f);
      s += p;
      cum[i] = s;
    }
    int m = k - 1;
    if (top_p < 1.0f)
      for (int i = 0; i < k; ++i)
        if (cum[i] >= top_p * s) { m = i; break; }
    const unsigned long long h = splitmix64(seed ^ ((unsigned long long)(unsigned)step * 0xD1B54A32D192ED03ull));
    const float u = (float)(h >> 40) * 5.9604644775390625e-08f;
    const float target = u * cum[m];
    int pick = m;
    for (int i = 0; i <= m; ++i)
      if (cum[i] > target) { pick = i; break; }
    const int tok = ri[pick];
    if (o.token) o.token[0] = tok;
    if (o.st) {
      const int pos = o.st->pos, slot = o.st->step - 1;
      if (pos <= o.max_seq) o.tokens[pos] = tok;
      if (slot >= 0 && slot < o.st->max_new) {
        o.out_dev[slot] = tok;
        if (o.out_host) *reinterpret_cast<volatile int*>(o.out_host + slot) = tok;
      }
    }
  }
}

int sample_candidates(int vocab) { return (vocab + kSampleChunk - 1) / kSampleChunk * kSampleK; }

size_t sample_workspace_bytes(int vocab) { return (size_t)sample_candidates(vocab) * 8 + 256; }

bool sampling_is_greedy(const qd_sampling& s) { return !(s.temperature > 0.0f) || s.top_k == 1; }

// The second level holds every first-level candidate in shared memory (48 KB).
constexpr int kSampleMaxVocab = 48 * 1024 / (kSampleK * 4) * kSampleChunk;

void check_sampling(const qd_sampling& s) {
  if (!(s.top_p > 0.0f) || s.top_p > 1.0f || s.top_k < 0 || !std::isfinite(s.temperature))
    throw QdError{QD_E_INVALID, "sampling: top_p must be in (0, 1], top_k >= 0, temperature finite"};
}

void enqueue_sample(const float* logits, int vocab, const qd_sampling& s, void* workspace, SampleOut o,
                    cudaStream_t stream) {
  const bool greedy = sampling_is_greedy(s);  // one candidate: the argmax
  const int K = greedy ? 1 : ((s.top_k >= 1 && s.top_k <= kSampleK) ? s.top_k : kSampleK);
  const float temperature = greedy ? 1.0f : s.temperature;
  const int chunks = (vocab + kSampleChunk - 1) / kSampleChunk;
  uint32_t* ck = static_cast<uint32_t*>(workspace);
  int* ci = reinterpret_cast<int*>(ck + (size_t)chunks * K);
  launch_ex(k_sample_partial, dim3(chunks), dim3(kSampleThreads), 0, stream, logits, vocab, K, ck, ci);
  const size_t smem = (size_t)chunks * K * 4;  // within the default 48 KB (checked by the callers)
  launch_ex(k_sample_final, dim3(1), dim3(kSampleThreads), smem, stream, (const uint32_t*)ck, (const int*)ci,
            chunks * K, K, std::min(K, vocab), temperature, s.top_p, (unsigned long long)s.seed, o);
}

void enqueue_engine_sample(qd_engine* e, const qd_sampling& s) {
  if (e->p.vocab > kSampleMaxVocab) throw QdError{QD_E_RANGE, "sampling: vocabulary beyond the sampler's limit"};
  if (!e->sample_ws) {
    if (cudaMalloc(&e->sample_ws, sample_workspace_bytes(e->p.vocab)) != cudaSuccess)
      throw QdError{QD_E_NOMEM, "cannot allocate the sampling workspace"};
  }
  SampleOut o{};
  o.st = e->st;
  o.tokens = e->tokens;
  o.out_dev = e->out_dev;
  o.out_host = e->out_host_dev;
  o.max_seq = e->opt.max_seq;
  enqueue_sample(e->logits, e->p.vocab, s, e->sample_ws, o, e->stream);
}

}  // namespace qd

extern "C" {

size_t qd_sample_workspace_bytes(uint32_t vocab) { return qd::sample_workspace_bytes((int)vocab); }

int qd_sample_logits(const float* logits, uint32_t vocab, const qd_sampling* s, uint32_t step, void* workspace,
                     int32_t* token, void* stream) {
  try {
    if (!logits || !s || !workspace || !token || vocab == 0) throw qd::QdError{QD_E_INVALID, "NULL argument"};
    if (vocab > (uint32_t)qd::kSampleMaxVocab)
      throw qd::QdError{QD_E_RANGE, "qd_sample_logits: vocab beyond " + std::to_string(qd::kSampleMaxVocab)};
    qd::check_sampling(*s);
    qd::SampleOut o{};
    o.token = token;
    o.step = (int)step;
    qd::enqueue_sample(logits, (int)vocab, *s, workspace, o, static_cast<cudaStream_t>(stream));
  } catch (const qd::QdError& err) {
    qd::set_thread_error(err.msg);
    return err.code;
  }
  return QD_OK;
}

}  // extern "C"
