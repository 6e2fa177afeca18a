// Top-K + temperature sampling on the device (llama-streaming.js:868-894
// sample(logits, topK, temperature)).
//
// The reference divides every logit by the temperature (double), sorts the
// (value, index) pairs by value descending with a stable sort, keeps topK,
// takes e_i = exp(v_i - v_0), sums them in order, normalises each, and
// returns the first index whose running sum of probabilities reaches
// r = Math.random().  Division by a positive temperature keeps the order of
// the f32 logits (distinct floats stay distinct in double), so the top K are
// the K largest logits with ties to the lower index, i.e. the K largest
// 64-bit keys (ordered float bits << 32 | ~index).  NaN logits get key 0 and
// are never sampled.  r comes from splitmix64(seed, counter), since the
// reference's Math.random is unseeded.
//
// 1. k_sample_cand: CTA per 2048 logits, bitonic sort of the keys in shared
//    memory, the chunk's K largest to the candidate list.
// 2. k_sample_pick: one CTA sorts the candidates (bitonic, shared memory),
//    then the reference's softmax and cumulative pick in double.  In a decode
//    graph it also advances the position and records the token, like the
//    greedy step end.
#include "pb_internal.cuh"

constexpr int SP_CHUNK = 2048;
constexpr int SP_THREADS = 1024;
constexpr int SP_MAX_K = 256;

__host__ __device__ __forceinline__ uint64_t sp_splitmix(uint64_t seed, uint64_t counter) {
  uint64_t z = seed + (counter + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// uniform double in [0, 1) with 53 random bits
__host__ __device__ __forceinline__ double sp_uniform(uint64_t seed, uint64_t counter) {
  return (double)(sp_splitmix(seed, counter) >> 11) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ uint64_t sp_key(float v, int idx) {
  const uint32_t b = __float_as_uint(v);
  if ((b & 0x7fffffffu) > 0x7f800000u) return 0ull;  // NaN
  const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)o << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)idx);
}

// Descending bitonic sort of n (a power of two) keys in shared memory.
__device__ void sp_sort_desc(uint64_t* keys, int n) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = keys[i], b = keys[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? a < b : a > b) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

__global__ void __launch_bounds__(SP_THREADS)
k_sample_cand(const float* __restrict__ logits, int V, int K, uint64_t* __restrict__ cand) {
  __shared__ uint64_t keys[SP_CHUNK];
  pb_pdl_trigger();
  pb_pdl_wait();  // logits come from the head
  const int base = blockIdx.x * SP_CHUNK;
  for (int i = threadIdx.x; i < SP_CHUNK; i += blockDim.x) {
    const int j = base + i;
    keys[i] = j < V ? sp_key(logits[j], j) : 0ull;
  }
  __syncthreads();
  sp_sort_desc(keys, SP_CHUNK);
  for (int i = threadIdx.x; i < K; i += blockDim.x) cand[(size_t)blockIdx.x * K + i] = keys[i];
}

// n_cand = chunks * K candidates; n2 = the next power of two.  The counter is
// ctr_dev[0] when given (then incremented), else `counter`.  With pos_dev the
// kernel ends a decode step: token to tok_dev[0] and hist[pos + 1], position
// advanced, the greedy argmax key cleared.
__global__ void __launch_bounds__(SP_THREADS)
k_sample_pick(const float* __restrict__ logits, int V, int K, double temperature, const uint64_t* __restrict__ cand,
              int n_cand, int n2, uint64_t seed, uint64_t counter, uint64_t* __restrict__ ctr_dev,
              int* __restrict__ tok_dev, int* __restrict__ pos_dev, int* __restrict__ hist, int hist_len,
              unsigned long long* __restrict__ key_reset) {
  extern __shared__ __align__(16) unsigned char sp_raw[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(sp_raw);  // [n2]
  __shared__ double ev[SP_MAX_K];
  __shared__ int sidx[SP_MAX_K];
  __shared__ double ssum;
  __shared__ int scount;
  pb_pdl_trigger();
  pb_pdl_wait();
  for (int i = threadIdx.x; i < n2; i += blockDim.x) keys[i] = i < n_cand ? cand[i] : 0ull;
  __syncthreads();
  sp_sort_desc(keys, n2);
  const int top = K < V ? K : V;  // topKItems = indexed.slice(0, topK)
  if (threadIdx.x == 0) {
    int c = 0;
    while (c < top && keys[c] != 0ull) ++c;
    scount = c;
  }
  __syncthreads();
  const int count = scount;
  if ((int)threadIdx.x < count) {
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)(keys[threadIdx.x] & 0xFFFFFFFFull));
    sidx[threadIdx.x] = idx;
    ev[threadIdx.x] = __ddiv_rn((double)logits[idx], temperature);  // v = logits[i] / temperature
  }
  __syncthreads();
  double vmax = count > 0 ? ev[0] : 0.0;
  __syncthreads();
  if ((int)threadIdx.x < count) ev[threadIdx.x] = exp(__dsub_rn(ev[threadIdx.x], vmax));  // Math.exp(v - maxV)
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < count; ++i) s = __dadd_rn(s, ev[i]);  // sum += e, in order
    ssum = s;
  }
  __syncthreads();
  if ((int)threadIdx.x < count) ev[threadIdx.x] = __ddiv_rn(ev[threadIdx.x], ssum);  // p / sum
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t ctr = ctr_dev ? *ctr_dev : counter;
    const double r = sp_uniform(seed, ctr);
    int tok = count > 0 ? sidx[0] : 0;
    double cum = 0.0;
    for (int i = 0; i < count; ++i) {
      cum = __dadd_rn(cum, ev[i]);
      if (r <= cum) {
        tok = sidx[i];
        break;
      }
    }
    if (ctr_dev) *ctr_dev = ctr + 1;
    tok_dev[0] = tok;
    if (pos_dev) {
      const int p = *pos_dev;
      if (hist && p + 1 >= 0 && p + 1 < hist_len) hist[p + 1] = tok;
      *pos_dev = p + 1;
    }
    if (key_reset) *key_reset = 0ull;
  }
}

static int sp_chunks(int V) { return (V + SP_CHUNK - 1) / SP_CHUNK; }
static int sp_pow2(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// Candidate keys a sampling launch over V logits needs (u64 count).
size_t pb_sample_cand_count(int V, int K) { return (size_t)sp_chunks(V) * (K < V ? K : V); }

int pb_launch_sample(pb_ctx* ctx, const float* logits, int V, int K, double temperature, uint64_t seed,
                     uint64_t counter, uint64_t* ctr_dev, uint64_t* cand, int* tok_dev, int* pos_dev, int* hist,
                     int hist_len, unsigned long long* key_reset) {
  if (V <= 0 || K <= 0 || K > SP_MAX_K || !(temperature > 0.0))
    return pb_set_error(ctx, PB_ERR_ARG, "sampling needs V > 0, 0 < topK <= %d and temperature > 0", SP_MAX_K);
  const int chunks = sp_chunks(V), kc = K < V ? K : V;
  const int n_cand = chunks * kc, n2 = sp_pow2(n_cand);
  if ((size_t)n2 * 8 > 200 * 1024)
    return pb_set_error(ctx, PB_ERR_ARG, "sampling: %d candidates exceed the selection kernel", n_cand);
  PB_TRY(pb_launch(ctx, "k_sample_cand", true, k_sample_cand, dim3(chunks), dim3(SP_THREADS), 0, logits, V, kc, cand));
  return pb_launch(ctx, "k_sample_pick", true, k_sample_pick, dim3(1), dim3(SP_THREADS), (size_t)n2 * 8, logits, V, K,
                   temperature, (const uint64_t*)cand, n_cand, n2, seed, counter, ctr_dev, tok_dev, pos_dev, hist,
                   hist_len, key_reset);
}

extern "C" double pb_sample_uniform(uint64_t seed, uint64_t counter) { return sp_uniform(seed, counter); }

extern "C" int pb_sample_topk(pb_ctx* ctx, const float* logits_dev, int V, int top_k, double temperature, uint64_t seed,
                              uint64_t counter, int* token_dev) {
  if (!ctx || !logits_dev || !token_dev) return PB_ERR_ARG;
  if (V > 0 && top_k > 0 && top_k <= SP_MAX_K) PB_TRY(pb_ensure_scratch(ctx, pb_sample_cand_count(V, top_k) * 8));
  return pb_launch_sample(ctx, logits_dev, V, top_k, temperature, seed, counter, nullptr, (uint64_t*)ctx->scratch,
                          token_dev, nullptr, nullptr, 0, nullptr);
}


// Early-exit confidence (llama-streaming.js:695-725 _checkEarlyExit): the 8
// largest logits (ties to the lower index), sumExp = sum_i exp(l_i - max) in
// order plus max(0, V - 8) * exp(-20) for the tail, topProb = exp(0) / sumExp.
__global__ void __launch_bounds__(SP_THREADS)
k_exit_prob(const float* __restrict__ logits, int V, const uint64_t* __restrict__ cand, int n_cand, int n2,
            double* __restrict__ prob) {
  extern __shared__ __align__(16) unsigned char sp_raw[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(sp_raw);
  pb_pdl_trigger();
  pb_pdl_wait();
  for (int i = threadIdx.x; i < n2; i += blockDim.x) keys[i] = i < n_cand ? cand[i] : 0ull;
  __syncthreads();
  sp_sort_desc(keys, n2);
  if (threadIdx.x == 0) {
    const int top = V < 8 ? V : 8;
    double s = 0.0, mx = 0.0;
    for (int i = 0; i < top && keys[i] != 0ull; ++i) {
      const double v = (double)logits[(int)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull))];
      if (i == 0) mx = v;
      s = __dadd_rn(s, exp(__dsub_rn(v, mx)));
    }
    const int tail = V - 8 > 0 ? V - 8 : 0;
    s = __dadd_rn(s, __dmul_rn((double)tail, exp(-20.0)));
    *prob = __ddiv_rn(exp(0.0), s);
  }
}

int pb_launch_exit_prob(pb_ctx* ctx, const float* logits, int V, uint64_t* cand, double* prob_dev) {
  const int chunks = sp_chunks(V), kc = V < 8 ? V : 8;
  const int n_cand = chunks * kc, n2 = sp_pow2(n_cand);
  if ((size_t)n2 * 8 > 200 * 1024) return pb_set_error(ctx, PB_ERR_ARG, "early exit: vocabulary too large");
  PB_TRY(pb_launch(ctx, "k_sample_cand", true, k_sample_cand, dim3(chunks), dim3(SP_THREADS), 0, logits, V, kc, cand));
  return pb_launch(ctx, "k_exit_prob", true, k_exit_prob, dim3(1), dim3(SP_THREADS), (size_t)n2 * 8, logits, V,
                   (const uint64_t*)cand, n_cand, n2, prob_dev);
}

int pb_setup_sample_kernels(void) {
  cudaError_t e = cudaFuncSetAttribute(k_sample_pick, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_exit_prob, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  return e == cudaSuccess ? PB_OK : PB_ERR_CUDA;
}
