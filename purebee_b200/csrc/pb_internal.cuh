// pb_internal.cuh - shared host/device internals of the sm_100a library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/purebee_cuda.h"

struct pb_ctx {
  int device = 0;
  int sm_count = 148;
  size_t l2_bytes = 0;
  cudaStream_t stream = nullptr;
  int timeout_ms = 10000;
  int* d_err = nullptr;         // device error word: 0 = ok
  int64_t launches = 0;
  std::string err;
  // scratch for one-shot host-buffer calls (grown on demand)
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
};

// Device layout of a quantized matrix.
//   qs: [N_pad/32 tiles][nb blocks][32 rows][QB bytes]  (QB = 16 for Q4, 32 for Q8)
//   d : [N_pad/32 tiles][nb blocks][32 rows] u16 scale (Q4_1: a second array m)
// A warp whose lanes are the 32 rows of a tile reads one block column with a
// single coalesced 512 B (Q4) / 1 KB (Q8) access.
struct pb_qmat {
  int type = 0;
  int N = 0, K = 0, N_pad = 0, nb = 0;
  uint8_t* qs = nullptr;
  uint16_t* d = nullptr;
  uint16_t* m = nullptr;  // Q4_1 min
};

// ---- host helpers ---------------------------------------------------------

int pb_set_error(pb_ctx* ctx, int code, const char* fmt, ...);
int pb_cuda_error(pb_ctx* ctx, cudaError_t e, const char* what);
int pb_wait(pb_ctx* ctx);  // bounded wait on the context stream
int pb_check_launch(pb_ctx* ctx, const char* what);
int pb_ensure_scratch(pb_ctx* ctx, size_t bytes);

#define PB_TRY_CUDA(ctx, expr)                               \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return pb_cuda_error(ctx, _e, #expr); \
  } while (0)

#define PB_TRY(expr)               \
  do {                             \
    int _rc = (expr);              \
    if (_rc != PB_OK) return _rc;  \
  } while (0)

#define PB_LAUNCHED(ctx, what) PB_TRY(pb_check_launch(ctx, what))

static inline int pb_cdiv(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// ---- device helpers -------------------------------------------------------

// gguf.js:55-70 full IEEE half decode (exact for every half, subnormals too).
__device__ __forceinline__ float pb_f16_exact(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}

// wasm-q4.js:88-109: exponent 0 -> +0, otherwise bits rebuilt without an
// inf/NaN case.
__device__ __forceinline__ float pb_f16_wasm(uint32_t bits) {
  uint32_t e = (bits >> 10) & 0x1f;
  uint32_t f = ((bits >> 15) << 31) | ((e + 112u) << 23) | ((bits & 0x3ffu) << 13);
  return e == 0 ? 0.0f : __uint_as_float(f);
}

// Record the first device-side error; the host reads it with pb_device_error.
__device__ __forceinline__ void pb_raise(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Device error codes (also reported as PB_ERR_DEVICE with this detail).
#define PB_DEVERR_BOUNDS 1
#define PB_DEVERR_WAIT 2
#define PB_DEVERR_TOKEN 3

// Ordered-key argmax: larger key = larger value, ties -> lower index.
// Values that are NaN or -inf never win (llama-streaming.js:899-909 uses a
// strict `>` from -Infinity and index 0).
__device__ __forceinline__ unsigned long long pb_argmax_key(float v, int idx) {
  if (!(v > -__int_as_float(0x7f800000))) return 0ull;  // NaN or -inf
  uint32_t b = __float_as_uint(v);
  uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int pb_argmax_index(unsigned long long key) {
  return key == 0ull ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

__device__ __forceinline__ double pb_warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float pb_warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide double sum with a fixed reduction tree: every block that sums
// the same values gets the same bits.  `red` needs blockDim.x/32 doubles.
__device__ __forceinline__ double pb_block_sum_d(double v, double* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = pb_warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  if (w == 0) {
    t = lane < nw ? red[lane] : 0.0;
    t = pb_warp_sum_d(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  t = red[0];
  return t;
}

// ---- launches shared between translation units ----------------------------

int pb_launch_matvec(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows,
                     const float* residual);
int pb_launch_head(pb_ctx* ctx, const pb_qmat* emb, const float* h, float* logits,
                   unsigned long long* argmax_key, int mode);
int pb_launch_argmax_finish(pb_ctx* ctx, const unsigned long long* key, int* idx);
int pb_qmat_alloc(pb_ctx* ctx, int type, int N, int K, pb_qmat** out);
int pb_qmat_pack_from_device(pb_ctx* ctx, pb_qmat* m, const void* gguf_dev);
int pb_setup_q4_kernels(void);
int pb_setup_ops_kernels(void);
