// pb_core.cu - context, device memory, errors, synthetic inputs, quantizers,
// GGUF decode and the device layout of quantized matrices.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <thread>

#include "pb_internal.cuh"
#include "pb_synth.h"

// ============================================================================
// errors and waits
// ============================================================================

int pb_set_error(pb_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return code;
}

int pb_cuda_error(pb_ctx* ctx, cudaError_t e, const char* what) {
  int code = (e == cudaErrorMemoryAllocation) ? PB_ERR_OOM : PB_ERR_CUDA;
  return pb_set_error(ctx, code, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int pb_check_launch(pb_ctx* ctx, const char* what) {
  ctx->launches++;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, what);
  return PB_OK;
}

// Poll the stream until it drains or the deadline passes (the reference's
// worker waits are bounded the same way, thread-pool.js:230-240).
int pb_wait(pb_ctx* ctx) {
  auto t0 = std::chrono::steady_clock::now();
  int spins = 0;
  for (;;) {
    cudaError_t e = cudaStreamQuery(ctx->stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return pb_cuda_error(ctx, e, "stream");
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms > ctx->timeout_ms)
      return pb_set_error(ctx, PB_ERR_TIMEOUT, "device work did not finish within %d ms", ctx->timeout_ms);
    if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  int code = 0;
  cudaError_t e = cudaMemcpy(&code, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, "read device error word");
  if (code != 0)
    return pb_set_error(ctx, PB_ERR_DEVICE, "a kernel raised device error %d (%s)", code,
                        code == PB_DEVERR_BOUNDS ? "index out of bounds"
                        : code == PB_DEVERR_WAIT ? "bounded wait expired"
                        : code == PB_DEVERR_TOKEN ? "token id out of range" : "unknown");
  return PB_OK;
}

int pb_ensure_gemm_scratch(pb_ctx* ctx, size_t bytes) {
  if (ctx->gemm_scratch_bytes >= bytes) return PB_OK;
  if (ctx->gemm_scratch) {
    PB_TRY(pb_wait(ctx));
    cudaFree(ctx->gemm_scratch);
    ctx->gemm_scratch = nullptr;
    ctx->gemm_scratch_bytes = 0;
  }
  PB_TRY_CUDA(ctx, cudaMalloc(&ctx->gemm_scratch, bytes));
  ctx->gemm_scratch_bytes = bytes;
  return PB_OK;
}

int pb_ensure_scratch(pb_ctx* ctx, size_t bytes) {
  if (ctx->scratch_bytes >= bytes) return PB_OK;
  if (ctx->scratch) {
    PB_TRY(pb_wait(ctx));
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  size_t sz = bytes < ((size_t)1 << 20) ? ((size_t)1 << 20) : bytes;
  PB_TRY_CUDA(ctx, cudaMalloc(&ctx->scratch, sz));
  ctx->scratch_bytes = sz;
  return PB_OK;
}

// ============================================================================
// context
// ============================================================================

extern "C" int pb_abi_version(void) { return PB_ABI_VERSION; }

extern "C" int pb_init(int device, pb_ctx** out) {
  if (!out) return PB_ERR_ARG;
  *out = nullptr;
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess || ndev == 0) return PB_ERR_CUDA;
  if (device < 0 || device >= ndev) return PB_ERR_ARG;
  pb_ctx* ctx = new pb_ctx();
  ctx->device = device;
  e = cudaSetDevice(device);
  if (e != cudaSuccess) { delete ctx; return PB_ERR_CUDA; }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) { delete ctx; return PB_ERR_CUDA; }
  if (prop.major != 10) {  // sm_100a code only
    delete ctx;
    return PB_ERR_STATE;
  }
  ctx->sm_count = prop.multiProcessorCount;
  // tuning override: matrix rows from which the fast mode takes the int8 tensor-core matvec
  if (const char* ev = getenv("PB_MVI_MIN_ROWS")) ctx->mvi_min_rows = atoi(ev);
  if (const char* ev = getenv("PB_MVT")) ctx->mvt = ev[0] == '1';  // tuning override: the tcgen05 matvec on
  if (const char* ev = getenv("PB_FUSE_ATTN")) ctx->fuse_attn = ev[0] == '1';  // tuning override: fused decode
  const char* nopdl = getenv("PB_NO_PDL");  // programmatic dependent launch off (debugging aid)
  ctx->pdl = !(nopdl && nopdl[0] == '1');

  ctx->l2_bytes = prop.l2CacheSize;
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) { delete ctx; return PB_ERR_CUDA; }
  if (cudaMalloc(&ctx->d_err, sizeof(int)) != cudaSuccess) { delete ctx; return PB_ERR_OOM; }
  cudaMemset(ctx->d_err, 0, sizeof(int));
  cudaDeviceSynchronize();
  if (pb_setup_q4_kernels() != PB_OK || pb_setup_ops_kernels() != PB_OK || pb_setup_gemm_kernels() != PB_OK ||
      pb_setup_mvi_kernels() != PB_OK || pb_setup_mvt_kernels() != PB_OK ||
      pb_setup_sample_kernels() != PB_OK ||
      pb_setup_noalloc(ctx) != PB_OK) {
    pb_shutdown(ctx);
    return PB_ERR_CUDA;
  }
  // Self-test of the Q4_0 kernel, as wasm-q4.js:673-704 does at init.
  const int K = 32, N = 2;
  float x[K];
  for (int i = 0; i < K; ++i) x[i] = 1.0f;
  uint8_t raw[36] = {0};
  raw[0] = 0x00; raw[1] = 0x3C;
  for (int j = 2; j < 18; ++j) raw[j] = 0x99;
  raw[18] = 0x00; raw[19] = 0x40;
  for (int j = 20; j < 36; ++j) raw[j] = 0xAA;
  float y[2] = {0, 0};
  int rc = pb_q4_0_matvec(ctx, x, raw, N, K, y);
  if (rc != PB_OK || y[0] != 32.0f || y[1] != 128.0f) {
    fprintf(stderr, "purebee_b200: Q4_0 self-test failed (rc=%d, got [%g, %g], want [32, 128])\n", rc, y[0], y[1]);
    pb_shutdown(ctx);
    return rc != PB_OK ? rc : PB_ERR_STATE;
  }
  *out = ctx;
  return PB_OK;
}

extern "C" int pb_shutdown(pb_ctx* ctx) {
  if (!ctx) return PB_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->gemm_scratch) cudaFree(ctx->gemm_scratch);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return PB_OK;
}

extern "C" const char* pb_last_error(const pb_ctx* ctx) { return ctx ? ctx->err.c_str() : "no context"; }

extern "C" int pb_set_matvec_mode(pb_ctx* ctx, int mode) {
  if (!ctx || (mode != PB_MATVEC_FAST && mode != PB_MATVEC_EXACT)) return PB_ERR_ARG;
  ctx->matvec_mode = mode;
  return PB_OK;
}

extern "C" int pb_matvec_mode(const pb_ctx* ctx) { return ctx ? ctx->matvec_mode : -1; }

extern "C" int pb_set_mvi_min_rows(pb_ctx* ctx, int rows) {
  if (!ctx || rows < 0) return PB_ERR_ARG;
  ctx->mvi_min_rows = rows;
  return PB_OK;
}

extern "C" int pb_set_fuse_attn(pb_ctx* ctx, int on) {
  if (!ctx || (on != 0 && on != 1)) return PB_ERR_ARG;
  ctx->fuse_attn = on == 1;
  return PB_OK;
}

extern "C" int pb_set_mvt(pb_ctx* ctx, int on) {
  if (!ctx || (on != 0 && on != 1)) return PB_ERR_ARG;
  ctx->mvt = on == 1;
  return PB_OK;
}

extern "C" int pb_set_timeout_ms(pb_ctx* ctx, int timeout_ms) {
  if (!ctx || timeout_ms <= 0) return PB_ERR_ARG;
  ctx->timeout_ms = timeout_ms;
  return PB_OK;
}

extern "C" int pb_sync(pb_ctx* ctx) {
  if (!ctx) return PB_ERR_ARG;
  return pb_wait(ctx);
}

extern "C" void* pb_stream(pb_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

extern "C" int pb_device_error(pb_ctx* ctx, int* code_out) {
  if (!ctx || !code_out) return PB_ERR_ARG;
  PB_TRY_CUDA(ctx, cudaMemcpy(code_out, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  return PB_OK;
}

extern "C" int64_t pb_launch_count(pb_ctx* ctx) { return ctx ? ctx->launches : 0; }

// ============================================================================
// capture / replay
// ============================================================================

struct pb_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

extern "C" int pb_capture_begin(pb_ctx* ctx) {
  if (!ctx) return PB_ERR_ARG;
  // thread-local mode: an unrelated thread's CUDA calls are not disturbed, and
  // a blocking call on this thread fails instead of being recorded
  PB_TRY_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  return PB_OK;
}

extern "C" int pb_capture_end(pb_ctx* ctx, pb_graph** out) {
  if (!ctx || !out) return PB_ERR_ARG;
  *out = nullptr;
  cudaGraph_t g = nullptr;
  cudaError_t ec = cudaStreamEndCapture(ctx->stream, &g);
  if (ec != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();  // the failed recording must not surface in a later launch check
    return pb_cuda_error(ctx, ec, "recording was invalidated (a blocking call was made while recording)");
  }
  pb_graph* pg = new pb_graph();
  pg->graph = g;
  cudaError_t e = cudaGraphInstantiate(&pg->exec, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    delete pg;
    return pb_cuda_error(ctx, e, "cudaGraphInstantiate");
  }
  *out = pg;
  return PB_OK;
}

extern "C" int pb_graph_launch(pb_ctx* ctx, pb_graph* g) {
  if (!ctx || !g) return PB_ERR_ARG;
  PB_TRY_CUDA(ctx, cudaGraphLaunch(g->exec, ctx->stream));
  return PB_OK;
}

extern "C" int pb_graph_free(pb_graph* g) {
  if (!g) return PB_OK;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
  return PB_OK;
}

// ============================================================================
// device memory
// ============================================================================

extern "C" int pb_malloc(pb_ctx* ctx, size_t bytes, void** dptr) {
  if (!ctx || !dptr) return PB_ERR_ARG;
  *dptr = nullptr;
  if (bytes == 0) bytes = 16;
  PB_TRY_CUDA(ctx, cudaMalloc(dptr, bytes));
  return PB_OK;
}

extern "C" int pb_free(pb_ctx* ctx, void* dptr) {
  if (!ctx) return PB_ERR_ARG;
  if (!dptr) return PB_OK;
  PB_TRY(pb_wait(ctx));
  PB_TRY_CUDA(ctx, cudaFree(dptr));
  return PB_OK;
}

extern "C" int pb_upload(pb_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || (!dst && bytes) || (!src && bytes)) return PB_ERR_ARG;
  if (!bytes) return PB_OK;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return pb_wait(ctx);
}

extern "C" int pb_download(pb_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || (!dst && bytes) || (!src && bytes)) return PB_ERR_ARG;
  if (!bytes) return PB_OK;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return pb_wait(ctx);
}

extern "C" int pb_memset(pb_ctx* ctx, void* dst, int value, size_t bytes) {
  if (!ctx || (!dst && bytes)) return PB_ERR_ARG;
  PB_TRY_CUDA(ctx, cudaMemsetAsync(dst, value, bytes, ctx->stream));
  return PB_OK;
}

extern "C" int pb_memcpy_d2d(pb_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || (!dst && bytes) || (!src && bytes)) return PB_ERR_ARG;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
  return PB_OK;
}

// ============================================================================
// synthetic inputs (pb_synth.h, identical bits to the CPU oracle)
// ============================================================================

__global__ void k_synth(float* out, int64_t n, uint64_t key, double stdev, int act) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    double v = pb_normal(key, (uint64_t)i);
    out[i] = act ? (float)v : (float)__dmul_rn(stdev, v);
  }
}

static int synth_launch(pb_ctx* ctx, float* out, int64_t n, uint64_t seed, uint64_t tid, double sd, int act) {
  if (!ctx || (!out && n) || n < 0) return PB_ERR_ARG;
  if (!n) return PB_OK;
  int64_t blocks = (n + 255) / 256;
  int grid = (int)(blocks < (int64_t)ctx->sm_count * 16 ? blocks : (int64_t)ctx->sm_count * 16);
  k_synth<<<grid, 256, 0, ctx->stream>>>(out, n, pb_stream_key(seed, tid), sd, act);
  PB_LAUNCHED(ctx, "k_synth");
  return PB_OK;
}

extern "C" int pb_synth_weights(pb_ctx* ctx, float* out, int64_t n, uint64_t seed, uint64_t tensor_id, double sd) {
  return synth_launch(ctx, out, n, seed, tensor_id, sd, 0);
}
extern "C" int pb_synth_activation(pb_ctx* ctx, float* out, int64_t n, uint64_t seed, uint64_t stream) {
  return synth_launch(ctx, out, n, seed, stream, 1.0, 1);
}
extern "C" int pb_synth_tokens(int* out, int n, uint64_t seed, int lo, int hi) {
  if ((!out && n) || hi <= lo) return PB_ERR_ARG;
  for (int i = 0; i < n; ++i) out[i] = pb_synth_token(seed, (uint64_t)i, lo, hi);
  return PB_OK;
}

// ============================================================================
// quantize.js format (a): quantize_q8 / quantize_q4 / dequantize (quantize.js:79-208)
// One warp per 32-value block; JS doubles and Math.round semantics.
// ============================================================================

// Math.round: nearest integer, ties toward +infinity.
__device__ __forceinline__ double js_round_d(double v) {
  double f = floor(v);
  return (__dsub_rn(v, f) >= 0.5) ? __dadd_rn(f, 1.0) : f;
}

__global__ void k_quantize_qa(const float* __restrict__ x, int64_t n, float* __restrict__ scales,
                              int8_t* __restrict__ q8, uint8_t* __restrict__ q4, int bits4) {
  int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  int64_t nblocks = (n + 31) / 32;
  if (b >= nblocks) return;
  int64_t i = b * 32 + lane;
  bool in = i < n;
  double v = in ? (double)x[i] : 0.0;
  double a = fabs(v);
  // maxAbs: JS loop `if (abs > maxAbs)` from 0 (NaN never wins)
  double m = (a > 0.0) ? a : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    double t = __shfl_xor_sync(0xffffffffu, m, o);
    m = t > m ? t : m;
  }
  double lim = bits4 ? 7.0 : 127.0;
  double scale = __ddiv_rn(m, lim);
  if (lane == 0) scales[b] = (float)scale;
  if (!bits4) {
    int8_t qv = 0;
    if (scale > 0.0 && in) {
      double inv = __ddiv_rn(lim, m);
      double r = js_round_d(__dmul_rn(v, inv));
      if (r == r && !isinf(r)) {  // ToInt8 (values are within [-127, 127] here)
        double t = fmod(trunc(r), 256.0);
        if (t < 0) t += 256.0;
        int iv = (int)t;
        qv = (int8_t)(iv >= 128 ? iv - 256 : iv);
      }
    }
    if (in || scale == 0.0 || i < nblocks * 32) q8[i] = qv;
  } else {
    int nib = 0;
    bool write = false;
    if (scale > 0.0 && in) {
      double inv = __ddiv_rn(lim, m);
      double r = js_round_d(__dmul_rn(v, inv));
      if (r == r) { r = r > 7.0 ? 7.0 : r; r = r < -8.0 ? -8.0 : r; }
      double u = __dadd_rn(r, 8.0);
      if (u == u && !isinf(u)) {
        double t = fmod(trunc(u), 16.0);
        if (t < 0) t += 16.0;
        nib = (int)t;
      }
      write = true;
    }
    // pair lanes (even, odd) into one byte; unwritten nibbles stay zero
    int nib_odd = __shfl_down_sync(0xffffffffu, nib, 1);
    int w_odd = __shfl_down_sync(0xffffffffu, (int)write, 1);
    if ((lane & 1) == 0 && i < nblocks * 32) {
      uint8_t byte = (uint8_t)((write ? (nib & 0x0F) : 0) | ((w_odd ? (nib_odd & 0x0F) : 0) << 4));
      q4[i / 2] = byte;
    }
  }
}

static int quantize_qa(pb_ctx* ctx, const float* x, int64_t n, float* scales, void* q, int bits4) {
  if (!ctx || n <= 0 || !x || !scales || !q) return PB_ERR_ARG;
  int64_t nblocks = (n + 31) / 32;
  int grid = pb_cdiv(nblocks, 8);
  k_quantize_qa<<<grid, 256, 0, ctx->stream>>>(x, n, scales, (int8_t*)q, (uint8_t*)q, bits4);
  PB_LAUNCHED(ctx, "k_quantize_qa");
  return PB_OK;
}

extern "C" int pb_quantize_q8a(pb_ctx* ctx, const float* x, int64_t n, float* scales, int8_t* q) {
  return quantize_qa(ctx, x, n, scales, q, 0);
}
extern "C" int pb_quantize_q4a(pb_ctx* ctx, const float* x, int64_t n, float* scales, uint8_t* q) {
  return quantize_qa(ctx, x, n, scales, q, 1);
}

__global__ void k_dequantize_qa(const float* __restrict__ scales, const void* __restrict__ q, int64_t n,
                                float* __restrict__ out, int bits4) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double s = scales[i / 32];
  double v;
  if (!bits4) {
    v = (double)((const int8_t*)q)[i];
  } else {
    uint8_t byte = ((const uint8_t*)q)[i / 2];
    int nib = (i & 1) ? ((byte >> 4) & 0x0F) : (byte & 0x0F);
    v = (double)(nib - 8);
  }
  out[i] = (float)__dmul_rn(v, s);
}

static int dequantize_qa(pb_ctx* ctx, const float* scales, const void* q, int64_t n, float* out, int bits4) {
  if (!ctx || n <= 0 || !scales || !q || !out) return PB_ERR_ARG;
  k_dequantize_qa<<<pb_cdiv(n, 256), 256, 0, ctx->stream>>>(scales, q, n, out, bits4);
  PB_LAUNCHED(ctx, "k_dequantize_qa");
  return PB_OK;
}
extern "C" int pb_dequantize_q8a(pb_ctx* ctx, const float* s, const int8_t* q, int64_t n, float* out) {
  return dequantize_qa(ctx, s, q, n, out, 0);
}
extern "C" int pb_dequantize_q4a(pb_ctx* ctx, const float* s, const uint8_t* q, int64_t n, float* out) {
  return dequantize_qa(ctx, s, q, n, out, 1);
}

// ============================================================================
// GGUF decode (gguf.js:219-315) and the build's GGUF encoders
// ============================================================================

__global__ void k_gguf_dequant(int type, const uint8_t* __restrict__ raw, int64_t n, float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (type == PB_TYPE_F32) {
    out[i] = ((const float*)raw)[i];
  } else if (type == PB_TYPE_F16) {
    out[i] = pb_f16_exact(((const uint16_t*)raw)[i]);
  } else {
    int64_t b = i / 32;
    int j = (int)(i % 32);
    if (type == PB_TYPE_Q4_0) {
      const uint8_t* blk = raw + b * 18;
      float d = pb_f16_exact((uint16_t)(blk[0] | (blk[1] << 8)));
      int byte = blk[2 + (j & 15)];
      int nib = j < 16 ? (byte & 15) : (byte >> 4);
      out[i] = __fmul_rn((float)(nib - 8), d);  // exact: 4-bit x 11-bit significands
    } else if (type == PB_TYPE_Q4_1) {
      const uint8_t* blk = raw + b * 20;
      double d = pb_f16_exact((uint16_t)(blk[0] | (blk[1] << 8)));
      double m = pb_f16_exact((uint16_t)(blk[2] | (blk[3] << 8)));
      int byte = blk[4 + (j & 15)];
      int nib = j < 16 ? (byte & 15) : (byte >> 4);
      out[i] = (float)__dadd_rn(__dmul_rn((double)nib, d), m);
    } else if (type == PB_TYPE_Q8_0) {
      const uint8_t* blk = raw + b * 34;
      float d = pb_f16_exact((uint16_t)(blk[0] | (blk[1] << 8)));
      out[i] = __fmul_rn((float)(int8_t)blk[2 + j], d);  // exact: 8-bit x 11-bit
    } else {  // Q6_K (gguf.js:317-355): [ql 128][qh 64][int8 scales 16][f16 d]
      const int64_t bk = i / 256;
      const int e = (int)(i % 256), half = e >> 7, r = e & 127, part = r >> 5, l = r & 31;
      const uint8_t* blk = raw + bk * 210;
      const uint8_t ql = blk[half * 64 + l + (part & 1) * 32];  // parts 0, 2 read byte l; 1, 3 byte l + 32
      const uint8_t qh = blk[128 + half * 32 + l];
      const int lo = (part < 2) ? (ql & 15) : (ql >> 4);
      const int q = (lo | (((qh >> (2 * part)) & 3) << 4)) - 32;
      const int sc = (int8_t)blk[192 + half * 8 + (l >> 4) + 2 * part];
      const float d = pb_f16_exact((uint16_t)(blk[208] | (blk[209] << 8)));
      // d * sc is exact in f32 (11 x 8 significant bits), so one rounding of
      // the exact product, like the reference's double product stored to f32
      out[i] = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
  }
}

extern "C" int pb_gguf_dequant(pb_ctx* ctx, int type, const void* raw, int64_t n, float* out) {
  if (!ctx || !raw || !out || n <= 0) return PB_ERR_ARG;
  if (type != PB_TYPE_F32 && type != PB_TYPE_F16 && type != PB_TYPE_Q4_0 && type != PB_TYPE_Q4_1 &&
      type != PB_TYPE_Q8_0 && type != PB_TYPE_Q6_K)
    return pb_set_error(ctx, PB_ERR_ARG, "unsupported tensor type %d", type);
  if (type != PB_TYPE_F32 && type != PB_TYPE_F16 && type != PB_TYPE_Q6_K && n % 32)
    return pb_set_error(ctx, PB_ERR_ARG, "quantized tensors need n %% 32 == 0");
  k_gguf_dequant<<<pb_cdiv(n, 256), 256, 0, ctx->stream>>>(type, (const uint8_t*)raw, n, out);
  PB_LAUNCHED(ctx, "k_gguf_dequant");
  return PB_OK;
}

// GGUF Q4_0 / Q8_0 encoders, one warp per block.  The definition: Q4_0 takes
// the signed element of largest magnitude m, d = m / -8, q = min(15,
// trunc(x/d + 8.5)); Q8_0 takes d = amax / 127, q = round-half-away(x/d);
// d is stored as an IEEE half (round to nearest even).
__global__ void k_gguf_quantize(int type, const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (b >= nblocks) return;
  float v = x[b * 32 + lane];
  float a = fabsf(v);
  if (type == PB_TYPE_Q4_0) {
    // signed value of the first element with the largest magnitude
    float am = a;
    int idx = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ta = __shfl_xor_sync(0xffffffffu, am, o);
      int ti = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ta > am || (ta == am && ti < idx)) { am = ta; idx = ti; }
    }
    // the oracle's strict `>` scan keeps the first index among equal maxima,
    // and only replaces on a strictly larger magnitude, starting from 0
    float mx = __shfl_sync(0xffffffffu, v, idx);
    if (!(am > 0.0f)) mx = 0.0f;
    float d = __fdiv_rn(mx, -8.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    float t = __fadd_rn(__fmul_rn(v, id), 8.5f);
    int q = (t != t) ? 0 : (int)fminf(fmaxf(t, 0.0f), 16.0f);
    q = q > 15 ? 15 : q;
    // element j (< 16) -> low nibble of byte j; element j+16 -> high nibble
    int qhi = __shfl_down_sync(0xffffffffu, q, 16);
    // byte j = element j (low nibble) | element j+16 (high nibble); pairs of
    // bytes go out as aligned 16-bit stores (a block starts on an even address)
    uint32_t byte = (uint32_t)(q | (qhi << 4)) & 0xFFu;
    uint32_t nxt = __shfl_down_sync(0xffffffffu, byte, 1);
    uint16_t* o16 = reinterpret_cast<uint16_t*>(out + b * 18);
    if (lane < 16 && (lane & 1) == 0) o16[1 + lane / 2] = (uint16_t)(byte | (nxt << 8));
    if (lane == 16) o16[0] = __half_as_ushort(__float2half_rn(d));
  } else {
    float am = a;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    float d = __fdiv_rn(am, 127.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    float t = __fmul_rn(v, id);
    float r = (t != t) ? 0.0f : roundf(t);
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    uint32_t byte = (uint32_t)(uint8_t)(int8_t)(int)r;
    uint32_t nxt = __shfl_down_sync(0xffffffffu, byte, 1);
    uint16_t* o16 = reinterpret_cast<uint16_t*>(out + b * 34);
    if ((lane & 1) == 0) o16[1 + lane / 2] = (uint16_t)(byte | (nxt << 8));
    if (lane == 1) o16[0] = __half_as_ushort(__float2half_rn(d));
  }
}

extern "C" int pb_gguf_quantize(pb_ctx* ctx, int type, const float* x, int64_t n, void* raw) {
  if (!ctx || !x || !raw || n <= 0 || n % 32) return PB_ERR_ARG;
  if (type != PB_TYPE_Q4_0 && type != PB_TYPE_Q8_0)
    return pb_set_error(ctx, PB_ERR_ARG, "GGUF encode supports Q4_0 and Q8_0 only");
  int64_t nb = n / 32;
  k_gguf_quantize<<<pb_cdiv(nb, 8), 256, 0, ctx->stream>>>(type, x, nb, (uint8_t*)raw);
  PB_LAUNCHED(ctx, "k_gguf_quantize");
  return PB_OK;
}

// ============================================================================
// device layout of quantized matrices (pb_qmat)
// ============================================================================

static int qbytes(int type) { return type == PB_TYPE_Q8_0 ? 32 : 16; }
static int gguf_block_bytes(int type) { return type == PB_TYPE_Q4_0 ? 18 : type == PB_TYPE_Q4_1 ? 20 : 34; }

int pb_qmat_alloc(pb_ctx* ctx, int type, int layout, int N, int K, pb_qmat** out) {
  if (!ctx || !out || N <= 0 || K <= 0 || K % 32) return pb_set_error(ctx, PB_ERR_ARG, "matrix shape %dx%d: K must be a multiple of 32", N, K);
  if (type != PB_TYPE_Q4_0 && type != PB_TYPE_Q4_1 && type != PB_TYPE_Q8_0)
    return pb_set_error(ctx, PB_ERR_ARG, "unsupported matrix type %d", type);
  pb_qmat* m = new pb_qmat();
  m->type = type;
  m->layout = layout;
  m->N = N;
  m->K = K;
  m->N_pad = (N + 31) / 32 * 32;
  m->nb = K / 32;
  size_t nblk = (size_t)m->N_pad * m->nb;
  cudaError_t e = cudaMalloc(&m->qs, nblk * qbytes(type));
  if (e == cudaSuccess) e = cudaMalloc(&m->d, nblk * 2);
  if (e == cudaSuccess && type == PB_TYPE_Q4_1) e = cudaMalloc(&m->m, nblk * 2);
  if (e != cudaSuccess) {
    cudaFree(m->qs); cudaFree(m->d); cudaFree(m->m);
    delete m;
    return pb_cuda_error(ctx, e, "pb_qmat allocation");
  }
  // padded rows: zero scales and zero payload
  cudaMemsetAsync(m->qs, 0, nblk * qbytes(type), ctx->stream);
  cudaMemsetAsync(m->d, 0, nblk * 2, ctx->stream);
  if (m->m) cudaMemsetAsync(m->m, 0, nblk * 2, ctx->stream);
  *out = m;
  return PB_OK;
}

// GGUF [N][nb][block] <-> the device layout; one thread per block.
__global__ void k_qmat_pack(int type, int layout, const uint8_t* __restrict__ src, int N, int nb,
                            uint8_t* __restrict__ qs, uint16_t* __restrict__ d, uint16_t* __restrict__ mn, int unpack) {
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = (int64_t)N * nb;
  if (t >= total) return;
  int n = (int)(t / nb), b = (int)(t % nb);
  int bb = type == PB_TYPE_Q4_0 ? 18 : type == PB_TYPE_Q4_1 ? 20 : 34;
  int hdr = type == PB_TYPE_Q4_1 ? 4 : 2;
  int pl = type == PB_TYPE_Q8_0 ? 32 : 16;
  uint8_t* g = (uint8_t*)src + t * bb;
  int64_t slot = pb_slot(layout, n, b, nb);
  uint8_t* p = qs + slot * pl;
  if (!unpack) {
    d[slot] = (uint16_t)(g[0] | (g[1] << 8));
    if (mn) mn[slot] = (uint16_t)(g[2] | (g[3] << 8));
    for (int i = 0; i < pl; ++i) p[i] = g[hdr + i];
  } else {
    uint16_t dv = d[slot];
    g[0] = (uint8_t)(dv & 0xff);
    g[1] = (uint8_t)(dv >> 8);
    if (mn) {
      uint16_t mv = mn[slot];
      g[2] = (uint8_t)(mv & 0xff);
      g[3] = (uint8_t)(mv >> 8);
    }
    for (int i = 0; i < pl; ++i) g[hdr + i] = p[i];
  }
}

int pb_qmat_pack_from_device(pb_ctx* ctx, pb_qmat* m, const void* gguf_dev) {
  int64_t total = (int64_t)m->N * m->nb;
  k_qmat_pack<<<pb_cdiv(total, 256), 256, 0, ctx->stream>>>(m->type, m->layout, (const uint8_t*)gguf_dev, m->N,
                                                            m->nb, m->qs, m->d, m->m, 0);
  PB_LAUNCHED(ctx, "k_qmat_pack");
  m->mma_ok = false;
  // matvec weights also get the tensor-core copy the fast matvec reads
  if (m->type == PB_TYPE_Q4_0 && m->layout == PB_LAYOUT_ROWS) return pb_qmat_build_mma(ctx, m);
  return PB_OK;
}

extern "C" int pb_qmat_from_device(pb_ctx* ctx, int type, const void* gguf_dev, int N, int K, pb_qmat** out) {
  if (!ctx || !gguf_dev || !out) return PB_ERR_ARG;
  const int layout = (type & PB_QMAT_TABLE) ? PB_LAYOUT_TILED8 : PB_LAYOUT_ROWS;
  type &= ~PB_QMAT_TABLE;
  PB_TRY(pb_qmat_alloc(ctx, type, layout, N, K, out));
  int rc = pb_qmat_pack_from_device(ctx, *out, gguf_dev);
  if (rc != PB_OK) { pb_qmat_free(ctx, *out); *out = nullptr; }
  return rc;
}

extern "C" int pb_qmat_upload(pb_ctx* ctx, int type, const void* gguf_host, int N, int K, pb_qmat** out) {
  if (!ctx || !gguf_host || !out) return PB_ERR_ARG;
  if (K % 32 || N <= 0) return pb_set_error(ctx, PB_ERR_ARG, "matrix shape %dx%d: K must be a multiple of 32", N, K);
  size_t bytes = (size_t)N * (K / 32) * gguf_block_bytes(type & ~PB_QMAT_TABLE);
  PB_TRY(pb_ensure_scratch(ctx, bytes));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(ctx->scratch, gguf_host, bytes, cudaMemcpyHostToDevice, ctx->stream));
  PB_TRY(pb_qmat_from_device(ctx, type, ctx->scratch, N, K, out));
  return pb_wait(ctx);
}

extern "C" int pb_qmat_download_gguf(pb_ctx* ctx, const pb_qmat* m, void* gguf_host) {
  if (!ctx || !m || !gguf_host) return PB_ERR_ARG;
  size_t bytes = (size_t)m->N * m->nb * gguf_block_bytes(m->type);
  PB_TRY(pb_ensure_scratch(ctx, bytes));
  int64_t total = (int64_t)m->N * m->nb;
  k_qmat_pack<<<pb_cdiv(total, 256), 256, 0, ctx->stream>>>(m->type, m->layout, (const uint8_t*)ctx->scratch, m->N,
                                                            m->nb, m->qs, m->d, m->m, 1);
  PB_LAUNCHED(ctx, "k_qmat_unpack");
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(gguf_host, ctx->scratch, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return pb_wait(ctx);
}

extern "C" int pb_qmat_free(pb_ctx* ctx, pb_qmat* m) {
  if (!m) return PB_OK;
  if (ctx) {
    int rc = pb_wait(ctx);
    if (rc != PB_OK) return rc;
  }
  cudaFree(m->qs);
  cudaFree(m->d);
  cudaFree(m->m);
  cudaFree(m->mq);
  cudaFree(m->md);
  cudaFree(m->tq);
  delete m;
  return PB_OK;
}

extern "C" int pb_qmat_info(const pb_qmat* m, int* type, int* N, int* K) {
  if (!m) return PB_ERR_ARG;
  if (type) *type = m->type;
  if (N) *N = m->N;
  if (K) *K = m->K;
  return PB_OK;
}
