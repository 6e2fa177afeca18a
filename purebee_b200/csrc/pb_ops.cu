// pb_ops.cu - engine.js operators and the per-token Llama ops on the device.
//
// The reference evaluates these ops in JavaScript doubles and rounds to f32
// on every Float32Array store; the kernels below do the same with explicit
// *_rn double intrinsics (no contraction).  Products of two f32 values are
// exact in double, so a DFMA that adds such a product equals the reference's
// separate multiply and add.  Sums over many terms use a fixed tree instead of
// the reference's left-to-right loop; the double result can differ in its last
// bits, which changes the f32-rounded output only in rare ties (the parity
// tests bound it).
#include <math.h>
#include <stdlib.h>

#include <vector>

#include <mutex>

#include <cooperative_groups.h>

#include "pb_attn_fast.cuh"
#include "pb_internal.cuh"

// ============================================================================
// RMSNorm (engine.js:429-449)
// ============================================================================

// With out16 (the batched path's f16 GEMM operand) the row is scaled in f32
// by 1/rms and rounded to f16 once; otherwise the reference's double
// arithmetic in f32 out.
// One row per CTA.  CH: x is stored in column chunks of width xc, chunk c at
// x + c * gridDim.x * xc (the row-split batch's replicated residual); the
// output rows are row-major either way.
template <bool CH>
__global__ void k_rmsnorm_t(const float* __restrict__ x, int dim, const float* __restrict__ w, double eps,
                            float* __restrict__ out, __half* __restrict__ out16, int xc, int hl) {
  __shared__ double red[32];
  pb_pdl_trigger();
  pb_pdl_wait();  // x comes from the previous kernel
  const size_t row = blockIdx.x;
  const float* xr = x + row * (CH ? xc : dim);
  const size_t cs = (size_t)gridDim.x * xc;
  auto X = [&](int d) { return CH ? xr[(size_t)(d / xc) * cs + d % xc] : xr[d]; };
  // each thread's values d = t, t + blockDim, ... are loaded once, together,
  // and kept (up to RMS_KEEP of them; longer rows read again below)
  constexpr int RMS_KEEP = 8;  // a 2048-wide row at 256 threads
  const int nt = blockDim.x;
  float xv[RMS_KEEP];
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < RMS_KEEP; ++k) {
    const int d = threadIdx.x + k * nt;
    if (d < dim) xv[k] = X(d);
  }
#pragma unroll
  for (int k = 0; k < RMS_KEEP; ++k) {
    const int d = threadIdx.x + k * nt;
    if (d < dim) {
      const double v = (double)xv[k];
      ss = __fma_rn(v, v, ss);
    }
  }
  for (int d = threadIdx.x + RMS_KEEP * nt; d < dim; d += nt) {
    const double v = (double)X(d);
    ss = __fma_rn(v, v, ss);
  }
  ss = pb_block_sum_d(ss, red);
  double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)dim), eps));
  auto XV = [&](int k, int d) { return k < RMS_KEEP ? xv[k] : X(d); };
  const float inv = (float)(1.0 / rms);
#pragma unroll
  for (int k = 0; k < RMS_KEEP; ++k) {
    const int d = threadIdx.x + k * nt;
    if (d < dim) {
      if (out16 && hl) pb_store_hl(out16, pb_hl_index((size_t)row * 2 * dim, d), xv[k] * inv * w[d]);
      else if (out16) out16[row * dim + d] = __float2half_rn(xv[k] * inv * w[d]);
      else out[row * dim + d] = (float)__dmul_rn(__ddiv_rn((double)xv[k], rms), (double)w[d]);
    }
  }
  for (int d = threadIdx.x + RMS_KEEP * nt, k = RMS_KEEP; d < dim; d += nt, ++k) {
    const float xd = XV(k, d);
    if (out16 && hl) pb_store_hl(out16, pb_hl_index((size_t)row * 2 * dim, d), xd * inv * w[d]);
    else if (out16) out16[row * dim + d] = __float2half_rn(xd * inv * w[d]);
    else out[row * dim + d] = (float)__dmul_rn(__ddiv_rn((double)xd, rms), (double)w[d]);
  }
}

// The RMSNorm that ends the row split's fused residual exchange (decode
// steps): row `row` of x is stored in column chunks of width xc (chunk c at
// x + c * rows * xc); this rank's chunk is local, every peer's arrives in
// this rank's slots as {v0, e, v1, e} packets from the peer's add epilogue
// (pb_xsend_pair).  The row goes to shared memory first -- the peers' values
// also into the local chunks -- then the arithmetic is k_rmsnorm_t's, so the
// output has the same bits as the unfused exchange followed by the norm.
// The last CTA advances the exchange counter.  Every poll is bounded by the
// context timeout (PB_DEVERR_WAIT).
__global__ void k_rmsnorm_xrecv(float* __restrict__ x, int dim, const float* __restrict__ w, double eps,
                                float* __restrict__ out, __half* __restrict__ out16, int xc, int hl, pb_xrecv xr) {
  extern __shared__ float xrow[];
  __shared__ double red[32];
  pb_pdl_trigger();
  pb_pdl_wait();  // this rank's chunk (and the exchange counter) come from the kernels before
  const int row = blockIdx.x, rows = gridDim.x;
  const unsigned int e = *xr.epoch + 1u;
  const size_t half = e & 1u;
  const unsigned long long t0 = pb_globaltimer_ns();
  bool ok = true;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    const int c = d / xc, k = d - c * xc;
    float* xl = x + (size_t)c * rows * xc + (size_t)row * xc + k;
    if (c == xr.rank) {
      xrow[d] = *xl;
      continue;
    }
    const uint4* src = xr.mine + (half * xr.world + c) * xr.cap_units + (((size_t)row * xc + k) >> 1);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    for (uint32_t it = 0; ok; ++it) {
      asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                   : "l"(src)
                   : "memory");
      if (v.y == e && v.w == e) break;
      if ((it & 63) == 63 && pb_globaltimer_ns() - t0 > xr.limit_ns) {
        pb_raise(xr.err, PB_DEVERR_WAIT);
        ok = false;
      }
    }
    const float val = __uint_as_float((k & 1) ? v.z : v.x);
    xrow[d] = val;
    *xl = val;  // the local copy of the peer's chunk
  }
  __syncthreads();
  double ss = 0.0;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    const double v = (double)xrow[d];
    ss = __fma_rn(v, v, ss);
  }
  ss = pb_block_sum_d(ss, red);
  double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)dim), eps));
  if (out16) {
    const float inv = (float)(1.0 / rms);
    if (hl) {
      for (int d = threadIdx.x; d < dim; d += blockDim.x)
        pb_store_hl(out16, pb_hl_index((size_t)row * 2 * dim, d), xrow[d] * inv * w[d]);
    } else {
      for (int d = threadIdx.x; d < dim; d += blockDim.x) out16[(size_t)row * dim + d] = __float2half_rn(xrow[d] * inv * w[d]);
    }
  } else {
    for (int d = threadIdx.x; d < dim; d += blockDim.x)
      out[(size_t)row * dim + d] = (float)__dmul_rn(__ddiv_rn((double)xrow[d], rms), (double)w[d]);
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(xr.done, 1u) == (unsigned)rows - 1) {
    *xr.done = 0u;
    *xr.epoch = e;
  }
}

int pb_launch_rmsnorm_xrecv(pb_ctx* ctx, float* x, int rows, int dim, const float* w, double eps, float* out,
                            __half* out16, int xc, int hl, const pb_xrecv& xr) {
  if (xc <= 0 || dim % xc || xc % 2 || (size_t)dim * 4 > 48 * 1024)
    return pb_set_error(ctx, PB_ERR_ARG, "fused residual exchange: chunks of %d over dim %d", xc, dim);
  pb_xrecv r = xr;
  r.limit_ns = (unsigned long long)ctx->timeout_ms * 1000000ull;
  r.err = ctx->d_err;
  return pb_launch(ctx, "k_rmsnorm_xrecv", true, k_rmsnorm_xrecv, dim3(rows), dim3(256), (size_t)dim * 4, x, dim, w,
                   eps, out, out16, xc, hl, r);
}

// The prefill-size form (rows >= PB_RMS_WARP_ROWS): a warp per row, 8 rows per
// CTA, float4 loads (the row read again for the output: it is in L1), the
// sum of squares over lane l's values 4(l + 32k) .. + 3 in order, then a warp
// tree.  A different partition from k_rmsnorm_t (within the rounding of a
// double sum); every path that normalises rows this many at a time takes it,
// the row split included, so they agree in bits.
constexpr int PB_RMS_WARP_ROWS = 4096;
template <bool CH>
__global__ void k_rmsnorm_w(const float* __restrict__ x, int dim, const float* __restrict__ w, double eps,
                            float* __restrict__ out, __half* __restrict__ out16, int xc, int hl, int rows) {
  pb_pdl_trigger();
  pb_pdl_wait();  // x comes from the previous kernel
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + (size_t)row * (CH ? xc : dim);
  const size_t cs = (size_t)rows * xc;
  auto X4 = [&](int d) {  // d % 4 == 0, xc % 4 == 0
    return *reinterpret_cast<const float4*>(CH ? xr + (size_t)(d / xc) * cs + d % xc : xr + d);
  };
  double ss = 0.0;
  for (int d = 4 * lane; d < dim; d += 128) {
    const float4 v = X4(d);
    ss = __fma_rn((double)v.x, (double)v.x, ss);
    ss = __fma_rn((double)v.y, (double)v.y, ss);
    ss = __fma_rn((double)v.z, (double)v.z, ss);
    ss = __fma_rn((double)v.w, (double)v.w, ss);
  }
  ss = pb_warp_sum_d(ss);
  const double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)dim), eps));
  const float inv = (float)(1.0 / rms);
  for (int d = 4 * lane; d < dim; d += 128) {
    const float4 v = X4(d);
    const float4 g = *reinterpret_cast<const float4*>(w + d);
    if (out16) {
      const float a0 = v.x * inv * g.x, a1 = v.y * inv * g.y, a2 = v.z * inv * g.z, a3 = v.w * inv * g.w;
      const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
      if (hl) {  // hi halves of the 64-group at +0, lo at +64 (pb_hl_index); 4 values stay in one group
        const size_t o = pb_hl_index((size_t)row * 2 * dim, d);
        *reinterpret_cast<uint2*>(out16 + o) = make_uint2(*reinterpret_cast<const uint32_t*>(&h01),
                                                          *reinterpret_cast<const uint32_t*>(&h23));
        const __half2 l01 = __floats2half2_rn(a0 - __low2float(h01), a1 - __high2float(h01));
        const __half2 l23 = __floats2half2_rn(a2 - __low2float(h23), a3 - __high2float(h23));
        *reinterpret_cast<uint2*>(out16 + o + 64) = make_uint2(*reinterpret_cast<const uint32_t*>(&l01),
                                                               *reinterpret_cast<const uint32_t*>(&l23));
      } else {
        *reinterpret_cast<uint2*>(out16 + (size_t)row * dim + d) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
      }
    } else {
      float4 o;
      o.x = (float)__dmul_rn(__ddiv_rn((double)v.x, rms), (double)g.x);
      o.y = (float)__dmul_rn(__ddiv_rn((double)v.y, rms), (double)g.y);
      o.z = (float)__dmul_rn(__ddiv_rn((double)v.z, rms), (double)g.z);
      o.w = (float)__dmul_rn(__ddiv_rn((double)v.w, rms), (double)g.w);
      *reinterpret_cast<float4*>(out + (size_t)row * dim + d) = o;
    }
  }
}

void pb_launch_rmsnorm(cudaStream_t st, const float* x, int rows, int dim, const float* w, double eps, float* out,
                       __half* out16, int xc, int hl, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const bool ch = xc > 0 && xc < dim;
  if (rows >= PB_RMS_WARP_ROWS && dim % 128 == 0 && (!ch || xc % 4 == 0)) {
    cfg.gridDim = dim3((rows + 7) / 8);
    if (ch) cudaLaunchKernelEx(&cfg, k_rmsnorm_w<true>, x, dim, w, eps, out, out16, xc, hl, rows);
    else cudaLaunchKernelEx(&cfg, k_rmsnorm_w<false>, x, dim, w, eps, out, out16, 0, hl, rows);
    return;
  }
  if (ch) cudaLaunchKernelEx(&cfg, k_rmsnorm_t<true>, x, dim, w, eps, out, out16, xc, hl);
  else cudaLaunchKernelEx(&cfg, k_rmsnorm_t<false>, x, dim, w, eps, out, out16, 0, hl);
}

extern "C" int pb_rmsnorm(pb_ctx* ctx, const float* x, int seq, int dim, const float* w, double eps, float* out) {
  if (!ctx || !x || !w || !out || seq <= 0 || dim <= 0) return PB_ERR_ARG;
  pb_launch_rmsnorm(ctx->stream, x, seq, dim, w, eps, out, nullptr, 0);
  PB_LAUNCHED(ctx, "k_rmsnorm");
  return PB_OK;
}

// ============================================================================
// softmax (engine.js:279-303), layerNorm (:315-344)
// ============================================================================

__global__ void k_softmax(const float* __restrict__ in, int cols, float* __restrict__ out) {
  __shared__ double red[32];
  __shared__ float fred[32];
  __shared__ int nanflag;
  const float* ir = in + (size_t)blockIdx.x * cols;
  float* orow = out + (size_t)blockIdx.x * cols;
  if (threadIdx.x == 0) nanflag = 0;
  __syncthreads();
  // Math.max over the row (NaN propagates)
  float m = -INFINITY;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float v = ir[c];
    if (v != v) nanflag = 1;
    m = fmaxf(m, v);
  }
  m = pb_warp_max_f(m);
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) fred[wid] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = -INFINITY;
    for (int i = 0; i < (blockDim.x + 31) / 32; ++i) t = fmaxf(t, fred[i]);
    fred[0] = nanflag ? __int_as_float(0x7fc00000) : t;
  }
  __syncthreads();
  double mx = fred[0];
  double s = 0.0;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float e = (float)exp(__dsub_rn((double)ir[c], mx));
    orow[c] = e;
    s = __dadd_rn(s, (double)e);
  }
  s = pb_block_sum_d(s, red);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) orow[c] = (float)__ddiv_rn((double)orow[c], s);
}

extern "C" int pb_softmax(pb_ctx* ctx, const float* in, int rows, int cols, float* out) {
  if (!ctx || !in || !out || rows <= 0 || cols <= 0) return PB_ERR_ARG;
  k_softmax<<<rows, 256, 0, ctx->stream>>>(in, cols, out);
  PB_LAUNCHED(ctx, "k_softmax");
  return PB_OK;
}

__global__ void k_layernorm(const float* __restrict__ x, int dim, const float* __restrict__ w,
                            const float* __restrict__ b, double eps, float* __restrict__ out) {
  __shared__ double red[32];
  const float* xr = x + (size_t)blockIdx.x * dim;
  double s = 0.0;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) s = __dadd_rn(s, (double)xr[d]);
  double mean = __ddiv_rn(pb_block_sum_d(s, red), (double)dim);
  // `variance += diff * diff`: diff*diff is not exact, so multiply then add
  double v = 0.0;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    double df = __dsub_rn((double)xr[d], mean);
    v = __dadd_rn(v, __dmul_rn(df, df));
  }
  double var = __ddiv_rn(pb_block_sum_d(v, red), (double)dim);
  double sd = __dsqrt_rn(__dadd_rn(var, eps));
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    double t = __dmul_rn(__ddiv_rn(__dsub_rn((double)xr[d], mean), sd), (double)w[d]);
    out[(size_t)blockIdx.x * dim + d] = (float)__dadd_rn(t, b ? (double)b[d] : 0.0);
  }
}

extern "C" int pb_layernorm(pb_ctx* ctx, const float* x, int seq, int dim, const float* w, const float* b, double eps,
                            float* out) {
  if (!ctx || !x || !w || !out || seq <= 0 || dim <= 0) return PB_ERR_ARG;
  k_layernorm<<<seq, 256, 0, ctx->stream>>>(x, dim, w, b, eps, out);
  PB_LAUNCHED(ctx, "k_layernorm");
  return PB_OK;
}

// ============================================================================
// elementwise ops (engine.js:96-106, 354-360, 459-484; llama-streaming.js:590-595)
// ============================================================================

enum { EW_ADD = 0, EW_MUL, EW_SILU, EW_GELU, EW_SWIGLU };

__global__ void k_elementwise(int op, const float* __restrict__ a, const float* __restrict__ b, int64_t n,
                              float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double x = a[i];
  double r;
  switch (op) {
    case EW_ADD: r = __dadd_rn(x, (double)b[i]); break;
    case EW_MUL: r = __dmul_rn(x, (double)b[i]); break;
    case EW_SILU: r = __ddiv_rn(x, __dadd_rn(1.0, exp(-x))); break;
    case EW_GELU: {
      const double c = __dsqrt_rn(__ddiv_rn(2.0, 3.141592653589793));  // Math.sqrt(2 / Math.PI)
      double x3 = __dmul_rn(__dmul_rn(__dmul_rn(0.044715, x), x), x);
      double inner = __dmul_rn(c, __dadd_rn(x, x3));
      r = __dmul_rn(__dmul_rn(0.5, x), __dadd_rn(1.0, tanh(inner)));
      break;
    }
    default: {  // fused SiLU(g) * u in double, one f32 rounding
      double silu = __ddiv_rn(x, __dadd_rn(1.0, exp(-x)));
      r = __dmul_rn(silu, (double)b[i]);
    }
  }
  out[i] = (float)r;
}

static int ew(pb_ctx* ctx, int op, const float* a, const float* b, int64_t n, float* out) {
  if (!ctx || !a || !out || n <= 0) return PB_ERR_ARG;
  if ((op == EW_ADD || op == EW_MUL || op == EW_SWIGLU) && !b) return PB_ERR_ARG;
  k_elementwise<<<pb_cdiv(n, 256), 256, 0, ctx->stream>>>(op, a, b, n, out);
  PB_LAUNCHED(ctx, "k_elementwise");
  return PB_OK;
}

extern "C" int pb_tensoradd(pb_ctx* ctx, const float* a, const float* b, int64_t n, float* out) { return ew(ctx, EW_ADD, a, b, n, out); }
extern "C" int pb_elementmul(pb_ctx* ctx, const float* a, const float* b, int64_t n, float* out) { return ew(ctx, EW_MUL, a, b, n, out); }
extern "C" int pb_silu(pb_ctx* ctx, const float* a, int64_t n, float* out) { return ew(ctx, EW_SILU, a, nullptr, n, out); }
extern "C" int pb_gelu(pb_ctx* ctx, const float* a, int64_t n, float* out) { return ew(ctx, EW_GELU, a, nullptr, n, out); }
extern "C" int pb_swiglu(pb_ctx* ctx, const float* g, const float* u, int n, float* out) { return ew(ctx, EW_SWIGLU, g, u, n, out); }

// ============================================================================
// f32 matmul in the WASM order (wasm-simd.js:71-91): C[m,n] = C[m,n] + a*B[k,n]
// ============================================================================

__global__ void k_matmul_f32(const float* __restrict__ A, int M, int K, const float* __restrict__ B, int N,
                             const float* __restrict__ bias, float* __restrict__ C) {
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  int m = blockIdx.y;
  if (n >= N) return;
  const float* ar = A + (size_t)m * K;
  float c = bias ? bias[n] : 0.0f;
  for (int k = 0; k < K; ++k) c = __fadd_rn(c, __fmul_rn(ar[k], B[(size_t)k * N + n]));
  C[(size_t)m * N + n] = c;
}

extern "C" int pb_matmul_f32(pb_ctx* ctx, const float* A, int M, int K, const float* B, int N, const float* bias,
                             float* C) {
  if (!ctx || !A || !B || !C || M <= 0 || K <= 0 || N <= 0) return PB_ERR_ARG;
  if (M > 65535) return pb_set_error(ctx, PB_ERR_ARG, "M=%d too large", M);
  dim3 grid(pb_cdiv(N, 128), M);
  k_matmul_f32<<<grid, 128, 0, ctx->stream>>>(A, M, K, B, N, bias, C);
  PB_LAUNCHED(ctx, "k_matmul_f32");
  return PB_OK;
}

// ============================================================================
// quantize.js:224-266 matmul_q8: out[m,n] += (a*scale)*q in double, f32 store,
// k ascending, zero activations skipped; the scale of a 32-column chunk is the
// block of its first flat element (quantize.js:256).
// ============================================================================

__global__ void k_matmul_q8a(const float* __restrict__ A, int M, int K, const float* __restrict__ scales,
                             const int8_t* __restrict__ q, int N, const float* __restrict__ bias,
                             float* __restrict__ out) {
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  int m = blockIdx.y;
  if (n >= N) return;
  const float* ar = A + (size_t)m * K;
  int64_t nstart = (int64_t)(n / 32) * 32;
  float o = bias ? bias[n] : 0.0f;
  for (int k = 0; k < K; ++k) {
    double a = ar[k];
    if (a == 0.0) continue;
    int64_t row = (int64_t)k * N;
    double sc = scales[(row + nstart) / 32];
    double as = __dmul_rn(a, sc);
    double t = __dmul_rn(as, (double)q[row + n]);
    o = (float)__dadd_rn((double)o, t);
  }
  out[(size_t)m * N + n] = o;
}

extern "C" int pb_matmul_q8a(pb_ctx* ctx, const float* A, int M, int K, const float* scales, const int8_t* q, int N,
                             const float* bias, float* out) {
  if (!ctx || !A || !scales || !q || !out || M <= 0 || K <= 0 || N <= 0) return PB_ERR_ARG;
  if (M > 65535) return pb_set_error(ctx, PB_ERR_ARG, "M=%d too large", M);
  dim3 grid(pb_cdiv(N, 128), M);
  k_matmul_q8a<<<grid, 128, 0, ctx->stream>>>(A, M, K, scales, q, N, bias, out);
  PB_LAUNCHED(ctx, "k_matmul_q8a");
  return PB_OK;
}

// ============================================================================
// generic attention (engine.js:374-415)
// ============================================================================

__global__ void k_attn_scores_generic(const float* __restrict__ Q, const float* __restrict__ Kt, int seqQ, int seqK,
                                      int dK, int causal, double scale, float* __restrict__ S) {
  int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
  if (j >= seqK) return;
  float v;
  if (causal && j > i) {
    v = -1e9f;
  } else {
    double dot = 0.0;
    for (int k = 0; k < dK; ++k) dot = __fma_rn((double)Q[(size_t)i * dK + k], (double)Kt[(size_t)j * dK + k], dot);
    v = (float)__dmul_rn(dot, scale);
  }
  S[(size_t)i * seqK + j] = v;
}

__global__ void k_attn_pv_generic(const float* __restrict__ W, const float* __restrict__ V, int seqK, int dV,
                                  float* __restrict__ out) {
  int d = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
  if (d >= dV) return;
  double s = 0.0;
  for (int j = 0; j < seqK; ++j) s = __fma_rn((double)W[(size_t)i * seqK + j], (double)V[(size_t)j * dV + d], s);
  out[(size_t)i * dV + d] = (float)s;
}

extern "C" int pb_attention(pb_ctx* ctx, const float* Q, const float* K, const float* V, int seqQ, int seqK, int dK,
                            int dV, int causal, float* out) {
  if (!ctx || !Q || !K || !V || !out || seqQ <= 0 || seqK <= 0 || dK <= 0 || dV <= 0) return PB_ERR_ARG;
  // one CTA row per query: grid.y is limited to 65535
  if (seqQ > 65535) return pb_set_error(ctx, PB_ERR_ARG, "seqQ = %d exceeds 65535", seqQ);
  size_t sb = (size_t)seqQ * seqK * 4;
  PB_TRY(pb_ensure_scratch(ctx, 2 * sb + 256));
  float* S = (float*)ctx->scratch;
  float* Wt = (float*)((char*)ctx->scratch + ((sb + 255) & ~(size_t)255));
  double scale = 1.0 / sqrt((double)dK);
  k_attn_scores_generic<<<dim3(pb_cdiv(seqK, 128), seqQ), 128, 0, ctx->stream>>>(Q, K, seqQ, seqK, dK, causal, scale, S);
  PB_LAUNCHED(ctx, "k_attn_scores_generic");
  PB_TRY(pb_softmax(ctx, S, seqQ, seqK, Wt));
  k_attn_pv_generic<<<dim3(pb_cdiv(dV, 64), seqQ), 64, 0, ctx->stream>>>(Wt, V, seqK, dV, out);
  PB_LAUNCHED(ctx, "k_attn_pv_generic");
  return PB_OK;
}

// The same attention with its scores S and probabilities W in a fixed device
// array instead of the context scratch, so the call allocates nothing.  S and
// W are written in full before they are read (every S[i, j], then every
// W[i, j] by the softmax), so nothing needs clearing between calls.  The array
// is one per device and shared by all contexts: overlapping calls race.
static __device__ __align__(256) unsigned char g_noalloc_attn[PB_NOALLOC_ATTN_BYTES];

constexpr int PB_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
static void* g_noalloc_attn_ptr[PB_MAX_DEVICES];

// Once per device, with that device current (pb_init): the array's address.
int pb_setup_noalloc(pb_ctx* ctx) {
  if (ctx->device < 0 || ctx->device >= PB_MAX_DEVICES)
    return pb_set_error(ctx, PB_ERR_ARG, "device %d out of range", ctx->device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_attn_ptr[ctx->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_attn);
    if (e != cudaSuccess || !p) return pb_cuda_error(ctx, e, "cudaGetSymbolAddress(g_noalloc_attn)");
    g_noalloc_attn_ptr[ctx->device] = p;
  }
  ctx->noalloc_attn = g_noalloc_attn_ptr[ctx->device];
  return PB_OK;
}

extern "C" int pb_attention_noalloc(pb_ctx* ctx, const float* Q, const float* K, const float* V, int seqQ, int seqK,
                                    int dK, int dV, int causal, float* out) {
  if (!ctx || !Q || !K || !V || !out || seqQ <= 0 || seqK <= 0 || dK <= 0 || dV <= 0) return PB_ERR_ARG;
  if (!ctx->noalloc_attn) return pb_set_error(ctx, PB_ERR_STATE, "no-alloc scratch not set up");
  if (seqQ > 65535) return pb_set_error(ctx, PB_ERR_ARG, "seqQ = %d exceeds 65535", seqQ);
  const size_t sb = (size_t)seqQ * seqK * 4, sb_al = (sb + 255) & ~(size_t)255;
  if (2 * sb_al > PB_NOALLOC_ATTN_BYTES)
    return pb_set_error(ctx, PB_ERR_ARG, "seqQ*seqK = %lld needs %zu bytes of scratch; the fixed array holds %u",
                        (long long)seqQ * seqK, 2 * sb_al, (unsigned)PB_NOALLOC_ATTN_BYTES);
  float* S = (float*)ctx->noalloc_attn;
  float* Wt = (float*)((char*)ctx->noalloc_attn + sb_al);
  double scale = 1.0 / sqrt((double)dK);
  k_attn_scores_generic<<<dim3(pb_cdiv(seqK, 128), seqQ), 128, 0, ctx->stream>>>(Q, K, seqQ, seqK, dK, causal, scale, S);
  PB_LAUNCHED(ctx, "k_attn_scores_generic");
  PB_TRY(pb_softmax(ctx, S, seqQ, seqK, Wt));
  k_attn_pv_generic<<<dim3(pb_cdiv(dV, 64), seqQ), 64, 0, ctx->stream>>>(Wt, V, seqK, dV, out);
  PB_LAUNCHED(ctx, "k_attn_pv_generic");
  return PB_OK;
}

// ============================================================================
// RoPE (llama-streaming.js:310-339) with a host-built rotation table
// ============================================================================

// tab[(pos - start) * (hd/2) + i/2] = {cos, sin} of pos / theta^(i/hd), in
// double, computed on the host exactly as the reference does.
__global__ void k_rope(float* __restrict__ q, float* __restrict__ k, int seq, int n_heads, int n_kv, int hd,
                       const double2* __restrict__ tab) {
  int t = blockIdx.y;
  int half = hd / 2;
  int nq = n_heads * half, nk = n_kv * half;
  int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nq + nk) return;
  bool isq = idx < nq;
  int rel = isq ? idx : idx - nq;
  int h = rel / half, pr = rel % half;
  double2 cs = tab[(size_t)t * half + pr];
  float* base = isq ? q + (size_t)t * n_heads * hd : k + (size_t)t * n_kv * hd;
  size_t off = (size_t)h * hd + 2 * pr;
  double x0 = base[off], x1 = base[off + 1];
  base[off] = (float)__dsub_rn(__dmul_rn(x0, cs.x), __dmul_rn(x1, cs.y));
  base[off + 1] = (float)__dadd_rn(__dmul_rn(x0, cs.y), __dmul_rn(x1, cs.x));
}

// Host table for positions [start, start + n): {cos, sin}(pos * 1/theta^(i/hd)).
void pb_rope_table(double theta, int hd, int start, int n, double2* out) {
  int half = hd / 2;
  for (int i = 0; i < hd; i += 2) {
    double freq = 1.0 / pow(theta, (double)i / hd);
    for (int p = 0; p < n; ++p) {
      double angle = (double)(start + p) * freq;
      out[(size_t)p * half + i / 2] = make_double2(cos(angle), sin(angle));
    }
  }
}

// Llama-3 RoPE frequency scaling, as Meta published it with Llama 3.1 / 3.2
// (the `rope_freqs` factors a GGUF file may carry).  For a pair frequency f
// with wavelength w = 2 pi / f, against the pre-training context C:
//   w < C / high_freq_factor   -> f            (high frequencies kept)
//   w > C / low_freq_factor    -> f / factor   (low frequencies stretched)
//   otherwise, with s = (C / w - low_freq_factor) / (high_freq_factor - low_freq_factor),
//                               -> (1 - s) f / factor + s f.
// The reference never applies it: llama-streaming.js:316-336 uses
// 1 / theta^(i / hd) as is, and gguf.js:378-410 never maps rope_freqs.weight.
// So it is off unless a caller turns it on, and off in every parity check.
extern "C" int pb_rope_freqs(double theta, int hd, double factor, double low_freq_factor, double high_freq_factor,
                             int original_max_pos, double* freqs_out) {
  if (hd <= 0 || (hd & 1) || !freqs_out || !(theta > 0)) return PB_ERR_ARG;
  const bool on = factor > 0;
  if (on && (!(low_freq_factor > 0) || !(high_freq_factor > low_freq_factor) || original_max_pos <= 0))
    return PB_ERR_ARG;
  const double two_pi = 6.283185307179586;
  const double ctx_len = (double)original_max_pos;
  for (int i = 0; i < hd; i += 2) {
    const double f = 1.0 / pow(theta, (double)i / hd);
    double g = f;
    if (on) {
      const double wavelen = two_pi / f;
      if (wavelen < ctx_len / high_freq_factor) {
        g = f;
      } else if (wavelen > ctx_len / low_freq_factor) {
        g = f / factor;
      } else {
        const double s = (ctx_len / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor);
        g = (1.0 - s) * f / factor + s * f;
      }
    }
    freqs_out[i / 2] = g;
  }
  return PB_OK;
}

// The rotation table for given pair frequencies (freqs[hd / 2]).
void pb_rope_table_freqs(const double* freqs, int hd, int start, int n, double2* out) {
  const int half = hd / 2;
  for (int j = 0; j < half; ++j)
    for (int p = 0; p < n; ++p) {
      const double angle = (double)(start + p) * freqs[j];
      out[(size_t)p * half + j] = make_double2(cos(angle), sin(angle));
    }
}

extern "C" int pb_rope(pb_ctx* ctx, float* q, float* k, int seq, int start_pos, int n_heads, int n_kv, int hd,
                       double theta) {
  if (!ctx || !q || !k || seq <= 0 || start_pos < 0 || n_heads <= 0 || n_kv <= 0 || hd <= 0 || (hd & 1))
    return PB_ERR_ARG;
  std::vector<double2> tab((size_t)seq * (hd / 2));
  pb_rope_table(theta, hd, start_pos, seq, tab.data());
  size_t tb = tab.size() * sizeof(double2);
  PB_TRY(pb_ensure_scratch(ctx, tb));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(ctx->scratch, tab.data(), tb, cudaMemcpyHostToDevice, ctx->stream));
  int tot = (n_heads + n_kv) * (hd / 2);
  k_rope<<<dim3(pb_cdiv(tot, 128), seq), 128, 0, ctx->stream>>>(q, k, seq, n_heads, n_kv, hd, (const double2*)ctx->scratch);
  PB_LAUNCHED(ctx, "k_rope");
  return pb_wait(ctx);  // the table lives in scratch until the kernel ran
}

// ============================================================================
// attention over the KV cache (llama-streaming.js:422-464 prefill, :543-573 decode)
// One CTA per (query row t, head h).
// ============================================================================

__global__ void k_attn_cached(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                              int q_stride, int start_pos, const int* __restrict__ pos_dev, int n_heads, int n_kv,
                              int hd, double scale, float* __restrict__ out, int max_len, pb_seq_geo geo, int* err) {
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ double red[32];
  __shared__ float fred[32];
  float* sc = (float*)sm;
  pb_pdl_trigger();  // the next matvec may start fetching its weights
  const int t = blockIdx.y, h = blockIdx.x;
  const int sp = pos_dev ? *pos_dev : start_pos;
  const int cache_len = sp + gridDim.y;
  if (cache_len > max_len) {
    pb_raise(err, PB_DEVERR_BOUNDS);
    return;
  }
  const int kv_dim = n_kv * hd, per = n_heads / n_kv, kh = h / per;
  q += blockIdx.z * geo.q;  // sequence of a batched launch
  kc += blockIdx.z * geo.kv;
  vc += blockIdx.z * geo.kv;
  out += blockIdx.z * geo.out;
  const float* qh = q + (size_t)t * q_stride + (size_t)h * hd;
  // scores (f32 stores of a double dot)
  for (int j = threadIdx.x; j < cache_len; j += blockDim.x) {
    float v;
    if (j > sp + t) {
      v = -INFINITY;
    } else {
      const float* kr = kc + (size_t)j * kv_dim + (size_t)kh * hd;
      double dot = 0.0;
      for (int d = 0; d < hd; ++d) dot = __fma_rn((double)qh[d], (double)kr[d], dot);
      v = (float)__dmul_rn(dot, scale);
    }
    sc[j] = v;
  }
  __syncthreads();
  // max: `if (scores[j] > maxScore)` from -Infinity
  float m = -INFINITY;
  for (int j = threadIdx.x; j < cache_len; j += blockDim.x) m = sc[j] > m ? sc[j] : m;
  m = pb_warp_max_f(m);
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  if (lane == 0) fred[wid] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t2 = -INFINITY;
    for (int i = 0; i < nw; ++i) t2 = fred[i] > t2 ? fred[i] : t2;
    fred[0] = t2;
  }
  __syncthreads();
  double mx = fred[0];
  double s = 0.0;
  for (int j = threadIdx.x; j < cache_len; j += blockDim.x) {
    float e = (float)exp(__dsub_rn((double)sc[j], mx));
    sc[j] = e;
    s = __dadd_rn(s, (double)e);
  }
  s = pb_block_sum_d(s, red);
  for (int j = threadIdx.x; j < cache_len; j += blockDim.x) sc[j] = (float)__ddiv_rn((double)sc[j], s);
  __syncthreads();
  // out[d] = sum_j p_j * V[j, d]: threads = hd dims x (blockDim/hd) j-slices
  int slices = blockDim.x / hd;
  int d = threadIdx.x % hd, sl = threadIdx.x / hd;
  double acc = 0.0;
  if (sl < slices) {
    const float* vb = vc + (size_t)kh * hd + d;
    for (int j = sl; j < cache_len; j += slices) acc = __fma_rn((double)sc[j], (double)vb[(size_t)j * kv_dim], acc);
  }
  double* part = (double*)(sc + ((max_len + 1) & ~1));
  __syncthreads();
  if (sl < slices) part[sl * hd + d] = acc;
  __syncthreads();
  if (threadIdx.x < hd) {
    double tot = 0.0;
    for (int i = 0; i < slices; ++i) tot = __dadd_rn(tot, part[i * hd + threadIdx.x]);
    out[(size_t)t * n_heads * hd + (size_t)h * hd + threadIdx.x] = (float)tot;
  }
}

// ============================================================================
// batched prefill attention on the tensor cores (the batched configuration only)
// ============================================================================
// A flash-attention forward with mma.sync m16n8k16 (f16 operands, f32
// accumulation).  CTA = (64 queries, head, sequence), four warps of 16 query
// rows.  Q, K and V tiles are converted from the f32 activations and cache to
// f16 in shared memory (rows padded to 72 halves so ldmatrix is conflict-free).
// TERMS == 3 (the batched model's default precision): every operand is kept
// as an f16 pair hi = f16(v), lo = f16(v - hi) -- Q, K and V in two tiles
// each, P split in registers -- and both products run as hi*hi + hi*lo +
// lo*hi, so the scores and the output carry about 22 bits instead of 11.
// Per 64-key tile: S = Q K^T in registers, scaled by log2(e)/sqrt(hd), causal
// mask, online softmax (running max and sum per row, exp2), P packed to f16
// straight from the S accumulators into A fragments, O += P V with V read by
// ldmatrix.trans.  The output is divided by the row sum at the end.  The
// batched path already runs its projections with f16 operands; this agrees
// with the reference's double-precision attention (llama-streaming.js:422-464)
// within that path's tolerance, and the one-sequence path keeps the exact
// kernels.
constexpr int FT_Q = 64, FT_KT = 64, FT_HD = 64, FT_LD = 72, FT_THREADS = 128;

__device__ __forceinline__ void ft_ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(pb_smem_addr(p)));
}
__device__ __forceinline__ void ft_ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(pb_smem_addr(p)));
}
__device__ __forceinline__ void ft_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t ft_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// 4 consecutive f32 of a row -> 4 halves in shared memory
__device__ __forceinline__ void ft_store4(__half* dst, float4 v) {
  uint2 u;
  u.x = ft_h2(v.x, v.y);
  u.y = ft_h2(v.z, v.w);
  *reinterpret_cast<uint2*>(dst) = u;
}
// the lo halves of (a, b) given their hi pair (each difference exact in f32)
__device__ __forceinline__ uint32_t ft_lo2(float a, float b, uint32_t hi) {
  const __half2 h = *reinterpret_cast<const __half2*>(&hi);
  return ft_h2(__fsub_rn(a, __low2float(h)), __fsub_rn(b, __high2float(h)));
}
// 4 consecutive f32 -> their hi halves at dst, their lo halves at dst_lo
__device__ __forceinline__ void ft_store4_hl(__half* dst, __half* dst_lo, float4 v) {
  uint2 u, l;
  u.x = ft_h2(v.x, v.y);
  u.y = ft_h2(v.z, v.w);
  l.x = ft_lo2(v.x, v.y, u.x);
  l.y = ft_lo2(v.z, v.w, u.y);
  *reinterpret_cast<uint2*>(dst) = u;
  *reinterpret_cast<uint2*>(dst_lo) = l;
}

template <int TERMS>
__global__ void __launch_bounds__(FT_THREADS)
k_attn_prefill_tc(const float* __restrict__ q, int q_stride, const float* __restrict__ kc,
                  const float* __restrict__ vc, int seq, int start_pos, int n_heads, int n_kv, float scale,
                  float* __restrict__ out, pb_seq_geo geo, const __half* __restrict__ khl,
                  const __half* __restrict__ vhl, int64_t hl_seq_stride, __half* __restrict__ out16) {
  // [hi, lo] tiles of Q, K, V (the lo tiles only with three terms)
  constexpr int T = TERMS == 3 ? 2 : 1;
  extern __shared__ __align__(16) unsigned char ft_raw[];
  __half(*Qs)[FT_LD] = reinterpret_cast<__half(*)[FT_LD]>(ft_raw);
  __half(*Ks)[FT_LD] = Qs + T * FT_Q;
  __half(*Vs)[FT_LD] = Ks + T * FT_KT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int q0 = blockIdx.x * FT_Q, h = blockIdx.y, z = blockIdx.z;
  const int per = n_heads / n_kv, kh = h / per, kv_dim = n_kv * FT_HD, dim = n_heads * FT_HD;
  q += z * geo.q;
  kc += z * geo.kv;
  vc += z * geo.kv;
  out += z * geo.out;
  if (out16) out16 += z * geo.out * 2;  // hi/lo pairs take the bytes of the f32 rows
  // khl / vhl (three terms): K and V already as hi/lo halves (k_rope_kv), copied
  // into the tiles by cp.async instead of converted here by every CTA
  const bool pre = TERMS == 3 && khl != nullptr;
  if (pre) {
    khl += z * hl_seq_stride + (size_t)kh * 2 * FT_HD;
    vhl += z * hl_seq_stride + (size_t)kh * 2 * FT_HD;
  }
  for (int i = tid; i < FT_Q * FT_HD / 4; i += FT_THREADS) {
    const int qr = i / (FT_HD / 4), d4 = i % (FT_HD / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + qr < seq) v = *reinterpret_cast<const float4*>(q + (size_t)(q0 + qr) * q_stride + (size_t)h * FT_HD + 4 * d4);
    if (TERMS == 3) ft_store4_hl(&Qs[qr][4 * d4], &Qs[FT_Q + qr][4 * d4], v);
    else ft_store4(&Qs[qr][4 * d4], v);
  }
  __syncthreads();
  uint32_t qa[4][4], ql[4][4];  // A fragments (hi, lo) of this warp's 16 rows, 4 steps of 16 dims
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, cc = kk * 16 + (lane >> 4) * 8;
    ft_ldsm_x4(&Qs[r][cc], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
    if (TERMS == 3) ft_ldsm_x4(&Qs[FT_Q + r][cc], ql[kk][0], ql[kk][1], ql[kk][2], ql[kk][3]);
  }
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};
  const float sl2 = scale * 1.4426950408889634f;
  const int qlast = (q0 + FT_Q < seq ? q0 + FT_Q : seq) - 1;
  const int kend = start_pos + qlast + 1;  // keys 0 .. start_pos + last query of the tile (causal)
  const int qp0 = start_pos + q0 + warp * 16 + g, qp1 = qp0 + 8;
  for (int k0 = 0; k0 < kend; k0 += FT_KT) {
    __syncthreads();  // the previous tile is no longer read
    if (pre) {  // 16-byte pieces: (row, hi / lo, 8 halves); rows past kend are zero
      for (int i = tid; i < FT_KT * 16; i += FT_THREADS) {
        const int kr = i >> 4, part = (i >> 3) & 1, c8 = (i & 7) * 8;
        __half* kd = &Ks[part * FT_KT + kr][c8];
        __half* vd = &Vs[part * FT_KT + kr][c8];
        if (k0 + kr < kend) {
          const size_t so = (size_t)(k0 + kr) * 2 * kv_dim + part * FT_HD + c8;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(pb_smem_addr(kd)), "l"(khl + so) : "memory");
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(pb_smem_addr(vd)), "l"(vhl + so) : "memory");
        } else {
          *reinterpret_cast<uint4*>(kd) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(vd) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
    }
    for (int i = tid; !pre && i < FT_KT * FT_HD / 4; i += FT_THREADS) {
      const int kr = i / (FT_HD / 4), d4 = i % (FT_HD / 4);
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (k0 + kr < kend) {
        kv4 = *reinterpret_cast<const float4*>(kc + (size_t)(k0 + kr) * kv_dim + (size_t)kh * FT_HD + 4 * d4);
        vv4 = *reinterpret_cast<const float4*>(vc + (size_t)(k0 + kr) * kv_dim + (size_t)kh * FT_HD + 4 * d4);
      }
      if (TERMS == 3) {
        ft_store4_hl(&Ks[kr][4 * d4], &Ks[FT_KT + kr][4 * d4], kv4);
        ft_store4_hl(&Vs[kr][4 * d4], &Vs[FT_KT + kr][4 * d4], vv4);
      } else {
        ft_store4(&Ks[kr][4 * d4], kv4);
        ft_store4(&Vs[kr][4 * d4], vv4);
      }
    }
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8, cc = kk * 16 + ((lane >> 3) & 1) * 8;
        ft_ldsm_x4(&Ks[r][cc], b0, b1, b2, b3);
        ft_mma(s[2 * np], qa[kk], b0, b1);
        ft_mma(s[2 * np + 1], qa[kk], b2, b3);
        if (TERMS == 3) {
          uint32_t l0, l1, l2, l3;
          ft_ldsm_x4(&Ks[FT_KT + r][cc], l0, l1, l2, l3);
          ft_mma(s[2 * np], qa[kk], l0, l1);
          ft_mma(s[2 * np + 1], qa[kk], l2, l3);
          ft_mma(s[2 * np], ql[kk], b0, b1);
          ft_mma(s[2 * np + 1], ql[kk], b2, b3);
        }
      }
    }
    float mt0 = -INFINITY, mt1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int key = k0 + 8 * j + 2 * t + c;
        const bool kin = key < kend;
        s[j][c] = (kin && key <= qp0) ? s[j][c] * sl2 : -INFINITY;
        s[j][2 + c] = (kin && key <= qp1) ? s[j][2 + c] * sl2 : -INFINITY;
        mt0 = fmaxf(mt0, s[j][c]);
        mt1 = fmaxf(mt1, s[j][2 + c]);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
      mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
    }
    const float mn0 = fmaxf(m_r[0], mt0), mn1 = fmaxf(m_r[1], mt1);
    const float al0 = mn0 == -INFINITY ? 1.0f : exp2f(m_r[0] - mn0);
    const float al1 = mn1 == -INFINITY ? 1.0f : exp2f(m_r[1] - mn1);
    float ls0 = 0.0f, ls1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        s[j][c] = mn0 == -INFINITY ? 0.0f : exp2f(s[j][c] - mn0);
        s[j][2 + c] = mn1 == -INFINITY ? 0.0f : exp2f(s[j][2 + c] - mn1);
        ls0 += s[j][c];
        ls1 += s[j][2 + c];
      }
      o[j][0] *= al0;
      o[j][1] *= al0;
      o[j][2] *= al1;
      o[j][3] *= al1;
    }
    l_r[0] = l_r[0] * al0 + ls0;
    l_r[1] = l_r[1] * al1 + ls1;
    m_r[0] = mn0;
    m_r[1] = mn1;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step: S n-tiles 2kk, 2kk+1 as the A fragment
      const uint32_t pa[4] = {ft_h2(s[2 * kk][0], s[2 * kk][1]), ft_h2(s[2 * kk][2], s[2 * kk][3]),
                              ft_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]), ft_h2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
      uint32_t pl[4] = {0u, 0u, 0u, 0u};
      if (TERMS == 3) {
        pl[0] = ft_lo2(s[2 * kk][0], s[2 * kk][1], pa[0]);
        pl[1] = ft_lo2(s[2 * kk][2], s[2 * kk][3], pa[1]);
        pl[2] = ft_lo2(s[2 * kk + 1][0], s[2 * kk + 1][1], pa[2]);
        pl[3] = ft_lo2(s[2 * kk + 1][2], s[2 * kk + 1][3], pa[3]);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, cc = np * 16 + (lane >> 4) * 8;
        ft_ldsm_x4_t(&Vs[r][cc], b0, b1, b2, b3);
        ft_mma(o[2 * np], pa, b0, b1);
        ft_mma(o[2 * np + 1], pa, b2, b3);
        if (TERMS == 3) {
          uint32_t l0, l1, l2, l3;
          ft_ldsm_x4_t(&Vs[FT_KT + r][cc], l0, l1, l2, l3);
          ft_mma(o[2 * np], pa, l0, l1);
          ft_mma(o[2 * np + 1], pa, l2, l3);
          ft_mma(o[2 * np], pl, b0, b1);
          ft_mma(o[2 * np + 1], pl, b2, b3);
        }
      }
    }
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], off);
    l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], off);
  }
  const float inv0 = 1.0f / l_r[0], inv1 = 1.0f / l_r[1];
  const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
  if (out16) {  // the wo GEMM's operand directly: hi/lo pairs (pb_hl_index), as k_f32_to_f16 forms them
    auto put = [&](int r, int d, float a, float b) {
      const size_t o = pb_hl_index((size_t)r * 2 * dim, h * FT_HD + d);
      const __half2 hi = __floats2half2_rn(a, b);
      *reinterpret_cast<__half2*>(out16 + o) = hi;
      *reinterpret_cast<__half2*>(out16 + o + 64) =
          __floats2half2_rn(__fsub_rn(a, __low2float(hi)), __fsub_rn(b, __high2float(hi)));
    };
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = 8 * j + 2 * t;
      if (r0 < seq) put(r0, d, o[j][0] * inv0, o[j][1] * inv0);
      if (r1 < seq) put(r1, d, o[j][2] * inv1, o[j][3] * inv1);
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int d = 8 * j + 2 * t;
    if (r0 < seq)
      *reinterpret_cast<float2*>(out + (size_t)r0 * dim + (size_t)h * FT_HD + d) =
          make_float2(o[j][0] * inv0, o[j][1] * inv0);
    if (r1 < seq)
      *reinterpret_cast<float2*>(out + (size_t)r1 * dim + (size_t)h * FT_HD + d) =
          make_float2(o[j][2] * inv1, o[j][3] * inv1);
  }
}

static size_t ft_smem(int terms) { return (size_t)(terms == 3 ? 2 : 1) * (FT_Q + 2 * FT_KT) * FT_LD * 2; }

int pb_launch_attn_prefill(pb_ctx* ctx, const float* q, int q_stride, const float* kc, const float* vc, int seq,
                           int start_pos, int n_heads, int n_kv, int hd, float* out, int nseq, pb_seq_geo geo,
                           int terms, const __half* khl, const __half* vhl, int64_t hl_seq_stride, __half* out16) {
  if (hd != FT_HD || (q_stride & 3) || (terms != 1 && terms != 3)) return PB_ERR_ARG;
  auto kern = terms == 3 ? k_attn_prefill_tc<3> : k_attn_prefill_tc<1>;
  kern<<<dim3(pb_cdiv(seq, FT_Q), n_heads, nseq), FT_THREADS, ft_smem(terms), ctx->stream>>>(
      q, q_stride, kc, vc, seq, start_pos, n_heads, n_kv, (float)(1.0 / sqrt((double)hd)), out, geo, khl, vhl,
      hl_seq_stride, terms == 3 ? out16 : nullptr);
  PB_LAUNCHED(ctx, "k_attn_prefill_tc");
  return PB_OK;
}

int pb_launch_attn_cached(pb_ctx* ctx, const float* q, int q_stride, const float* kc, const float* vc, int seq,
                          int start_pos, const int* pos_dev, int n_heads, int n_kv, int hd, float* out, int max_len,
                          int nseq, pb_seq_geo geo) {
  int threads = hd * 4 <= 1024 ? hd * 4 : hd;
  if (threads < 64) threads = 64;
  size_t smem = (size_t)((max_len + 1) & ~1) * 4 + (size_t)(threads / hd + 1) * hd * 8 + 16;
  if (smem > 200 * 1024) return pb_set_error(ctx, PB_ERR_ARG, "cache length %d too long for one CTA", max_len);
  double scale = 1.0 / sqrt((double)hd);
  k_attn_cached<<<dim3(n_heads, seq, nseq), threads, smem, ctx->stream>>>(q, kc, vc, q_stride, start_pos, pos_dev,
                                                                          n_heads, n_kv, hd, scale, out, max_len, geo,
                                                                          ctx->d_err);
  PB_LAUNCHED(ctx, "k_attn_cached");
  return PB_OK;
}

extern "C" int pb_attn_cached(pb_ctx* ctx, const float* q, const float* kc, const float* vc, int seq, int start_pos,
                              int n_heads, int n_kv, int hd, float* out) {
  if (!ctx || !q || !kc || !vc || !out || seq <= 0 || start_pos < 0 || n_heads <= 0 || n_kv <= 0 || hd <= 0 ||
      n_heads % n_kv)
    return PB_ERR_ARG;
  return pb_launch_attn_cached(ctx, q, n_heads * hd, kc, vc, seq, start_pos, nullptr, n_heads, n_kv, hd, out,
                               start_pos + seq, 1, pb_seq_geo());
}

// ============================================================================
// model-step kernels
// ============================================================================

// RoPE on q (in place, row stride q_stride) and k, then KV append
// (llama-streaming.js:531-541): rows t = 0..seq-1 at position pos0 + t,
// pos0 = *pos_dev when pos_dev is set.  tab has one entry per position.
// The batched prefill attention's K / V operands, converted once: per position,
// per kv head, its hd hi halves then its hd lo halves (hi = f16(v), lo =
// f16(v - hi), as the attention converts them); off = head * hd + d, d even.
__device__ __forceinline__ void ft_store_hl_pair(__half* row, size_t off, int hd, float a, float b) {
  const size_t o = (off / hd) * 2 * hd + off % hd;
  const __half2 hi = __floats2half2_rn(a, b);
  *reinterpret_cast<__half2*>(row + o) = hi;
  *reinterpret_cast<__half2*>(row + o + hd) =
      __floats2half2_rn(__fsub_rn(a, __low2float(hi)), __fsub_rn(b, __high2float(hi)));
}

__global__ void k_rope_kv(float* __restrict__ q, int q_stride, const float* __restrict__ k, int k_stride,
                          const float* __restrict__ v, int v_stride, int n_heads, int n_kv, int hd,
                          const double2* __restrict__ tab, int start_pos, const int* __restrict__ pos_dev,
                          float* __restrict__ kc, float* __restrict__ vc, int max_len, int rows_per_seq,
                          int64_t cache_seq_stride, int* err, int rows, int rows_per_cta, __half* __restrict__ khl,
                          __half* __restrict__ vhl, int64_t hl_seq_stride) {
  pb_pdl_trigger();
  pb_pdl_wait();  // q, k, v come from the projection
  const int half = hd / 2, kv_dim = n_kv * hd;
  const int nq = n_heads * half, nk = n_kv * half;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int p0 = pos_dev ? *pos_dev : start_pos;
  // rows_per_cta rows of the same element columns per CTA (prefill sizes: fewer, longer CTAs)
  for (int rr = 0; rr < rows_per_cta; ++rr) {
    const int t = blockIdx.y * rows_per_cta + rr;  // row; rows of sequence s are s*rows_per_seq .. +rows_per_seq-1
    if (t >= rows) break;
    const int sq = t / rows_per_seq;
    float* kcs = kc + sq * cache_seq_stride;
    float* vcs = vc + sq * cache_seq_stride;
    const int pos = p0 + (t - sq * rows_per_seq);
    if (pos < 0 || pos >= max_len) {
      if (threadIdx.x == 0 && blockIdx.x == 0) pb_raise(err, PB_DEVERR_BOUNDS);
      return;
    }
    if (idx < nq + nk) {
      const bool isq = idx < nq;
      const int rel = isq ? idx : idx - nq;
      const int h = rel / half, pr = rel % half;
      const double2 cs = tab[(size_t)pos * half + pr];
      const size_t off = (size_t)h * hd + 2 * pr;
      const float2 xv = *reinterpret_cast<const float2*>(isq ? q + (size_t)t * q_stride + off
                                                              : k + (size_t)t * k_stride + off);
      const double x0 = xv.x, x1 = xv.y;
      float2 r;
      r.x = (float)__dsub_rn(__dmul_rn(x0, cs.x), __dmul_rn(x1, cs.y));
      r.y = (float)__dadd_rn(__dmul_rn(x0, cs.y), __dmul_rn(x1, cs.x));
      *reinterpret_cast<float2*>(isq ? q + (size_t)t * q_stride + off : kcs + (size_t)pos * kv_dim + off) = r;
      if (!isq && khl) ft_store_hl_pair(khl + sq * hl_seq_stride + (size_t)pos * 2 * kv_dim, off, hd, r.x, r.y);
    } else if (idx < nq + nk + kv_dim) {
      const int dd = idx - nq - nk;
      const float vv = v[(size_t)t * v_stride + dd];
      vcs[(size_t)pos * kv_dim + dd] = vv;
      if (vhl) {
        __half* row = vhl + sq * hl_seq_stride + (size_t)pos * 2 * kv_dim + (size_t)(dd / hd) * 2 * hd + dd % hd;
        const __half hi = __float2half_rn(vv);
        row[0] = hi;
        row[hd] = __float2half_rn(__fsub_rn(vv, __half2float(hi)));
      }
    }
  }
}

// SwiGLU: mode 0 = fused f32((g/(1+e^-g))*u) (llama-streaming.js:590-595);
// mode 1 = SILU then ELEMENT_MUL, two f32 roundings (llama.js:329-332,
// llama-streaming.js:478-481).
// interleave4: g and u are columns of one [g4 | u4]-tiled output row.
__global__ void k_glu(const float* __restrict__ g, int g_stride, const float* __restrict__ u, int u_stride, int F,
                      int mode, int interleave4, float* __restrict__ out) {
  int i = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
  if (i >= F) return;
  int gi = interleave4 ? 8 * (i >> 2) + (i & 3) : i;
  int ui = interleave4 ? gi + 4 : i;
  double gv = g[(size_t)m * g_stride + gi], uv = u[(size_t)m * u_stride + ui];
  double silu = __ddiv_rn(gv, __dadd_rn(1.0, exp(-gv)));
  if (mode == 1) silu = (double)(float)silu;
  out[(size_t)m * F + i] = (float)__dmul_rn(silu, uv);
}

// Embedding lookup (llama-streaming.js:748-759): x[i] = dequantized row tok_i
// of a tiled Q4_0 / Q8_0 table (exact f16 decode, gguf.js:55-70) or f32 tiles.
// When key_dev is set the token is the argmax of the previous step.
__global__ void k_embed(int type, const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc,
                        const float* __restrict__ f32tiles, int V, int dim, const int* __restrict__ toks,
                        const unsigned long long* __restrict__ key_dev, int* __restrict__ tok_out,
                        unsigned long long* __restrict__ key_reset, float* __restrict__ x, int* err) {
  pb_pdl_trigger();
  int i = blockIdx.y;
  int tok = key_dev ? pb_argmax_index(*key_dev) : toks[i];
  if (tok < 0 || tok >= V) {
    if (threadIdx.x == 0 && blockIdx.x == 0) pb_raise(err, PB_DEVERR_TOKEN);
    return;
  }
  int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d < dim) {
    int nb = dim / 32, tile = tok >> 5, r = tok & 31;
    float v;
    if (type == PB_TYPE_F32) {
      v = f32tiles[((size_t)tile * dim + d) * 32 + r];
    } else {
      int b = d >> 5, j = d & 31;
      size_t slot = (size_t)pb_qslot(tok, b, nb);
      float sc = pb_f16_exact(dsc[slot]);
      if (type == PB_TYPE_Q4_0) {
        uint8_t byte = qs[slot * 16 + (j & 15)];
        int nib = j < 16 ? (byte & 15) : (byte >> 4);
        v = __fmul_rn((float)(nib - 8), sc);
      } else {
        v = __fmul_rn((float)(int8_t)qs[slot * 32 + j], sc);
      }
    }
    x[(size_t)i * dim + d] = v;
  }
  __syncthreads();
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
    if (tok_out) *tok_out = tok;
  }
}

// End of a device-resident decode step: record the greedy token, advance the
// position and clear the argmax key for the next step.
__global__ void k_step_end(unsigned long long* __restrict__ key, int* __restrict__ tok_dev, int* __restrict__ pos_dev,
                           int* __restrict__ hist, int hist_len) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int next = pb_argmax_index(*key);
    *tok_dev = next;
    int p = *pos_dev;
    if (hist && p + 1 >= 0 && p + 1 < hist_len) hist[p + 1] = next;
    *pos_dev = p + 1;
    *key = 0ull;
  }
}


// ============================================================================
// decode attention (one query, llama-streaming.js:543-573) in one kernel
// ============================================================================
// k_attn_dec: CTA (query head h, sequence z), AF_THREADS threads.
//   1. scores: thread per position j (j = tid, tid + AF_THREADS, ...): the K
//      row's float4 loads all in flight, then the reference's order: double
//      dot, d ascending, then f32(dot * scale);
//   2. max over the f32 scores (`if (scores[j] > maxScore)` from -Infinity:
//      NaN never wins, so a tree of the same comparison gives the same value);
//   3. e_j = f32(exp(s_j - max)), the double sum of e_j (per-thread running
//      sums, then a fixed block tree), p_j = f32(e_j / sum);
//   4. out[d] = f32(sum_j p_j * V[j, d]) in double: thread (float4 lane d4,
//      position group jg), V rows prefetched into L2 while the scores run,
//      then the groups summed in a fixed two-level order.
// The four query heads of a kv head read the same K and V rows; L2 serves the
// repeats.  Scores and probabilities stay in shared memory: no scratch.

constexpr int AF_THREADS = 512;
constexpr int AF_MAX_HD = 256;
// PV partials [groups][hd] (groups * hd <= 4 * AF_THREADS) and their first-level
// sums [ceil(groups / 4)][hd] (<= AF_THREADS + AF_MAX_HD), in doubles
constexpr int AF_PART = AF_THREADS * 5 + AF_MAX_HD;

__global__ void __launch_bounds__(AF_THREADS, 1)
k_attn_dec(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
           const int* __restrict__ pos_dev, int n_heads, int n_kv, int hd, double scale, float* __restrict__ out,
           int max_len, pb_seq_geo geo, int* err) {
  extern __shared__ __align__(16) unsigned char af_raw[];
  double* part = reinterpret_cast<double*>(af_raw);     // [AF_PART] PV partials and their sums
  float* sp = reinterpret_cast<float*>(part + AF_PART);  // [max_len] scores, then probabilities
  __shared__ __align__(16) float qs[AF_MAX_HD];
  __shared__ double red[AF_THREADS / 32];
  __shared__ float wmax[AF_THREADS / 32];
  pb_pdl_trigger();  // the output projection may start fetching its weights
  pb_pdl_wait();     // q and the new cache row come from the projection matvec
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = *pos_dev;
  const int cache_len = pos + 1;
  if (pos < 0 || cache_len > max_len) {
    if (tid == 0 && h == 0 && blockIdx.y == 0) pb_raise(err, PB_DEVERR_BOUNDS);
    return;
  }
  const int per = n_heads / n_kv, g = h / per, kv_dim = n_kv * hd, h4 = hd / 4;
  q += blockIdx.y * geo.q;  // sequence of a batched launch
  kc += blockIdx.y * geo.kv;
  vc += blockIdx.y * geo.kv;
  out += blockIdx.y * geo.out;
  const float* vb = vc + (size_t)g * hd;
  for (int j = tid; j < cache_len; j += AF_THREADS) pb_l2_prefetch(vb + (size_t)j * kv_dim, (uint32_t)hd * 4);
  if (tid < h4) reinterpret_cast<float4*>(qs)[tid] = reinterpret_cast<const float4*>(q + (size_t)h * hd)[tid];
  __syncthreads();

  float m = -INFINITY;
  for (int j = tid; j < cache_len; j += AF_THREADS) {
    const float4* kr = reinterpret_cast<const float4*>(kc + (size_t)j * kv_dim + (size_t)g * hd);
    double dot = 0.0;
    for (int c0 = 0; c0 < h4; c0 += 16) {
      float4 k4[16];
#pragma unroll
      for (int u = 0; u < 16; ++u)
        if (c0 + u < h4) k4[u] = kr[c0 + u];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        if (c0 + u < h4) {
          const float4 a = reinterpret_cast<const float4*>(qs)[c0 + u];
          dot = __fma_rn((double)a.x, (double)k4[u].x, dot);  // exact product: one rounding per term
          dot = __fma_rn((double)a.y, (double)k4[u].y, dot);
          dot = __fma_rn((double)a.z, (double)k4[u].z, dot);
          dot = __fma_rn((double)a.w, (double)k4[u].w, dot);
        }
      }
    }
    const float s = (float)__dmul_rn(dot, scale);
    sp[j] = s;
    m = s > m ? s : m;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, m, o);
    m = t > m ? t : m;
  }
  if (lane == 0) wmax[warp] = m;
  __syncthreads();
  m = wmax[0];
  for (int w = 1; w < AF_THREADS / 32; ++w) m = wmax[w] > m ? wmax[w] : m;
  const double mx = m;

  double s = 0.0;
  for (int j = tid; j < cache_len; j += AF_THREADS) {
    const float e = (float)exp(__dsub_rn((double)sp[j], mx));
    sp[j] = e;
    s = __dadd_rn(s, (double)e);
  }
  s = pb_block_sum_d(s, red);
  for (int j = tid; j < cache_len; j += AF_THREADS) sp[j] = (float)__ddiv_rn((double)sp[j], s);
  __syncthreads();

  const int jgroups = AF_THREADS / h4, d4 = tid % h4, jg = tid / h4;
  double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
  if (jg < jgroups) {
    const float* vl = vb + 4 * d4;
    for (int base = jg; base < cache_len; base += 8 * jgroups) {
      float4 vv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = base + u * jgroups;
        if (j < cache_len) vv[u] = *reinterpret_cast<const float4*>(vl + (size_t)j * kv_dim);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = base + u * jgroups;
        if (j < cache_len) {
          const double pj = (double)sp[j];
          a0 = __fma_rn(pj, (double)vv[u].x, a0);
          a1 = __fma_rn(pj, (double)vv[u].y, a1);
          a2 = __fma_rn(pj, (double)vv[u].z, a2);
          a3 = __fma_rn(pj, (double)vv[u].w, a3);
        }
      }
    }
    double* pr = part + (size_t)jg * hd + 4 * d4;  // part[jg][d]
    pr[0] = a0;
    pr[1] = a1;
    pr[2] = a2;
    pr[3] = a3;
  }
  __syncthreads();
  // fixed two-level sum over the position groups: sums of 4 consecutive groups, then those in order
  const int n1 = (jgroups + 3) / 4;
  double* lvl = part + (size_t)jgroups * hd;  // [n1][hd], past the partials
  for (int idx = tid; idx < hd * n1; idx += AF_THREADS) {
    const int d = idx % hd, k = idx / hd;
    double t = part[(size_t)(4 * k) * hd + d];
    for (int i = 4 * k + 1; i < 4 * k + 4 && i < jgroups; ++i) t = __dadd_rn(t, part[(size_t)i * hd + d]);
    lvl[idx] = t;
  }
  __syncthreads();
  if (tid < hd) {
    double o = 0.0;
    for (int k = 0; k < n1; ++k) o = __dadd_rn(o, lvl[(size_t)k * hd + tid]);
    out[(size_t)h * hd + tid] = (float)o;
  }
}

// ============================================================================
// decode attention of one sequence split over positions (llama-streaming.js
// :543-573 in double, as the reference computes it)
// ============================================================================
// k_attn_dec1<PER>: CTA (kv head g, split sp) over the positions
// [sp * P, (sp + 1) * P) of the cache, P = ceil(cache_len / nsplit), for the
// PER query heads of the group (each K and V row is read once).  Up to 8
// splits per kv head (64 CTAs for 8 kv heads): each CTA walks an eighth of
// the cache instead of one CTA per head walking all of it, and the merge
// stays short.
//   - before griddepcontrol.wait: the position (written by the step before),
//     this split's K rows j < pos into registers and its V rows into L2
//     (only row pos is written by the projection this step);
//   - scores: thread per position, s_j = f32(dot * scale) with the double dot
//     in the reference's order (d ascending, exact products);
//   - per head the split's max m_c, e_j = f32(exp(s_j - m_c)) (the
//     reference's f32 store), S_c = sum e_j and O_c[d] = sum_j e_j V[j, d]
//     in double;
//   - the last split of a kv head to finish (an atomic counter; no waiting)
//     merges in split order: M = max m_c, S = sum S_c exp(m_c - M),
//     out[d] = f32(sum O_c[d] exp(m_c - M) / S), and resets the counter.
// Against the reference this moves the division by the sum after the
// products and rescales a split's f32 e_j when its max is not the global
// one: differences of an f32 rounding, within the attention tolerance.
constexpr int AD1_THREADS = 128;
constexpr int AD1_MAX_P = 512;   // positions per split
constexpr int AD1_MAX_HD = 128;
constexpr int AD1_GROUPS = AD1_THREADS / 16;  // PV position groups (16 float4 lanes cover hd <= 64 per pass)

template <int PER>
__global__ void __launch_bounds__(AD1_THREADS)
k_attn_dec1(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
            const int* __restrict__ pos_dev, int n_kv, int hd, double scale, float* __restrict__ out, int max_len,
            int nsplit, double* __restrict__ ws, unsigned int* __restrict__ counters, int* err) {
  extern __shared__ __align__(16) double ad1_sm[];
  const int g = blockIdx.x, sp = blockIdx.y, tid = threadIdx.x;
  const int pos = *pos_dev;  // final: the step's first kernel starts after the previous step ended
  const int cache_len = pos + 1;
  if (pos < 0 || cache_len > max_len) {
    pb_pdl_trigger();
    pb_pdl_wait();  // a dependent grid ends after the one before it, on every path
    if (tid == 0 && g == 0 && sp == 0) pb_raise(err, PB_DEVERR_BOUNDS);
    return;
  }
  const int kv_dim = n_kv * hd, h4 = hd >> 2;
  const int P = (cache_len + nsplit - 1) / nsplit;
  const int j0 = sp * P, j1 = min(j0 + P, cache_len);
  const int n = j1 > j0 ? j1 - j0 : 0;
  const float* kb = kc + (size_t)g * hd;
  const float* vb = vc + (size_t)g * hd;
  // K rows already in the cache (j < pos) into registers, V rows into L2
  constexpr int KR = 16;  // float4 per thread held across the wait (hd <= 64)
  float4 kr[KR];
  const int jt = j0 + tid;
  const bool has_row = tid < n;
  if (has_row && jt < pos) {
#pragma unroll
    for (int u = 0; u < KR; ++u)
      if (u < h4) kr[u] = reinterpret_cast<const float4*>(kb + (size_t)jt * kv_dim)[u];
  }
  for (int j = j0 + tid; j < j1 && j < pos; j += AD1_THREADS) pb_l2_prefetch(vb + (size_t)j * kv_dim, (uint32_t)hd * 4);
  pb_pdl_trigger();
  pb_pdl_wait();  // q and the cache row at pos come from the projection

  double* e = ad1_sm;                                             // [PER][AD1_MAX_P]: e_j, then unused
  double* pv = e + (size_t)PER * AD1_MAX_P;                       // [AD1_GROUPS][PER][hd]
  float* qs = reinterpret_cast<float*>(pv + (size_t)AD1_GROUPS * PER * hd);  // [PER][hd]
  __shared__ float smax[PER][AD1_THREADS / 32];
  __shared__ double ssum[PER][AD1_THREADS / 32];
  __shared__ unsigned int last_flag;
  for (int i = tid; i < PER * h4; i += AD1_THREADS)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(q + (size_t)g * PER * hd)[i];
  __syncthreads();

  // scores, thread per position
  for (int t = tid; t < n; t += AD1_THREADS) {
    const int j = j0 + t;
    const float4* krow = reinterpret_cast<const float4*>(kb + (size_t)j * kv_dim);
    double dot[PER];
#pragma unroll
    for (int h = 0; h < PER; ++h) dot[h] = 0.0;
    for (int c0 = 0; c0 < h4; c0 += KR) {
      float4 k4[KR];
      const bool reg = t == tid && j < pos && c0 == 0;  // held from before the wait
#pragma unroll
      for (int u = 0; u < KR; ++u)
        if (c0 + u < h4) k4[u] = reg ? kr[u] : krow[c0 + u];
#pragma unroll
      for (int u = 0; u < KR; ++u) {
        if (c0 + u < h4) {
#pragma unroll
          for (int h = 0; h < PER; ++h) {
            const float4 a = reinterpret_cast<const float4*>(qs + h * hd)[c0 + u];
            dot[h] = __fma_rn((double)a.x, (double)k4[u].x, dot[h]);  // exact products, one rounding each
            dot[h] = __fma_rn((double)a.y, (double)k4[u].y, dot[h]);
            dot[h] = __fma_rn((double)a.z, (double)k4[u].z, dot[h]);
            dot[h] = __fma_rn((double)a.w, (double)k4[u].w, dot[h]);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < PER; ++h) {
      const float s_ = (float)__dmul_rn(dot[h], scale);
      e[h * AD1_MAX_P + t] = (double)s_;
    }
  }
  // the split's max per head (`s > m` from -Infinity: NaN never wins)
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int h = 0; h < PER; ++h) {
    float m = -INFINITY;
    for (int t = tid; t < n; t += AD1_THREADS) {
      const float s_ = (float)e[h * AD1_MAX_P + t];
      m = s_ > m ? s_ : m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float o_ = __shfl_xor_sync(0xffffffffu, m, o);
      m = o_ > m ? o_ : m;
    }
    if (lane == 0) smax[h][warp] = m;
  }
  __syncthreads();
  float mc[PER];
#pragma unroll
  for (int h = 0; h < PER; ++h) {
    float m = smax[h][0];
    for (int w = 1; w < AD1_THREADS / 32; ++w) m = smax[h][w] > m ? smax[h][w] : m;
    mc[h] = m;
  }
  // e_j = f32(exp(s_j - m_c)) and the split's double sum
#pragma unroll
  for (int h = 0; h < PER; ++h) {
    double acc = 0.0;
    for (int t = tid; t < n; t += AD1_THREADS) {
      const float ej = (float)exp(__dsub_rn(e[h * AD1_MAX_P + t], (double)mc[h]));
      e[h * AD1_MAX_P + t] = (double)ej;
      acc = __dadd_rn(acc, (double)ej);
    }
    acc = pb_warp_sum_d(acc);
    if (lane == 0) ssum[h][warp] = acc;
  }
  __syncthreads();
  // O_c[h][d] = sum_j e_j V[j, d]: thread (float4 lane d4, position group jg)
  const int d4 = tid & 15, jg = tid >> 4;
  for (int dc = 0; dc < h4; dc += 16) {
    const int dd = dc + d4;
    double a[PER][4];
#pragma unroll
    for (int h = 0; h < PER; ++h) a[h][0] = a[h][1] = a[h][2] = a[h][3] = 0.0;
    if (dd < h4) {
      for (int t = jg; t < n; t += AD1_GROUPS) {
        const float4 v = reinterpret_cast<const float4*>(vb + (size_t)(j0 + t) * kv_dim)[dd];
#pragma unroll
        for (int h = 0; h < PER; ++h) {
          const double p = e[h * AD1_MAX_P + t];
          a[h][0] = __fma_rn(p, (double)v.x, a[h][0]);
          a[h][1] = __fma_rn(p, (double)v.y, a[h][1]);
          a[h][2] = __fma_rn(p, (double)v.z, a[h][2]);
          a[h][3] = __fma_rn(p, (double)v.w, a[h][3]);
        }
      }
#pragma unroll
      for (int h = 0; h < PER; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) pv[((size_t)jg * PER + h) * hd + 4 * dd + c] = a[h][c];
    }
  }
  __syncthreads();
  // this split's partial: [m_c, S_c, O_c[hd]] per head, groups summed in order
  double* wsp = ws + ((size_t)g * nsplit + sp) * PER * (2 + hd);
  for (int i = tid; i < PER * hd; i += AD1_THREADS) {
    const int h = i / hd, d = i - h * hd;
    double o = pv[(size_t)h * hd + d];
    for (int k = 1; k < AD1_GROUPS; ++k) o = __dadd_rn(o, pv[((size_t)k * PER + h) * hd + d]);
    wsp[(size_t)h * (2 + hd) + 2 + d] = o;
  }
  if (tid < PER) {
    double sacc = ssum[tid][0];
    for (int w = 1; w < AD1_THREADS / 32; ++w) sacc = __dadd_rn(sacc, ssum[tid][w]);
    wsp[(size_t)tid * (2 + hd)] = (double)mc[tid];
    wsp[(size_t)tid * (2 + hd) + 1] = sacc;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last_flag = atomicAdd(counters + g, 1u) == (unsigned)nsplit - 1;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  // the last split merges every split of this kv head, in split order:
  // the splits' maxima and sums into shared memory, one scale factor
  // f_c = exp(m_c - M) per (head, split), then the partial outputs in
  // batches of loads issued before use
  const double* wg = ws + (size_t)g * nsplit * PER * (2 + hd);
  double* fm = e;                          // [PER][nsplit]: m_c, then f_c
  double* fs = e + (size_t)PER * nsplit;   // [PER][nsplit]: S_c (0: an empty split)
  __shared__ double mh[PER], sh[PER];
  for (int i = tid; i < PER * nsplit; i += AD1_THREADS) {
    const int h = i / nsplit, c = i - h * nsplit;
    const double* w = wg + ((size_t)c * PER + h) * (2 + hd);
    fm[i] = __ldcg(w);
    fs[i] = __ldcg(w + 1);
  }
  __syncthreads();
  if (tid < PER) {
    double M = -INFINITY;
    for (int c = 0; c < nsplit; ++c)
      if (fs[tid * nsplit + c] != 0.0 && fm[tid * nsplit + c] > M) M = fm[tid * nsplit + c];
    mh[tid] = M;
  }
  __syncthreads();
  for (int i = tid; i < PER * nsplit; i += AD1_THREADS) {
    const double M = mh[i / nsplit], m_ = fm[i];
    fm[i] = fs[i] == 0.0 ? 0.0 : (m_ == M ? 1.0 : exp(__dsub_rn(m_, M)));
  }
  __syncthreads();
  if (tid < PER) {  // a non-empty split has S_c >= 1 or NaN (which then reaches the output)
    double S = 0.0;
    for (int c = 0; c < nsplit; ++c)
      if (fs[tid * nsplit + c] != 0.0) S = __fma_rn(fs[tid * nsplit + c], fm[tid * nsplit + c], S);
    sh[tid] = S;
  }
  __syncthreads();
  for (int i = tid; i < PER * hd; i += AD1_THREADS) {
    const int h = i / hd, d = i - h * hd;
    double O = 0.0;
    for (int c0 = 0; c0 < nsplit; c0 += 8) {
      double v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = c0 + j < nsplit ? __ldcg(wg + ((size_t)(c0 + j) * PER + h) * (2 + hd) + 2 + d) : 0.0;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < nsplit && fs[h * nsplit + c0 + j] != 0.0) O = __fma_rn(v[j], fm[h * nsplit + c0 + j], O);
    }
    out[((size_t)g * PER + h) * hd + d] = (float)__ddiv_rn(O, sh[h]);
  }
  if (tid == 0) counters[g] = 0u;  // ready for the next launch
}

// k_attn_dec_group: the batched form (configs with many sequences), in f32 like
// the batched prefill attention.  CTA (kv head g, sequence z), AG_THREADS
// threads, all `per` query heads of the group at once so each K and V row is
// read once per CTA:
//   1. scores: thread per position, f32 dots (d ascending) for every head;
//   2. per-head max and f32 sum of e_j = exp(s_j - max) (warp then block tree),
//      p_j = e_j / sum;
//   3. out[h][d] = sum_j p_j[h] * V[j, d]: thread (float4 lane d4, position
//      group jg) for every head, the groups summed in order.
constexpr int AG_THREADS = 256;
constexpr int AD_MAX_GROUP = 8;  // query heads per kv head

__global__ void __launch_bounds__(AG_THREADS)
k_attn_dec_group(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                 const int* __restrict__ pos_dev, int n_heads, int n_kv, int hd, float scale, float* __restrict__ out,
                 int max_len, pb_seq_geo geo, int* err) {
  extern __shared__ __align__(16) unsigned char ag_raw[];
  const int per = n_heads / n_kv, h4 = hd / 4;
  float* qs = reinterpret_cast<float*>(ag_raw);  // [per][hd]
  float* sp = qs + per * hd;                      // [per][max_len] scores, then probabilities
  float* part = sp + (size_t)per * max_len;       // [jgroups][per][hd]
  __shared__ float wred[AD_MAX_GROUP][AG_THREADS / 32];
  __shared__ float hstat[AD_MAX_GROUP];
  pb_pdl_trigger();
  pb_pdl_wait();
  const int g = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = *pos_dev;
  const int cache_len = pos + 1;
  if (pos < 0 || cache_len > max_len) {
    if (tid == 0 && g == 0 && blockIdx.y == 0) pb_raise(err, PB_DEVERR_BOUNDS);
    return;
  }
  const int kv_dim = n_kv * hd;
  q += blockIdx.y * geo.q + (size_t)g * per * hd;
  kc += blockIdx.y * geo.kv + (size_t)g * hd;
  vc += blockIdx.y * geo.kv + (size_t)g * hd;
  out += blockIdx.y * geo.out + (size_t)g * per * hd;
  for (int j = tid; j < cache_len; j += AG_THREADS) pb_l2_prefetch(vc + (size_t)j * kv_dim, (uint32_t)hd * 4);
  for (int i = tid; i < per * h4; i += AG_THREADS)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(q)[i];
  __syncthreads();

  float mloc[AD_MAX_GROUP];
#pragma unroll
  for (int hl = 0; hl < AD_MAX_GROUP; ++hl) mloc[hl] = -INFINITY;
  for (int j = tid; j < cache_len; j += AG_THREADS) {
    const float4* kr = reinterpret_cast<const float4*>(kc + (size_t)j * kv_dim);
    float dot[AD_MAX_GROUP];
#pragma unroll
    for (int hl = 0; hl < AD_MAX_GROUP; ++hl) dot[hl] = 0.0f;
    for (int c0 = 0; c0 < h4; c0 += 8) {
      float4 k4[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u < h4) k4[u] = kr[c0 + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (c0 + u < h4) {
#pragma unroll
          for (int hl = 0; hl < AD_MAX_GROUP; ++hl) {
            if (hl < per) {
              const float4 a = reinterpret_cast<const float4*>(qs + hl * hd)[c0 + u];
              dot[hl] = __fmaf_rn(a.x, k4[u].x, dot[hl]);
              dot[hl] = __fmaf_rn(a.y, k4[u].y, dot[hl]);
              dot[hl] = __fmaf_rn(a.z, k4[u].z, dot[hl]);
              dot[hl] = __fmaf_rn(a.w, k4[u].w, dot[hl]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int hl = 0; hl < AD_MAX_GROUP; ++hl) {
      if (hl < per) {
        const float sv = __fmul_rn(dot[hl], scale);
        sp[(size_t)hl * max_len + j] = sv;
        mloc[hl] = sv > mloc[hl] ? sv : mloc[hl];
      }
    }
  }
#pragma unroll
  for (int hl = 0; hl < AD_MAX_GROUP; ++hl) {
    if (hl < per) {
      float m = mloc[hl];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, m, o);
        m = t > m ? t : m;
      }
      if (lane == 0) wred[hl][warp] = m;
    }
  }
  __syncthreads();
  if (tid < per) {
    float m = wred[tid][0];
    for (int w = 1; w < AG_THREADS / 32; ++w) m = wred[tid][w] > m ? wred[tid][w] : m;
    hstat[tid] = m;
  }
  __syncthreads();
  float sloc[AD_MAX_GROUP];
#pragma unroll
  for (int hl = 0; hl < AD_MAX_GROUP; ++hl) {
    sloc[hl] = 0.0f;
    if (hl < per) {
      const float mx = hstat[hl];
      for (int j = tid; j < cache_len; j += AG_THREADS) {
        const float e = expf(__fsub_rn(sp[(size_t)hl * max_len + j], mx));
        sp[(size_t)hl * max_len + j] = e;
        sloc[hl] = __fadd_rn(sloc[hl], e);
      }
    }
  }
  __syncthreads();  // every thread has read hstat
#pragma unroll
  for (int hl = 0; hl < AD_MAX_GROUP; ++hl) {
    if (hl < per) {
      float t = sloc[hl];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
      if (lane == 0) wred[hl][warp] = t;
    }
  }
  __syncthreads();
  if (tid < per) {
    float t = wred[tid][0];
    for (int w = 1; w < AG_THREADS / 32; ++w) t = __fadd_rn(t, wred[tid][w]);
    hstat[tid] = t;
  }
  __syncthreads();
  for (int i = tid; i < per * cache_len; i += AG_THREADS) {
    const int hl = i / cache_len, j = i - hl * cache_len;
    sp[(size_t)hl * max_len + j] = __fdiv_rn(sp[(size_t)hl * max_len + j], hstat[hl]);
  }
  __syncthreads();

  const int jgroups = AG_THREADS / h4, d4 = tid % h4, jg = tid / h4;
  if (jg < jgroups) {
    float4 acc[AD_MAX_GROUP];
#pragma unroll
    for (int hl = 0; hl < AD_MAX_GROUP; ++hl) acc[hl] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* vl = vc + 4 * d4;
    for (int base = jg; base < cache_len; base += 8 * jgroups) {
      float4 vv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = base + u * jgroups;
        if (j < cache_len) vv[u] = *reinterpret_cast<const float4*>(vl + (size_t)j * kv_dim);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = base + u * jgroups;
        if (j < cache_len) {
#pragma unroll
          for (int hl = 0; hl < AD_MAX_GROUP; ++hl) {
            if (hl < per) {
              const float pj = sp[(size_t)hl * max_len + j];
              acc[hl].x = __fmaf_rn(pj, vv[u].x, acc[hl].x);
              acc[hl].y = __fmaf_rn(pj, vv[u].y, acc[hl].y);
              acc[hl].z = __fmaf_rn(pj, vv[u].z, acc[hl].z);
              acc[hl].w = __fmaf_rn(pj, vv[u].w, acc[hl].w);
            }
          }
        }
      }
    }
#pragma unroll
    for (int hl = 0; hl < AD_MAX_GROUP; ++hl)
      if (hl < per) reinterpret_cast<float4*>(part + ((size_t)jg * per + hl) * hd)[d4] = acc[hl];
  }
  __syncthreads();
  for (int i = tid; i < per * hd; i += AG_THREADS) {
    float t = part[i];
    for (int k = 1; k < jgroups; ++k) t = __fadd_rn(t, part[(size_t)k * per * hd + i]);
    out[i] = t;
  }
}

// k_attn_dec_split: flash-decoding form of the batched decode attention for
// head_dim 64.  CTA (kv head g, sequence z, split s) takes cache positions
// [s * AS_SPLIT, (s + 1) * AS_SPLIT); its four warps take blocks of AS_BLK
// positions in turn.  A block's K and V rows (256 bytes each) are brought into
// the warp's shared memory by bulk copies, one row per lane, completing on the
// buffer's mbarrier; two buffers per warp, so the next block loads while this
// one is used.  Per block: lane (position p = lane % 8, dim quarter lane / 8)
// dots its 16 dims of the K row with every query head of the group, two
// shuffles complete the dots; each warp keeps an online softmax per head
// (running max, sum and output, rescaled when the max grows) and accumulates
// p_j V_j with lane l owning dims 2l, 2l + 1.  The warps merge in order 0..3,
// and the last CTA of (g, z) to finish merges the splits in order
// s = 0, 1, ...  The split is fixed by position, not by the grid, so the
// result does not depend on scheduling or on how many kv heads share the
// launch.
constexpr int AS_SPLIT = 256, AS_BLK = 8, AS_WARPS = 4, AS_HD = 64, AS_KLD = AS_HD + 4;

struct as_warp_smem {
  float k[2][AS_BLK][AS_KLD];  // padded rows: lanes reading rows p..p+7 hit distinct banks
  float v[2][AS_BLK][AS_HD];
  float p[AS_BLK][AD_MAX_GROUP];
  uint64_t bar[2];
};

template <int PER>
__global__ void __launch_bounds__(AS_WARPS * 32)
k_attn_dec_split(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                 const int* __restrict__ pos_dev, int n_kv, float scale, float* __restrict__ out,
                 __half* __restrict__ out16, int hl, int max_len, pb_seq_geo geo, float* __restrict__ ws,
                 int* __restrict__ counters, int* err) {
  extern __shared__ __align__(16) unsigned char as_raw[];
  float* qs = reinterpret_cast<float*>(as_raw);  // [per][64]
  as_warp_smem* stage = reinterpret_cast<as_warp_smem*>(as_raw + AD_MAX_GROUP * AS_HD * 4);
  __shared__ int last_cta;
  pb_pdl_trigger();
  pb_pdl_wait();
  constexpr int per = PER;
  const int g = blockIdx.x, z = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = *pos_dev, cache_len = pos + 1;
  if (pos < 0 || cache_len > max_len) {
    if (tid == 0 && g == 0 && z == 0 && s == 0) pb_raise(err, PB_DEVERR_BOUNDS);
    return;
  }
  const int nsplit = (cache_len + AS_SPLIT - 1) / AS_SPLIT;
  if (s >= nsplit) return;  // past the cache: no work, not counted
  const int j0 = s * AS_SPLIT, j1 = min(cache_len, j0 + AS_SPLIT);
  const int kv_dim = n_kv * AS_HD;
  q += z * geo.q + (size_t)g * per * AS_HD;
  kc += z * geo.kv + (size_t)g * AS_HD;
  vc += z * geo.kv + (size_t)g * AS_HD;
  as_warp_smem* w = stage + warp;
  if (lane == 0) {
    pb_mbar_init(&w->bar[0], 1);
    pb_mbar_init(&w->bar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < per * (AS_HD / 4); i += AS_WARPS * 32)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(q)[i];
  __syncthreads();

  const int nblk = (j1 - j0 + AS_BLK - 1) / AS_BLK;
  // block b's live K rows (lanes 0..7) and V rows (lanes 8..15) into buffer buf
  auto issue = [&](int b, int buf) {
    const int jb = j0 + b * AS_BLK, live = min(AS_BLK, j1 - jb);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // after the warp's reads of this buffer
    if (lane == 0) pb_mbar_arrive_tx(&w->bar[buf], (uint32_t)live * AS_HD * 4 * 2);
    __syncwarp();
    const int r = lane & 7;
    if (lane < 16 && r < live) {
      const size_t row = (size_t)(jb + r) * kv_dim;
      if (lane < 8) pb_bulk_g2s(&w->k[buf][r][0], kc + row, AS_HD * 4, &w->bar[buf]);
      else pb_bulk_g2s(&w->v[buf][r][0], vc + row, AS_HD * 4, &w->bar[buf]);
    }
  };
  float m[PER], l[PER], acc[PER][2];
#pragma unroll
  for (int h = 0; h < PER; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
    acc[h][0] = acc[h][1] = 0.0f;
  }
  const int p = lane & 7, qd = lane >> 3;
  if (warp < nblk) issue(warp, 0);
  int it = 0;
  bool ok = true;
  for (int b = warp; b < nblk && ok; b += AS_WARPS, ++it) {
    const int buf = it & 1;
    if (b + AS_WARPS < nblk) issue(b + AS_WARPS, buf ^ 1);
    if (!(ok = pb_mbar_wait_sleep(&w->bar[buf], (it >> 1) & 1, err))) break;
    const int jb = j0 + b * AS_BLK;
    const bool live = jb + p < j1;
    float dot[PER];
#pragma unroll
    for (int h = 0; h < PER; ++h) dot[h] = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 k4 = *reinterpret_cast<const float4*>(&w->k[buf][p][qd * 16 + 4 * c]);
#pragma unroll
      for (int h = 0; h < PER; ++h) {
        const float4 a = *reinterpret_cast<const float4*>(qs + h * AS_HD + qd * 16 + 4 * c);
        dot[h] = __fmaf_rn(a.x, k4.x, dot[h]);
        dot[h] = __fmaf_rn(a.y, k4.y, dot[h]);
        dot[h] = __fmaf_rn(a.z, k4.z, dot[h]);
        dot[h] = __fmaf_rn(a.w, k4.w, dot[h]);
      }
    }
    float e[PER];
#pragma unroll
    for (int h = 0; h < PER; ++h) {
      float d = __fadd_rn(dot[h], __shfl_xor_sync(0xffffffffu, dot[h], 8));
      d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 16));
      const float sc = live ? __fmul_rn(d, scale) : -INFINITY;
      float bm = sc;
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float mn = fmaxf(m[h], bm);  // finite: the block's first position is live
      const float corr = __expf(__fsub_rn(m[h], mn));  // 0 while m is -inf
      e[h] = live ? __expf(__fsub_rn(sc, mn)) : 0.0f;
      float bs = e[h];
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) bs = __fadd_rn(bs, __shfl_xor_sync(0xffffffffu, bs, o));
      l[h] = __fmaf_rn(l[h], corr, bs);
      acc[h][0] = __fmul_rn(acc[h][0], corr);
      acc[h][1] = __fmul_rn(acc[h][1], corr);
      m[h] = mn;
    }
    if (qd == 0) {
#pragma unroll
      for (int h = 0; h < PER; ++h) w->p[p][h] = e[h];
    }
    __syncwarp();
    const int nlive = min(AS_BLK, j1 - jb);  // rows past the cache were not loaded
#pragma unroll
    for (int jj = 0; jj < AS_BLK; ++jj) {
      if (jj < nlive) {
        const float2 v = *reinterpret_cast<const float2*>(&w->v[buf][jj][2 * lane]);
        float pj[PER];
        if constexpr (PER % 4 == 0) {
#pragma unroll
          for (int h = 0; h < PER; h += 4) {
            const float4 t = *reinterpret_cast<const float4*>(&w->p[jj][h]);
            pj[h] = t.x;
            pj[h + 1] = t.y;
            pj[h + 2] = t.z;
            pj[h + 3] = t.w;
          }
        } else {
#pragma unroll
          for (int h = 0; h < PER; ++h) pj[h] = w->p[jj][h];
        }
#pragma unroll
        for (int h = 0; h < PER; ++h) {
          acc[h][0] = __fmaf_rn(pj[h], v.x, acc[h][0]);
          acc[h][1] = __fmaf_rn(pj[h], v.y, acc[h][1]);
        }
      }
    }
    __syncwarp();  // the block's buffers and p are free for the next issue
  }
  if (!ok) {
    // a copy that never completed: wait (bounded) for the warp's other buffer
    // too, so no bulk copy is in flight when the CTA exits
    pb_mbar_wait_sleep(&w->bar[(it + 1) & 1], ((it + 1) >> 1) & 1, err);
  }
  __syncthreads();  // every warp is done with its staging: reuse it for the merge
  float* mg = reinterpret_cast<float*>(stage);  // [warp][per][2 + 64]: max, sum, output
  const int rec = 2 + AS_HD;
#pragma unroll
  for (int h = 0; h < PER; ++h) {
    float* r = mg + ((size_t)warp * per + h) * rec;
    if (lane == 0) {
      r[0] = m[h];
      r[1] = l[h];
    }
    r[2 + 2 * lane] = acc[h][0];
    r[3 + 2 * lane] = acc[h][1];
  }
  __syncthreads();
  const bool split = nsplit > 1;
  float* part = ws + (((size_t)z * n_kv + g) * ((max_len + AS_SPLIT - 1) / AS_SPLIT) + s) * per * rec;
  for (int i = tid; i < per * AS_HD; i += AS_WARPS * 32) {
    const int h = i / AS_HD, d = i % AS_HD;
    float M = -INFINITY;
    for (int wi = 0; wi < AS_WARPS; ++wi) M = fmaxf(M, mg[((size_t)wi * per + h) * rec]);
    float L = 0.0f, O = 0.0f;
    for (int wi = 0; wi < AS_WARPS; ++wi) {
      const float* r = mg + ((size_t)wi * per + h) * rec;
      const float f = r[0] == -INFINITY ? 0.0f : __expf(__fsub_rn(r[0], M));
      L = __fmaf_rn(r[1], f, L);
      O = __fmaf_rn(r[2 + d], f, O);
    }
    if (!split) {
      const int c = g * per * AS_HD + i;
      if (out16 && hl) pb_store_hl(out16, pb_hl_index(z * 2 * geo.out, c), __fdiv_rn(O, L));
      else if (out16) out16[z * geo.out + c] = __float2half_rn(__fdiv_rn(O, L));
      else out[z * geo.out + c] = __fdiv_rn(O, L);
    } else {
      if (d == 0) {
        part[(size_t)h * rec] = M;
        part[(size_t)h * rec + 1] = L;
      }
      part[(size_t)h * rec + 2 + d] = O;
    }
  }
  if (!split) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) last_cta = atomicAdd(counters + (size_t)z * n_kv + g, 1) == nsplit - 1;
  __syncthreads();
  if (!last_cta) return;
  __threadfence();
  const float* parts = ws + ((size_t)z * n_kv + g) * ((max_len + AS_SPLIT - 1) / AS_SPLIT) * per * rec;
  for (int i = tid; i < per * AS_HD; i += AS_WARPS * 32) {
    const int h = i / AS_HD, d = i % AS_HD;
    float M = -INFINITY;
    for (int si = 0; si < nsplit; ++si) M = fmaxf(M, __ldcg(parts + ((size_t)si * per + h) * rec));
    float L = 0.0f, O = 0.0f;
    for (int si = 0; si < nsplit; ++si) {
      const float* r = parts + ((size_t)si * per + h) * rec;
      const float f = __expf(__fsub_rn(__ldcg(r), M));
      L = __fmaf_rn(__ldcg(r + 1), f, L);
      O = __fmaf_rn(__ldcg(r + 2 + d), f, O);
    }
    const int c = g * per * AS_HD + i;
    if (out16 && hl) pb_store_hl(out16, pb_hl_index(z * 2 * geo.out, c), __fdiv_rn(O, L));
    else if (out16) out16[z * geo.out + c] = __float2half_rn(__fdiv_rn(O, L));
    else out[z * geo.out + c] = __fdiv_rn(O, L);
  }
  if (tid == 0) counters[(size_t)z * n_kv + g] = 0;  // for the next launch
}

static size_t as_smem() { return (size_t)AD_MAX_GROUP * AS_HD * 4 + AS_WARPS * sizeof(as_warp_smem); }

// Workspace floats and counters k_attn_dec_split needs for nseq sequences.
size_t pb_attn_split_ws_floats(int n_heads, int n_kv, int max_len, int nseq) {
  return (size_t)nseq * n_kv * ((max_len + AS_SPLIT - 1) / AS_SPLIT) * (n_heads / n_kv) * (2 + AS_HD);
}

static size_t ag_smem(int per, int hd, int max_len) {
  return ((size_t)per * hd + (size_t)per * max_len + (size_t)(AG_THREADS / (hd / 4)) * per * hd) * 4;
}

// Whether k_attn_dec takes this shape (the callers fall back to the general
// cached attention otherwise).
bool pb_attn_decode_ok(int n_heads, int n_kv, int hd, int max_len) {
  return n_kv > 0 && n_heads % n_kv == 0 && hd % 4 == 0 && hd <= AF_MAX_HD &&
         (size_t)AF_PART * 8 + (size_t)max_len * 4 <= 200 * 1024;
}

// The batched form also needs <= AD_MAX_GROUP query heads per kv head and its
// per-head scores in shared memory.
bool pb_attn_decode_group_ok(int n_heads, int n_kv, int hd, int max_len) {
  return pb_attn_decode_ok(n_heads, n_kv, hd, max_len) && n_heads / n_kv <= AD_MAX_GROUP && hd / 4 <= AG_THREADS &&
         ag_smem(n_heads / n_kv, hd, max_len) <= 200 * 1024;
}

// Decode attention for one query at *pos_dev over the cache (nseq sequences
// of a batched launch, `geo` apart).
int pb_launch_attn_decode(pb_ctx* ctx, const float* q, const float* kc, const float* vc, const int* pos_dev,
                          int n_heads, int n_kv, int hd, float* out, int max_len, int nseq, pb_seq_geo geo,
                          float* ws, size_t ws_floats, int* counters, __half* out16, int hl16) {
  if (!(nseq > 1 ? pb_attn_decode_group_ok(n_heads, n_kv, hd, max_len) : pb_attn_decode_ok(n_heads, n_kv, hd, max_len)))
    return pb_set_error(ctx, PB_ERR_ARG, "decode attention needs n_heads %% n_kv == 0, head_dim %% 4 == 0, "
                                         "head_dim <= %d and max_len <= %d", AF_MAX_HD, (200 * 1024 - AF_PART * 8) / 4);
  const double scale = 1.0 / sqrt((double)hd);  // llama-streaming.js:546
  if (nseq > 1) {
    const int per = n_heads / n_kv;
    if (hd == AS_HD && ws && counters && ws_floats >= pb_attn_split_ws_floats(n_heads, n_kv, max_len, nseq)) {
      const dim3 grid(n_kv, nseq, (max_len + AS_SPLIT - 1) / AS_SPLIT);
      switch (per) {
#define PB_AS_CASE(P)                                                                                              \
  case P:                                                                                                          \
    return pb_launch(ctx, "k_attn_dec_split", true, k_attn_dec_split<P>, grid, dim3(AS_WARPS * 32), as_smem(), q, \
                     kc, vc, pos_dev, n_kv, (float)scale, out, out16, hl16, max_len, geo, ws, counters, ctx->d_err);
        PB_AS_CASE(1) PB_AS_CASE(2) PB_AS_CASE(3) PB_AS_CASE(4) PB_AS_CASE(5) PB_AS_CASE(6) PB_AS_CASE(7)
        PB_AS_CASE(8)
#undef PB_AS_CASE
        default: break;
      }
    }
    if (out16) return pb_set_error(ctx, PB_ERR_ARG, "f16 attention output needs the split decode attention");
    return pb_launch(ctx, "k_attn_dec_group", true, k_attn_dec_group, dim3(n_kv, nseq), dim3(AG_THREADS),
                     ag_smem(per, hd, max_len), q, kc, vc, pos_dev, n_heads, n_kv, hd, (float)scale, out, max_len, geo,
                     ctx->d_err);
  }
  const size_t smem = (size_t)AF_PART * 8 + (size_t)max_len * 4;
  return pb_launch(ctx, "k_attn_dec", true, k_attn_dec, dim3(n_heads, nseq), dim3(AF_THREADS), smem, q, kc, vc,
                   pos_dev, n_heads, n_kv, hd, scale, out, max_len, geo, ctx->d_err);
}

// Splits of the one-sequence decode attention: at most 8 per kv head and at
// most AD1_MAX_P positions each.
int pb_attn_dec1_splits(int n_kv, int max_len, int sm_count) {
  // up to 8 splits per kv head: more splits shorten each CTA's walk over the
  // cache but lengthen the merge; 8 measured best at 128-640 positions
  int ns = sm_count / n_kv;
  if (ns > 8) ns = 8;
  if (ns < 1) ns = 1;
  const int need = (max_len + AD1_MAX_P - 1) / AD1_MAX_P;
  return ns < need ? need : ns;
}

size_t pb_attn_dec1_ws_doubles(int n_heads, int n_kv, int hd, int nsplit) {
  return (size_t)n_kv * nsplit * (n_heads / n_kv) * (2 + hd);
}

static size_t ad1_smem(int per, int hd) {
  return (size_t)per * AD1_MAX_P * 8 + (size_t)AD1_GROUPS * per * hd * 8 + (size_t)per * hd * 4;
}

bool pb_attn_dec1_ok(int n_heads, int n_kv, int hd) {
  return n_kv > 0 && n_heads % n_kv == 0 && n_heads / n_kv <= 8 && hd % 4 == 0 && hd <= AD1_MAX_HD &&
         ad1_smem(n_heads / n_kv, hd) <= 200 * 1024;
}

// The position-split decode attention of one sequence; ws holds
// pb_attn_dec1_ws_doubles doubles, counters n_kv zeroed words (the kernel
// leaves them zero).
int pb_launch_attn_dec1(pb_ctx* ctx, const float* q, const float* kc, const float* vc, const int* pos_dev,
                        int n_heads, int n_kv, int hd, float* out, int max_len, int nsplit, double* ws,
                        unsigned int* counters) {
  if (!pb_attn_dec1_ok(n_heads, n_kv, hd) || nsplit <= 0 || nsplit > AD1_MAX_P / 2 ||
      (size_t)(max_len + nsplit - 1) / nsplit > AD1_MAX_P)
    return pb_set_error(ctx, PB_ERR_ARG, "split decode attention: unsupported shape");
  const double scale = 1.0 / sqrt((double)hd);  // llama-streaming.js:546
  const dim3 grid(n_kv, nsplit);
  const int per = n_heads / n_kv;
  switch (per) {
#define PB_AD1_CASE(P)                                                                                          \
  case P:                                                                                                       \
    return pb_launch(ctx, "k_attn_dec1", true, k_attn_dec1<P>, grid, dim3(AD1_THREADS), ad1_smem(P, hd), q, kc, \
                     vc, pos_dev, n_kv, hd, scale, out, max_len, nsplit, ws, counters, ctx->d_err);
    PB_AD1_CASE(1) PB_AD1_CASE(2) PB_AD1_CASE(3) PB_AD1_CASE(4) PB_AD1_CASE(5) PB_AD1_CASE(6) PB_AD1_CASE(7)
    PB_AD1_CASE(8)
#undef PB_AD1_CASE
    default:
      return pb_set_error(ctx, PB_ERR_ARG, "split decode attention: at most 8 query heads per kv head");
  }
}

// k_attn_dec_fast<PER>: the fast mode's decode attention for one query
// (head_dim 64), the f32 form of k_attn_dec1 above: CTA (kv head g, split sp)
// of a cluster per kv head (pb_attn_fast.cuh).
//   - before griddepcontrol.wait: the split's K and V rows j < pos (final:
//     written by earlier steps) into shared memory by cp.async, so their
//     latency overlaps the projection that is still running;
//   - after it: q and the row at pos (this step's), then aq_attend.
template <int PER>
__global__ void __launch_bounds__(AQ_THREADS)
k_attn_dec_fast(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                const int* __restrict__ pos_dev, int n_kv, float scale, float* __restrict__ out, int max_len, int pmax,
                int* err) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ __align__(16) float aq_sm[];
  float* ks = aq_sm;                                  // [pmax][AQ_KLD] (padded: conflict-free row reads)
  float* vs = ks + (size_t)pmax * AQ_KLD;             // [pmax][64]
  float* sc = vs + (size_t)pmax * AQ_HD;              // [PER][pmax]: scores, then p
  float* qs = sc + (size_t)PER * pmax;                // [PER][64]
  float* gp = qs + PER * AQ_HD;                       // [4][PER][64]: PV partials of the position groups
  __shared__ aq_parts<PER> pt;
  const int g = blockIdx.x, sp = (int)cl.block_rank(), nsplit = (int)cl.num_blocks(), tid = threadIdx.x;
  const int pos = *pos_dev;  // final: the step's first kernel starts after the previous step ended
  const int cache_len = pos + 1;
  const int P = (cache_len + nsplit - 1) / nsplit;
  if (pos < 0 || cache_len > max_len || P > pmax) {  // the same for every CTA: all leave before any barrier
    pb_pdl_trigger();
    pb_pdl_wait();  // a dependent grid ends after the one before it, on every path
    if (tid == 0 && g == 0 && sp == 0) pb_raise(err, PB_DEVERR_BOUNDS);
    return;
  }
  const int kv_dim = n_kv * AQ_HD;
  const int j0 = sp * P;
  const int n = cache_len - j0 < 0 ? 0 : (cache_len - j0 < P ? cache_len - j0 : P);
  const bool has_pos = pos >= j0 && pos < j0 + n;
  const int npre = has_pos ? n - 1 : n;  // rows before pos: final already
  const float* kb = kc + (size_t)g * AQ_HD;
  const float* vb = vc + (size_t)g * AQ_HD;
  for (int i = tid; i < npre * 16; i += AQ_THREADS) {
    const int r = i >> 4, c = i & 15;
    const size_t src = (size_t)(j0 + r) * kv_dim + 4 * c;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(pb_smem_addr(ks + r * AQ_KLD + 4 * c)),
                 "l"(kb + src) : "memory");
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(pb_smem_addr(vs + r * AQ_HD + 4 * c)),
                 "l"(vb + src) : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  pb_pdl_trigger();
  pb_pdl_wait();  // q and the cache row at pos come from the projection
  if (has_pos && tid < 32) {
    const int r = pos - j0, c = tid & 15;
    const float* src = (tid < 16 ? kb : vb) + (size_t)pos * kv_dim + 4 * c;
    float* dst = tid < 16 ? ks + r * AQ_KLD + 4 * c : vs + r * AQ_HD + 4 * c;
    *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src);
  }
  for (int i = tid; i < PER * AQ_HD / 4; i += AQ_THREADS)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(q + (size_t)g * PER * AQ_HD)[i];
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  aq_attend<PER>(cl, ks, vs, sc, qs, gp, pt, n, pmax, scale, out + (size_t)g * PER * AQ_HD);
}

// Whether the fast decode attention takes this shape (max_len positions in
// at most AQ_MAX_SPLIT splits of at most AQ_MAXP).
bool pb_attn_dec_fast_ok(int n_heads, int n_kv, int hd, int max_len) {
  return n_kv > 0 && n_heads % n_kv == 0 && n_heads / n_kv <= 8 && hd == AQ_HD &&
         (max_len + AQ_MAX_SPLIT - 1) / AQ_MAX_SPLIT <= AQ_MAXP;
}

int pb_launch_attn_dec_fast(pb_ctx* ctx, const float* q, const float* kc, const float* vc, const int* pos_dev,
                            int n_heads, int n_kv, int hd, float* out, int max_len) {
  if (!pb_attn_dec_fast_ok(n_heads, n_kv, hd, max_len))
    return pb_set_error(ctx, PB_ERR_ARG, "fast decode attention: unsupported shape");
  const int nsplit = AQ_MAX_SPLIT, pmax = (max_len + nsplit - 1) / nsplit, per = n_heads / n_kv;
  const float scale = (float)(1.0 / sqrt((double)hd));  // llama-streaming.js:546
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_kv, nsplit);
  cfg.blockDim = dim3(AQ_THREADS);
  cfg.dynamicSmemBytes = aq_smem(per, pmax);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = nsplit;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ctx->pdl ? 2 : 1;
  cudaError_t e = cudaErrorInvalidValue;
  switch (per) {
#define PB_AQ_CASE(P) \
  case P: e = cudaLaunchKernelEx(&cfg, k_attn_dec_fast<P>, q, kc, vc, pos_dev, n_kv, scale, out, max_len, pmax, ctx->d_err); break;
    PB_AQ_CASE(1) PB_AQ_CASE(2) PB_AQ_CASE(3) PB_AQ_CASE(4) PB_AQ_CASE(5) PB_AQ_CASE(6) PB_AQ_CASE(7) PB_AQ_CASE(8)
#undef PB_AQ_CASE
    default: break;
  }
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, "k_attn_dec_fast");
  return pb_check_launch(ctx, "k_attn_dec_fast");
}

extern "C" int pb_attn_decode(pb_ctx* ctx, const float* q, const float* kc, const float* vc, int pos, int n_heads,
                              int n_kv, int hd, int max_len, float* out) {
  if (!ctx || !q || !kc || !vc || !out || n_heads <= 0 || n_kv <= 0 || hd <= 0 || pos < 0 || pos >= max_len)
    return pb_set_error(ctx, PB_ERR_ARG, "pb_attn_decode: bad arguments (pos %d, max_len %d)", pos, max_len);
  if (!pb_attn_dec1_ok(n_heads, n_kv, hd))
    return pb_set_error(ctx, PB_ERR_ARG, "pb_attn_decode: needs n_heads %% n_kv == 0, at most 8 query heads per kv "
                                         "head, head_dim %% 4 == 0 and head_dim <= %d", AD1_MAX_HD);
  const bool fast = ctx->matvec_mode == PB_MATVEC_FAST && pb_attn_dec_fast_ok(n_heads, n_kv, hd, max_len);
  const int nsplit = pb_attn_dec1_splits(n_kv, max_len, ctx->sm_count);
  const size_t wsb = fast ? 0 : pb_attn_dec1_ws_doubles(n_heads, n_kv, hd, nsplit) * 8;
  PB_TRY(pb_ensure_scratch(ctx, wsb + 256 + (size_t)n_kv * 4 + 16));
  double* ws = (double*)ctx->scratch;
  unsigned int* cnt = (unsigned int*)((char*)ctx->scratch + ((wsb + 255) & ~(size_t)255));
  int* pos_dev = (int*)(cnt + n_kv);
  PB_TRY_CUDA(ctx, cudaMemsetAsync(cnt, 0, (size_t)n_kv * 4, ctx->stream));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(pos_dev, &pos, 4, cudaMemcpyHostToDevice, ctx->stream));
  if (fast) PB_TRY(pb_launch_attn_dec_fast(ctx, q, kc, vc, pos_dev, n_heads, n_kv, hd, out, max_len));
  else PB_TRY(pb_launch_attn_dec1(ctx, q, kc, vc, pos_dev, n_heads, n_kv, hd, out, max_len, nsplit, ws, cnt));
  return pb_wait(ctx);  // the position's host copy must outlive the transfer
}

int pb_setup_ops_kernels(void) {
  for (auto k : {k_attn_prefill_tc<1>, k_attn_prefill_tc<3>})
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ft_smem(3)) != cudaSuccess)
      return PB_ERR_CUDA;
  cudaError_t e = cudaFuncSetAttribute(k_attn_cached, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_attn_dec, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_attn_dec_group, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  for (auto k : {k_attn_dec_split<1>, k_attn_dec_split<2>, k_attn_dec_split<3>, k_attn_dec_split<4>,
                 k_attn_dec_split<5>, k_attn_dec_split<6>, k_attn_dec_split<7>, k_attn_dec_split<8>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)as_smem());
  for (auto k : {k_attn_dec_fast<1>, k_attn_dec_fast<2>, k_attn_dec_fast<3>, k_attn_dec_fast<4>,
                 k_attn_dec_fast<5>, k_attn_dec_fast<6>, k_attn_dec_fast<7>, k_attn_dec_fast<8>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  for (auto k : {k_attn_dec1<1>, k_attn_dec1<2>, k_attn_dec1<3>, k_attn_dec1<4>, k_attn_dec1<5>, k_attn_dec1<6>,
                 k_attn_dec1<7>, k_attn_dec1<8>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  return e == cudaSuccess ? PB_OK : PB_ERR_CUDA;
}
