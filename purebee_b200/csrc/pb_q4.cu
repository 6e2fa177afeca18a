// pb_q4.cu - quantized matvec and LM-head kernels for sm_100a.
//
// Matvec (wasm-q4.js:118-267 Q4_0, :275-435 Q4_1).  The reference computes,
// per row and per lane L in 0..3, a per-block partial
//     blockAcc[L] = sum over g in {0,4,8,12} of  (lo-8)*x[g+L], (hi-8)*x[g+16+L]
// in f32 with a separate multiply and add, then the in-order chain
//     acc[L] = acc[L] + blockAcc[L]*d        (blocks b = 0, 1, 2, ...)
// and y = (acc1 + acc3) + (acc0 + acc2).  The per-block partials are
// independent, so eight producer warps compute them for all (row, block)
// pairs of a row tile in parallel (lanes = rows, one coalesced 16 B load per
// lane); one consumer warp runs the in-order chains from a shared-memory ring
// as chunks of blocks complete (mbarrier handshake, bounded waits).  The
// result is bit-identical to the reference's WASM kernel.
//
// Head (wasm-q4.js:447-566 batch_dot over the table gguf.js:239-286
// dequantizes).  The reference's lane L chain runs over k = L, L+4, ... of
// the f32 table.  Each lane of a warp owns one vocab row and walks all blocks;
// the dequantized value (q-8)*d is rebuilt exactly with one FFMA from a
// magic-exponent float, then p = h[k]*e and acc[L] += p as in the reference.
// The greedy argmax (llama-streaming.js:899-909) is fused as an ordered-key
// atomicMax.
#include <stdio.h>

#include "pb_internal.cuh"

// ---------------------------------------------------------------------------
// mbarrier helpers with bounded waits
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar)) : "memory");
}
// Wait for the phase with the given parity to complete; gives up after about
// two seconds of device clock, records PB_DEVERR_WAIT and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  uint32_t addr = smem_u32(bar);
  long long t0 = clock64();
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 255) == 255 && clock64() - t0 > 4000000000LL) {
      pb_raise(err, PB_DEVERR_WAIT);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// exact nibble -> float conversions
// ---------------------------------------------------------------------------
// A float whose exponent makes the mantissa bit at position p worth 1 holds
// 2^(23-p) + n when the nibble n sits at bits p..p+3; subtracting 2^(23-p) + 8
// leaves exactly n - 8.

#define PB_MAG0 0x4B000000u   // p = 0  -> 2^23
#define PB_MAG4 0x49000000u   // p = 4  -> 2^19
#define PB_MAG8 0x47000000u   // p = 8  -> 2^15
#define PB_MAG12 0x45000000u  // p = 12 -> 2^11
#define PB_MAG16 0x43000000u  // p = 16 -> 2^7

__device__ __forceinline__ float mag(uint32_t w, uint32_t mask, uint32_t e) { return __uint_as_float((w & mask) | e); }

// x chunk (4 floats) i of block b in the swizzled shared copy of x.
__device__ __forceinline__ float4 xchunk(const float4* xs, int b, int i) { return xs[b * 8 + (i ^ (b & 7))]; }

// Partial sums of one Q4_0 block for the four lanes (wasm-q4.js:193-229),
// already multiplied by d.
__device__ __forceinline__ float4 q4_0_block(uint4 pl, float d, const float4* xs, int b) {
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  uint32_t wv[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t w = wv[g], w2 = w >> 16;
    float4 xl = xchunk(xs, b, g), xh = xchunk(xs, b, 4 + g);
    float l0 = __fsub_rn(mag(w, 0xFu, PB_MAG0), 8388616.0f);
    float h0 = __fsub_rn(mag(w, 0xF0u, PB_MAG4), 524296.0f);
    float l1 = __fsub_rn(mag(w, 0xF00u, PB_MAG8), 32776.0f);
    float h1 = __fsub_rn(mag(w, 0xF000u, PB_MAG12), 2056.0f);
    float l2 = __fsub_rn(mag(w, 0xF0000u, PB_MAG16), 136.0f);
    float h2 = __fsub_rn(mag(w2, 0xF0u, PB_MAG4), 524296.0f);
    float l3 = __fsub_rn(mag(w2, 0xF00u, PB_MAG8), 32776.0f);
    float h3 = __fsub_rn(mag(w2, 0xF000u, PB_MAG12), 2056.0f);
    a0 = __fadd_rn(a0, __fmul_rn(l0, xl.x));
    a1 = __fadd_rn(a1, __fmul_rn(l1, xl.y));
    a2 = __fadd_rn(a2, __fmul_rn(l2, xl.z));
    a3 = __fadd_rn(a3, __fmul_rn(l3, xl.w));
    a0 = __fadd_rn(a0, __fmul_rn(h0, xh.x));
    a1 = __fadd_rn(a1, __fmul_rn(h1, xh.y));
    a2 = __fadd_rn(a2, __fmul_rn(h2, xh.z));
    a3 = __fadd_rn(a3, __fmul_rn(h3, xh.w));
  }
  return make_float4(__fmul_rn(a0, d), __fmul_rn(a1, d), __fmul_rn(a2, d), __fmul_rn(a3, d));
}

// Q4_1 (wasm-q4.js:357-398): nibAcc += n*x, xAcc += x per lane (lo then hi),
// block value nibAcc*delta + xAcc*min.
__device__ __forceinline__ float4 q4_1_block(uint4 pl, float dl, float mn, const float4* xs, int b) {
  float n0 = 0, n1 = 0, n2 = 0, n3 = 0, s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  uint32_t wv[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t w = wv[g], w2 = w >> 16;
    float4 xl = xchunk(xs, b, g), xh = xchunk(xs, b, 4 + g);
    float l0 = __fsub_rn(mag(w, 0xFu, PB_MAG0), 8388608.0f);
    float h0 = __fsub_rn(mag(w, 0xF0u, PB_MAG4), 524288.0f);
    float l1 = __fsub_rn(mag(w, 0xF00u, PB_MAG8), 32768.0f);
    float h1 = __fsub_rn(mag(w, 0xF000u, PB_MAG12), 2048.0f);
    float l2 = __fsub_rn(mag(w, 0xF0000u, PB_MAG16), 128.0f);
    float h2 = __fsub_rn(mag(w2, 0xF0u, PB_MAG4), 524288.0f);
    float l3 = __fsub_rn(mag(w2, 0xF00u, PB_MAG8), 32768.0f);
    float h3 = __fsub_rn(mag(w2, 0xF000u, PB_MAG12), 2048.0f);
    n0 = __fadd_rn(n0, __fmul_rn(l0, xl.x)); s0 = __fadd_rn(s0, xl.x);
    n1 = __fadd_rn(n1, __fmul_rn(l1, xl.y)); s1 = __fadd_rn(s1, xl.y);
    n2 = __fadd_rn(n2, __fmul_rn(l2, xl.z)); s2 = __fadd_rn(s2, xl.z);
    n3 = __fadd_rn(n3, __fmul_rn(l3, xl.w)); s3 = __fadd_rn(s3, xl.w);
    n0 = __fadd_rn(n0, __fmul_rn(h0, xh.x)); s0 = __fadd_rn(s0, xh.x);
    n1 = __fadd_rn(n1, __fmul_rn(h1, xh.y)); s1 = __fadd_rn(s1, xh.y);
    n2 = __fadd_rn(n2, __fmul_rn(h2, xh.z)); s2 = __fadd_rn(s2, xh.z);
    n3 = __fadd_rn(n3, __fmul_rn(h3, xh.w)); s3 = __fadd_rn(s3, xh.w);
  }
  return make_float4(__fadd_rn(__fmul_rn(n0, dl), __fmul_rn(s0, mn)), __fadd_rn(__fmul_rn(n1, dl), __fmul_rn(s1, mn)),
                     __fadd_rn(__fmul_rn(n2, dl), __fmul_rn(s2, mn)), __fadd_rn(__fmul_rn(n3, dl), __fmul_rn(s3, mn)));
}

// ---------------------------------------------------------------------------
// matvec kernel
// ---------------------------------------------------------------------------

constexpr int MV_NP = 8;     // producer warps
constexpr int MV_SLOTS = 4;  // ring depth (chunks)
constexpr int MV_PF = 2;     // chunks of weights prefetched into registers

template <int R>
struct MvShape {
  static constexpr int G = 32 / R;        // blocks per producer warp step
  static constexpr int CH = MV_NP * G;    // blocks per chunk
  static constexpr int PS_FLOAT4 = MV_SLOTS * CH * R;
};

// Epilogue flags
#define MV_EPI_RESIDUAL 1

template <int R, int TYPE>
__global__ void __launch_bounds__((MV_NP + 1) * 32)
k_matvec(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, const uint16_t* __restrict__ msc,
         int N, int nb, const float* __restrict__ x, float* __restrict__ y, const float* __restrict__ residual,
         int row_begin, int row_end, int* err) {
  using S = MvShape<R>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* bar_full = (uint64_t*)smem_raw;
  uint64_t* bar_empty = bar_full + MV_SLOTS;
  float4* ps = (float4*)(smem_raw + 128);
  float4* xs = ps + S::PS_FLOAT4;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = row_begin + blockIdx.x * R;
  const int tile = row0 >> 5, r_in_tile0 = row0 & 31;
  const int K = nb * 32;

  if (tid == 0) {
    for (int s = 0; s < MV_SLOTS; ++s) {
      mbar_init(&bar_full[s], MV_NP * 32);
      mbar_init(&bar_empty[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // x -> shared memory, float4 chunks swizzled within each 32-value block
  for (int c = tid; c < K / 4; c += blockDim.x) {
    int b = c >> 3, i = c & 7;
    xs[b * 8 + (i ^ (b & 7))] = reinterpret_cast<const float4*>(x)[c];
  }
  __syncthreads();

  const int nchunks = (nb + S::CH - 1) / S::CH;

  if (warp < MV_NP) {
    // ---------------- producers ----------------
    const int r = lane % R, s = lane / R;
    const int grow = row0 + r;
    const size_t tile_base = (size_t)tile * nb;
    uint4 pf_q[MV_PF];
    uint16_t pf_d[MV_PF], pf_m[MV_PF];
    auto load = [&](int c, int k) {
      int b = c * S::CH + warp * S::G + s;
      if (c < nchunks && b < nb) {
        size_t slot = (tile_base + b) * 32 + r_in_tile0 + r;
        pf_q[k] = __ldg(reinterpret_cast<const uint4*>(qs) + slot);
        pf_d[k] = __ldg(dsc + slot);
        if (TYPE == PB_TYPE_Q4_1) pf_m[k] = __ldg(msc + slot);
      }
    };
#pragma unroll
    for (int k = 0; k < MV_PF; ++k) load(k, k);
    bool ok = true;
    for (int c0 = 0; c0 < nchunks; c0 += MV_PF) {
#pragma unroll
      for (int k = 0; k < MV_PF; ++k) {
        int c = c0 + k;
        if (c >= nchunks) break;
        int slot = c % MV_SLOTS;
        if (c >= MV_SLOTS && ok) ok = mbar_wait(&bar_empty[slot], ((c / MV_SLOTS) - 1) & 1, err);
        int b = c * S::CH + warp * S::G + s;
        float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b < nb) {
          if (TYPE == PB_TYPE_Q4_0) p = q4_0_block(pf_q[k], pb_f16_wasm(pf_d[k]), xs, b);
          else p = q4_1_block(pf_q[k], pb_f16_wasm(pf_d[k]), pb_f16_wasm(pf_m[k]), xs, b);
        }
        (void)grow;
        ps[(slot * S::CH + warp * S::G + s) * R + r] = p;
        load(c + MV_PF, k);
        mbar_arrive(&bar_full[slot]);
      }
    }
  } else {
    // ---------------- consumer: in-order chains ----------------
    constexpr int CPL = (R * 4) / 32;  // chains per lane
    const int L = lane & 3, rq = lane >> 2;
    float acc[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) acc[j] = 0.0f;
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      int slot = c % MV_SLOTS;
      if (ok) ok = mbar_wait(&bar_full[slot], (c / MV_SLOTS) & 1, err);
      int nblk = nb - c * S::CH;
      nblk = nblk < S::CH ? nblk : S::CH;
      const float* pslot = reinterpret_cast<const float*>(ps + slot * S::CH * R);
      for (int bb = 0; bb < nblk; ++bb) {
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[j] = __fadd_rn(acc[j], pslot[(bb * R + rq + 8 * j) * 4 + L]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_empty[slot]);
    }
    // y = (acc1 + acc3) + (acc0 + acc2) across the four lanes of a row
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      float a0 = __shfl_sync(0xffffffffu, acc[j], (lane & ~3) + 0);
      float a1 = __shfl_sync(0xffffffffu, acc[j], (lane & ~3) + 1);
      float a2 = __shfl_sync(0xffffffffu, acc[j], (lane & ~3) + 2);
      float a3 = __shfl_sync(0xffffffffu, acc[j], (lane & ~3) + 3);
      float v = __fadd_rn(__fadd_rn(a1, a3), __fadd_rn(a0, a2));
      int row = row0 + rq + 8 * j;
      if (L == 0 && row < row_end && row < N) {
        if (residual) v = __fadd_rn(residual[row], v);
        y[row] = v;
      }
    }
  }
}

template <int R, int TYPE>
static int launch_mv(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row_begin, int row_end,
                     const float* residual) {
  using S = MvShape<R>;
  size_t smem = 128 + (size_t)S::PS_FLOAT4 * 16 + (size_t)w->K * 4;
  int grid = pb_cdiv(row_end - row_begin, R);
  k_matvec<R, TYPE><<<grid, (MV_NP + 1) * 32, smem, ctx->stream>>>(w->qs, w->d, w->m, w->N, w->nb, x, y, residual,
                                                                    row_begin, row_end, ctx->d_err);
  PB_LAUNCHED(ctx, "k_matvec");
  return PB_OK;
}

int pb_launch_matvec(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows,
                     const float* residual) {
  if (!ctx || !w || !x || !y) return PB_ERR_ARG;
  if (w->type != PB_TYPE_Q4_0 && w->type != PB_TYPE_Q4_1)
    return pb_set_error(ctx, PB_ERR_ARG, "matvec supports Q4_0 and Q4_1 matrices");
  if (w->K > 32768) return pb_set_error(ctx, PB_ERR_ARG, "K=%d exceeds the 32768 supported", w->K);
  if (rows <= 0) { row0 = 0; rows = w->N; }
  if (row0 < 0 || row0 + rows > w->N || (row0 & 31))
    return pb_set_error(ctx, PB_ERR_ARG, "row range [%d, %d) invalid (start must be a multiple of 32)", row0, row0 + rows);
  int row_end = row0 + rows;
  int n = rows;
  // Rows per CTA: small matrices use 8-row CTAs for parallelism, tall ones
  // 32-row CTAs to amortise the in-order chain.
  int R = n >= 32 * ctx->sm_count * 2 ? 32 : (n >= 16 * ctx->sm_count * 2 ? 16 : 8);
  if (w->type == PB_TYPE_Q4_0) {
    if (R == 32) return launch_mv<32, PB_TYPE_Q4_0>(ctx, w, x, y, row0, row_end, residual);
    if (R == 16) return launch_mv<16, PB_TYPE_Q4_0>(ctx, w, x, y, row0, row_end, residual);
    return launch_mv<8, PB_TYPE_Q4_0>(ctx, w, x, y, row0, row_end, residual);
  }
  return launch_mv<8, PB_TYPE_Q4_1>(ctx, w, x, y, row0, row_end, residual);
}

extern "C" int pb_qmat_matvec(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows) {
  return pb_launch_matvec(ctx, w, x, y, row0, rows, nullptr);
}

static int host_matvec(pb_ctx* ctx, int type, const float* x, const uint8_t* raw, int N, int K, float* y) {
  if (!ctx || !x || !raw || !y || N <= 0 || K <= 0 || K % 32)
    return pb_set_error(ctx, PB_ERR_ARG, "q4 matvec: bad arguments (N=%d, K=%d; K must be a multiple of 32)", N, K);
  pb_qmat* m = nullptr;
  PB_TRY(pb_qmat_upload(ctx, type, raw, N, K, &m));
  float *dx = nullptr, *dy = nullptr;
  int rc = PB_OK;
  cudaError_t e = cudaMalloc(&dx, (size_t)K * 4);
  if (e == cudaSuccess) e = cudaMalloc(&dy, (size_t)N * 4);
  if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "matvec buffers");
  if (rc == PB_OK) {
    e = cudaMemcpyAsync(dx, x, (size_t)K * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "upload x");
  }
  if (rc == PB_OK) rc = pb_launch_matvec(ctx, m, dx, dy, 0, N, nullptr);
  if (rc == PB_OK) {
    e = cudaMemcpyAsync(y, dy, (size_t)N * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "download y");
  }
  if (rc == PB_OK) rc = pb_wait(ctx);
  cudaStreamSynchronize(ctx->stream);
  cudaFree(dx);
  cudaFree(dy);
  pb_qmat_free(nullptr, m);
  return rc;
}

extern "C" int pb_q4_0_matvec(pb_ctx* ctx, const float* x, const uint8_t* raw, int N, int K, float* y) {
  return host_matvec(ctx, PB_TYPE_Q4_0, x, raw, N, K, y);
}
extern "C" int pb_q4_1_matvec(pb_ctx* ctx, const float* x, const uint8_t* raw, int N, int K, float* y) {
  return host_matvec(ctx, PB_TYPE_Q4_1, x, raw, N, K, y);
}

// ---------------------------------------------------------------------------
// head kernels
// ---------------------------------------------------------------------------

constexpr int HD_WARPS = 8;
constexpr int HD_PF = 4;

// One lane per vocab row; lanes of a warp = the 32 rows of a tile.
// mode 0: batch_dot order (wasm-q4.js:467-549) over Q4_0 / Q8_0 tiles.
template <int TYPE>
__global__ void __launch_bounds__(HD_WARPS * 32)
k_head(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int N, int nb, const float* __restrict__ h,
       float* __restrict__ logits, unsigned long long* __restrict__ amax) {
  extern __shared__ __align__(16) float hs[];
  const int K = nb * 32;
  for (int i = threadIdx.x; i < K / 4; i += blockDim.x) reinterpret_cast<float4*>(hs)[i] = reinterpret_cast<const float4*>(h)[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = blockIdx.x * HD_WARPS + warp;
  const int row = tile * 32 + lane;
  const int ntiles = (N + 31) >> 5;
  float result = 0.0f;
  if (tile < ntiles) {
    constexpr int PL = TYPE == PB_TYPE_Q8_0 ? 2 : 1;  // uint4 per block payload
    const uint4* q4 = reinterpret_cast<const uint4*>(qs);
    uint4 pq[HD_PF][PL];
    uint16_t pd[HD_PF];
    auto load = [&](int b, int k) {
      if (b < nb) {
        size_t slot = ((size_t)tile * nb + b) * 32 + lane;
#pragma unroll
        for (int u = 0; u < PL; ++u) pq[k][u] = __ldcs(q4 + slot * PL + u);
        pd[k] = __ldcs(dsc + slot);
      }
    };
#pragma unroll
    for (int k = 0; k < HD_PF; ++k) load(k, k);
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    for (int b0 = 0; b0 < nb; b0 += HD_PF) {
#pragma unroll
      for (int k = 0; k < HD_PF; ++k) {
        int b = b0 + k;
        if (b >= nb) break;
        float d = pb_f16_exact(pd[k]);
        const float4* hb = reinterpret_cast<const float4*>(hs) + b * 8;
        if (TYPE == PB_TYPE_Q4_0) {
          uint32_t wv[4] = {pq[k][0].x, pq[k][0].y, pq[k][0].z, pq[k][0].w};
          float e[8][4];  // e[i][L]: element 4i+L of the block
          if (isfinite(d)) {
            float c15 = __fmul_rn(-32776.0f, d), c11 = __fmul_rn(-2056.0f, d), c7 = __fmul_rn(-136.0f, d);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint32_t w = wv[g], wa = w << 8, wb = w >> 12;
              // lo nibbles (elements g*4+L) and hi nibbles (elements 16+g*4+L)
              e[g][0] = __fmaf_rn(mag(wa, 0xF00u, PB_MAG8), d, c15);
              e[g + 4][0] = __fmaf_rn(mag(wa, 0xF000u, PB_MAG12), d, c11);
              e[g][1] = __fmaf_rn(mag(w, 0xF00u, PB_MAG8), d, c15);
              e[g + 4][1] = __fmaf_rn(mag(w, 0xF000u, PB_MAG12), d, c11);
              e[g][2] = __fmaf_rn(mag(w, 0xF0000u, PB_MAG16), d, c7);
              e[g + 4][2] = __fmaf_rn(mag(wb, 0xF00u, PB_MAG8), d, c15);
              e[g][3] = __fmaf_rn(mag(wb, 0xF000u, PB_MAG12), d, c11);
              e[g + 4][3] = __fmaf_rn(mag(wb, 0xF0000u, PB_MAG16), d, c7);
            }
          } else {  // inf / NaN scale: the plain product, as gguf.js computes it
#pragma unroll
            for (int g = 0; g < 4; ++g)
#pragma unroll
              for (int L = 0; L < 4; ++L) {
                uint32_t byte = (wv[g] >> (8 * L)) & 0xFFu;
                e[g][L] = __fmul_rn((float)((int)(byte & 15u) - 8), d);
                e[g + 4][L] = __fmul_rn((float)((int)(byte >> 4) - 8), d);
              }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float4 hv = hb[i];
            acc0 = __fadd_rn(acc0, __fmul_rn(hv.x, e[i][0]));
            acc1 = __fadd_rn(acc1, __fmul_rn(hv.y, e[i][1]));
            acc2 = __fadd_rn(acc2, __fmul_rn(hv.z, e[i][2]));
            acc3 = __fadd_rn(acc3, __fmul_rn(hv.w, e[i][3]));
          }
        } else {  // Q8_0: element j = byte j of the 32-byte payload
          uint32_t wv[8] = {pq[k][0].x, pq[k][0].y, pq[k][0].z, pq[k][0].w,
                            pq[k][1].x, pq[k][1].y, pq[k][1].z, pq[k][1].w};
          bool fin = isfinite(d);
          float c = __fmul_rn(-32896.0f, d);  // -(2^15 + 128) * d, exact
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            uint32_t u = wv[i] ^ 0x80808080u;  // biased bytes: q + 128
            float4 hv = hb[i];
            float e0, e1, e2, e3;
            if (fin) {
              e0 = __fmaf_rn(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7504)), d, c);
              e1 = __fmaf_rn(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7514)), d, c);
              e2 = __fmaf_rn(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7524)), d, c);
              e3 = __fmaf_rn(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7534)), d, c);
            } else {
              e0 = __fmul_rn((float)(int8_t)(wv[i] & 0xFF), d);
              e1 = __fmul_rn((float)(int8_t)((wv[i] >> 8) & 0xFF), d);
              e2 = __fmul_rn((float)(int8_t)((wv[i] >> 16) & 0xFF), d);
              e3 = __fmul_rn((float)(int8_t)((wv[i] >> 24) & 0xFF), d);
            }
            acc0 = __fadd_rn(acc0, __fmul_rn(hv.x, e0));
            acc1 = __fadd_rn(acc1, __fmul_rn(hv.y, e1));
            acc2 = __fadd_rn(acc2, __fmul_rn(hv.z, e2));
            acc3 = __fadd_rn(acc3, __fmul_rn(hv.w, e3));
          }
        }
        load(b + HD_PF, k);
      }
    }
    result = __fadd_rn(__fadd_rn(acc1, acc3), __fadd_rn(acc0, acc2));
    if (row < N) logits[row] = result;
  }
  if (amax) {
    unsigned long long key = (tile < ntiles && row < N) ? pb_argmax_key(result, row) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long t = __shfl_xor_sync(0xffffffffu, key, o);
      key = t > key ? t : key;
    }
    if (lane == 0 && key) atomicMax(amax, key);
  }
}

// llama.js:359-367 head: logit = f32(sum_d h[d]*E[v,d]) in double over an f32
// table stored as tiles [V/32][D][32] (lanes = rows; coalesced 128 B loads).
__global__ void __launch_bounds__(HD_WARPS * 32)
k_head_f32_double(const float* __restrict__ E, int N, int D, const float* __restrict__ h, float* __restrict__ logits,
                  unsigned long long* __restrict__ amax) {
  extern __shared__ __align__(16) float hs[];
  for (int i = threadIdx.x; i < D; i += blockDim.x) hs[i] = h[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = blockIdx.x * HD_WARPS + warp;
  const int row = tile * 32 + lane;
  const int ntiles = (N + 31) >> 5;
  float result = 0.0f;
  if (tile < ntiles) {
    const float* tp = E + (size_t)tile * D * 32 + lane;
    double dot = 0.0;
    int d = 0;
    for (; d + 8 <= D; d += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcs(tp + (size_t)(d + u) * 32);
#pragma unroll
      for (int u = 0; u < 8; ++u) dot = __fma_rn((double)hs[d + u], (double)v[u], dot);  // exact product: one rounding
    }
    for (; d < D; ++d) dot = __fma_rn((double)hs[d], (double)__ldcs(tp + (size_t)d * 32), dot);
    result = (float)dot;
    if (row < N) logits[row] = result;
  }
  if (amax) {
    unsigned long long key = (tile < ntiles && row < N) ? pb_argmax_key(result, row) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long t = __shfl_xor_sync(0xffffffffu, key, o);
      key = t > key ? t : key;
    }
    if (lane == 0 && key) atomicMax(amax, key);
  }
}

// wasm-q4.js:798-839 lmHead over a row-major f32 table (one-shot host API).
__global__ void k_head_f32_rowmajor(const float* __restrict__ E, int N, int D, const float* __restrict__ h,
                                    float* __restrict__ logits) {
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float* w = E + (size_t)n * D;
  int K4 = D & ~3;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int k = 0; k < K4; k += 4) {
    a0 = __fadd_rn(a0, __fmul_rn(h[k], w[k]));
    a1 = __fadd_rn(a1, __fmul_rn(h[k + 1], w[k + 1]));
    a2 = __fadd_rn(a2, __fmul_rn(h[k + 2], w[k + 2]));
    a3 = __fadd_rn(a3, __fmul_rn(h[k + 3], w[k + 3]));
  }
  float s = __fadd_rn(__fadd_rn(a1, a3), __fadd_rn(a0, a2));
  for (int k = K4; k < D; ++k) s = __fadd_rn(s, __fmul_rn(h[k], w[k]));
  logits[n] = s;
}

__global__ void k_argmax_finish(const unsigned long long* key, int* idx) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *idx = pb_argmax_index(*key);
}

// mode: 0 = batch_dot order over Q4_0/Q8_0 tiles; 1 = double order over f32 tiles
int pb_launch_head(pb_ctx* ctx, const pb_qmat* emb, const float* h, float* logits, unsigned long long* amax, int mode) {
  int ntiles = (emb->N + 31) / 32;
  int grid = pb_cdiv(ntiles, HD_WARPS);
  size_t smem = (size_t)emb->K * 4;
  if (smem > 200 * 1024) return pb_set_error(ctx, PB_ERR_ARG, "head dim %d too large", emb->K);
  if (mode == 1) {
    k_head_f32_double<<<grid, HD_WARPS * 32, smem, ctx->stream>>>((const float*)emb->qs, emb->N, emb->K, h, logits, amax);
  } else if (emb->type == PB_TYPE_Q4_0) {
    k_head<PB_TYPE_Q4_0><<<grid, HD_WARPS * 32, smem, ctx->stream>>>(emb->qs, emb->d, emb->N, emb->nb, h, logits, amax);
  } else if (emb->type == PB_TYPE_Q8_0) {
    k_head<PB_TYPE_Q8_0><<<grid, HD_WARPS * 32, smem, ctx->stream>>>(emb->qs, emb->d, emb->N, emb->nb, h, logits, amax);
  } else {
    return pb_set_error(ctx, PB_ERR_ARG, "head table type %d not supported", emb->type);
  }
  PB_LAUNCHED(ctx, "k_head");
  return PB_OK;
}

int pb_launch_argmax_finish(pb_ctx* ctx, const unsigned long long* key, int* idx) {
  k_argmax_finish<<<1, 32, 0, ctx->stream>>>(key, idx);
  PB_LAUNCHED(ctx, "k_argmax_finish");
  return PB_OK;
}

extern "C" int pb_qmat_head(pb_ctx* ctx, const pb_qmat* emb, const float* h, float* logits, int* argmax_dev) {
  if (!ctx || !emb || !h || !logits) return PB_ERR_ARG;
  if (emb->type != PB_TYPE_Q4_0 && emb->type != PB_TYPE_Q8_0)
    return pb_set_error(ctx, PB_ERR_ARG, "head table must be Q4_0 or Q8_0");
  unsigned long long* key = nullptr;
  if (argmax_dev) {
    PB_TRY(pb_ensure_scratch(ctx, 64));
    key = (unsigned long long*)ctx->scratch;
    PB_TRY_CUDA(ctx, cudaMemsetAsync(key, 0, 8, ctx->stream));
  }
  PB_TRY(pb_launch_head(ctx, emb, h, logits, key, 0));
  if (argmax_dev) PB_TRY(pb_launch_argmax_finish(ctx, key, argmax_dev));
  return PB_OK;
}

__global__ void k_argmax(const float* __restrict__ v, int n, unsigned long long* key) {
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    unsigned long long k = pb_argmax_key(v[i], i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0 && best) atomicMax(key, best);
}

extern "C" int pb_argmax(pb_ctx* ctx, const float* logits, int n, int* idx) {
  if (!ctx || !logits || !idx || n <= 0) return PB_ERR_ARG;
  PB_TRY(pb_ensure_scratch(ctx, 64));
  unsigned long long* key = (unsigned long long*)ctx->scratch;
  PB_TRY_CUDA(ctx, cudaMemsetAsync(key, 0, 8, ctx->stream));
  int grid = pb_cdiv(n, 256);
  grid = grid > ctx->sm_count * 4 ? ctx->sm_count * 4 : grid;
  k_argmax<<<grid, 256, 0, ctx->stream>>>(logits, n, key);
  PB_LAUNCHED(ctx, "k_argmax");
  return pb_launch_argmax_finish(ctx, key, idx);
}

extern "C" int pb_lm_head(pb_ctx* ctx, const float* h, const float* emb, int V, int D, float* logits) {
  if (!ctx || !h || !emb || !logits || V <= 0 || D <= 0) return PB_ERR_ARG;
  size_t eb = (size_t)V * D * 4;
  float *dE = nullptr, *dh = nullptr, *dl = nullptr;
  int rc = PB_OK;
  cudaError_t e = cudaMalloc(&dE, eb);
  if (e == cudaSuccess) e = cudaMalloc(&dh, (size_t)D * 4);
  if (e == cudaSuccess) e = cudaMalloc(&dl, (size_t)V * 4);
  if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "lm_head buffers");
  if (rc == PB_OK) {
    e = cudaMemcpyAsync(dE, emb, eb, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dh, h, (size_t)D * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "lm_head upload");
  }
  if (rc == PB_OK) {
    k_head_f32_rowmajor<<<pb_cdiv(V, 128), 128, 0, ctx->stream>>>(dE, V, D, dh, dl);
    rc = pb_check_launch(ctx, "k_head_f32_rowmajor");
  }
  if (rc == PB_OK) {
    e = cudaMemcpyAsync(logits, dl, (size_t)V * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "lm_head download");
  }
  if (rc == PB_OK) rc = pb_wait(ctx);
  cudaStreamSynchronize(ctx->stream);
  cudaFree(dE);
  cudaFree(dh);
  cudaFree(dl);
  return rc;
}

// ---------------------------------------------------------------------------
// prefill GEMM over a Q4_0 matrix in the reference's prefill arithmetic:
// the weights are dequantized exactly (gguf.js:259-286) and the WASM matmul
// accumulates C[m,n] = C[m,n] + x[m,k]*W[n,k] in f32, k ascending
// (wasm-simd.js:71-91, reached from llama-streaming.js:398 via
// engine.js:180-190).  Lanes = 32 rows n of a tile, MT query rows per thread,
// x staged in shared memory a chunk of blocks at a time.
// ---------------------------------------------------------------------------

constexpr int PF_WARPS = 8;
constexpr int PF_MT = 16;
constexpr int PF_KC = 8;  // blocks per x chunk

__global__ void __launch_bounds__(PF_WARPS * 32)
k_prefill_q4(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int N, int nb,
             const float* __restrict__ X, int ldx, int M, float* __restrict__ C, int ldc) {
  __shared__ __align__(16) float xs[PF_MT][PF_KC * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = blockIdx.x * PF_WARPS + warp;
  const int ntiles = (N + 31) >> 5;
  const int m0 = blockIdx.y * PF_MT;
  const int K = nb * 32;
  float acc[PF_MT];
#pragma unroll
  for (int i = 0; i < PF_MT; ++i) acc[i] = 0.0f;
  for (int b0 = 0; b0 < nb; b0 += PF_KC) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < PF_MT * PF_KC * 32; idx += blockDim.x) {
      int mm = idx / (PF_KC * 32), kk = idx % (PF_KC * 32);
      int k = b0 * 32 + kk;
      xs[mm][kk] = (m0 + mm < M && k < K) ? X[(size_t)(m0 + mm) * ldx + k] : 0.0f;
    }
    __syncthreads();
    if (tile < ntiles) {
      for (int bb = 0; bb < PF_KC && b0 + bb < nb; ++bb) {
        size_t slot = ((size_t)tile * nb + b0 + bb) * 32 + lane;
        uint4 pl = __ldg(reinterpret_cast<const uint4*>(qs) + slot);
        float d = pb_f16_exact(__ldg(dsc + slot));
        float e[32];
        uint32_t wv[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
        for (int g = 0; g < 4; ++g)
#pragma unroll
          for (int L = 0; L < 4; ++L) {
            uint32_t byte = (wv[g] >> (8 * L)) & 0xFFu;
            e[4 * g + L] = __fmul_rn(__fsub_rn(__uint_as_float((byte & 15u) | PB_MAG0), 8388616.0f), d);
            e[16 + 4 * g + L] = __fmul_rn(__fsub_rn(__uint_as_float((byte >> 4) | PB_MAG0), 8388616.0f), d);
          }
#pragma unroll
        for (int mm = 0; mm < PF_MT; ++mm) {
          const float4* xr = reinterpret_cast<const float4*>(&xs[mm][bb * 32]);
          float a = acc[mm];
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            float4 xv = xr[c4];
            a = __fadd_rn(a, __fmul_rn(xv.x, e[4 * c4 + 0]));
            a = __fadd_rn(a, __fmul_rn(xv.y, e[4 * c4 + 1]));
            a = __fadd_rn(a, __fmul_rn(xv.z, e[4 * c4 + 2]));
            a = __fadd_rn(a, __fmul_rn(xv.w, e[4 * c4 + 3]));
          }
          acc[mm] = a;
        }
      }
    }
  }
  int n = tile * 32 + lane;
  if (tile < ntiles && n < N) {
#pragma unroll
    for (int mm = 0; mm < PF_MT; ++mm)
      if (m0 + mm < M) C[(size_t)(m0 + mm) * ldc + n] = acc[mm];
  }
}

int pb_launch_prefill_q4(pb_ctx* ctx, const pb_qmat* w, const float* X, int ldx, int M, float* C, int ldc) {
  if (w->type != PB_TYPE_Q4_0) return pb_set_error(ctx, PB_ERR_ARG, "prefill GEMM needs a Q4_0 matrix");
  int ntiles = (w->N + 31) / 32;
  dim3 grid(pb_cdiv(ntiles, PF_WARPS), pb_cdiv(M, PF_MT));
  if (grid.y > 65535) return pb_set_error(ctx, PB_ERR_ARG, "M=%d too large", M);
  k_prefill_q4<<<grid, PF_WARPS * 32, 0, ctx->stream>>>(w->qs, w->d, w->N, w->nb, X, ldx, M, C, ldc);
  PB_LAUNCHED(ctx, "k_prefill_q4");
  return PB_OK;
}

// Opt every kernel with a large dynamic shared-memory footprint in once, at
// context creation (never during stream capture).
int pb_setup_q4_kernels(void) {
  const int lim = 200 * 1024;
  cudaError_t e = cudaSuccess;
  e = e ? e : cudaFuncSetAttribute(k_matvec<8, PB_TYPE_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_matvec<16, PB_TYPE_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_matvec<32, PB_TYPE_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_matvec<8, PB_TYPE_Q4_1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_head<PB_TYPE_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_head<PB_TYPE_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_head_f32_double, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  return e == cudaSuccess ? PB_OK : PB_ERR_CUDA;
}
