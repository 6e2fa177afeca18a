// pb_q4.cu - quantized matvec and LM-head kernels for sm_100a.
//
// Matvec (wasm-q4.js:118-267 Q4_0, :275-435 Q4_1).  The reference computes,
// per row and per lane L in 0..3, a per-block partial
//     blockAcc[L] = sum over g in {0,4,8,12} of  (lo-8)*x[g+L], (hi-8)*x[g+16+L]
// in f32 with a separate multiply and add, then the in-order chain
//     acc[L] = acc[L] + blockAcc[L]*d        (blocks b = 0, 1, 2, ...)
// and y = (acc1 + acc3) + (acc0 + acc2).  Two modes run it (pb_set_matvec_mode):
//   - exact (k_matvec, k_matvec_ws): the per-block partials are independent,
//     so warps compute them for all (row, block) pairs of an 8-row tile in
//     parallel and the in-order acc[L] chains run over them from shared
//     memory: bit-identical to the reference's WASM kernel;
//   - fast, the default (k_mvf here; k_mvi, the int8 tensor-core kernel in
//     pb_mvi.cu, for matrices of at least ctx->mvi_min_rows rows): the same
//     exact (q-8)*x products summed in another order with one FMA per
//     weight, a warp per (8-row tile, 32-block chunk) unit with the payload
//     streamed through per-warp cp.async stages, chunk partials summed in
//     order: within an f32 relative tolerance of the reference.
// Both take the same fused prologues (RMSNorm of x) and epilogues (residual
// add, RoPE + KV append, SwiGLU of interleaved gate|up tiles, argmax).
//
// Head (wasm-q4.js:447-566 batch_dot over the table gguf.js:239-286
// dequantizes).  The reference's lane L chain runs over k = L, L+4, ... of
// the f32 table.  Each lane of a warp owns one vocab row and walks all blocks;
// the dequantized value (q-8)*d is rebuilt exactly with one FFMA from a
// magic-exponent float, then p = h[k]*e and acc[L] += p as in the reference.
// The greedy argmax (llama-streaming.js:899-909) is fused as an ordered-key
// atomicMax.
#include <stdio.h>
#include <stdlib.h>

#include <cooperative_groups.h>

#include "pb_attn_fast.cuh"
#include "pb_internal.cuh"

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

// (w & MASK) | e as one three-input logic op, e held in a register (the
// exponent patterns come in as kernel arguments, so they stay in registers
// instead of being rebuilt from immediates).
template <uint32_t MASK>
__device__ __forceinline__ float magr(uint32_t w, uint32_t e) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "n"(MASK), "r"(e));
  return __uint_as_float(r);
}

struct pb_magics {
  uint32_t m0, m4, m8, m12, m16;
};

// ---------------------------------------------------------------------------
// matvec kernel
// ---------------------------------------------------------------------------
// Persistent CTAs of MV_THREADS threads, one per SM.  A tile is 8 consecutive
// rows (contiguous in the row-major device layout); a CTA works on
// S = MV_THREADS / (2 nb) tiles at a time ("slots").
//   - thread (slot s, half h, block b) keeps x[32b .. 32b+31] in registers for
//     the whole kernel (RMS-normalised in the prologue when the epilogue asks
//     for it) and, for each tile of its slot, loads block b of rows
//     4h .. 4h+3, so a warp reads 512 contiguous bytes per row;
//   - every CTA first issues bulk L2 prefetches for all of its tiles and its
//     share of the region the next kernel reads (before griddepcontrol.wait:
//     weights never depend on the previous kernel), then keeps the next
//     iteration's blocks in flight in registers while it computes;
//   - the block partials of the WASM lane order (wasm-q4.js:193-229) go to
//     shared memory (double-buffered); warp s then runs slot s's 32 in-order
//     chains acc[L] += partial (8 rows x 4 lanes, wasm-q4.js:225-229) and the
//     fused epilogue.

constexpr int MV_THREADS = 512;
constexpr int MV_RPT = 4;      // rows per thread
constexpr int MV_PF_DIST = 4;  // iterations of L2 prefetch ahead of the loads

// Tiles in flight per CTA ("slots"): 2 nb threads each, rounded up to whole
// warps (a slot syncs on its own named barrier, ids 1..15).
__host__ __device__ __forceinline__ int mv_slot_threads(int nb) { return (2 * nb + 31) / 32 * 32; }
__host__ __device__ __forceinline__ int mv_slots(int nb, int nt) {
  const int s = nt / mv_slot_threads(nb);
  return s < 15 ? s : 15;
}

// Packed f32x2 arithmetic, each component rounded to nearest like the scalar
// instruction.  The code generator fuses a packed multiply that feeds a packed
// add into a packed FMA (one rounding instead of the reference's two), even
// with .rn and --fmad=false.  So a product that is summed afterwards is formed
// as f2fma(a, b, nz) with nz = -0.0 passed in from the host: fma(a, b, -0)
// rounds a*b exactly like mul.rn does (the -0 leaves +0 and -0 products
// alone), and an FMA is never contracted into the add that follows.  nz comes
// from a kernel argument so the compiler cannot turn the FMA back into a
// multiply.
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
  float2 r;
  asm("{ .reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd; }"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 f2add(float2 a, float2 b) {
  float2 r;
  asm("{ .reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd; }"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{ .reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd; }"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}


// f32 pairs held as 64-bit registers, so packed operands never need moves.
__device__ __forceinline__ uint64_t p2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 up2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t p2add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t p2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t p2mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Two rows of the same block at once, x of the block as 16 pairs
// xp[i] = (x[2i], x[2i+1]).  Same arithmetic as q4_0_row2.
__device__ __forceinline__ void q4_0_row2p(uint4 pa, uint4 pb, float da, float db, const uint64_t (&xp)[16],
                                           uint64_t nz, const pb_magics& M, float4& ra, float4& rb) {
  const uint64_t c_l01 = p2(-8388616.0f, -32776.0f), c_l23 = p2(-136.0f, -32776.0f);
  const uint64_t c_h = p2(-524296.0f, -2056.0f);
  uint64_t a01 = 0, a23 = 0, b01 = 0, b23 = 0;  // +0.0f pairs
  const uint32_t wa[4] = {pa.x, pa.y, pa.z, pa.w}, wb[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t w = wa[g], w2 = w >> 16, v = wb[g], v2 = v >> 16;
    const uint64_t la01 = p2add(p2(magr<0xFu>(w, M.m0), magr<0xF00u>(w, M.m8)), c_l01);
    const uint64_t lb01 = p2add(p2(magr<0xFu>(v, M.m0), magr<0xF00u>(v, M.m8)), c_l01);
    const uint64_t la23 = p2add(p2(magr<0xF0000u>(w, M.m16), magr<0xF00u>(w2, M.m8)), c_l23);
    const uint64_t lb23 = p2add(p2(magr<0xF0000u>(v, M.m16), magr<0xF00u>(v2, M.m8)), c_l23);
    a01 = p2add(a01, p2fma(la01, xp[2 * g], nz));
    b01 = p2add(b01, p2fma(lb01, xp[2 * g], nz));
    a23 = p2add(a23, p2fma(la23, xp[2 * g + 1], nz));
    b23 = p2add(b23, p2fma(lb23, xp[2 * g + 1], nz));
    const uint64_t ha01 = p2add(p2(magr<0xF0u>(w, M.m4), magr<0xF000u>(w, M.m12)), c_h);
    const uint64_t hb01 = p2add(p2(magr<0xF0u>(v, M.m4), magr<0xF000u>(v, M.m12)), c_h);
    const uint64_t ha23 = p2add(p2(magr<0xF0u>(w2, M.m4), magr<0xF000u>(w2, M.m12)), c_h);
    const uint64_t hb23 = p2add(p2(magr<0xF0u>(v2, M.m4), magr<0xF000u>(v2, M.m12)), c_h);
    a01 = p2add(a01, p2fma(ha01, xp[8 + 2 * g], nz));
    b01 = p2add(b01, p2fma(hb01, xp[8 + 2 * g], nz));
    a23 = p2add(a23, p2fma(ha23, xp[9 + 2 * g], nz));
    b23 = p2add(b23, p2fma(hb23, xp[9 + 2 * g], nz));
  }
  const uint64_t dA = p2(da, da), dB = p2(db, db);
  const float2 ra01 = up2(p2mul(a01, dA)), ra23 = up2(p2mul(a23, dA));
  const float2 rb01 = up2(p2mul(b01, dB)), rb23 = up2(p2mul(b23, dB));
  ra = make_float4(ra01.x, ra01.y, ra23.x, ra23.y);
  rb = make_float4(rb01.x, rb01.y, rb23.x, rb23.y);
}

// Two rows of the same block at once (the four accumulation chains of the two
// rows are independent, so their adds overlap).
__device__ __forceinline__ void q4_0_row2(uint4 pa, uint4 pb, float da, float db, const float (&xr)[32], float2 nz,
                                          const pb_magics& M, float4& ra, float4& rb) {
  float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
  float2 b01 = make_float2(0.f, 0.f), b23 = make_float2(0.f, 0.f);
  const uint32_t wa[4] = {pa.x, pa.y, pa.z, pa.w}, wb[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float2 xl01 = make_float2(xr[4 * g], xr[4 * g + 1]), xl23 = make_float2(xr[4 * g + 2], xr[4 * g + 3]);
    const float2 xh01 = make_float2(xr[16 + 4 * g], xr[16 + 4 * g + 1]);
    const float2 xh23 = make_float2(xr[16 + 4 * g + 2], xr[16 + 4 * g + 3]);
    const uint32_t w = wa[g], w2 = w >> 16, v = wb[g], v2 = v >> 16;
    const float2 la01 = f2add(make_float2(magr<0xFu>(w, M.m0), magr<0xF00u>(w, M.m8)), make_float2(-8388616.0f, -32776.0f));
    const float2 lb01 = f2add(make_float2(magr<0xFu>(v, M.m0), magr<0xF00u>(v, M.m8)), make_float2(-8388616.0f, -32776.0f));
    const float2 la23 = f2add(make_float2(magr<0xF0000u>(w, M.m16), magr<0xF00u>(w2, M.m8)), make_float2(-136.0f, -32776.0f));
    const float2 lb23 = f2add(make_float2(magr<0xF0000u>(v, M.m16), magr<0xF00u>(v2, M.m8)), make_float2(-136.0f, -32776.0f));
    a01 = f2add(a01, f2fma(la01, xl01, nz));
    b01 = f2add(b01, f2fma(lb01, xl01, nz));
    a23 = f2add(a23, f2fma(la23, xl23, nz));
    b23 = f2add(b23, f2fma(lb23, xl23, nz));
    const float2 ha01 = f2add(make_float2(magr<0xF0u>(w, M.m4), magr<0xF000u>(w, M.m12)), make_float2(-524296.0f, -2056.0f));
    const float2 hb01 = f2add(make_float2(magr<0xF0u>(v, M.m4), magr<0xF000u>(v, M.m12)), make_float2(-524296.0f, -2056.0f));
    const float2 ha23 = f2add(make_float2(magr<0xF0u>(w2, M.m4), magr<0xF000u>(w2, M.m12)), make_float2(-524296.0f, -2056.0f));
    const float2 hb23 = f2add(make_float2(magr<0xF0u>(v2, M.m4), magr<0xF000u>(v2, M.m12)), make_float2(-524296.0f, -2056.0f));
    a01 = f2add(a01, f2fma(ha01, xh01, nz));
    b01 = f2add(b01, f2fma(hb01, xh01, nz));
    a23 = f2add(a23, f2fma(ha23, xh23, nz));
    b23 = f2add(b23, f2fma(hb23, xh23, nz));
  }
  const float2 dA = make_float2(da, da), dB = make_float2(db, db);
  const float2 ra01 = f2mul(a01, dA), ra23 = f2mul(a23, dA), rb01 = f2mul(b01, dB), rb23 = f2mul(b23, dB);
  ra = make_float4(ra01.x, ra01.y, ra23.x, ra23.y);
  rb = make_float4(rb01.x, rb01.y, rb23.x, rb23.y);
}

// Q4_1 (wasm-q4.js:357-398): nibAcc[L] += n*x (lo then hi), xAcc[L] += x;
// block value nibAcc*delta + xAcc*min.  xAcc depends only on x, so sx holds
// it for the thread's block.
__device__ __forceinline__ float4 q4_1_row(uint4 pl, float dl, float mn, const float (&xr)[32], float4 sx,
                                           float2 nz, const pb_magics& M) {
  float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
  const uint32_t wv[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t w = wv[g], w2 = w >> 16;
    const float2 l01 = f2add(make_float2(magr<0xFu>(w, M.m0), magr<0xF00u>(w, M.m8)),
                             make_float2(-8388608.0f, -32768.0f));
    const float2 l23 = f2add(make_float2(magr<0xF0000u>(w, M.m16), magr<0xF00u>(w2, M.m8)),
                             make_float2(-128.0f, -32768.0f));
    const float2 h01 = f2add(make_float2(magr<0xF0u>(w, M.m4), magr<0xF000u>(w, M.m12)),
                             make_float2(-524288.0f, -2048.0f));
    const float2 h23 = f2add(make_float2(magr<0xF0u>(w2, M.m4), magr<0xF000u>(w2, M.m12)),
                             make_float2(-524288.0f, -2048.0f));
    a01 = f2add(a01, f2fma(l01, make_float2(xr[4 * g], xr[4 * g + 1]), nz));
    a23 = f2add(a23, f2fma(l23, make_float2(xr[4 * g + 2], xr[4 * g + 3]), nz));
    a01 = f2add(a01, f2fma(h01, make_float2(xr[16 + 4 * g], xr[16 + 4 * g + 1]), nz));
    a23 = f2add(a23, f2fma(h23, make_float2(xr[16 + 4 * g + 2], xr[16 + 4 * g + 3]), nz));
  }
  return make_float4(__fadd_rn(__fmul_rn(a01.x, dl), __fmul_rn(sx.x, mn)),
                     __fadd_rn(__fmul_rn(a01.y, dl), __fmul_rn(sx.y, mn)),
                     __fadd_rn(__fmul_rn(a23.x, dl), __fmul_rn(sx.z, mn)),
                     __fadd_rn(__fmul_rn(a23.y, dl), __fmul_rn(sx.w, mn)));
}

// x, RMS-normalised with the gains w when w is set (engine.js:429-449), into
// the shared copy whose float4 chunks are swizzled within each 32-value block.
// Every global load of a thread is issued before any is used: one memory
// latency for the prologue instead of one per element.  The sum of squares
// runs per thread over its float4 chunks in order, then through the block's
// fixed reduction tree, so every CTA forms the same value.  Needs
// K / 4 <= MV_STAGE_CH * nthreads.
constexpr int MV_STAGE_CH = 4;

__device__ __forceinline__ void mv_stage_x(const float* __restrict__ x, const float* __restrict__ w, double eps, int K,
                                           float4* xs4, double* red) {
  const int tid = threadIdx.x, nt = blockDim.x, nc = K / 4;
  float4 xv[MV_STAGE_CH], wv[MV_STAGE_CH];
#pragma unroll
  for (int i = 0; i < MV_STAGE_CH; ++i) {
    const int c = tid + i * nt;
    if (c < nc) {
      xv[i] = reinterpret_cast<const float4*>(x)[c];
      if (w) wv[i] = reinterpret_cast<const float4*>(w)[c];
    }
  }
  double rms = 0.0;
  if (w) {
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < MV_STAGE_CH; ++i) {
      if (tid + i * nt < nc) {
        ss = __fma_rn((double)xv[i].x, (double)xv[i].x, ss);
        ss = __fma_rn((double)xv[i].y, (double)xv[i].y, ss);
        ss = __fma_rn((double)xv[i].z, (double)xv[i].z, ss);
        ss = __fma_rn((double)xv[i].w, (double)xv[i].w, ss);
      }
    }
    ss = pb_block_sum_d(ss, red);
    rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)K), eps));
  }
#pragma unroll
  for (int i = 0; i < MV_STAGE_CH; ++i) {
    const int c = tid + i * nt;
    if (c < nc) {
      float4 v = xv[i];
      if (w) {
        v.x = (float)__dmul_rn(__ddiv_rn((double)v.x, rms), (double)wv[i].x);
        v.y = (float)__dmul_rn(__ddiv_rn((double)v.y, rms), (double)wv[i].y);
        v.z = (float)__dmul_rn(__ddiv_rn((double)v.z, rms), (double)wv[i].z);
        v.w = (float)__dmul_rn(__ddiv_rn((double)v.w, rms), (double)wv[i].w);
      }
      const int bj = c >> 3, ci = c & 7;
      xs4[bj * 8 + (ci ^ (bj & 7))] = v;
    }
  }
}

struct MvBuf {
  uint4 q[MV_RPT];
  uint32_t d[MV_RPT];
  uint32_t m[MV_RPT];
};

template <int TYPE>
__device__ __forceinline__ void mv_load(MvBuf& R, const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc,
                                        const uint16_t* __restrict__ msc, int tile, int h, int b, int nb) {
#pragma unroll
  for (int i = 0; i < MV_RPT; ++i) {
    const size_t slot = (size_t)(tile * 8 + h * MV_RPT + i) * nb + b;
    R.q[i] = __ldcs(reinterpret_cast<const uint4*>(qs) + slot);
    R.d[i] = __ldcs(dsc + slot);
    if (TYPE == PB_TYPE_Q4_1) R.m[i] = __ldcs(msc + slot);
  }
}

// Chain of slot `slot`'s tile over the nb block partials, then the epilogue.
// Lane = 4 * row + L.
__device__ __forceinline__ void mv_chain(const float* __restrict__ pc, int nb, int tile, int N, int row_end,
                                         float* __restrict__ y, const pb_mv_epi& epi, int* err) {
  const int lane = threadIdx.x & 31, rr = lane >> 2, L = lane & 3;
  float acc = 0.0f;
  int b = 0;
  for (; b + 8 <= nb; b += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = pc[(b + u) * 32 + ((rr ^ u) << 2) + L];  // (b + u) & 7 == u
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
  }
  for (; b < nb; ++b) acc = __fadd_rn(acc, pc[b * 32 + ((rr ^ (b & 7)) << 2) + L]);
  // y = (acc1 + acc3) + (acc0 + acc2)  (wasm-q4.js:236-245)
  const int base = lane & ~3;
  const float a0 = __shfl_sync(0xffffffffu, acc, base + 0);
  const float a1 = __shfl_sync(0xffffffffu, acc, base + 1);
  const float a2 = __shfl_sync(0xffffffffu, acc, base + 2);
  const float a3 = __shfl_sync(0xffffffffu, acc, base + 3);
  const float v = __fadd_rn(__fadd_rn(a1, a3), __fadd_rn(a0, a2));
  pb_mv_epilogue(v, tile, N, 0, row_end, y, epi, err);
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(NT, 1)
k_matvec(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, const uint16_t* __restrict__ msc, int N,
         int nb, int tile_begin, int tile_end, int row_end, const float* __restrict__ x, float* __restrict__ y,
         pb_mv_epi epi, float nzf, pb_magics M, int* err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ double red[NT / 32];
  const int S = mv_slots(nb, NT), stride = mv_slot_threads(nb);
  const int K = nb * 32;
  float* ps = reinterpret_cast<float*>(smem_raw);  // [S][2][nb][8 rows (swizzled)][4 lanes]
  float4* xs4 = reinterpret_cast<float4*>(ps + (size_t)2 * S * nb * 32);  // x, chunks swizzled per block
  const int tid = threadIdx.x;
  const int s = tid / stride, rem = tid - s * stride, h = rem / nb, b = h < 2 ? rem - h * nb : 0;
  const bool worker = s < S && h < 2;
  const int per_iter = gridDim.x * S;
  const float2 nz = make_float2(nzf, nzf);

  // L2 prefetch of the slot's first MV_PF_DIST tiles (a tile is contiguous;
  // each iteration then prefetches the tile MV_PF_DIST ahead) and of this
  // CTA's share of the later kernels' operands, then the first tile's blocks
  const size_t tq = (size_t)8 * nb * 16, td = (size_t)8 * nb * 2;
  auto prefetch_tile = [&](int t) {
    if (t < tile_end) {
      pb_l2_prefetch(qs + (size_t)t * tq, (uint32_t)tq);
      pb_l2_prefetch(dsc + (size_t)t * td / 2, (uint32_t)td);
      if (TYPE == PB_TYPE_Q4_1) pb_l2_prefetch(msc + (size_t)t * td / 2, (uint32_t)td);
    }
  };
  const bool pf_thread = s < S && rem == 0;
  if (pf_thread)
    for (int i = 0; i < MV_PF_DIST; ++i) prefetch_tile(tile_begin + i * per_iter + s * gridDim.x + blockIdx.x);
  if (tid == 0)
    for (int i = 0; i < PB_MAX_L2_NEXT; ++i) pb_l2_prefetch_share(epi.l2_next[i], epi.l2_next_bytes[i], blockIdx.x, gridDim.x);
  MvBuf A, B;
  {
    const int t0 = tile_begin + s * gridDim.x + blockIdx.x;
    if (worker && t0 < tile_end) mv_load<TYPE>(A, qs, dsc, msc, t0, h, b, nb);
  }
  pb_pdl_trigger();
  pb_pdl_wait();  // x (and the residual) come from the previous kernel

  // x (RMS-normalised when asked: engine.js:429-449 with a fixed reduction
  // tree, identical in every CTA) into shared memory, then the block into
  // registers
  mv_stage_x(x, epi.norm_w, epi.eps, K, xs4, red);
  __syncthreads();
  if (s >= S) return;  // threads beyond the last slot have no further part
  float xr[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = xs4[b * 8 + (i ^ (b & 7))];
    xr[4 * i] = v.x;
    xr[4 * i + 1] = v.y;
    xr[4 * i + 2] = v.z;
    xr[4 * i + 3] = v.w;
  }
  float4 sx = make_float4(0.f, 0.f, 0.f, 0.f);
  if (TYPE == PB_TYPE_Q4_1) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      sx.x = __fadd_rn(__fadd_rn(sx.x, xr[4 * g]), xr[16 + 4 * g]);
      sx.y = __fadd_rn(__fadd_rn(sx.y, xr[4 * g + 1]), xr[16 + 4 * g + 1]);
      sx.z = __fadd_rn(__fadd_rn(sx.z, xr[4 * g + 2]), xr[16 + 4 * g + 2]);
      sx.w = __fadd_rn(__fadd_rn(sx.w, xr[4 * g + 3]), xr[16 + 4 * g + 3]);
    }
  }

  // The slots run independently, each with its own named barrier (ids 1..S)
  // and double-buffered partials; the slot's first warp runs the chains.
  float* pslot = ps + (size_t)s * 2 * nb * 32;
  const bool chain_warp = rem < 32;
  auto iteration = [&](MvBuf& cur, MvBuf& nxt, int it) -> bool {
    const int tc = tile_begin + it * per_iter + s * gridDim.x + blockIdx.x;  // slot-uniform
    if (tc >= tile_end) return false;
    if (pf_thread) prefetch_tile(tc + MV_PF_DIST * per_iter);
    if (worker && tc + per_iter < tile_end) mv_load<TYPE>(nxt, qs, dsc, msc, tc + per_iter, h, b, nb);
    float* pbuf = pslot + (size_t)(it & 1) * nb * 32;
    if (worker) {
      float* pw = pbuf + (size_t)b * 32;
#pragma unroll
      for (int i = 0; i < MV_RPT; i += 2) {  // two rows at a time: independent chains interleave
        const int r = h * MV_RPT + i;
        float4 p0, p1;
        if (TYPE == PB_TYPE_Q4_0) {
          q4_0_row2(cur.q[i], cur.q[i + 1], pb_f16_wasm(cur.d[i]), pb_f16_wasm(cur.d[i + 1]), xr, nz, M, p0, p1);
        } else {
          p0 = q4_1_row(cur.q[i], pb_f16_wasm(cur.d[i]), pb_f16_wasm(cur.m[i]), xr, sx, nz, M);
          p1 = q4_1_row(cur.q[i + 1], pb_f16_wasm(cur.d[i + 1]), pb_f16_wasm(cur.m[i + 1]), xr, sx, nz, M);
        }
        *reinterpret_cast<float4*>(pw + ((r ^ (b & 7)) << 2)) = p0;
        *reinterpret_cast<float4*>(pw + (((r + 1) ^ (b & 7)) << 2)) = p1;
      }
    }
    asm volatile("bar.sync %0, %1;" ::"r"(1 + s), "r"(stride) : "memory");
    if (chain_warp) mv_chain(pbuf, nb, tc, N, row_end, y, epi, err);
    return true;
  };
  for (int it = 0;; it += 2) {
    if (!iteration(A, B, it)) break;
    if (!iteration(B, A, it + 1)) break;
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised matvec for K <= 4096 (nb <= 128).  Each slot is Cs =
// roundup(2 nb, 32) compute threads plus one chain warp.  The compute threads
// never wait for the chain: they hand each tile's partials over through a
// two-buffer ring guarded by named barriers (FULL: compute arrives, chain
// syncs; EMPTY: chain arrives, compute syncs before reusing a buffer).
// ---------------------------------------------------------------------------

constexpr int MVW_MAX_SLOTS = 3;  // 4 named barriers per slot, ids 1..12

__host__ __device__ __forceinline__ int mvw_compute_threads(int nb) { return (2 * nb + 31) / 32 * 32; }
__host__ __device__ __forceinline__ int mvw_slots(int nb) {
  const int s = 512 / (mvw_compute_threads(nb) + 32);
  return s < MVW_MAX_SLOTS ? s : MVW_MAX_SLOTS;
}
__host__ __device__ __forceinline__ int mvw_threads(int nb) { return mvw_slots(nb) * (mvw_compute_threads(nb) + 32); }

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void named_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <int TYPE>
__global__ void __launch_bounds__(512, 1)
k_matvec_ws(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, const uint16_t* __restrict__ msc, int N,
            int nb, int tile_begin, int tile_end, int row_end, const float* __restrict__ x, float* __restrict__ y,
            pb_mv_epi epi, float nzf, pb_magics M, int* err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ double red[16];
  const int S = mvw_slots(nb), Cs = mvw_compute_threads(nb), stride = Cs + 32;
  const int K = nb * 32;
  float* ps = reinterpret_cast<float*>(smem_raw);                         // [S][2][nb][8 rows (swizzled)][4]
  float4* xs4 = reinterpret_cast<float4*>(ps + (size_t)2 * S * nb * 32);  // x, chunks swizzled per block
  const int tid = threadIdx.x;
  const int s = tid / stride, rem = tid - s * stride;
  const bool chain = rem >= Cs;                 // the slot's last warp
  const int h = chain ? 2 : rem / nb, b = (!chain && h < 2) ? rem - h * nb : 0;
  const bool worker = !chain && h < 2;
  const int per_iter = gridDim.x * S;
  const float2 nz = make_float2(nzf, nzf);
  const int first = tile_begin + s * gridDim.x + blockIdx.x;
  const int n_iter = first < tile_end ? (tile_end - first + per_iter - 1) / per_iter : 0;  // slot-uniform

  const size_t tq = (size_t)8 * nb * 16, td = (size_t)8 * nb * 2;
  auto prefetch_tile = [&](int t) {
    if (t < tile_end) {
      pb_l2_prefetch(qs + (size_t)t * tq, (uint32_t)tq);
      pb_l2_prefetch(dsc + (size_t)t * td / 2, (uint32_t)td);
      if (TYPE == PB_TYPE_Q4_1) pb_l2_prefetch(msc + (size_t)t * td / 2, (uint32_t)td);
    }
  };
  const bool pf_thread = rem == 0;
  if (pf_thread)
    for (int i = 0; i < MV_PF_DIST; ++i) prefetch_tile(first + i * per_iter);
  if (tid == 0)
    for (int i = 0; i < PB_MAX_L2_NEXT; ++i) pb_l2_prefetch_share(epi.l2_next[i], epi.l2_next_bytes[i], blockIdx.x, gridDim.x);
  MvBuf A, B;
  if (worker && n_iter > 0) mv_load<TYPE>(A, qs, dsc, msc, first, h, b, nb);
  pb_pdl_trigger();
  pb_pdl_wait();

  mv_stage_x(x, epi.norm_w, epi.eps, K, xs4, red);
  __syncthreads();
  float* pslot = ps + (size_t)s * 2 * nb * 32;
  const int bar = 1 + 4 * s;  // FULL0, FULL1, EMPTY0, EMPTY1

  if (chain) {
    for (int it = 0; it < n_iter; ++it) {
      named_sync(bar + (it & 1), stride);
      mv_chain(pslot + (size_t)(it & 1) * nb * 32, nb, first + it * per_iter, N, row_end, y, epi, err);
      if (it + 2 < n_iter) named_arrive(bar + 2 + (it & 1), stride);
    }
    return;
  }

  float xr[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = xs4[b * 8 + (i ^ (b & 7))];
    xr[4 * i] = v.x;
    xr[4 * i + 1] = v.y;
    xr[4 * i + 2] = v.z;
    xr[4 * i + 3] = v.w;
  }
  float4 sx = make_float4(0.f, 0.f, 0.f, 0.f);
  if (TYPE == PB_TYPE_Q4_1) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      sx.x = __fadd_rn(__fadd_rn(sx.x, xr[4 * g]), xr[16 + 4 * g]);
      sx.y = __fadd_rn(__fadd_rn(sx.y, xr[4 * g + 1]), xr[16 + 4 * g + 1]);
      sx.z = __fadd_rn(__fadd_rn(sx.z, xr[4 * g + 2]), xr[16 + 4 * g + 2]);
      sx.w = __fadd_rn(__fadd_rn(sx.w, xr[4 * g + 3]), xr[16 + 4 * g + 3]);
    }
  }
  uint64_t xp[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) xp[i] = p2(xr[2 * i], xr[2 * i + 1]);
  const uint64_t nz64 = p2(nzf, nzf);
  auto iteration = [&](MvBuf& cur, MvBuf& nxt, int it) {
    const int tc = first + it * per_iter;
    if (pf_thread) prefetch_tile(tc + MV_PF_DIST * per_iter);
    if (worker && it + 1 < n_iter) mv_load<TYPE>(nxt, qs, dsc, msc, tc + per_iter, h, b, nb);
    if (it >= 2) named_sync(bar + 2 + (it & 1), stride);  // the chain is done with this buffer
    if (worker) {
      float* pw = pslot + (size_t)(it & 1) * nb * 32 + (size_t)b * 32;
#pragma unroll
      for (int i = 0; i < MV_RPT; i += 2) {
        const int r = h * MV_RPT + i;
        float4 p0, p1;
        if (TYPE == PB_TYPE_Q4_0) {
          q4_0_row2p(cur.q[i], cur.q[i + 1], pb_f16_wasm(cur.d[i]), pb_f16_wasm(cur.d[i + 1]), xp, nz64, M, p0, p1);
        } else {
          p0 = q4_1_row(cur.q[i], pb_f16_wasm(cur.d[i]), pb_f16_wasm(cur.m[i]), xr, sx, nz, M);
          p1 = q4_1_row(cur.q[i + 1], pb_f16_wasm(cur.d[i + 1]), pb_f16_wasm(cur.m[i + 1]), xr, sx, nz, M);
        }
        *reinterpret_cast<float4*>(pw + ((r ^ (b & 7)) << 2)) = p0;
        *reinterpret_cast<float4*>(pw + (((r + 1) ^ (b & 7)) << 2)) = p1;
      }
    }
    named_arrive(bar + (it & 1), stride);
  };
  for (int it = 0; it < n_iter; it += 2) {
    iteration(A, B, it);
    if (it + 1 < n_iter) iteration(B, A, it + 1);
  }
}

// ---------------------------------------------------------------------------
// Fast Q4_0 matvec (the default decode path).  The same products as the
// reference, (q - 8) * x with q - 8 exact, summed with one FMA per weight
// instead of the reference's separate multiply and add and in a different
// order, so y agrees with wasm-q4.js:118-267 within an f32 tolerance, not
// bit for bit (the exact kernels above stay the parity mode).
//
// A warp works on one (8-row tile, 32-block K chunk): lane l takes block
// 32 c + l of the tile's 8 rows (16-byte coalesced loads, 512 contiguous
// bytes per row), keeps that block's x as 16 f32 pairs, and forms per row
// the block sum with packed f32x2 arithmetic: a nibble becomes the exact
// float 2^k + q by one logic op, a packed add removes 2^k + 8, a packed FMA
// accumulates.  That is one integer and two f32 lane operations per weight.
// The block sum times the f16 scale (decoded the WASM way, wasm-q4.js
// :88-109) is added into the row's partial.  The 8 row partials of the warp
// are summed across lanes by a transposed butterfly (lane 4r ends with row
// r), the K chunks of a tile are added in chunk order in shared memory, and
// the tile's epilogue is the one of the exact kernels.  Each CTA prefetches
// its tiles into L2 a few iterations ahead (bulk prefetch), so the register
// loads find them there.
// ---------------------------------------------------------------------------
constexpr int MVF_MAX_WARPS = 16;
constexpr int MVF_PF = 3;  // CTA iterations of L2 prefetch ahead

__device__ __forceinline__ float q4_0_block_fast(uint4 p, const uint64_t (&xp)[16], const pb_magics& M) {
  const uint64_t c_l01 = p2(-8388616.0f, -32776.0f), c_l23 = p2(-136.0f, -32776.0f);
  const uint64_t c_h = p2(-524296.0f, -2056.0f);
  uint64_t a = 0, b = 0;  // two independent FMA chains of f32 pairs
  const uint32_t wv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t w = wv[g], w2 = w >> 16;
    // elements 4g, 4g+1 (low nibbles of bytes 0, 1), 4g+2, 4g+3 (bytes 2, 3),
    // then the high nibbles: elements 16 + 4g .. 16 + 4g + 3
    const uint64_t l01 = p2add(p2(magr<0xFu>(w, M.m0), magr<0xF00u>(w, M.m8)), c_l01);
    const uint64_t l23 = p2add(p2(magr<0xF0000u>(w, M.m16), magr<0xF00u>(w2, M.m8)), c_l23);
    const uint64_t h01 = p2add(p2(magr<0xF0u>(w, M.m4), magr<0xF000u>(w, M.m12)), c_h);
    const uint64_t h23 = p2add(p2(magr<0xF0u>(w2, M.m4), magr<0xF000u>(w2, M.m12)), c_h);
    a = p2fma(l01, xp[2 * g], a);
    b = p2fma(l23, xp[2 * g + 1], b);
    a = p2fma(h01, xp[8 + 2 * g], a);
    b = p2fma(h23, xp[9 + 2 * g], b);
  }
  const float2 s = up2(p2add(a, b));
  return __fadd_rn(s.x, s.y);
}

// Two nibbles into one f32 pair and the magic offsets removed, in one asm
// block, so the pair is built in place rather than moved together.
template <uint32_t MA, uint32_t MB>
__device__ __forceinline__ uint64_t nib_pair(uint32_t wa, uint32_t wb, uint32_t ea, uint32_t eb, uint64_t c) {
  uint64_t r;
  asm("{\n\t.reg .b32 a, b;\n\t.reg .b64 t;\n\t"
      "lop3.b32 a, %1, %5, %3, 0xEA;\n\t"
      "lop3.b32 b, %2, %6, %4, 0xEA;\n\t"
      "mov.b64 t, {a, b};\n\t"
      "add.rn.f32x2 %0, t, %7;\n\t}"
      : "=l"(r)
      : "r"(wa), "r"(wb), "r"(ea), "r"(eb), "n"(MA), "n"(MB), "l"(c));
  return r;
}

// The same block sum with the pairs built by nib_pair.
__device__ __forceinline__ float q4_0_block_fast2(uint4 p, const uint64_t (&xp)[16], const pb_magics& M) {
  const uint64_t c_l01 = p2(-8388616.0f, -32776.0f), c_l23 = p2(-136.0f, -32776.0f);
  const uint64_t c_h = p2(-524296.0f, -2056.0f);
  uint64_t a = 0, b = 0;
  const uint32_t wv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t w = wv[g], w2 = w >> 16;
    a = p2fma(nib_pair<0xFu, 0xF00u>(w, w, M.m0, M.m8, c_l01), xp[2 * g], a);
    b = p2fma(nib_pair<0xF0000u, 0xF00u>(w, w2, M.m16, M.m8, c_l23), xp[2 * g + 1], b);
    a = p2fma(nib_pair<0xF0u, 0xF000u>(w, w, M.m4, M.m12, c_h), xp[8 + 2 * g], a);
    b = p2fma(nib_pair<0xF0u, 0xF000u>(w2, w2, M.m4, M.m12, c_h), xp[9 + 2 * g], b);
  }
  const float2 s = up2(p2add(a, b));
  return __fadd_rn(s.x, s.y);
}

// Scalar form: one logic op, one add and one FMA per weight, no pairs.
__device__ __forceinline__ float q4_0_block_scalar(uint4 p, const uint64_t (&xp)[16], const pb_magics& M) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  const uint32_t wv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t w = wv[g], w2 = w >> 16;
    const float2 xl01 = up2(xp[2 * g]), xl23 = up2(xp[2 * g + 1]), xh01 = up2(xp[8 + 2 * g]), xh23 = up2(xp[9 + 2 * g]);
    a0 = __fmaf_rn(__fadd_rn(magr<0xFu>(w, M.m0), -8388616.0f), xl01.x, a0);
    a1 = __fmaf_rn(__fadd_rn(magr<0xF00u>(w, M.m8), -32776.0f), xl01.y, a1);
    a2 = __fmaf_rn(__fadd_rn(magr<0xF0000u>(w, M.m16), -136.0f), xl23.x, a2);
    a3 = __fmaf_rn(__fadd_rn(magr<0xF00u>(w2, M.m8), -32776.0f), xl23.y, a3);
    a0 = __fmaf_rn(__fadd_rn(magr<0xF0u>(w, M.m4), -524296.0f), xh01.x, a0);
    a1 = __fmaf_rn(__fadd_rn(magr<0xF000u>(w, M.m12), -2056.0f), xh01.y, a1);
    a2 = __fmaf_rn(__fadd_rn(magr<0xF0u>(w2, M.m4), -524296.0f), xh23.x, a2);
    a3 = __fmaf_rn(__fadd_rn(magr<0xF000u>(w2, M.m12), -2056.0f), xh23.y, a3);
  }
  return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}

// Q8_0 block (gguf.js:239-257): byte j is element j; a byte becomes the
// exact float 2^15 + (q + 128) by one byte permute with the exponent
// pattern (q biased by 128 first), a packed add removes 2^15 + 128.
__device__ __forceinline__ float q8_0_block_fast(uint4 p0, uint4 p1, const uint64_t (&xp)[16]) {
  const uint64_t c = p2(-32896.0f, -32896.0f);
  uint64_t a = 0, b = 0;
  const uint32_t wv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t u = wv[i] ^ 0x80808080u;
    const uint64_t e01 = p2add(p2(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7504)),
                                  __uint_as_float(__byte_perm(u, PB_MAG8, 0x7514))), c);
    const uint64_t e23 = p2add(p2(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7524)),
                                  __uint_as_float(__byte_perm(u, PB_MAG8, 0x7534))), c);
    a = p2fma(e01, xp[2 * i], a);
    b = p2fma(e23, xp[2 * i + 1], b);
  }
  const float2 s = up2(p2add(a, b));
  return __fadd_rn(s.x, s.y);
}

// x (RMS-normalised when w is set) into shared memory, float4 chunks
// swizzled within each 32-value block (bank-conflict-free reads of one block
// per lane).  Any K: the threads loop over the chunks.
// The sum of squares runs over a fixed partition (128 lanes, chunk c on lane
// c % 128 in ascending order, then a fixed tree), so it does not depend on
// the CTA size: every launch shape of the same vector normalises it to the
// same bits.  Loads go out in batches of 4 per thread before any is used, so
// staging costs one memory latency per batch, not one per chunk.
constexpr int MVF_XB = 4;
__device__ __forceinline__ void mvf_stage_x(const float* __restrict__ x, const float* __restrict__ w, double eps, int K,
                                            float4* xs4, double* red) {
  const int tid = threadIdx.x, nt = blockDim.x, nc = K / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  double rms = 0.0;
  if (w) {
    if (tid < 128) {
      double ss = 0.0;
      for (int c0 = tid; c0 < nc; c0 += 128 * MVF_XB) {
        float4 v[MVF_XB];
#pragma unroll
        for (int j = 0; j < MVF_XB; ++j)
          if (c0 + 128 * j < nc) v[j] = x4[c0 + 128 * j];
#pragma unroll
        for (int j = 0; j < MVF_XB; ++j) {
          if (c0 + 128 * j < nc) {
            ss = __fma_rn((double)v[j].x, (double)v[j].x, ss);
            ss = __fma_rn((double)v[j].y, (double)v[j].y, ss);
            ss = __fma_rn((double)v[j].z, (double)v[j].z, ss);
            ss = __fma_rn((double)v[j].w, (double)v[j].w, ss);
          }
        }
      }
      ss = pb_warp_sum_d(ss);
      if ((tid & 31) == 0) red[tid >> 5] = ss;
    }
    __syncthreads();
    const double ss = __dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3]));
    rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)K), eps));
  }
  // the fast path scales in f32 by 1 / rms (rms itself in double): two f32
  // roundings per element instead of the reference's double (x / rms) * w
  const float inv = w ? (float)(1.0 / rms) : 1.0f;
  for (int c0 = tid; c0 < nc; c0 += nt * MVF_XB) {
    float4 v[MVF_XB], wv[MVF_XB];
#pragma unroll
    for (int j = 0; j < MVF_XB; ++j) {
      const int c = c0 + nt * j;
      if (c < nc) {
        v[j] = x4[c];
        if (w) wv[j] = w4[c];
      }
    }
#pragma unroll
    for (int j = 0; j < MVF_XB; ++j) {
      const int c = c0 + nt * j;
      if (c < nc) {
        float4 o = v[j];
        if (w) {
          o.x = __fmul_rn(__fmul_rn(o.x, inv), wv[j].x);
          o.y = __fmul_rn(__fmul_rn(o.y, inv), wv[j].y);
          o.z = __fmul_rn(__fmul_rn(o.z, inv), wv[j].z);
          o.w = __fmul_rn(__fmul_rn(o.w, inv), wv[j].w);
        }
        const int bj = c >> 3, ci = c & 7;
        xs4[bj * 8 + (ci ^ (bj & 7))] = o;
      }
    }
  }
}

// The same staging for K <= 2048 with the norm (the qkv and gate-up
// prologues): threads below 128 hold their chunks of x -- one batch, so the
// same chunks and order as above -- in registers from the sum of squares to
// the scaling, and the norm weights arrive in wr before the dependency wait:
// one pass over x in L2 instead of two, the same bits.
__device__ __forceinline__ bool mvf_x_in_regs(const float* w, int K) { return w && K / 4 <= 128 * MVF_XB; }
__device__ __forceinline__ void mvf_load_w(const float* __restrict__ w, int K, float4 (&wr)[MVF_XB]) {
  const int tid = threadIdx.x, nc = K / 4;
  if (tid < 128)
#pragma unroll
    for (int j = 0; j < MVF_XB; ++j)
      if (tid + 128 * j < nc) wr[j] = reinterpret_cast<const float4*>(w)[tid + 128 * j];
}
__device__ __forceinline__ void mvf_stage_x_regs(const float* __restrict__ x, double eps, int K, const float4 (&wr)[MVF_XB],
                                                 float4* xs4, double* red) {
  const int tid = threadIdx.x, nc = K / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4 v[MVF_XB];
  if (tid < 128) {
#pragma unroll
    for (int j = 0; j < MVF_XB; ++j)
      if (tid + 128 * j < nc) v[j] = x4[tid + 128 * j];
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < MVF_XB; ++j) {
      if (tid + 128 * j < nc) {
        ss = __fma_rn((double)v[j].x, (double)v[j].x, ss);
        ss = __fma_rn((double)v[j].y, (double)v[j].y, ss);
        ss = __fma_rn((double)v[j].z, (double)v[j].z, ss);
        ss = __fma_rn((double)v[j].w, (double)v[j].w, ss);
      }
    }
    ss = pb_warp_sum_d(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
  }
  __syncthreads();
  if (tid < 128) {
    const double ss = __dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3]));
    const double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)K), eps));
    const float inv = (float)(1.0 / rms);
#pragma unroll
    for (int j = 0; j < MVF_XB; ++j) {
      const int c = tid + 128 * j;
      if (c < nc) {
        float4 o = v[j];
        o.x = __fmul_rn(__fmul_rn(o.x, inv), wr[j].x);
        o.y = __fmul_rn(__fmul_rn(o.y, inv), wr[j].y);
        o.z = __fmul_rn(__fmul_rn(o.z, inv), wr[j].z);
        o.w = __fmul_rn(__fmul_rn(o.w, inv), wr[j].w);
        const int bj = c >> 3, ci = c & 7;
        xs4[bj * 8 + (ci ^ (bj & 7))] = o;
      }
    }
  }
}

constexpr int MVF_NS = 2;  // shared-memory stages of weight payload per warp

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// CTA of W warps = TPC tiles x KC chunks per iteration (TPC = W / KC).
// TYPE Q4_0 or Q8_0; LAYOUT ROWS (matvec weights) or TILED8 (a head table:
// block b of the tile's 8 rows is 8 consecutive slots).
// The payload streams through shared memory: each lane copies its own 16-byte
// pieces with cp.async into its warp's stage buffer, MVF_NS units ahead, and
// reads back only what it copied (no cross-lane hand-off, so no barrier); the
// scales are loaded into registers one unit ahead.  The loads of the next
// units are therefore in flight while a unit is computed, and the CTA's
// later tiles are bulk-prefetched into L2 further ahead still.
template <int TYPE, int LAYOUT, int VAR = 0>
__global__ void __launch_bounds__(MVF_MAX_WARPS * 32, 1)
k_mvf(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int N, int nb, int tile_begin, int tile_end,
      int row_end, const float* __restrict__ x, float* __restrict__ y, pb_mv_epi epi, pb_magics M, int* err) {
  constexpr int QB = TYPE == PB_TYPE_Q8_0 ? 32 : 16;  // payload bytes per block
  constexpr int PL = QB / 16;                          // 16-byte pieces per block
  constexpr int STAGE = 8 * 32 * QB;                   // one unit: 8 rows x 32 lanes
  extern __shared__ __align__(16) unsigned char mvf_raw[];
  __shared__ double red[MVF_MAX_WARPS];
  const int K = nb * 32, KC = (nb + 31) >> 5, W = blockDim.x >> 5, TPC = W / KC;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tl = warp / KC, ch = warp - tl * KC;  // this warp's tile slot and K chunk
  const bool active = tl < TPC;
  const int b = ch * 32 + lane;
  const bool has_b = active && b < nb;
  float4* xs4 = reinterpret_cast<float4*>(mvf_raw);                  // [K / 4] swizzled
  float* part = reinterpret_cast<float*>(mvf_raw + (size_t)K * 4);   // [2][TPC][KC][8]
  unsigned char* wst = mvf_raw + (size_t)K * 4 + (((size_t)2 * TPC * KC * 8 * 4 + 15) & ~(size_t)15) +
                       (size_t)warp * MVF_NS * STAGE;                // this warp's stages
  const int per_iter = gridDim.x * TPC;
  const int n_iter = (tile_end - tile_begin + per_iter - 1) / per_iter;  // CTA-uniform
  const uint4* q4 = reinterpret_cast<const uint4*>(qs);
  const size_t tq = (size_t)8 * nb * QB, td = (size_t)8 * nb * 2;
  auto tile_of = [&](int it) { return tile_begin + it * per_iter + blockIdx.x * TPC + tl; };
  auto live = [&](int it) { return has_b && it < n_iter && tile_of(it) < tile_end; };
  auto slot_of = [&](int t, int r) {
    return LAYOUT == PB_LAYOUT_TILED8 ? ((size_t)t * nb + b) * 8 + r : (size_t)(t * 8 + r) * nb + b;
  };
  // L2 prefetch: the chunk-0 warp of each tile slot fetches its tile (payload
  // and scales are contiguous per tile) MVF_PF iterations ahead
  auto prefetch = [&](int it) {
    const int t = tile_of(it);
    if (active && ch == 0 && lane == 0 && it < n_iter && t < tile_end) {
      pb_l2_prefetch(qs + (size_t)t * tq, (uint32_t)tq);
      pb_l2_prefetch(dsc + (size_t)t * td / 2, (uint32_t)td);
    }
  };
  // unit `it`'s payload into stage it % MVF_NS (one commit group per unit,
  // empty when the unit is past the end, so the group count stays regular)
  auto issue = [&](int it) {
    if (live(it)) {
      const int t = tile_of(it);
      unsigned char* st = wst + (size_t)(it % MVF_NS) * STAGE;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const size_t slot = slot_of(t, r);
#pragma unroll
        for (int u = 0; u < PL; ++u) cp_async16(st + ((size_t)(r * 32 + lane) * PL + u) * 16, q4 + slot * PL + u);
      }
    }
    cp_async_commit();
  };
  auto scales = [&](int it, uint32_t (&pd)[8]) {
    if (live(it)) {
      const int t = tile_of(it);
#pragma unroll
      for (int r = 0; r < 8; ++r) pd[r] = __ldcs(dsc + slot_of(t, r));
    }
  };
  for (int i = 0; i < MVF_PF; ++i) prefetch(i);
  if (tid == 0)
    for (int i = 0; i < PB_MAX_L2_NEXT; ++i) pb_l2_prefetch_share(epi.l2_next[i], epi.l2_next_bytes[i], blockIdx.x, gridDim.x);
  // weights do not depend on the previous kernel: the first units go out before the wait
#pragma unroll
  for (int i = 0; i < MVF_NS; ++i) issue(i);
  uint32_t pd[8], pdn[8];
  scales(0, pd);
  const bool xr = mvf_x_in_regs(epi.norm_w, K);
  float4 wr[MVF_XB];
  if (xr) mvf_load_w(epi.norm_w, K, wr);
  pb_pdl_trigger();
  pb_pdl_wait();  // x (and the residual) come from the previous kernel
  if (xr) mvf_stage_x_regs(x, epi.eps, K, wr, xs4, red);
  else mvf_stage_x(x, epi.norm_w, epi.eps, K, xs4, red);
  __syncthreads();
  // a residual epilogue's rows are loaded one tile ahead, during the sums
  // (independent loads: nothing waits on them until the store)
  auto res_row = [&](int it) -> float {
    const int row = tile_of(it) * 8 + (lane >> 2);
    return epi.kind == PB_EPI_RESIDUAL && active && ch == 0 && (lane & 3) == 0 && it < n_iter &&
                   tile_of(it) < tile_end && row < row_end && row < N
               ? epi.residual[row]
               : 0.0f;
  };
  float res = res_row(0);
  uint64_t xp[16];
  if (has_b) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = xs4[b * 8 + (i ^ (b & 7))];
      xp[2 * i] = p2(v.x, v.y);
      xp[2 * i + 1] = p2(v.z, v.w);
    }
  }
  for (int it = 0; it < n_iter; ++it) {
    prefetch(it + MVF_PF);
    scales(it + 1, pdn);
    asm volatile("cp.async.wait_group %0;" ::"n"(MVF_NS - 1) : "memory");  // unit it has landed
    const int t = tile_of(it);
    float v[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) v[r] = 0.0f;
    if (live(it)) {
      const unsigned char* st = wst + (size_t)(it % MVF_NS) * STAGE;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint4* pp = reinterpret_cast<const uint4*>(st + (size_t)(r * 32 + lane) * QB);
        // the scale as the kernel being replaced decodes it: the WASM matvec's
        // (wasm-q4.js:88-109) for matvec weights, the exact one of the table
        // the reference's head reads (gguf.js:55-70)
        const float d = LAYOUT == PB_LAYOUT_TILED8 ? pb_f16_exact(pd[r]) : pb_f16_wasm(pd[r]);
        const float bs = TYPE == PB_TYPE_Q8_0 ? q8_0_block_fast(pp[0], pp[PL - 1], xp)
                         : VAR == 1 ? q4_0_block_fast2(pp[0], xp, M)
                         : VAR == 2 ? q4_0_block_scalar(pp[0], xp, M)
                                    : q4_0_block_fast(pp[0], xp, M);
        v[r] = __fmul_rn(bs, d);
      }
    }
    issue(it + MVF_NS);  // this lane read its own pieces of the stage: refill it
#pragma unroll
    for (int r = 0; r < 8; ++r) pd[r] = pdn[r];
    // transposed butterfly over the lanes: lane 4r ends with row r's sum
    float w4[4], w2[2];
    const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = b16 ? v[i] : v[i + 4], keep = b16 ? v[i + 4] : v[i];
      w4[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 16));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = b8 ? w4[i] : w4[i + 2], keep = b8 ? w4[i + 2] : w4[i];
      w2[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 8));
    }
    float z;
    {
      const float send = b4 ? w2[0] : w2[1], keep = b4 ? w2[1] : w2[0];
      z = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
    }
    z = __fadd_rn(z, __shfl_xor_sync(0xffffffffu, z, 2));
    z = __fadd_rn(z, __shfl_xor_sync(0xffffffffu, z, 1));
    // lane 4r: row r = 4 bit4 + 2 bit3 + bit2 of the lane
    const int row_of_lane = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    float* pbuf = part + (size_t)(it & 1) * TPC * KC * 8;
    if (active && (lane & 3) == 0) pbuf[((size_t)tl * KC + ch) * 8 + row_of_lane] = z;
    __syncthreads();
    if (active && ch == 0 && t < tile_end) {
      const int rr = lane >> 2;
      float s_ = pbuf[(size_t)tl * KC * 8 + rr];
      for (int c = 1; c < KC; ++c) s_ = __fadd_rn(s_, pbuf[((size_t)tl * KC + c) * 8 + rr]);
      if (epi.kind == PB_EPI_RESIDUAL) {  // pb_mv_epilogue's residual store, the row loaded above
        const int row = t * 8 + rr;
        if ((lane & 3) == 0 && row < row_end && row < N) y[row] = __fadd_rn(res, s_);
        res = res_row(it + 1);
      } else {
        pb_mv_epilogue(s_, t, N, 0, row_end, y, epi, err);
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // no copy outlives the CTA
}

static size_t mvf_smem(const pb_qmat* w, int W) {
  const int KC = (w->nb + 31) / 32, TPC = W / KC, QB = w->type == PB_TYPE_Q8_0 ? 32 : 16;
  return (size_t)w->K * 4 + (((size_t)2 * TPC * KC * 8 * 4 + 15) & ~(size_t)15) + (size_t)W * MVF_NS * 8 * 32 * QB;
}

// Warps per CTA: small matrices get small CTAs (more SMs share the rows),
// large ones up to 16 warps; at least one warp per K chunk; within the
// shared-memory budget.
static int mvf_warps(const pb_qmat* w, int ntiles, int sm_count) {
  const int KC = (w->nb + 31) / 32;
  int W = 4;
  while (W < MVF_MAX_WARPS && (int64_t)ntiles * KC / W >= 2 * sm_count) W *= 2;
  while (W < KC) W *= 2;
  while (W > KC && W > 4 && mvf_smem(w, W) > (size_t)200 * 1024) W /= 2;
  return W;
}

static int launch_mvf(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int tile_begin, int ntiles,
                      int row_end, const pb_mv_epi& epi) {
  const int KC = (w->nb + 31) / 32;
  const int W = mvf_warps(w, ntiles, ctx->sm_count), TPC = W / KC;
  const size_t smem = mvf_smem(w, W);
  if (smem > (size_t)200 * 1024)
    return pb_set_error(ctx, PB_ERR_ARG, "fast matvec: K=%d needs %zu bytes of shared memory", w->K, smem);
  const int groups = (ntiles + TPC - 1) / TPC;
  int per_sm = MVF_MAX_WARPS / W;  // CTAs resident at once: registers ...
  const int by_smem = (int)((size_t)220 * 1024 / (smem + 1024));
  per_sm = per_sm < by_smem ? per_sm : by_smem;  // ... and shared memory
  if (per_sm < 1) per_sm = 1;
  const int cap = ctx->sm_count * per_sm;
  const int grid = groups < cap ? groups : cap;
  static const int var = getenv("PB_MVF_VARIANT") ? atoi(getenv("PB_MVF_VARIANT")) : 0;  // arithmetic form (tuning)
  auto kern = w->type == PB_TYPE_Q8_0
                  ? (w->layout == PB_LAYOUT_TILED8 ? k_mvf<PB_TYPE_Q8_0, PB_LAYOUT_TILED8> : k_mvf<PB_TYPE_Q8_0, PB_LAYOUT_ROWS>)
                  : w->layout == PB_LAYOUT_TILED8 ? k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_TILED8>
                  : var == 1 ? k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_ROWS, 1>
                  : var == 2 ? k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_ROWS, 2> : k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_ROWS>;
  return pb_launch(ctx, "k_mvf", true, kern, dim3(grid), dim3(W * 32), smem, (const uint8_t*)w->qs,
                   (const uint16_t*)w->d, w->N, w->nb, tile_begin, tile_begin + ntiles, row_end, x, y, epi,
                   pb_magics{PB_MAG0, PB_MAG4, PB_MAG8, PB_MAG12, PB_MAG16}, ctx->d_err);
}

// ---------------------------------------------------------------------------
// Fused decode projection + attention (fast mode, one sequence,
// llama-streaming.js:505-573): the RMSNorm -> [wq; wk; wv] matvec with RoPE
// and the KV write at pos, and the decode attention, in one kernel.  Separate,
// the attention waits for the whole projection grid to finish (a dependent
// launch costs about 2 us per link); here the 8 CTAs that attend for kv head
// g (one cluster, as k_attn_dec_fast) first compute g's own rows of the
// projection -- PER q heads, k and v, (PER + 2) x 64 rows, PER + 2 8-row
// tiles per CTA -- and meet at a cluster barrier.
//   - before griddepcontrol.wait: the CTA's weight payloads and scales
//     (final) and its split's K/V rows before pos into shared memory;
//   - after it: x into shared memory, RMS-normalised as k_mvf does; each warp
//     computes (8-row tile, 32-block chunk) units with k_mvf's block sums,
//     scales and transposed reduction, the chunks added in order, and the
//     tile goes through the matvec epilogue (RoPE on q and k, k and v into the
//     cache at pos, q to y): the same bits as k_mvf;
//   - cluster barrier (the group's q, k and v are written), then q and the
//     row at pos (L2 reads: written by the other CTAs) and aq_attend, the
//     attention of k_attn_dec_fast on the first 128 threads: the same bits.
// Measured at the Llama-3.2-1B shape it is slower than the two kernels (15.6
// against 6.3 + 5.8 us of marginal time per layer, 0.617 against 0.561 ms
// per decode step): the projection's 768 units of 8 rows x 32 blocks run on
// the 64 SMs of the clusters (12 per SM instead of about 5), and the
// clusters (206 KB of shared memory per CTA with a 2048-position cache) start
// only when 8 SMs of a GPC are free.  Off by default (pb_set_fuse_attn).
// ---------------------------------------------------------------------------
constexpr int QA_THREADS = 256;
constexpr int QA_SMEM_MAX = 220 * 1024;  // dynamic shared memory (the static part is about 1 KB)

static size_t qa_smem(const pb_qmat* w, int per, int pmax) {
  const int KC = w->nb / 32, units = (per + 2) * KC;
  return (size_t)w->K * 4 + (size_t)units * 256 * 16 + (size_t)units * 256 * 2 + (size_t)(per + 2) * KC * 8 * 4 +
         aq_smem(per, pmax);
}

template <int PER>
__global__ void __launch_bounds__(QA_THREADS)
k_qkv_attn(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int N, int nb,
           const float* __restrict__ x, float* __restrict__ y, pb_mv_epi epi, float scale, float* __restrict__ out,
           int pmax, pb_magics M, int* err) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  constexpr int TPC = PER + 2;  // 8-row tiles per CTA: (PER + 2) x 64 rows over the 8 CTAs of the group
  extern __shared__ __align__(16) unsigned char qa_raw[];
  const int K = nb * 32, KC = nb / 32, units = TPC * KC;
  float4* xs4 = reinterpret_cast<float4*>(qa_raw);                                  // [K / 4] swizzled
  unsigned char* wst = qa_raw + (size_t)K * 4;                                      // [unit][8 rows][32 lanes] x 16 B
  uint16_t* dst_s = reinterpret_cast<uint16_t*>(wst + (size_t)units * 4096);      // [unit][8 rows][32 lanes]
  float* cpart = reinterpret_cast<float*>(dst_s + (size_t)units * 256);           // [tile][chunk][8]
  float* ks = cpart + (size_t)TPC * KC * 8;                                         // attention: K, V, scores, q, PV
  float* vs = ks + (size_t)pmax * AQ_KLD;
  float* sc = vs + (size_t)pmax * AQ_HD;
  float* qsm = sc + (size_t)PER * pmax;
  float* gp = qsm + PER * AQ_HD;
  __shared__ aq_parts<PER> pt;
  __shared__ double red[4];
  const int g = blockIdx.x, sp = (int)cl.block_rank(), nsplit = (int)cl.num_blocks(), tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int pos = *epi.pos_dev;
  const int cache_len = pos + 1, max_len = epi.max_len;
  const int P = (cache_len + nsplit - 1) / nsplit;
  if (pos < 0 || cache_len > max_len || P > pmax) {  // the same for every CTA: all leave before any barrier
    pb_pdl_trigger();
    pb_pdl_wait();
    if (tid == 0 && g == 0 && sp == 0) pb_raise(err, PB_DEVERR_BOUNDS);
    return;
  }
  const int qt = epi.q_rows / 8, kt = epi.kv_rows / 8;
  auto gtile = [&](int lt) {  // local tile of the group -> 8-row tile of the matrix
    return lt < PER * 8 ? g * PER * 8 + lt : lt < PER * 8 + 8 ? qt + g * 8 + (lt - PER * 8) : qt + kt + g * 8 + (lt - PER * 8 - 8);
  };
  // the CTA's weight payloads and scales: item (unit u, row r, lane), unit u =
  // (tile u / KC, chunk u % KC), lane = block (u % KC) * 32 + lane
  for (int i = tid; i < units * 256; i += QA_THREADS) {
    const int u = i >> 8, r = (i >> 5) & 7, b = (u % KC) * 32 + (i & 31);
    const int t = gtile(sp * TPC + u / KC);
    cp_async16(wst + (size_t)i * 16, qs + ((size_t)(t * 8 + r) * nb + b) * 16);
  }
  for (int i = tid; i < units * 32; i += QA_THREADS) {  // 8 scales per 16-byte piece
    const int u = i >> 5, r = (i >> 2) & 7, c = i & 3;
    const int t = gtile(sp * TPC + u / KC);
    cp_async16(dst_s + ((size_t)u * 8 + r) * 32 + c * 8, dsc + (size_t)(t * 8 + r) * nb + (u % KC) * 32 + c * 8);
  }
  // the split's K and V rows before pos (final: written by earlier steps)
  const int kv_dim = epi.kv_rows;
  const int j0 = sp * P;
  const int n = cache_len - j0 < 0 ? 0 : (cache_len - j0 < P ? cache_len - j0 : P);
  const bool has_pos = pos >= j0 && pos < j0 + n;
  const int npre = has_pos ? n - 1 : n;
  const float* kb = epi.kc + (size_t)g * AQ_HD;
  const float* vb = epi.vc + (size_t)g * AQ_HD;
  for (int i = tid; i < npre * 16; i += QA_THREADS) {
    const int r = i >> 4, c = i & 15;
    const size_t src = (size_t)(j0 + r) * kv_dim + 4 * c;
    cp_async16(ks + r * AQ_KLD + 4 * c, kb + src);
    cp_async16(vs + r * AQ_HD + 4 * c, vb + src);
  }
  cp_async_commit();
  if (tid == 0) {
    const int cta = (int)(blockIdx.y * gridDim.x + blockIdx.x), ncta = (int)(gridDim.x * gridDim.y);
    for (int i = 0; i < PB_MAX_L2_NEXT; ++i) pb_l2_prefetch_share(epi.l2_next[i], epi.l2_next_bytes[i], cta, ncta);
  }
  pb_pdl_trigger();
  pb_pdl_wait();  // x comes from the previous kernel
  mvf_stage_x(x, epi.norm_w, epi.eps, K, xs4, red);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  // the units, k_mvf's arithmetic: warp w takes units w, w + 8, ...
  for (int u = warp; u < units; u += QA_THREADS / 32) {
    const int lt = u / KC, ch = u % KC, b = ch * 32 + lane;
    uint64_t xp[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = xs4[b * 8 + (i ^ (b & 7))];
      xp[2 * i] = p2(v.x, v.y);
      xp[2 * i + 1] = p2(v.z, v.w);
    }
    float v[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint4 pp = *reinterpret_cast<const uint4*>(wst + ((size_t)u * 256 + r * 32 + lane) * 16);
      const float d = pb_f16_wasm(dst_s[((size_t)u * 8 + r) * 32 + lane]);
      v[r] = __fmul_rn(q4_0_block_fast(pp, xp, M), d);
    }
    // transposed butterfly over the lanes: lane 4r ends with row r's sum
    float w4[4], w2[2];
    const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = b16 ? v[i] : v[i + 4], keep = b16 ? v[i + 4] : v[i];
      w4[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 16));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = b8 ? w4[i] : w4[i + 2], keep = b8 ? w4[i + 2] : w4[i];
      w2[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 8));
    }
    float z;
    {
      const float send = b4 ? w2[0] : w2[1], keep = b4 ? w2[1] : w2[0];
      z = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
    }
    z = __fadd_rn(z, __shfl_xor_sync(0xffffffffu, z, 2));
    z = __fadd_rn(z, __shfl_xor_sync(0xffffffffu, z, 1));
    const int row_of_lane = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    if ((lane & 3) == 0) cpart[((size_t)lt * KC + ch) * 8 + row_of_lane] = z;
  }
  __syncthreads();
  // each tile: the chunks added in order, then the matvec epilogue
  for (int lt = warp; lt < TPC; lt += QA_THREADS / 32) {
    const int rr = lane >> 2;
    float s_ = cpart[(size_t)lt * KC * 8 + rr];
    for (int c = 1; c < KC; ++c) s_ = __fadd_rn(s_, cpart[((size_t)lt * KC + c) * 8 + rr]);
    pb_mv_epilogue(s_, gtile(sp * TPC + lt), N, 0, N, y, epi, err);
  }
  cl.sync();  // the group's q, k and v rows are written
  if (has_pos && tid < 32) {
    const int r = pos - j0, c = tid & 15;
    const float* src = (tid < 16 ? kb : vb) + (size_t)pos * kv_dim + 4 * c;
    float* dst = tid < 16 ? ks + r * AQ_KLD + 4 * c : vs + r * AQ_HD + 4 * c;
    *reinterpret_cast<float4*>(dst) = __ldcg(reinterpret_cast<const float4*>(src));
  }
  for (int i = tid; i < PER * AQ_HD / 4; i += QA_THREADS)
    reinterpret_cast<float4*>(qsm)[i] = __ldcg(reinterpret_cast<const float4*>(y + (size_t)g * PER * AQ_HD) + i);
  __syncthreads();
  aq_attend<PER>(cl, ks, vs, sc, qsm, gp, pt, n, pmax, scale, out + (size_t)g * PER * AQ_HD);
}

// Whether the fused projection + attention takes the layer: the fast decode
// attention's shape, a Q4_0 row-layout [q | k | v] matrix with K a multiple of
// 1024, and its shared memory.
bool pb_qkv_attn_ok(const pb_qmat* w, int n_heads, int n_kv, int hd, int max_len) {
  if (!w || w->type != PB_TYPE_Q4_0 || w->layout != PB_LAYOUT_ROWS || w->nb % 32 || hd != AQ_HD || n_kv <= 0 ||
      n_heads % n_kv || n_heads / n_kv > AQ_MAX_SPLIT || w->N != (n_heads + 2 * n_kv) * hd)
    return false;
  const int pmax = (max_len + AQ_MAX_SPLIT - 1) / AQ_MAX_SPLIT;
  return pmax <= AQ_MAXP && qa_smem(w, n_heads / n_kv, pmax) <= (size_t)QA_SMEM_MAX;
}

// The projection of e (RoPE + KV epilogue, its norm and L2 hints) and the
// decode attention into out, in one launch.
int pb_launch_qkv_attn(pb_ctx* ctx, const pb_qmat* w, const float* x, float* qkv_out, const pb_mv_epi& e, int n_heads,
                       int n_kv, float* out) {
  if (e.kind != PB_EPI_ROPE_KV || !e.pos_dev || !pb_qkv_attn_ok(w, n_heads, n_kv, e.head_dim, e.max_len))
    return pb_set_error(ctx, PB_ERR_ARG, "fused projection + attention: unsupported shape");
  const int per = n_heads / n_kv, pmax = (e.max_len + AQ_MAX_SPLIT - 1) / AQ_MAX_SPLIT;
  const float scale = (float)(1.0 / sqrt((double)e.head_dim));  // llama-streaming.js:546
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_kv, AQ_MAX_SPLIT);
  cfg.blockDim = dim3(QA_THREADS);
  cfg.dynamicSmemBytes = qa_smem(w, per, pmax);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = AQ_MAX_SPLIT;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ctx->pdl ? 2 : 1;
  const pb_magics M{PB_MAG0, PB_MAG4, PB_MAG8, PB_MAG12, PB_MAG16};
  cudaError_t err = cudaErrorInvalidValue;
  switch (per) {
#define PB_QA_CASE(P)                                                                                           \
  case P:                                                                                                       \
    err = cudaLaunchKernelEx(&cfg, k_qkv_attn<P>, (const uint8_t*)w->qs, (const uint16_t*)w->d, w->N, w->nb, x, \
                             qkv_out, e, scale, out, pmax, M, ctx->d_err);                                      \
    break;
    PB_QA_CASE(1) PB_QA_CASE(2) PB_QA_CASE(3) PB_QA_CASE(4) PB_QA_CASE(5) PB_QA_CASE(6) PB_QA_CASE(7) PB_QA_CASE(8)
#undef PB_QA_CASE
    default: break;
  }
  if (err != cudaSuccess) return pb_cuda_error(ctx, err, "k_qkv_attn");
  return pb_check_launch(ctx, "k_qkv_attn");
}

// The LM head in the fast mode: the fast kernel over the head table (Q4_0 /
// Q8_0, either layout) with the final RMSNorm prologue and the logits +
// greedy argmax epilogue.  The exact kernel (k_head) keeps batch_dot's order.
int pb_launch_head_fast(pb_ctx* ctx, const pb_qmat* t, const float* h, const float* norm_w, double eps, float* logits,
                        unsigned long long* amax) {
  if ((t->type != PB_TYPE_Q4_0 && t->type != PB_TYPE_Q8_0) || t->nb > 32 * MVF_MAX_WARPS)
    return pb_set_error(ctx, PB_ERR_ARG, "fast head: Q4_0 or Q8_0 table, K <= %d", 32 * 32 * MVF_MAX_WARPS);
  pb_mv_epi e;
  e.kind = amax ? PB_EPI_ARGMAX : PB_EPI_STORE;
  e.norm_w = norm_w;
  e.eps = eps;
  e.amax = amax;
  if (ctx->mvt && pb_mvt_ok(t)) return pb_launch_mvt(ctx, t, h, logits, 0, t->N, e);
  if (t->mq && t->mma_ok && t->layout == PB_LAYOUT_ROWS && t->type == PB_TYPE_Q4_0 && t->N >= ctx->mvi_min_rows)
    return pb_launch_mvi(ctx, t, h, logits, 0, t->N, e);
  return launch_mvf(ctx, t, h, logits, 0, (t->N + 7) / 8, t->N, e);
}

static size_t mvw_smem(const pb_qmat* w) {
  return (size_t)2 * mvw_slots(w->nb) * w->nb * 32 * 4 + (size_t)w->nb * 32 * 4;
}

static size_t mv_smem(const pb_qmat* w, int nt) {
  return (size_t)2 * mv_slots(w->nb, nt) * w->nb * 32 * 4 + (size_t)w->nb * 32 * 4;
}

template <int TYPE, int NT>
static int launch_mv_nt(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int tile_begin, int ntiles,
                        int row_end, const pb_mv_epi& epi) {
  // persistent, at most one CTA per SM; a small matrix leaves SMs free, where
  // the next kernel's CTAs start early (programmatic dependent launch)
  const int S = mv_slots(w->nb, NT), groups = (ntiles + S - 1) / S;
  const int grid = groups < ctx->sm_count ? groups : ctx->sm_count;
  return pb_launch(ctx, "k_matvec", true, k_matvec<TYPE, NT>, dim3(grid), dim3(NT), mv_smem(w, NT),
                   (const uint8_t*)w->qs, (const uint16_t*)w->d, (const uint16_t*)w->m, w->N, w->nb, tile_begin,
                   tile_begin + ntiles, row_end, x, y, epi, -0.0f,
                   pb_magics{PB_MAG0, PB_MAG4, PB_MAG8, PB_MAG12, PB_MAG16}, ctx->d_err);
}

template <int TYPE>
static int launch_mv(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int tile_begin, int ntiles, int row_end,
                     const pb_mv_epi& epi) {
  if (w->nb <= 128) {
    const int S = mvw_slots(w->nb), groups = (ntiles + S - 1) / S;
    const int grid = groups < ctx->sm_count ? groups : ctx->sm_count;
    return pb_launch(ctx, "k_matvec_ws", true, k_matvec_ws<TYPE>, dim3(grid), dim3(mvw_threads(w->nb)), mvw_smem(w),
                     (const uint8_t*)w->qs, (const uint16_t*)w->d, (const uint16_t*)w->m, w->N, w->nb, tile_begin,
                     tile_begin + ntiles, row_end, x, y, epi, -0.0f,
                     pb_magics{PB_MAG0, PB_MAG4, PB_MAG8, PB_MAG12, PB_MAG16}, ctx->d_err);
  }
  return launch_mv_nt<TYPE, MV_THREADS>(ctx, w, x, y, tile_begin, ntiles, row_end, epi);
}

bool pb_fast_uses_mvf(const pb_ctx* ctx, const pb_qmat* w) {
  return !(ctx->mvt && pb_mvt_ok(w)) && !(w->mq && w->mma_ok && w->layout == PB_LAYOUT_ROWS && w->N >= ctx->mvi_min_rows);
}

int pb_launch_matvec(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows,
                     const pb_mv_epi* epi_in) {
  if (!ctx || !w || !x) return PB_ERR_ARG;
  if (w->type != PB_TYPE_Q4_0 && w->type != PB_TYPE_Q4_1)
    return pb_set_error(ctx, PB_ERR_ARG, "matvec supports Q4_0 and Q4_1 matrices");
  if (w->layout != PB_LAYOUT_ROWS)
    return pb_set_error(ctx, PB_ERR_ARG, "matrix was uploaded as a head table (PB_QMAT_TABLE); the matvec needs the "
                                         "row layout");
  const bool fast = w->type == PB_TYPE_Q4_0 && ctx->matvec_mode == PB_MATVEC_FAST;
  if (w->nb > (fast ? 32 * MVF_MAX_WARPS : MV_THREADS / 2))
    return pb_set_error(ctx, PB_ERR_ARG, "K=%d exceeds the %d the matvec kernel supports", w->K,
                        fast ? 1024 * MVF_MAX_WARPS : MV_THREADS * 16);
  if (rows <= 0) { row0 = 0; rows = w->N; }
  if (row0 < 0 || row0 + rows > w->N || (row0 & 7))
    return pb_set_error(ctx, PB_ERR_ARG, "row range [%d, %d) invalid (start must be a multiple of 8)", row0, row0 + rows);
  pb_mv_epi epi = epi_in ? *epi_in : pb_mv_epi();
  if (!y && epi.kind != PB_EPI_SWIGLU4) return PB_ERR_ARG;
  const int tile_begin = row0 / 8, ntiles = pb_cdiv(rows, 8);
  if (fast) {
    // the tcgen05 int8 kernel where it is on and takes the matrix; else the mma.sync int8
    // kernel on the matrix's current tensor-core copy (large matrices: on small
    // ones its per-launch staging of x costs more than it saves), else the f32
    // one; chosen per matrix, so row slices of one matrix agree in bits
    if (ctx->mvt && pb_mvt_ok(w)) return pb_launch_mvt(ctx, w, x, y, row0, rows, epi);
    if (w->mq && w->mma_ok && w->layout == PB_LAYOUT_ROWS && w->N >= ctx->mvi_min_rows)
      return pb_launch_mvi(ctx, w, x, y, row0, rows, epi);
    return launch_mvf(ctx, w, x, y, tile_begin, ntiles, row0 + rows, epi);
  }
  if (w->type == PB_TYPE_Q4_0) return launch_mv<PB_TYPE_Q4_0>(ctx, w, x, y, tile_begin, ntiles, row0 + rows, epi);
  return launch_mv<PB_TYPE_Q4_1>(ctx, w, x, y, tile_begin, ntiles, row0 + rows, epi);
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
  if (rc == PB_OK) {  // the module functions keep the reference's exact lane order
    const int mode = ctx->matvec_mode;
    ctx->matvec_mode = PB_MATVEC_EXACT;
    rc = pb_launch_matvec(ctx, m, dx, dy, 0, N, nullptr);
    ctx->matvec_mode = mode;
  }
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
constexpr int HD_PF_Q4 = 8, HD_PF_Q8 = 4;  // blocks of loads in flight per lane

// The hidden vector into shared memory, RMS-normalised with the final norm
// gains when norm_w is set (engine.js:429-449; a fixed reduction tree, so all
// CTAs get identical values).  A thread's global loads are all issued before
// any is used (K <= 16 * blockDim.x).
__device__ __forceinline__ void load_hidden(const float* __restrict__ h, const float* __restrict__ norm_w, double eps,
                                            int K, float* hs) {
  __shared__ double red[HD_WARPS];
  const int tid = threadIdx.x, nt = blockDim.x, nc = K / 4;
  float4 hv[4], wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + i * nt;
    if (c < nc) {
      hv[i] = reinterpret_cast<const float4*>(h)[c];
      if (norm_w) wv[i] = reinterpret_cast<const float4*>(norm_w)[c];
    }
  }
  double rms = 0.0;
  if (norm_w) {
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (tid + i * nt < nc) {
        ss = __fma_rn((double)hv[i].x, (double)hv[i].x, ss);
        ss = __fma_rn((double)hv[i].y, (double)hv[i].y, ss);
        ss = __fma_rn((double)hv[i].z, (double)hv[i].z, ss);
        ss = __fma_rn((double)hv[i].w, (double)hv[i].w, ss);
      }
    }
    ss = pb_block_sum_d(ss, red);
    rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)K), eps));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + i * nt;
    if (c < nc) {
      float4 v = hv[i];
      if (norm_w) {
        v.x = (float)__dmul_rn(__ddiv_rn((double)v.x, rms), (double)wv[i].x);
        v.y = (float)__dmul_rn(__ddiv_rn((double)v.y, rms), (double)wv[i].y);
        v.z = (float)__dmul_rn(__ddiv_rn((double)v.z, rms), (double)wv[i].z);
        v.w = (float)__dmul_rn(__ddiv_rn((double)v.w, rms), (double)wv[i].w);
      }
      reinterpret_cast<float4*>(hs)[c] = v;
    }
  }
  __syncthreads();
}

// acc[L] += h[4i + L] * e[4i + L] for L = 0..3: packed products, scalar sums
// (a packed add of packed products would be contracted into an FMA).
__device__ __forceinline__ void head_acc(float& a0, float& a1, float& a2, float& a3, float4 hv, float2 e01,
                                         float2 e23) {
  const float2 p01 = f2mul(make_float2(hv.x, hv.y), e01), p23 = f2mul(make_float2(hv.z, hv.w), e23);
  a0 = __fadd_rn(a0, p01.x);
  a1 = __fadd_rn(a1, p01.y);
  a2 = __fadd_rn(a2, p23.x);
  a3 = __fadd_rn(a3, p23.y);
}

// One lane per vocab row; lanes of a warp = the 32 rows of a tile.
// mode 0: batch_dot order (wasm-q4.js:467-549) over Q4_0 / Q8_0 tiles.
template <int TYPE>
__global__ void __launch_bounds__(HD_WARPS * 32)
k_head(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int N, int nb, const float* __restrict__ h,
       const float* __restrict__ norm_w, double eps, float* __restrict__ logits, unsigned long long* __restrict__ amax) {
  extern __shared__ __align__(16) float hs[];
  const int K = nb * 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = blockIdx.x * HD_WARPS + warp;
  const int row = tile * 32 + lane;
  const int ntiles = (N + 31) >> 5;
  constexpr int PL = TYPE == PB_TYPE_Q8_0 ? 2 : 1;  // uint4 per block payload
  const uint4* q4 = reinterpret_cast<const uint4*>(qs);
  constexpr int HD_PF = TYPE == PB_TYPE_Q8_0 ? HD_PF_Q8 : HD_PF_Q4;
  uint4 pq[HD_PF][PL];
  uint16_t pd[HD_PF];
  auto load = [&](int b, int k) {
    if (b < nb) {
      size_t slot = (size_t)pb_qslot(tile * 32 + lane, b, nb);
#pragma unroll
      for (int u = 0; u < PL; ++u) pq[k][u] = __ldcs(q4 + slot * PL + u);
      pd[k] = __ldcs(dsc + slot);
    }
  };
  // the table does not depend on the previous kernel: fetch before waiting
  if (tile < ntiles) {
#pragma unroll
    for (int k = 0; k < HD_PF; ++k) load(k, k);
  }
  pb_pdl_trigger();
  pb_pdl_wait();
  load_hidden(h, norm_w, eps, K, hs);
  float result = 0.0f;
  if (tile < ntiles) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;  // acc[k % 4] of batch_dot
    for (int b0 = 0; b0 < nb; b0 += HD_PF) {
#pragma unroll
      for (int k = 0; k < HD_PF; ++k) {
        int b = b0 + k;
        if (b >= nb) break;
        float d = pb_f16_exact(pd[k]);
        const float4* hb = reinterpret_cast<const float4*>(hs) + b * 8;
        if (TYPE == PB_TYPE_Q4_0) {
          const uint32_t wv[4] = {pq[k][0].x, pq[k][0].y, pq[k][0].z, pq[k][0].w};
          if (isfinite(d)) {
            // e = (q - 8) * d rebuilt exactly: fma(2^k + q, d, -(2^k + 8) * d)
            const float c15 = __fmul_rn(-32776.0f, d), c11 = __fmul_rn(-2056.0f, d), c7 = __fmul_rn(-136.0f, d);
            const float2 dd = make_float2(d, d);
            float2 e01[8], e23[8];  // element 4i+L for lanes (0,1) and (2,3)
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const uint32_t w = wv[g], wa = w << 8, wb = w >> 12;
              e01[g] = f2fma(make_float2(mag(wa, 0xF00u, PB_MAG8), mag(w, 0xF00u, PB_MAG8)), dd, make_float2(c15, c15));
              e23[g] = f2fma(make_float2(mag(w, 0xF0000u, PB_MAG16), mag(wb, 0xF000u, PB_MAG12)), dd, make_float2(c7, c11));
              e01[g + 4] = f2fma(make_float2(mag(wa, 0xF000u, PB_MAG12), mag(w, 0xF000u, PB_MAG12)), dd,
                                 make_float2(c11, c11));
              e23[g + 4] = f2fma(make_float2(mag(wb, 0xF00u, PB_MAG8), mag(wb, 0xF0000u, PB_MAG16)), dd,
                                 make_float2(c15, c7));
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 hv = hb[i];
              head_acc(a0, a1, a2, a3, hv, e01[i], e23[i]);
            }
          } else {  // inf / NaN scale: the plain product, as gguf.js computes it
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 hv = hb[i];
              float e[4];
#pragma unroll
              for (int L = 0; L < 4; ++L) {
                const uint32_t byte = (wv[i & 3] >> (8 * L)) & 0xFFu;
                const int q = i < 4 ? (int)(byte & 15u) : (int)(byte >> 4);
                e[L] = __fmul_rn((float)(q - 8), d);
              }
              head_acc(a0, a1, a2, a3, hv, make_float2(e[0], e[1]), make_float2(e[2], e[3]));
            }
          }
        } else {  // Q8_0: element j = byte j of the 32-byte payload
          const uint32_t wv[8] = {pq[k][0].x, pq[k][0].y, pq[k][0].z, pq[k][0].w,
                                  pq[k][1].x, pq[k][1].y, pq[k][1].z, pq[k][1].w};
          const bool fin = isfinite(d);
          const float c = __fmul_rn(-32896.0f, d);  // -(2^15 + 128) * d, exact
          const float2 dd = make_float2(d, d), cc = make_float2(c, c);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t u = wv[i] ^ 0x80808080u;  // biased bytes: q + 128
            const float4 hv = hb[i];
            float2 e01, e23;
            if (fin) {
              e01 = f2fma(make_float2(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7504)),
                                      __uint_as_float(__byte_perm(u, PB_MAG8, 0x7514))), dd, cc);
              e23 = f2fma(make_float2(__uint_as_float(__byte_perm(u, PB_MAG8, 0x7524)),
                                      __uint_as_float(__byte_perm(u, PB_MAG8, 0x7534))), dd, cc);
            } else {
              e01 = make_float2(__fmul_rn((float)(int8_t)(wv[i] & 0xFF), d), __fmul_rn((float)(int8_t)((wv[i] >> 8) & 0xFF), d));
              e23 = make_float2(__fmul_rn((float)(int8_t)((wv[i] >> 16) & 0xFF), d), __fmul_rn((float)(int8_t)(wv[i] >> 24), d));
            }
            head_acc(a0, a1, a2, a3, hv, e01, e23);
          }
        }
        load(b + HD_PF, k);
      }
    }
    result = __fadd_rn(__fadd_rn(a1, a3), __fadd_rn(a0, a2));
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
k_head_f32_double(const float* __restrict__ E, int N, int D, const float* __restrict__ h,
                  const float* __restrict__ norm_w, double eps, float* __restrict__ logits,
                  unsigned long long* __restrict__ amax) {
  extern __shared__ __align__(16) float hs[];
  load_hidden(h, norm_w, eps, D, hs);
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

// batch_dot (wasm-q4.js:467-549) over an f32 table stored as tiles
// [V/32][D][32]: lanes = rows, acc[k % 4] += h[k] * E[v, k] with a separate
// multiply and add, k ascending, then (acc1 + acc3) + (acc0 + acc2).  This is
// the head of a streaming model whose table the reference dequantizes to f32
// (streaming-loader.js:324-335) from a type the device keeps as f32 (Q6_K,
// F16, F32).
__global__ void __launch_bounds__(HD_WARPS * 32)
k_head_f32_bd(const float* __restrict__ E, int N, int D, const float* __restrict__ h,
              const float* __restrict__ norm_w, double eps, float* __restrict__ logits,
              unsigned long long* __restrict__ amax) {
  extern __shared__ __align__(16) float hs[];
  pb_pdl_trigger();
  pb_pdl_wait();
  load_hidden(h, norm_w, eps, D, hs);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = blockIdx.x * HD_WARPS + warp;
  const int row = tile * 32 + lane;
  const int ntiles = (N + 31) >> 5;
  float result = 0.0f;
  if (tile < ntiles) {
    const float* tp = E + (size_t)tile * D * 32 + lane;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int d = 0; d < D; d += 8) {  // D % 32 == 0
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcs(tp + (size_t)(d + u) * 32);
#pragma unroll
      for (int u = 0; u < 8; u += 4) {
        const float4 hv = *reinterpret_cast<const float4*>(hs + d + u);
        head_acc(a0, a1, a2, a3, hv, make_float2(v[u], v[u + 1]), make_float2(v[u + 2], v[u + 3]));
      }
    }
    result = __fadd_rn(__fadd_rn(a1, a3), __fadd_rn(a0, a2));
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

// mode: 0 = batch_dot order over Q4_0/Q8_0 tiles; 1 = double order over f32
// tiles (llama.js); 2 = batch_dot order over f32 tiles
int pb_launch_head(pb_ctx* ctx, const pb_qmat* emb, const float* h, float* logits, unsigned long long* amax, int mode) {
  return pb_launch_head_norm(ctx, emb, h, nullptr, 0.0, logits, amax, mode);
}

int pb_launch_head_norm(pb_ctx* ctx, const pb_qmat* emb, const float* h, const float* norm_w, double eps, float* logits,
                        unsigned long long* amax, int mode) {
  int ntiles = (emb->N + 31) / 32;
  int grid = pb_cdiv(ntiles, HD_WARPS);
  size_t smem = (size_t)emb->K * 4;
  if (emb->K > 16 * HD_WARPS * 32 || (emb->K & 3))
    return pb_set_error(ctx, PB_ERR_ARG, "head dim %d: at most %d and a multiple of 4", emb->K, 16 * HD_WARPS * 32);
  if (mode == 1) {
    k_head_f32_double<<<grid, HD_WARPS * 32, smem, ctx->stream>>>((const float*)emb->qs, emb->N, emb->K, h, norm_w, eps,
                                                                   logits, amax);
  } else if (mode == 2) {
    if (emb->type != PB_TYPE_F32 || (emb->K & 31))
      return pb_set_error(ctx, PB_ERR_ARG, "f32 head table: type F32 and dim a multiple of 32");
    return pb_launch(ctx, "k_head_f32_bd", true, k_head_f32_bd, dim3(grid), dim3(HD_WARPS * 32), smem,
                     (const float*)emb->qs, emb->N, emb->K, h, norm_w, eps, logits, amax);
  } else if (emb->type == PB_TYPE_Q4_0 || emb->type == PB_TYPE_Q8_0) {
    if (emb->layout != PB_LAYOUT_TILED8)
      return pb_set_error(ctx, PB_ERR_ARG, "head table must be uploaded with PB_QMAT_TABLE");
    return pb_launch(ctx, "k_head", true, emb->type == PB_TYPE_Q4_0 ? k_head<PB_TYPE_Q4_0> : k_head<PB_TYPE_Q8_0>,
                     dim3(grid), dim3(HD_WARPS * 32), smem, (const uint8_t*)emb->qs, (const uint16_t*)emb->d, emb->N,
                     emb->nb, h, norm_w, eps, logits, amax);
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
constexpr int PF_KC = 8;                        // blocks per chunk
constexpr int PF_ROWS = PF_WARPS * 32;          // weight rows per CTA
constexpr int PF_WSTRIDE = PF_KC * 16 + 16;     // bytes per staged row (padded: conflict-free lane reads)

// Weight rows arrive in the row-major layout: a CTA stages its 256 rows x 8
// blocks (coalesced: 8 threads per 128-byte row segment) in shared memory,
// and lane n then reads its own row's blocks from there.
__global__ void __launch_bounds__(PF_WARPS * 32)
k_prefill_q4(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int N, int N_pad, int nb,
             const float* __restrict__ X, int ldx, int M, float* __restrict__ C, int ldc) {
  extern __shared__ __align__(16) unsigned char pf_raw[];
  float(*xs)[PF_KC * 32] = reinterpret_cast<float(*)[PF_KC * 32]>(pf_raw);            // [PF_MT][256]
  uint8_t* ws = pf_raw + sizeof(float) * PF_MT * PF_KC * 32;                           // [256][PF_WSTRIDE]
  uint16_t* ds = reinterpret_cast<uint16_t*>(ws + (size_t)PF_ROWS * PF_WSTRIDE);       // [256][PF_KC]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row0 = blockIdx.x * PF_ROWS;
  const int n = row0 + warp * 32 + lane;
  const int m0 = blockIdx.y * PF_MT;
  const int K = nb * 32;
  float acc[PF_MT];
#pragma unroll
  for (int i = 0; i < PF_MT; ++i) acc[i] = 0.0f;
  for (int b0 = 0; b0 < nb; b0 += PF_KC) {
    const int kc = nb - b0 < PF_KC ? nb - b0 : PF_KC;
    __syncthreads();
    for (int idx = threadIdx.x; idx < PF_MT * PF_KC * 32; idx += blockDim.x) {
      int mm = idx / (PF_KC * 32), kk = idx % (PF_KC * 32);
      int k = b0 * 32 + kk;
      xs[mm][kk] = (m0 + mm < M && k < K) ? X[(size_t)(m0 + mm) * ldx + k] : 0.0f;
    }
    for (int idx = threadIdx.x; idx < PF_ROWS * PF_KC; idx += blockDim.x) {
      const int r = idx / PF_KC, bb = idx % PF_KC;
      const int row = row0 + r;
      if (bb < kc && row < N_pad) {
        const size_t slot = (size_t)row * nb + b0 + bb;
        *reinterpret_cast<uint4*>(ws + (size_t)r * PF_WSTRIDE + bb * 16) = __ldcs(reinterpret_cast<const uint4*>(qs) + slot);
        ds[r * PF_KC + bb] = __ldcs(dsc + slot);
      }
    }
    __syncthreads();
    if (n < N) {
      const int r = warp * 32 + lane;
      for (int bb = 0; bb < kc; ++bb) {
        const uint4 pl = *reinterpret_cast<const uint4*>(ws + (size_t)r * PF_WSTRIDE + bb * 16);
        float d = pb_f16_exact(ds[r * PF_KC + bb]);
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
  if (n < N) {
#pragma unroll
    for (int mm = 0; mm < PF_MT; ++mm)
      if (m0 + mm < M) C[(size_t)(m0 + mm) * ldc + n] = acc[mm];
  }
}

static size_t pf_smem() {
  return sizeof(float) * PF_MT * PF_KC * 32 + (size_t)PF_ROWS * PF_WSTRIDE + (size_t)PF_ROWS * PF_KC * 2;
}

int pb_launch_prefill_q4(pb_ctx* ctx, const pb_qmat* w, const float* X, int ldx, int M, float* C, int ldc) {
  if (w->type != PB_TYPE_Q4_0 || w->layout != PB_LAYOUT_ROWS)
    return pb_set_error(ctx, PB_ERR_ARG, "prefill GEMM needs a Q4_0 matrix in the row layout");
  dim3 grid(pb_cdiv(w->N, PF_ROWS), pb_cdiv(M, PF_MT));
  if (grid.y > 65535) return pb_set_error(ctx, PB_ERR_ARG, "M=%d too large", M);
  k_prefill_q4<<<grid, PF_WARPS * 32, pf_smem(), ctx->stream>>>(w->qs, w->d, w->N, w->N_pad, w->nb, X, ldx, M, C, ldc);
  PB_LAUNCHED(ctx, "k_prefill_q4");
  return PB_OK;
}

// Opt every kernel with a large dynamic shared-memory footprint in once, at
// context creation (never during stream capture).
int pb_setup_q4_kernels(void) {
  const int lim = 200 * 1024;
  cudaError_t e = cudaSuccess;
  e = e ? e : cudaFuncSetAttribute(k_matvec<PB_TYPE_Q4_0, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  e = e ? e : cudaFuncSetAttribute(k_matvec<PB_TYPE_Q4_1, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  e = e ? e : cudaFuncSetAttribute(k_matvec_ws<PB_TYPE_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  e = e ? e : cudaFuncSetAttribute(k_matvec_ws<PB_TYPE_Q4_1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  e = e ? e : cudaFuncSetAttribute(k_prefill_q4, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  e = e ? e : cudaFuncSetAttribute(k_head<PB_TYPE_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_head<PB_TYPE_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_head_f32_double, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_head_f32_bd, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  for (auto k : {k_qkv_attn<1>, k_qkv_attn<2>, k_qkv_attn<3>, k_qkv_attn<4>, k_qkv_attn<5>, k_qkv_attn<6>,
                 k_qkv_attn<7>, k_qkv_attn<8>})
    e = e ? e : cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, QA_SMEM_MAX);
  e = e ? e : cudaFuncSetAttribute(k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_ROWS, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_ROWS, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_mvf<PB_TYPE_Q4_0, PB_LAYOUT_TILED8>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_mvf<PB_TYPE_Q8_0, PB_LAYOUT_ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e = e ? e : cudaFuncSetAttribute(k_mvf<PB_TYPE_Q8_0, PB_LAYOUT_TILED8>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  return e == cudaSuccess ? PB_OK : PB_ERR_CUDA;
}
