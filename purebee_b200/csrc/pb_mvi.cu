// pb_mvi.cu - the int8 tensor-core Q4_0 matvec of the fast mode (k_mvi).
//
// y[n] = sum_b d[n][b] * sum_{k in block b} (q[n][k] - 8) * x[k]  (wasm-q4.js
// :118-267 computes the same sum in its own f32 order; this path agrees with
// it within an f32 tolerance, the exact kernels in pb_q4.cu stay the parity
// mode).
//
// The 4-bit codes go to the tensor cores as unsigned bytes and x as signed
// bytes: mma.sync m16n8k32 (u8 x s8 -> s32) sums exact integer products.  x
// is written per 32-value block b as three signed digits,
//     x[k] ~= 2^e_b / 127 * (d0 + d1 / 254 + d2 / 254^2),
// each in [-127, 127] (e_b: the block maximum's binary exponent, so 2^-e_b
// scales exactly); the representation error is about 1e-7 of the block's
// largest |x|.  The -8 of the codes is applied through T_b = the sum of
// each digit over the block, also exact.
//
// Fragments: a warp takes a 16-row tile.  For the 8 blocks of a span (256 k)
// the MMA's 8 columns are the 8 blocks: at step j (block 8s + j) only the
// lanes of column j (group g == j) supply their digits, the others zeros, so
// column j of the accumulator collects block 8s + j alone.  After the span
// each lane holds four distinct (row, block) integer sums per digit and
// applies that block's scale d (the f16 scale, decoded as the WASM matvec
// decodes it, wasm-q4.js:88-109) and 2^e_b / 127 in f32.  Per weight this is
// one quarter of a logic op to unpack codes (w & 0x0F0F0F0F gives 4 codes),
// against about four instructions per weight on the f32 pipes.
//
// Layout of the copy (pb_qmat mq / md), 16-row tiles T, nbp = blocks per row
// padded to a multiple of 8 (the padding holds zero codes and scales):
//   mq [T][nbp/2][32 lanes][16 B]: lane (g = lane/4, t = lane%4), block
//      b = 2 * pair + h at bytes 8h .. 8h+7 as two words:
//        w0 byte i: low nibble q(16T+g, 32b+4t+i), high nibble q(16T+g+8, 32b+4t+i)
//        w1 byte i: low nibble q(16T+g, 32b+16+4t+i), high nibble q(16T+g+8, 32b+16+4t+i)
//      so w0 & 0x0F0F0F0F and w0 & 0xF0F0F0F0 are the A fragment registers
//      of rows g and g+8 (the latter carrying 16 q, undone in the scale).
//   md [T][nbp/8][32 lanes][4] u16: d(g, 8s+2t), d(g, 8s+2t+1), d(g+8, 8s+2t),
//      d(g+8, 8s+2t+1): the scales of the accumulator entries the lane holds.
#include "pb_internal.cuh"

// Rebuild the copy from the matrix's current payload and scales (either layout).
__global__ void k_pack_mma(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int layout, int N, int nb,
                           int nbp, int nt16, uint8_t* __restrict__ mq, uint16_t* __restrict__ md) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t npay = (int64_t)nt16 * (nbp / 2) * 32, nsc = (int64_t)nt16 * (nbp / 8) * 32;
  const int lane = (int)(i & 31), g = lane >> 2, t = lane & 3;
  if (i < npay) {
    const int64_t r = i >> 5;
    const int pair = (int)(r % (nbp / 2)), T = (int)(r / (nbp / 2));
    const int r0 = 16 * T + g, r1 = r0 + 8;
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int b = 2 * pair + h;
      uint32_t w0 = 0, w1 = 0;
      if (b < nb) {
        const uint8_t* p0 = r0 < N ? qs + pb_slot(layout, r0, b, nb) * 16 : nullptr;
        const uint8_t* p1 = r1 < N ? qs + pb_slot(layout, r1, b, nb) * 16 : nullptr;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t b0 = p0 ? p0[4 * t + k] : 0u, b1 = p1 ? p1[4 * t + k] : 0u;
          w0 |= ((b0 & 15u) | ((b1 & 15u) << 4)) << (8 * k);  // elements 4t+k (low nibbles)
          w1 |= ((b0 >> 4) | ((b1 >> 4) << 4)) << (8 * k);     // elements 16+4t+k (high nibbles)
        }
      }
      o[2 * h] = w0;
      o[2 * h + 1] = w1;
    }
    reinterpret_cast<uint4*>(mq)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  } else if (i < npay + nsc) {
    const int64_t j = i - npay, r = j >> 5;
    const int s = (int)(r % (nbp / 8)), T = (int)(r / (nbp / 8));
    const int r0 = 16 * T + g, r1 = r0 + 8, b0 = 8 * s + 2 * t, b1 = b0 + 1;
    auto dv = [&](int row, int b) -> uint16_t { return row < N && b < nb ? dsc[pb_slot(layout, row, b, nb)] : 0; };
    const uint16_t v[4] = {dv(r0, b0), dv(r0, b1), dv(r1, b0), dv(r1, b1)};
    reinterpret_cast<uint2*>(md)[j] = make_uint2(v[0] | ((uint32_t)v[1] << 16), v[2] | ((uint32_t)v[3] << 16));
  }
}

int pb_qmat_build_mma(pb_ctx* ctx, pb_qmat* m) {
  if (m->type != PB_TYPE_Q4_0) return pb_set_error(ctx, PB_ERR_ARG, "the tensor-core copy is for Q4_0 matrices");
  const int nbp = (m->nb + 7) / 8 * 8, nt16 = (m->N + 15) / 16;
  if (!m->mq) {
    if (cudaMalloc(&m->mq, (size_t)nt16 * nbp * 256) != cudaSuccess ||
        cudaMalloc(&m->md, (size_t)nt16 * (nbp / 8) * 32 * 8) != cudaSuccess) {
      cudaFree(m->mq);
      m->mq = nullptr;
      return pb_set_error(ctx, PB_ERR_OOM, "tensor-core matvec copy");
    }
  }
  m->nbp = nbp;
  const int64_t tot = (int64_t)nt16 * (nbp / 2) * 32 + (int64_t)nt16 * (nbp / 8) * 32;
  k_pack_mma<<<pb_cdiv(tot, 256), 256, 0, ctx->stream>>>(m->qs, m->d, m->layout, m->N, m->nb, nbp, nt16, m->mq, m->md);
  PB_LAUNCHED(ctx, "k_pack_mma");
  PB_TRY(pb_qmat_build_mvt(ctx, m));
  m->mma_ok = true;
  return PB_OK;
}

namespace {

constexpr int MVI_MAX_WARPS = 16;
constexpr int MVI_PF = 2;  // CTA iterations of L2 prefetch ahead

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Per-block digits of x (RMS-normalised when w is set) into shared memory:
//   dig[b][i][t] = {word t, word 4+t} of digit i of block b (the B fragment
//   registers of lane t), tinfo[b] = {T0, T1, T2, 2^e / 127}.
// One warp per block, one element per lane.  The sum of squares runs over a
// fixed 128-lane partition (chunk c on lane c % 128), so every launch shape
// normalises a vector to the same bits.
__device__ __forceinline__ void mvi_stage(const float* __restrict__ x, const float* __restrict__ w, double eps, int K,
                                          int nbp, uint2* dig, int4* tinfo, double* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, W = blockDim.x >> 5, nb = K / 32;
  float inv = 1.0f;
  if (w) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    if (tid < 128) {
      double ss = 0.0;
      for (int c0 = tid; c0 < K / 4; c0 += 128 * 4) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c0 + 128 * j < K / 4) v[j] = x4[c0 + 128 * j];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (c0 + 128 * j < K / 4) {
            ss = __fma_rn((double)v[j].x, (double)v[j].x, ss);
            ss = __fma_rn((double)v[j].y, (double)v[j].y, ss);
            ss = __fma_rn((double)v[j].z, (double)v[j].z, ss);
            ss = __fma_rn((double)v[j].w, (double)v[j].w, ss);
          }
        }
      }
      ss = pb_warp_sum_d(ss);
      if (lane == 0) red[warp] = ss;
    }
    __syncthreads();
    const double ss = __dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3]));
    inv = (float)(1.0 / __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)K), eps)));
  }
  for (int b0 = warp; b0 < nbp; b0 += W * 4) {
    float xv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // four blocks' loads in flight per lane
      const int b = b0 + W * u;
      xv[u] = 0.0f;
      if (b < nb) {
        xv[u] = x[32 * b + lane];
        if (w) xv[u] = __fmul_rn(__fmul_rn(xv[u], inv), w[32 * b + lane]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = b0 + W * u;
      if (b >= nbp) break;
      int i0, i1, i2;
      const float f = pb_x_digits(xv[u], i0, i1, i2);
      // byte `lane` of each digit: word lane / 4; lane t of the fragment keeps words t and 4 + t
      const int wd = lane >> 2, tt = wd & 3, hh = wd >> 2;
      unsigned char* base = reinterpret_cast<unsigned char*>(dig + (size_t)b * 12);
      base[(0 * 4 + tt) * 8 + hh * 4 + (lane & 3)] = (unsigned char)(int8_t)i0;
      base[(1 * 4 + tt) * 8 + hh * 4 + (lane & 3)] = (unsigned char)(int8_t)i1;
      base[(2 * 4 + tt) * 8 + hh * 4 + (lane & 3)] = (unsigned char)(int8_t)i2;
      const int s0 = __reduce_add_sync(0xffffffffu, i0), s1 = __reduce_add_sync(0xffffffffu, i1),
                s2 = __reduce_add_sync(0xffffffffu, i2);
      if (lane == 0) tinfo[b] = make_int4(s0, s1, s2, __float_as_int(f));
    }
  }
}

}  // namespace

// CTA of W warps = TPC tiles x KCH span chunks per iteration; a warp's unit is
// (16-row tile, spans [ch * spc, ...)).  The chunks of a tile are summed in
// chunk order in shared memory and the tile's two 8-row halves go through the
// exact kernels' epilogue.
__global__ void __launch_bounds__(MVI_MAX_WARPS * 32, 1)
k_mvi(const uint8_t* __restrict__ mq, const uint16_t* __restrict__ md, int N, int nb, int nbp, int t_begin,
      int t_end, int row_begin, int row_end, int spc, const float* __restrict__ x, float* __restrict__ y, pb_mv_epi epi,
      int* err) {
  extern __shared__ __align__(16) unsigned char mvi_raw[];
  __shared__ double red[MVI_MAX_WARPS];
  const int K = nb * 32, nspan = nbp / 8, KCH = (nspan + spc - 1) / spc, W = blockDim.x >> 5, TPC = W / KCH;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int tl = warp / KCH, ch = warp - tl * KCH;
  const bool active = tl < TPC;
  const int s_lo = ch * spc, s_hi = s_lo + spc < nspan ? s_lo + spc : nspan;
  uint2* dig = reinterpret_cast<uint2*>(mvi_raw);                          // [nbp][3][4] uint2
  int4* tinfo = reinterpret_cast<int4*>(mvi_raw + (size_t)nbp * 96);        // [nbp]
  float* part = reinterpret_cast<float*>(mvi_raw + (size_t)nbp * 112);      // [2][TPC][KCH][16]
  const int per_iter = gridDim.x * TPC;
  const int n_iter = (t_end - t_begin + per_iter - 1) / per_iter;  // CTA-uniform
  auto tile_of = [&](int it) { return t_begin + it * per_iter + blockIdx.x * TPC + tl; };
  const size_t tile_q = (size_t)nbp * 256, tile_d = (size_t)nspan * 256;
  auto prefetch = [&](int it) {
    const int T = tile_of(it);
    if (active && ch == 0 && lane == 0 && it < n_iter && T < t_end) {
      pb_l2_prefetch(mq + (size_t)T * tile_q, (uint32_t)tile_q);
      pb_l2_prefetch(md + (size_t)T * tile_d / 2, (uint32_t)tile_d);
    }
  };
  for (int i = 0; i < MVI_PF; ++i) prefetch(i);
  if (tid == 0)
    for (int i = 0; i < PB_MAX_L2_NEXT; ++i) pb_l2_prefetch_share(epi.l2_next[i], epi.l2_next_bytes[i], blockIdx.x, gridDim.x);
  const uint4* q4 = reinterpret_cast<const uint4*>(mq);
  const uint2* d2 = reinterpret_cast<const uint2*>(md);
  // one span's codes (4 block pairs) and scales in registers
  uint4 qa[4];
  uint2 da;
  auto load = [&](int T, int s) {
#pragma unroll
    for (int q = 0; q < 4; ++q) qa[q] = __ldcs(q4 + ((size_t)T * (nbp / 2) + 4 * s + q) * 32 + lane);
    da = __ldcs(d2 + ((size_t)T * nspan + s) * 32 + lane);
  };
  if (active && n_iter > 0 && tile_of(0) < t_end && s_lo < s_hi) load(tile_of(0), s_lo);
  pb_pdl_trigger();
  pb_pdl_wait();  // x (and the residual) come from the previous kernel
  mvi_stage(x, epi.norm_w, epi.eps, K, nbp, dig, tinfo, red);
  __syncthreads();
  for (int it = 0; it < n_iter; ++it) {
    prefetch(it + MVI_PF);
    const int T = tile_of(it);
    const bool live = active && T < t_end;
    float acc_lo = 0.0f, acc_hi = 0.0f;  // rows g and g + 8 of the tile, this lane's blocks
    if (live) {
      for (int s = s_lo; s < s_hi; ++s) {
        const uint4 q0 = qa[0], q1 = qa[1], q2 = qa[2], q3 = qa[3];
        const uint2 dd = da;
        // the next span's (or the next tile's first span's) codes while this one runs
        if (s + 1 < s_hi) load(T, s + 1);
        else if (it + 1 < n_iter && tile_of(it + 1) < t_end) load(tile_of(it + 1), s_lo);
        const uint2* bd = dig + (size_t)(8 * s + g) * 12 + t;  // this lane's column: block 8s + g
        const uint2 b0 = bd[0], b1 = bd[4], b2 = bd[8];
        int D0[4] = {0, 0, 0, 0}, D1[4] = {0, 0, 0, 0}, D2[4] = {0, 0, 0, 0};
        const uint32_t w[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                                q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t w0 = w[2 * j], w1 = w[2 * j + 1];
          const uint32_t a0 = w0 & 0x0F0F0F0Fu, a1 = w0 & 0xF0F0F0F0u, a2 = w1 & 0x0F0F0F0Fu, a3 = w1 & 0xF0F0F0F0u;
          const bool mine = g == j;  // column j = block 8s + j: only its lanes supply digits
          mma_u8s8(D0, a0, a1, a2, a3, mine ? b0.x : 0u, mine ? b0.y : 0u);
          mma_u8s8(D1, a0, a1, a2, a3, mine ? b1.x : 0u, mine ? b1.y : 0u);
          mma_u8s8(D2, a0, a1, a2, a3, mine ? b2.x : 0u, mine ? b2.y : 0u);
        }
        // entries: (row g, block 8s+2t), (row g, 8s+2t+1), (row g+8, 8s+2t), (row g+8, 8s+2t+1)
        const int4 ti0 = tinfo[8 * s + 2 * t], ti1 = tinfo[8 * s + 2 * t + 1];
        const uint32_t dw[4] = {dd.x & 0xFFFFu, dd.x >> 16, dd.y & 0xFFFFu, dd.y >> 16};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int4 ti = (c & 1) ? ti1 : ti0;
          const int off = c < 2 ? 8 : 128;  // 8 * T, and 16 * 8 * T for the rows carrying 16 q
          const int e0 = D0[c] - off * ti.x, e1 = D1[c] - off * ti.y, e2 = D2[c] - off * ti.z;
          float v = __fmaf_rn((float)e2, 1.0f / 64516.0f, __fmaf_rn((float)e1, 1.0f / 254.0f, (float)e0));
          if (c >= 2) v = __fmul_rn(v, 1.0f / 16.0f);
          const float sc = __fmul_rn(pb_f16_wasm(dw[c]), __int_as_float(ti.w));
          if (c < 2) acc_lo = __fmaf_rn(v, sc, acc_lo);
          else acc_hi = __fmaf_rn(v, sc, acc_hi);
        }
      }
    }
    // the four lanes of a group hold different blocks of the same rows
    acc_lo = __fadd_rn(acc_lo, __shfl_xor_sync(0xffffffffu, acc_lo, 1));
    acc_hi = __fadd_rn(acc_hi, __shfl_xor_sync(0xffffffffu, acc_hi, 1));
    acc_lo = __fadd_rn(acc_lo, __shfl_xor_sync(0xffffffffu, acc_lo, 2));
    acc_hi = __fadd_rn(acc_hi, __shfl_xor_sync(0xffffffffu, acc_hi, 2));
    float* pbuf = part + (size_t)(it & 1) * TPC * KCH * 16;
    if (active && t == 0) {
      pbuf[((size_t)tl * KCH + ch) * 16 + g] = acc_lo;
      pbuf[((size_t)tl * KCH + ch) * 16 + g + 8] = acc_hi;
    }
    __syncthreads();
    if (active && ch == 0 && T < t_end) {
      const int rr = lane >> 2;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v = pbuf[(size_t)tl * KCH * 16 + 8 * h + rr];
        for (int c = 1; c < KCH; ++c) v = __fadd_rn(v, pbuf[((size_t)tl * KCH + c) * 16 + 8 * h + rr]);
        pb_mv_epilogue(v, 2 * T + h, N, row_begin, row_end, y, epi, err);
      }
    }
  }
}

static size_t mvi_smem(int nbp, int TPC, int KCH) { return (size_t)nbp * 112 + (size_t)2 * TPC * KCH * 16 * 4; }

int pb_launch_mvi(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows, const pb_mv_epi& epi) {
  if (!w->mq || !w->mma_ok) return pb_set_error(ctx, PB_ERR_STATE, "the matrix has no current tensor-core copy");
  const int nspan = w->nbp / 8;
  int spc = 2;
  while ((nspan + spc - 1) / spc > MVI_MAX_WARPS) spc *= 2;
  const int KCH = (nspan + spc - 1) / spc;
  const int t_begin = row0 / 16, t_end = (row0 + rows + 15) / 16, ntiles = t_end - t_begin;
  int W = 4;
  while (W < KCH) W *= 2;
  while (W < MVI_MAX_WARPS && (int64_t)ntiles * KCH / W >= 2 * ctx->sm_count) W *= 2;
  const int TPC = W / KCH;
  const size_t smem = mvi_smem(w->nbp, TPC, KCH);
  if (smem > (size_t)200 * 1024) return pb_set_error(ctx, PB_ERR_ARG, "K=%d too large for the tensor-core matvec", w->K);
  const int groups = (ntiles + TPC - 1) / TPC;
  int per_sm = MVI_MAX_WARPS / W;
  const int by_smem = (int)((size_t)220 * 1024 / (smem + 1024));
  per_sm = per_sm < by_smem ? per_sm : by_smem;
  if (per_sm < 1) per_sm = 1;
  const int cap = ctx->sm_count * per_sm;
  const int grid = groups < cap ? groups : cap;
  return pb_launch(ctx, "k_mvi", true, k_mvi, dim3(grid), dim3(W * 32), smem, (const uint8_t*)w->mq,
                   (const uint16_t*)w->md, w->N, w->nb, w->nbp, t_begin, t_end, row0, row0 + rows, spc, x, y, epi,
                   ctx->d_err);
}

int pb_setup_mvi_kernels(void) {
  return cudaFuncSetAttribute(k_mvi, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) == cudaSuccess
             ? PB_OK : PB_ERR_CUDA;
}
