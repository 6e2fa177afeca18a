// pb_gemm.cu - tensor-core Q4_0 x f16 GEMM for the batched configuration.
//
// C[M tokens][N rows] = X[M][K] . W[N][K]^T, W a resident Q4_0 matrix (either
// device layout; the batched LM head runs it over the tiled table).  This is the batched prefill / batched decode form of the
// reference's per-row matvec (wasm-q4.js:118-267) and of its prefill matmul
// (llama-streaming.js:398 -> wasm-simd.js:71-91).  It does not reproduce the
// reference's f32 operation order.  The scale is decoded as the reference
// decodes it (wasm-q4.js:88-109: a zero exponent is +0), and the weight value
// (q-8)*d is exact in f32.  One term (pb_gemm_epi terms == 1): each operand
// is rounded to f16 once.  Three terms (the batched model's default): each
// operand v becomes the f16 pair hi = f16(v), lo = f16(v - hi) -- exact for
// the weights, about 22 bits for x -- and hi*hi + hi*lo + lo*hi run on the
// tensor cores.  Products are exact and the sums run in f32 on the tensor
// cores, so results agree with the reference within a stated relative
// tolerance (about 3e-3 with one term, the accumulation bound with three),
// not bit for bit; the batch-1 decode path keeps the exact kernels.  Values
// past the f16 range (a scale with exponent 31, |x| > 65504) overflow the
// operands.
//
// One CTA computes a 128-row x 128-token tile with tcgen05.mma (kind::f16,
// M = 128, N = 128, K = 16 per instruction), the accumulator in 128 TMEM
// columns.  Per 64-wide K step all 256 threads stage the operands into a
// double-buffered shared-memory ring in the K-major 128-byte-swizzled layout
// the MMA descriptors name: the weight tile is dequantized on the fly
// (2 Q4_0 blocks per row), the activations are rounded to f16.  One thread
// issues the four MMAs of a step and commits them to the stage's mbarrier;
// the stage is rewritten only after that mbarrier's phase completes.  Every
// wait is bounded and records PB_DEVERR_WAIT instead of hanging.

#include <cuda_fp16.h>

#include <stdlib.h>

#include "pb_tc.cuh"

namespace {

constexpr int GM_ROWS = 128;    // weight rows per CTA (MMA M)
constexpr int GM_TOK = 128;     // tokens per CTA (MMA N)
constexpr int GM_KSTEP = 64;    // K per stage: one 128-byte swizzle row of f16
constexpr int GM_THREADS = 256;
constexpr int GM_TILE_BYTES = GM_ROWS * GM_KSTEP * 2;  // 16 KB, A and B alike
constexpr int GM_STAGE_BYTES = 2 * GM_TILE_BYTES;
constexpr int PB_GEMM_TMA_MIN_M = 512;  // from here on the f16 copy of W pays for itself

// Instruction descriptor: D f32, A and B f16, both K-major, M = 128, N = tok.
__host__ __device__ constexpr uint32_t gm_idesc(int tok) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(tok >> 3) << 17) | ((uint32_t)(GM_ROWS >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The lo halves of (a, b) given their hi pair: f16(a - hi_a), f16(b - hi_b)
// (each difference exact in f32).
__device__ __forceinline__ uint32_t pack_lo2(float a, float b, uint32_t hi) {
  const __half2 h = *reinterpret_cast<const __half2*>(&hi);
  return pack_h2(__fsub_rn(a, __low2float(h)), __fsub_rn(b, __high2float(h)));
}

}  // namespace

// One TMEM row (weight row `row`) of 32 token columns m0c .. m0c+31 through
// the epilogue.  Every lane of the warp calls it (the SwiGLU partner row is
// row ^ 4, lane ^ 4 of the same warp).
__device__ __forceinline__ void gemm_emit32(const uint32_t (&v)[32], bool zero, int row, int N, int m0c, int M,
                                            float* __restrict__ C, int ldc, const pb_gemm_epi& epi) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float r = zero ? 0.0f : __uint_as_float(v[j]);
    const int m = m0c + j;
    if (epi.mode == PB_GEMM_SWIGLU) {
      const float partner = __shfl_xor_sync(0xffffffffu, r, 4);
      if (row < N && m < M && (row & 4) == 0) {
        const float silu = __fdividef(r, 1.0f + __expf(-r));
        const float h = __fmul_rn(silu, partner);
        const int f = 4 * (row >> 3) + (row & 3);
        if (epi.h16 && epi.terms == 3) pb_store_hl(epi.h16, pb_hl_index((size_t)m * N, f), h);
        else if (epi.h16) epi.h16[(size_t)m * (N / 2) + f] = __float2half_rn(h);
        else epi.h32[(size_t)m * (N / 2) + f] = h;
      }
    } else {
      float v = r;
      if (row < N && m < M) {
        float* c = C + (size_t)m * ldc + row;
        v = epi.mode == PB_GEMM_ADD ? __fadd_rn(*c, r) : r;
        *c = v;
      }
      if (epi.xs.world > 0) {  // the fused residual exchange: lanes (row, row ^ 1) form a packet
        const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
        if (row < N && m < M && (row & 1) == 0) pb_xsend_pair(epi.xs, m, row, v, partner);
      }
    }
  }
}

// TOK tokens per CTA (MMA N = 64 or 128).  grid.z splits K: CTA z covers K
// steps [z*kper, (z+1)*kper) and, when gridDim.z > 1, writes its partial tile
// to C + z*M*ldc (a workspace the reduce kernel sums in order of z).
// TERMS == 3: a stage holds the hi and lo tiles of both operands (the weight
// value splits exactly, x to about 22 bits) and each 16-wide K slice issues
// hi*hi, hi*lo and lo*hi into the accumulator.
template <int TOK, bool XCH, int TERMS>
__global__ void __launch_bounds__(GM_THREADS, 1)
k_q4_gemm_tc(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int layout, int N, int N_pad, int nb,
             const float* __restrict__ X, int ldx, int M, float* __restrict__ C, int ldc, int kper, pb_gemm_epi epi,
             int* err) {
  extern __shared__ __align__(1024) unsigned char gm_raw[];
  __shared__ uint64_t bars[2];
  __shared__ uint32_t tmem_base;
  // 1024-byte alignment of the swizzled tiles (the swizzle repeats every 1024 bytes)
  unsigned char* ring = gm_raw + ((1024 - (pb_smem_addr(gm_raw) & 1023)) & 1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * GM_ROWS, m0 = blockIdx.y * TOK;
  const int K = nb * 32, ktot = (K + GM_KSTEP - 1) / GM_KSTEP;
  const int kbeg = blockIdx.z * kper, kend_ = kbeg + kper < ktot ? kbeg + kper : ktot;
  const int ksteps = kend_ > kbeg ? kend_ - kbeg : 0;
  C += (size_t)blockIdx.z * M * ldc;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(pb_smem_addr(&tmem_base)),
                 "r"(TOK)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    pb_mbar_init(&bars[0], 1);
    pb_mbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_d = tmem_base;

  // The CTA's whole weight slice into L2 first (row layout: one contiguous run
  // per row), then a register double buffer: step ks + 1's weights and
  // activations are loaded before step ks's MMAs are issued.
  if (layout == PB_LAYOUT_ROWS && tid < GM_ROWS && ksteps > 0) {
    const int row = n0 + tid, b0 = 2 * kbeg, b1 = 2 * kend_ < nb ? 2 * kend_ : nb;
    if (row < N_pad && b1 > b0) pb_l2_prefetch(qs + ((size_t)row * nb + b0) * 16, (uint32_t)(b1 - b0) * 16);
  }
  const int wr = tid >> 1, wblk = tid & 1;  // weights: (row, block) of the two Q4_0 blocks of a step
  const int xr_ = tid >> 1, xh = tid & 1;   // activations: (token, half of the 64-wide step)
  const bool xlive_row = xr_ < TOK && m0 + xr_ < M;
  pb_pdl_trigger();
  pb_pdl_wait();  // the activations (and C) come from the previous kernels
  uint4 pl;
  float dsv;
  float4 xa[8];
  auto load_step = [&](int kg) {
    const int b = kg * 2 + wblk, row = n0 + wr;
    pl = make_uint4(0, 0, 0, 0);
    dsv = 0.0f;
    if (b < nb && row < N_pad) {
      const size_t slot = (size_t)pb_slot(layout, row, b, nb);
      pl = __ldg(reinterpret_cast<const uint4*>(qs) + slot);
      dsv = pb_f16_wasm(__ldg(dsc + slot));  // the reference's scale decode
    }
    const int k = kg * GM_KSTEP + xh * 32;
    const bool live = xlive_row && k < K;
    // XCH: X in column chunks; a 32-wide half step never straddles one (x_chunk % 64 == 0)
    const int xc = epi.x_chunk;
    const float4* xr = reinterpret_cast<const float4*>(
        XCH ? X + (size_t)(k / xc) * M * xc + (size_t)(m0 + xr_) * xc + k % xc : X + (size_t)(m0 + xr_) * ldx + k);
#pragma unroll
    for (int c = 0; c < 8; ++c) xa[c] = live ? __ldg(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  if (ksteps > 0) load_step(kbeg);

  bool ok = true;
  // stage tiles: A hi, B hi, then (TERMS == 3) A lo, B lo
  constexpr int STAGE = (TERMS == 3 ? 4 : 2) * GM_TILE_BYTES;
  for (int ks = 0; ks < ksteps && ok; ++ks) {
    const int st = ks & 1;
    unsigned char* sA = ring + st * STAGE;
    unsigned char* sB = sA + GM_TILE_BYTES;
    unsigned char* sAl = sA + 2 * GM_TILE_BYTES;
    unsigned char* sBl = sA + 3 * GM_TILE_BYTES;
    if (ks >= 2) ok = pb_mbar_wait(&bars[st], ((ks >> 1) - 1) & 1, err);  // MMAs of step ks-2 are done with it
    if (!ok) break;
    {
      const uint32_t wv[4] = {pl.x, pl.y, pl.z, pl.w};
      float e[32];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t byte = (wv[j >> 2] >> (8 * (j & 3))) & 0xFFu;
        e[j] = (float)((int)(byte & 15u) - 8) * dsv;       // exact in f32
        e[16 + j] = (float)((int)(byte >> 4) - 8) * dsv;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 v;
        v.x = pack_h2(e[8 * c + 0], e[8 * c + 1]);
        v.y = pack_h2(e[8 * c + 2], e[8 * c + 3]);
        v.z = pack_h2(e[8 * c + 4], e[8 * c + 5]);
        v.w = pack_h2(e[8 * c + 6], e[8 * c + 7]);
        *reinterpret_cast<uint4*>(sA + pb_sw128(wr, wblk * 4 + c)) = v;
        if (TERMS == 3) {
          uint4 l;
          l.x = pack_lo2(e[8 * c + 0], e[8 * c + 1], v.x);
          l.y = pack_lo2(e[8 * c + 2], e[8 * c + 3], v.y);
          l.z = pack_lo2(e[8 * c + 4], e[8 * c + 5], v.z);
          l.w = pack_lo2(e[8 * c + 6], e[8 * c + 7], v.w);
          *reinterpret_cast<uint4*>(sAl + pb_sw128(wr, wblk * 4 + c)) = l;
        }
      }
    }
    if (xr_ < TOK) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 v;
        v.x = pack_h2(xa[2 * c].x, xa[2 * c].y);
        v.y = pack_h2(xa[2 * c].z, xa[2 * c].w);
        v.z = pack_h2(xa[2 * c + 1].x, xa[2 * c + 1].y);
        v.w = pack_h2(xa[2 * c + 1].z, xa[2 * c + 1].w);
        *reinterpret_cast<uint4*>(sB + pb_sw128(xr_, xh * 4 + c)) = v;
        if (TERMS == 3) {
          uint4 l;
          l.x = pack_lo2(xa[2 * c].x, xa[2 * c].y, v.x);
          l.y = pack_lo2(xa[2 * c].z, xa[2 * c].w, v.y);
          l.z = pack_lo2(xa[2 * c + 1].x, xa[2 * c + 1].y, v.z);
          l.w = pack_lo2(xa[2 * c + 1].z, xa[2 * c + 1].w, v.w);
          *reinterpret_cast<uint4*>(sBl + pb_sw128(xr_, xh * 4 + c)) = l;
        }
      }
    }
    if (ks + 1 < ksteps) load_step(kbeg + ks + 1);
    // generic-proxy writes -> visible to the tensor core's async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t da = pb_sw128_desc(pb_smem_addr(sA)), db = pb_sw128_desc(pb_smem_addr(sB));
      const uint64_t dal = pb_sw128_desc(pb_smem_addr(sAl)), dbl = pb_sw128_desc(pb_smem_addr(sBl));
#pragma unroll
      for (int kk = 0; kk < GM_KSTEP / 16; ++kk) {  // +32 bytes (16 f16) along K per MMA
        mma_f16(tmem_d, da + 2 * kk, db + 2 * kk, gm_idesc(TOK), (ks > 0 || kk > 0) ? 1u : 0u);
        if (TERMS == 3) {
          mma_f16(tmem_d, da + 2 * kk, dbl + 2 * kk, gm_idesc(TOK), 1u);
          mma_f16(tmem_d, dal + 2 * kk, db + 2 * kk, gm_idesc(TOK), 1u);
        }
      }
      pb_umma_commit(&bars[st]);
    }
  }
  // the last step's commit covers every MMA issued before it
  if (ok && ksteps > 0) ok = pb_mbar_wait(&bars[(ksteps - 1) & 1], ((ksteps - 1) >> 1) & 1, err);
  const bool empty_split = ksteps == 0;  // no MMA wrote the accumulator: the partial is zero
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (ok && warp < 4) {
    // warp w reads TMEM lanes 32w .. 32w+31 (weight rows), 32 token columns at a time
    const int row = n0 + warp * 32 + lane;
#pragma unroll 1
    for (int c0 = 0; c0 < TOK; c0 += 32) {
      uint32_t v[32];
      pb_tmem_ld32(tmem_d + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
      gemm_emit32(v, empty_split, row, N, m0 + c0, M, C, ldc, epi);  // split-K partials always STORE
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(TOK) : "memory");
  }
}

static size_t gm_smem(int terms) { return (size_t)2 * (terms == 3 ? 2 : 1) * GM_STAGE_BYTES + 1024; }

// ---------------------------------------------------------------------------
// Large batches: a plain f16 GEMM fed by TMA.  The Q4_0 weights are first
// dequantized to an f16 copy ((q-8)*d exact in f32, rounded once, the same
// values the fused kernel stages) and x is rounded to f16 once; both then
// stream through a 4-stage ring of 128-byte-swizzled tiles loaded by
// cp.async.bulk.tensor.  Persistent CTAs, one per SM, walk the 128 x 256
// output tiles.  Warp roles: warp 0 lane 0 issues the TMA loads (one ring
// across all of the CTA's tiles), warp 1 lane 0 issues the MMAs (128 x 256 x
// 16 per instruction) and commits each stage back to its "empty" barrier.
// The accumulator alternates between two 256-column TMEM buffers, so warps
// 4-11 (lane quadrant (w - 4) % 4, half (w - 4) / 4 of the columns) drain
// tile i through the epilogue while the MMAs of tile i + 1 run.  The dequant
// copy costs N*K*2 bytes, about 1% of the GEMM time when M >= 512.
// ---------------------------------------------------------------------------

constexpr int TG_ROWS = 128, TG_TOK = 256, TG_K = 64, TG_STAGES = 4, TG_THREADS = 384;
constexpr int TG_EPI_WARPS = 8;  // warps 4..11
constexpr int TG_A_BYTES = TG_ROWS * TG_K * 2, TG_B_BYTES = TG_TOK * TG_K * 2;
constexpr int TG_STAGE_BYTES = TG_A_BYTES + TG_B_BYTES;
constexpr uint32_t TG_IDESC = (1u << 4) | ((uint32_t)(TG_TOK >> 3) << 17) | ((uint32_t)(TG_ROWS >> 4) << 24);

namespace {

// Tile t of the persistent GEMM in panel order: panels of TG_PANEL weight-row
// blocks, within a panel the token blocks in turn and the panel's row blocks
// within each, so the tiles in flight at once (one per SM) share a panel of
// W and a few token blocks of X that L2 holds.  (Row blocks fastest swept the
// whole weight for every token block.)  Only the schedule changes.
constexpr int TG_PANEL = 16;
__device__ __forceinline__ void tg_tile(int t, int ntn, int ntm, int& n0, int& m0) {
  const int panel = t / (TG_PANEL * ntm);
  const int pn = ntn - panel * TG_PANEL < TG_PANEL ? ntn - panel * TG_PANEL : TG_PANEL;
  const int within = t - panel * TG_PANEL * ntm;
  n0 = (panel * TG_PANEL + within % pn) * TG_ROWS;
  m0 = (within / pn) * TG_TOK;
}

__device__ __forceinline__ void mma_f16_n256(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(TG_IDESC), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

}  // namespace

// terms == 3: the row is written as hi/lo pairs in 64-wide groups
// (pb_hl_index), [N_pad][2K] halves; the pair is exact: hi + lo == (q-8)*d.
__global__ void k_dequant_q4_f16(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int layout, int nb,
                                 int64_t nblocks, __half* __restrict__ out, int terms) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // output block (row-major) per thread
  pb_pdl_trigger();
  pb_pdl_wait();  // the scratch it writes may still be read by the GEMM before
  if (b >= nblocks) return;
  const int row = (int)(b / nb), blk = (int)(b % nb);
  const int64_t slot = pb_slot(layout, row, blk, nb);
  const uint4 pl = __ldg(reinterpret_cast<const uint4*>(qs) + slot);
  const float d = pb_f16_wasm(__ldg(dsc + slot));  // the reference's scale decode
  const uint32_t wv[4] = {pl.x, pl.y, pl.z, pl.w};
  float e[32];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t byte = (wv[j >> 2] >> (8 * (j & 3))) & 0xFFu;
    e[j] = (float)((int)(byte & 15u) - 8) * d;  // exact in f32
    e[16 + j] = (float)((int)(byte >> 4) - 8) * d;
  }
  uint32_t h[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) h[j] = pack_h2(e[2 * j], e[2 * j + 1]);
  uint4* o = reinterpret_cast<uint4*>(
      terms == 3 ? out + (size_t)row * 2 * nb * 32 + (size_t)(blk >> 1) * 128 + (blk & 1) * 32 : out + b * 32);
#pragma unroll
  for (int c = 0; c < 4; ++c) o[c] = make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
  if (terms == 3) {
    uint32_t l[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) l[j] = pack_lo2(e[2 * j], e[2 * j + 1], h[j]);
#pragma unroll
    for (int c = 0; c < 4; ++c) o[8 + c] = make_uint4(l[4 * c], l[4 * c + 1], l[4 * c + 2], l[4 * c + 3]);  // +64 halves
  }
}

// f32 X (row-major with stride ldx, or in column chunks of width kc) ->
// row-major f16 [M][K], or (terms == 3) hi/lo pairs [M][2K] (pb_hl_index)
__global__ void k_f32_to_f16(const float* __restrict__ x, int M, int K, int ldx, int kc, __half* __restrict__ out,
                             int terms) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;  // 4 values per thread
  pb_pdl_trigger();
  pb_pdl_wait();
  if (i >= (int64_t)M * K) return;
  const int m = (int)(i / K), k = (int)(i % K);
  const float* src = kc ? x + (size_t)(k / kc) * M * kc + (size_t)m * kc + k % kc : x + (size_t)m * ldx + k;
  const float4 v = __ldg(reinterpret_cast<const float4*>(src));
  const uint2 hi = make_uint2(pack_h2(v.x, v.y), pack_h2(v.z, v.w));
  if (terms != 3) {
    reinterpret_cast<uint2*>(out)[i / 4] = hi;
    return;
  }
  const size_t o = (size_t)m * 2 * K + (size_t)(k >> 6) * 128 + (k & 63);  // k % 4 == 0: 8-byte stores
  *reinterpret_cast<uint2*>(out + o) = hi;
  *reinterpret_cast<uint2*>(out + o + 64) = make_uint2(pack_lo2(v.x, v.y, hi.x), pack_lo2(v.z, v.w, hi.y));
}

// TERMS == 3: both operands are hi/lo pair rows ([rows][2K] halves, 64-wide
// groups), a stage holds A hi, B hi, A lo, B lo (two stages fit), and each
// 16-wide K slice issues hi*hi, hi*lo and lo*hi.
template <int TERMS>
__global__ void __launch_bounds__(TG_THREADS, 1)
k_gemm_f16_tma(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, int N, int M,
               int K, int xkc, float* __restrict__ C, int ldc, pb_gemm_epi epi, int* err) {
  constexpr int NST = TERMS == 3 ? 2 : TG_STAGES;
  constexpr int SB = TERMS == 3 ? 2 * TG_STAGE_BYTES : TG_STAGE_BYTES;
  extern __shared__ __align__(1024) unsigned char tg_raw[];
  __shared__ uint64_t full[NST], empty[NST], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  unsigned char* ring = tg_raw + ((1024 - (pb_smem_addr(tg_raw) & 1023)) & 1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ksteps = K / TG_K;
  const int ntn = (N + TG_ROWS - 1) / TG_ROWS, ntm = (M + TG_TOK - 1) / TG_TOK, ntiles = ntn * ntm;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(pb_smem_addr(&tmem_base)),
                 "r"(2 * TG_TOK)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int s = 0; s < NST; ++s) {
      pb_mbar_init(&full[s], 1);
      pb_mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      pb_mbar_init(&acc_full[b], 1);
      pb_mbar_init(&acc_empty[b], TG_EPI_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_d = tmem_base;
  pb_pdl_trigger();
  pb_pdl_wait();  // both operands and C come from the previous kernels

  if (warp == 0 && lane == 0) {
    // producer: stage s is free once the MMAs that read it committed to empty[s]
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      int n0, m0;
      tg_tile(t, ntn, ntm, n0, m0);
      for (int ks = 0; ks < ksteps; ++ks, ++g) {
        const int s = g % NST;
        if (g >= NST && !(ok = pb_mbar_wait(&empty[s], ((g / NST) - 1) & 1, err))) break;
        unsigned char* sA = ring + s * SB;
        pb_mbar_arrive_tx(&full[s], SB);
        // X: column chunk (k / xkc), x coordinate k % xkc (a multiple of 64 elements);
        // hi/lo rows: the hi group at 2x, the lo group 64 halves after it
        const int xk = (ks * TG_K) % xkc, xz = (ks * TG_K) / xkc;
        if (TERMS == 3) {
          pb_tma_load_2d(sA, &map_w, 2 * ks * TG_K, n0, &full[s]);
          pb_tma_load_3d(sA + TG_A_BYTES, &map_x, 2 * xk, m0, xz, &full[s]);
          pb_tma_load_2d(sA + TG_STAGE_BYTES, &map_w, 2 * ks * TG_K + 64, n0, &full[s]);
          pb_tma_load_3d(sA + TG_STAGE_BYTES + TG_A_BYTES, &map_x, 2 * xk + 64, m0, xz, &full[s]);
        } else {
          pb_tma_load_2d(sA, &map_w, ks * TG_K, n0, &full[s]);
          pb_tma_load_3d(sA + TG_A_BYTES, &map_x, xk, m0, xz, &full[s]);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: tile i accumulates into buffer i % 2 once the epilogue has drained tile i - 2
    int g = 0, i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++i) {
      const int b = i & 1;
      if (i >= 2 && !(ok = pb_mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1, err))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc = tmem_d + (uint32_t)(b * TG_TOK);
      for (int ks = 0; ks < ksteps; ++ks, ++g) {
        const int s = g % NST;
        if (!(ok = pb_mbar_wait(&full[s], (g / NST) & 1, err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        unsigned char* sA = ring + s * SB;
        const uint64_t da = pb_sw128_desc(pb_smem_addr(sA)), db = pb_sw128_desc(pb_smem_addr(sA + TG_A_BYTES));
        const uint64_t dal = pb_sw128_desc(pb_smem_addr(sA + TG_STAGE_BYTES));
        const uint64_t dbl = pb_sw128_desc(pb_smem_addr(sA + TG_STAGE_BYTES + TG_A_BYTES));
#pragma unroll
        for (int kk = 0; kk < TG_K / 16; ++kk) {
          mma_f16_n256(acc, da + 2 * kk, db + 2 * kk, (ks > 0 || kk > 0) ? 1u : 0u);
          if (TERMS == 3) {
            mma_f16_n256(acc, da + 2 * kk, dbl + 2 * kk, 1u);
            mma_f16_n256(acc, dal + 2 * kk, db + 2 * kk, 1u);
          }
        }
        pb_umma_commit(&empty[s]);
      }
      pb_umma_commit(&acc_full[b]);  // fires when every MMA of the tile has completed
    }
  } else if (warp >= 4) {
    // epilogue: lane quadrant q of the accumulator, half of its 256 columns
    const int q = (warp - 4) & 3, half = (warp - 4) >> 2;
    int i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      if (!pb_mbar_wait(&acc_full[b], (i >> 1) & 1, err)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int n0, m0;
      tg_tile(t, ntn, ntm, n0, m0);
      const int row = n0 + q * 32 + lane;
#pragma unroll 1
      for (int c0 = half * (TG_TOK / 2); c0 < (half + 1) * (TG_TOK / 2); c0 += 32) {
        uint32_t v[32];
        pb_tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * TG_TOK + c0), v);
        gemm_emit32(v, false, row, N, m0 + c0, M, C, ldc, epi);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(pb_smem_addr(&acc_empty[b])) : "memory");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(2 * TG_TOK) : "memory");
  }
}

static size_t tg_smem(int terms) {
  return (terms == 3 ? (size_t)2 * 2 * TG_STAGE_BYTES : (size_t)TG_STAGES * TG_STAGE_BYTES) + 1024;
}

// Row-major f16 [rows][K] with a box of box_rows x 64 elements, 128-byte swizzle.
static int make_map(pb_ctx* ctx, CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
  auto enc = pb_tensor_map_encoder(ctx);
  if (!enc) return PB_ERR_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)TG_K, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return pb_set_error(ctx, PB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PB_OK;
}

// f16 X as [K / kc][rows][kc] (kc == K: plain row-major [rows][K]) with a box
// of box_rows x 64 elements of one chunk, 128-byte swizzle.
static int make_map_x(pb_ctx* ctx, CUtensorMap* map, const void* base, int rows, int K, int kc, int box_rows) {
  auto enc = pb_tensor_map_encoder(ctx);
  if (!enc) return PB_ERR_CUDA;
  cuuint64_t dims[3] = {(cuuint64_t)kc, (cuuint64_t)rows, (cuuint64_t)(K / kc)};
  cuuint64_t strides[2] = {(cuuint64_t)kc * 2, (cuuint64_t)rows * kc * 2};
  cuuint32_t box[3] = {(cuuint32_t)TG_K, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return pb_set_error(ctx, PB_ERR_CUDA, "cuTensorMapEncodeTiled (3d) failed (%d)", (int)r);
  return PB_OK;
}

static int launch_gemm_tma(pb_ctx* ctx, const pb_qmat* w, const float* X, const __half* Xh, int ldx, int M, float* C,
                           int ldc, const pb_gemm_epi& epi) {
  const int K = w->K, tw = epi.terms == 3 ? 2 : 1;  // halves per value: hi (and lo)
  const size_t wbytes = (size_t)w->N_pad * K * 2 * tw, xbytes = Xh ? 0 : (size_t)M * K * 2 * tw;
  const size_t off_x = (wbytes + 1023) & ~(size_t)1023;
  PB_TRY(pb_ensure_gemm_scratch(ctx, off_x + xbytes));
  __half* w16 = reinterpret_cast<__half*>(ctx->gemm_scratch);
  const __half* x16 = Xh;
  const int64_t nblk = (int64_t)w->N_pad * w->nb;
  PB_TRY(pb_launch(ctx, "k_dequant_q4_f16", true, k_dequant_q4_f16, dim3((unsigned)pb_cdiv(nblk, 256)), dim3(256), 0,
                   (const uint8_t*)w->qs, (const uint16_t*)w->d, w->layout, w->nb, nblk, w16, epi.terms));
  if (!Xh) {  // the activations rounded to f16 once (or split into hi/lo pairs)
    __half* xs = reinterpret_cast<__half*>(static_cast<char*>(ctx->gemm_scratch) + off_x);
    PB_TRY(pb_launch(ctx, "k_f32_to_f16", true, k_f32_to_f16, dim3((unsigned)pb_cdiv((int64_t)M * K / 4, 256)),
                     dim3(256), 0, X, M, K, ldx, epi.x_chunk, xs, epi.terms));
    x16 = xs;
  }
  // the f32 conversion writes whole rows; an f16 operand keeps its chunks
  const int xkc = (Xh && epi.x_chunk) ? epi.x_chunk : K;
  CUtensorMap mw, mx;
  PB_TRY(make_map(ctx, &mw, w16, w->N_pad, K * tw, TG_ROWS));
  PB_TRY(make_map_x(ctx, &mx, const_cast<__half*>(x16), M, K * tw, xkc * tw, TG_TOK));
  const int64_t ntiles = (int64_t)pb_cdiv(w->N, TG_ROWS) * pb_cdiv(M, TG_TOK);
  if (ntiles > (1ll << 30)) return pb_set_error(ctx, PB_ERR_ARG, "M=%d too large", M);
  const int grid = (int)(ntiles < ctx->sm_count ? ntiles : ctx->sm_count);  // persistent: one CTA per SM
  auto kern = epi.terms == 3 ? k_gemm_f16_tma<3> : k_gemm_f16_tma<1>;
  return pb_launch(ctx, "k_gemm_f16_tma", true, kern, dim3(grid), dim3(TG_THREADS), tg_smem(epi.terms), mw, mx, w->N, M,
                   K, xkc, C, ldc, epi, ctx->d_err);
}

// C[m][n] = sum over z (ascending) of the split-K partials ws[z][m][n], then
// the epilogue: stored, added to C, or (SwiGLU, one thread per output f) the
// gate and up rows of f summed and combined.
__global__ void k_splitk_reduce(const float* __restrict__ ws, int splits, int M, int N, float* __restrict__ C,
                                int ldc, pb_gemm_epi epi) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
  pb_pdl_trigger();
  pb_pdl_wait();  // the partials come from the GEMM before
  if (epi.mode == PB_GEMM_SWIGLU) {
    if (i >= N / 2) return;
    const int ng = 8 * (i >> 2) + (i & 3), nu = ng + 4;
    float g = 0.0f, u = 0.0f;
    for (int z = 0; z < splits; ++z) {
      g += ws[((size_t)z * M + m) * N + ng];
      u += ws[((size_t)z * M + m) * N + nu];
    }
    const float h = __fdividef(g, 1.0f + __expf(-g)) * u;
    if (epi.h16 && epi.terms == 3) pb_store_hl(epi.h16, pb_hl_index((size_t)m * N, i), h);
    else if (epi.h16) epi.h16[(size_t)m * (N / 2) + i] = __float2half_rn(h);
    else epi.h32[(size_t)m * (N / 2) + i] = h;
    return;
  }
  float v = 0.0f;
  if (i < N) {
    float acc = 0.0f;
    for (int z = 0; z < splits; ++z) acc += ws[((size_t)z * M + m) * N + i];
    float* c = C + (size_t)m * ldc + i;
    v = epi.mode == PB_GEMM_ADD ? __fadd_rn(*c, acc) : acc;
    *c = v;
  }
  if (epi.xs.world > 0) {  // the fused residual exchange: threads (i, i ^ 1) form a packet
    const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
    if (i < N && (i & 1) == 0) pb_xsend_pair(epi.xs, m, i, v, partner);
  }
}

// k_splitk_reduce for a STORE / ADD GEMM followed by an RMSNorm (epi.norm_w):
// one CTA of 1024 threads per row m.  Each value is k_splitk_reduce's (the
// splits' partials summed in ascending order from 0, four loads in flight at
// a time, then stored or added to C) and goes to shared memory; the row is then normalised with
// k_rmsnorm_t's arithmetic: its first 256 threads take k_rmsnorm_t's values
// (d = t, t + 256, ...) for the sum of squares, the other warps add exact
// zeros to the same block sum.  So the output has the bits of the reduce and
// the norm launched apart.
constexpr int RN_THREADS = 1024, RN_NORM_THREADS = 256;
__global__ void __launch_bounds__(RN_THREADS)
k_splitk_reduce_norm(const float* __restrict__ ws, int splits, int M, int N, float* __restrict__ C, pb_gemm_epi epi) {
  extern __shared__ float rn_row[];  // [N]
  __shared__ double red[32];
  const int m = blockIdx.x, tid = threadIdx.x;
  pb_pdl_trigger();
  pb_pdl_wait();  // the partials come from the GEMM before
  for (int d = tid; d < N; d += RN_THREADS) {
    // the splits in ascending order, four loads in flight at a time
    const float* src = ws + (size_t)m * N + d;
    const size_t zs = (size_t)M * N;
    float acc = 0.0f;
    int z = 0;
    for (; z + 4 <= splits; z += 4) {
      const float p0 = src[z * zs], p1 = src[(z + 1) * zs], p2 = src[(z + 2) * zs], p3 = src[(z + 3) * zs];
      acc += p0;
      acc += p1;
      acc += p2;
      acc += p3;
    }
    for (; z < splits; ++z) acc += src[z * zs];
    float* c = C + (size_t)m * N + d;
    const float v = epi.mode == PB_GEMM_ADD ? __fadd_rn(*c, acc) : acc;
    *c = v;
    rn_row[d] = v;
  }
  __syncthreads();
  double ss = 0.0;
  if (tid < RN_NORM_THREADS)
    for (int d = tid; d < N; d += RN_NORM_THREADS) {
      const double dv = (double)rn_row[d];
      ss = __fma_rn(dv, dv, ss);
    }
  ss = pb_block_sum_d(ss, red);
  const double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)N), epi.norm_eps));
  const float inv = (float)(1.0 / rms);
  const float* w = epi.norm_w;
  for (int d = tid; d < N; d += RN_THREADS) {
    const float v = rn_row[d];
    if (epi.norm_out16 && epi.norm_hl) pb_store_hl(epi.norm_out16, pb_hl_index((size_t)m * 2 * N, d), v * inv * w[d]);
    else if (epi.norm_out16) epi.norm_out16[(size_t)m * N + d] = __float2half_rn(v * inv * w[d]);
    else epi.norm_out[(size_t)m * N + d] = (float)__dmul_rn(__ddiv_rn((double)v, rms), (double)w[d]);
  }
}

// The split-K partials of ws summed into C (and, when the GEMM is followed
// by its RMSNorm and the shapes allow, normalised in the same kernel:
// *norm_done).
static int launch_reduce(pb_ctx* ctx, const float* ws, int splits, int M, int N, float* C, int ldc,
                         const pb_gemm_epi& epi, bool* norm_done) {
  if (epi.norm_w && epi.mode != PB_GEMM_SWIGLU && epi.xs.world == 0 && ldc == N && (size_t)N * 4 <= 48 * 1024) {
    *norm_done = true;
    return pb_launch(ctx, "k_splitk_reduce_norm", true, k_splitk_reduce_norm, dim3(M), dim3(RN_THREADS), (size_t)N * 4,
                     ws, splits, M, N, C, epi);
  }
  const int cols = epi.mode == PB_GEMM_SWIGLU ? N / 2 : N;
  return pb_launch(ctx, "k_splitk_reduce", true, k_splitk_reduce, dim3(pb_cdiv(cols, 256), M), dim3(256), 0, ws,
                   splits, M, N, C, ldc, epi);
}

bool pb_gemm_uses_tma(const pb_qmat* w, int M) { return M >= PB_GEMM_TMA_MIN_M && w->K % TG_K == 0; }
static int launch_gemm_ws(pb_ctx* ctx, const pb_qmat* w, const __half* Xh, int M, float* C, int ldc, float* ws,
                          size_t ws_bytes, const pb_gemm_epi& epi, bool* norm_done);

static int launch_q4_gemm(pb_ctx* ctx, const pb_qmat* w, const float* X, int ldx, int M, float* C, int ldc, float* ws,
                          size_t ws_bytes, const pb_gemm_epi& epi, const __half* Xh, bool* norm_done);

int pb_launch_q4_gemm(pb_ctx* ctx, const pb_qmat* w, const float* X, int ldx, int M, float* C, int ldc, float* ws,
                      size_t ws_bytes, const pb_gemm_epi* epi_in, const __half* Xh) {
  const pb_gemm_epi epi = epi_in ? *epi_in : pb_gemm_epi();
  if (epi.norm_w && (epi.mode == PB_GEMM_SWIGLU || epi.xs.world > 0 || ldc != (w ? w->N : 0) ||
                     !(epi.norm_out || epi.norm_out16)))
    return pb_set_error(ctx, PB_ERR_ARG, "a GEMM's RMSNorm needs a STORE / ADD row-major C and an output");
  bool norm_done = false;
  PB_TRY(launch_q4_gemm(ctx, w, X, ldx, M, C, ldc, ws, ws_bytes, epi, Xh, &norm_done));
  if (epi.norm_w && !norm_done) {
    pb_launch_rmsnorm(ctx->stream, C, M, w->N, epi.norm_w, epi.norm_eps, epi.norm_out, epi.norm_out16, 0, epi.norm_hl,
                      ctx->pdl);
    PB_LAUNCHED(ctx, "k_rmsnorm");
  }
  return PB_OK;
}

static int launch_q4_gemm(pb_ctx* ctx, const pb_qmat* w, const float* X, int ldx, int M, float* C, int ldc, float* ws,
                          size_t ws_bytes, const pb_gemm_epi& epi, const __half* Xh, bool* norm_done) {
  if (!ctx || !w || !(X || Xh) || M <= 0) return PB_ERR_ARG;
  if (epi.mode == PB_GEMM_SWIGLU ? (!(epi.h16 || epi.h32) || w->N % 8) : !C) return PB_ERR_ARG;
  if (w->type != PB_TYPE_Q4_0) return pb_set_error(ctx, PB_ERR_ARG, "the tensor-core GEMM needs a Q4_0 matrix");
  if (X && ((ldx & 3) || ((uintptr_t)X & 15)))
    return pb_set_error(ctx, PB_ERR_ARG, "X must be 16-byte aligned with a row stride that is a multiple of 4");
  if (epi.x_chunk && (epi.x_chunk % 64 || w->K % epi.x_chunk))
    return pb_set_error(ctx, PB_ERR_ARG, "column chunks of %d do not tile K=%d in steps of 64", epi.x_chunk, w->K);
  if (Xh && ((uintptr_t)Xh & 15)) return pb_set_error(ctx, PB_ERR_ARG, "f16 X must be 16-byte aligned");
  if (pb_gemm_uses_tma(w, M)) return launch_gemm_tma(ctx, w, X, Xh, ldx, M, C, ldc, epi);
  if (Xh && pb_gemm_uses_ws(w, M)) return launch_gemm_ws(ctx, w, Xh, M, C, ldc, ws, ws_bytes, epi, norm_done);
  if (!X)
    return pb_set_error(ctx, PB_ERR_ARG, "f16 activations need M >= %d or M <= 64", PB_GEMM_TMA_MIN_M);
  const int tok = M <= 64 ? 64 : GM_TOK;
  dim3 grid(pb_cdiv(w->N, GM_ROWS), pb_cdiv(M, tok), 1);
  if (grid.y > 65535) return pb_set_error(ctx, PB_ERR_ARG, "M=%d too large", M);
  // With a workspace, split K over CTAs until the grid covers the SMs twice;
  // the partial tiles are summed in split order, so the result does not
  // depend on scheduling.
  const int ktot = pb_cdiv(w->K, GM_KSTEP);
  int splits = 1;
  if (ws) {
    // planned for split_n rows when set (a row slice keeps the whole matrix's plan)
    const int plan_n = epi.split_n > 0 ? epi.split_n : w->N;
    const int base = pb_cdiv(plan_n, GM_ROWS) * grid.y;
    // until the grid covers the SMs twice, or once with the three-term stages (one CTA per SM)
    splits = pb_cdiv((epi.terms == 3 ? 1 : 2) * ctx->sm_count, base);
    const int max_by_k = ktot / 4 > 1 ? ktot / 4 : 1;
    const int max_by_ws = (int)(ws_bytes / ((size_t)M * plan_n * 4));
    const int fit = (int)(ws_bytes / ((size_t)M * w->N * 4));  // the partials of this matrix must fit
    splits = splits < max_by_k ? splits : max_by_k;
    splits = splits < max_by_ws ? splits : max_by_ws;
    splits = splits < fit ? splits : fit;
    if (splits < 1) splits = 1;
  }
  const int kper = pb_cdiv(ktot, splits);
  splits = pb_cdiv(ktot, kper);
  grid.z = splits;
  float* dst = splits > 1 ? ws : C;
  const int ldd = splits > 1 ? w->N : ldc;
  pb_gemm_epi kepi = epi;  // split partials are stored (same X layout), the reduce finishes
  if (splits > 1) {
    kepi.mode = PB_GEMM_STORE;
    kepi.h16 = nullptr;
    kepi.h32 = nullptr;
    kepi.xs.world = 0;  // the reduce sends the finished values
  }
  auto kern = epi.terms == 3
                  ? (tok == 64 ? (epi.x_chunk ? k_q4_gemm_tc<64, true, 3> : k_q4_gemm_tc<64, false, 3>)
                               : (epi.x_chunk ? k_q4_gemm_tc<128, true, 3> : k_q4_gemm_tc<128, false, 3>))
                  : (tok == 64 ? (epi.x_chunk ? k_q4_gemm_tc<64, true, 1> : k_q4_gemm_tc<64, false, 1>)
                               : (epi.x_chunk ? k_q4_gemm_tc<128, true, 1> : k_q4_gemm_tc<128, false, 1>));
  PB_TRY(pb_launch(ctx, "k_q4_gemm_tc", true, kern, grid, dim3(GM_THREADS), gm_smem(epi.terms), (const uint8_t*)w->qs,
                   (const uint16_t*)w->d, w->layout, w->N, w->N_pad, w->nb, X, ldx, M, dst, ldd, kper, kepi,
                   ctx->d_err));
  if (splits > 1) PB_TRY(launch_reduce(ctx, ws, splits, M, w->N, C, ldc, epi, norm_done));
  return PB_OK;
}

extern "C" int pb_q4_gemm_f16(pb_ctx* ctx, const pb_qmat* w, const void* x16_dev, int M, float* c_dev, int ldc) {
  if (!ctx || !w || !x16_dev || !c_dev || M <= 0) return PB_ERR_ARG;
  if (ldc < w->N) return pb_set_error(ctx, PB_ERR_ARG, "row stride smaller than the matrix");
  if (!pb_gemm_uses_ws(w, M) && !pb_gemm_uses_tma(w, M))
    return pb_set_error(ctx, PB_ERR_ARG, "f16 activations take M <= 64 or M >= %d rows and K %% 64 == 0",
                        PB_GEMM_TMA_MIN_M);
  return pb_launch_q4_gemm(ctx, w, nullptr, w->K, M, c_dev, ldc, nullptr, 0, nullptr,
                           static_cast<const __half*>(x16_dev));
}

extern "C" int pb_q4_gemm(pb_ctx* ctx, const pb_qmat* w, const float* x_dev, int M, int ldx, float* c_dev, int ldc) {
  return pb_q4_gemm_ex(ctx, w, x_dev, M, ldx, c_dev, ldc, 1);
}

extern "C" int pb_q4_gemm_ex(pb_ctx* ctx, const pb_qmat* w, const float* x_dev, int M, int ldx, float* c_dev, int ldc,
                             int terms) {
  if (!w || (terms != 1 && terms != 3)) return PB_ERR_ARG;
  if (ldx < w->K || ldc < w->N) return pb_set_error(ctx, PB_ERR_ARG, "row strides smaller than the matrix");
  pb_gemm_epi e;
  e.terms = terms;
  return pb_launch_q4_gemm(ctx, w, x_dev, ldx, M, c_dev, ldc, nullptr, 0, &e);
}

extern "C" int pb_q4_gemm_hl(pb_ctx* ctx, const pb_qmat* w, const void* xhl_dev, int M, float* c_dev, int ldc) {
  if (!ctx || !w || !xhl_dev || !c_dev || M <= 0) return PB_ERR_ARG;
  if (ldc < w->N) return pb_set_error(ctx, PB_ERR_ARG, "row stride smaller than the matrix");
  if (!pb_gemm_uses_ws(w, M) && !pb_gemm_uses_tma(w, M))
    return pb_set_error(ctx, PB_ERR_ARG, "hi/lo activations take M <= 64 or M >= %d rows and K %% 64 == 0",
                        PB_GEMM_TMA_MIN_M);
  pb_gemm_epi e;
  e.terms = 3;
  return pb_launch_q4_gemm(ctx, w, nullptr, w->K, M, c_dev, ldc, nullptr, 0, &e, static_cast<const __half*>(xhl_dev));
}

// ---------------------------------------------------------------------------
// Decode-size batches (M <= 64 tokens, f16 activations): a warp-specialised
// form of the fused-dequant GEMM.  CTA = 128 weight rows x 64 tokens, K split
// over grid.z as in k_q4_gemm_tc.  Per 64-wide K step a 6-stage ring holds the
// raw Q4_0 payload tile (4 KB, TMA from the resident layout) and the
// activation tile (TMA, 128-byte swizzle), so about 70 KB per SM stream in
// flight; the dequantized f16 weight tile is double-buffered apart from it:
//   warp 0 lane 0: TMA producer (payload + activations, one mbarrier);
//   warp 1 lane 0: MMA issuer (four 128 x 64 x 16 MMAs per step, committed
//     to the stage's "empty" and the weight buffer's "free" mbarriers);
//   warps 2-5: dequant, thread t = row t: its 2 blocks from shared memory,
//     value (q - 8) * d in half precision: the nibble is OR-ed into the f16
//     1024.0 (0x6400), 1032 is subtracted (exact) and the product with d is
//     rounded once, the same bits as rounding the exact f32 product; the f16
//     row goes to the swizzled tile; then the epilogue of its TMEM quadrant.
// The weight values are the ones k_q4_gemm_tc stages; the K steps accumulate
// in the same order, so both kernels give the same partial sums.
// ---------------------------------------------------------------------------

constexpr int GW_ROWS = 128, GW_TOK = 64, GW_K = 64, GW_STAGES = 6, GW_ABUF = 2, GW_THREADS = 320;
constexpr int GW_DQ = GW_THREADS - 64;  // dequant threads: one per (row, block) of a 64-wide K step
static_assert(GW_DQ == 2 * GW_ROWS && GW_TOK == 64 && GW_K == 64,
              "the dequant threads cover a step's two blocks of every row; two warps share a TMEM quadrant's columns");
constexpr int GW_RAW_BYTES = GW_ROWS * 32;               // 2 Q4_0 payloads (16 B) per row
constexpr int GW_X_BYTES = GW_TOK * GW_K * 2;            // f16 activations, swizzled
constexpr int GW_A_BYTES = GW_ROWS * GW_K * 2;           // f16 weights, swizzled
// [GW_ABUF dequantized tiles][GW_STAGES (activations, payload) stages], the
// activations first in a stage (1024-aligned); with three terms each weight
// tile and each activation tile is a hi, lo pair
static size_t gw_smem(int terms) {
  const int t = terms == 3 ? 2 : 1;
  return (size_t)GW_ABUF * GW_A_BYTES * t + (size_t)GW_STAGES * (GW_X_BYTES * t + GW_RAW_BYTES) + 1024;
}

namespace {
__device__ __forceinline__ uint32_t h2_sub_mul(uint32_t v, uint32_t magic, uint32_t d2) {
  // (v - magic) * d2 on f16 pairs: the subtraction is exact, the product rounded once
  uint32_t r;
  asm("{\n\t.reg .b32 t;\n\tsub.rn.f16x2 t, %1, %2;\n\tmul.rn.f16x2 %0, t, %3;\n\t}"
      : "=r"(r)
      : "r"(v), "r"(magic), "r"(d2));
  return r;
}

// hi = f16((v - magic) * d2) and lo = (v - magic) * d2 - hi on f16 pairs.  The
// fused multiply-add rounds once, and the remainder is exact in f16: the
// product is an integer multiple of d's last place with at most 14
// significant bits, so hi (11 bits) leaves a multiple of that place of at
// most 4 bits.
__device__ __forceinline__ void h2_sub_mul_hl(uint32_t v, uint32_t magic, uint32_t d2, uint32_t& hi, uint32_t& lo) {
  asm("{\n\t.reg .b32 t, n;\n\tsub.rn.f16x2 t, %2, %3;\n\tmul.rn.f16x2 %0, t, %4;\n\t"
      "neg.f16x2 n, %0;\n\tfma.rn.f16x2 %1, t, %4, n;\n\t}"
      : "=r"(hi), "=r"(lo)
      : "r"(v), "r"(magic), "r"(d2));
}
}  // namespace

// TERMS == 3: the activations are hi/lo pair rows (two TMA boxes per step),
// the dequant warps write the weight tile's hi and lo halves, and each
// 16-wide K slice issues hi*hi, hi*lo and lo*hi.
template <int TERMS>
__global__ void __launch_bounds__(GW_THREADS, 1)
k_q4_gemm_ws(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_x,
             const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int layout, int N, int N_pad, int nb, int M, int xkc,
             float* __restrict__ C, int ldc, int kper, pb_gemm_epi epi, int* err) {
  constexpr int TW = TERMS == 3 ? 2 : 1;
  constexpr int XB = GW_X_BYTES * TW, SB = XB + GW_RAW_BYTES, AB = GW_A_BYTES * TW;
  extern __shared__ __align__(1024) unsigned char gw_raw[];
  __shared__ uint64_t full[GW_STAGES], empty[GW_STAGES], aready[GW_ABUF], afree[GW_ABUF], accf;
  __shared__ uint32_t tmem_base;
  unsigned char* ring = gw_raw + ((1024 - (pb_smem_addr(gw_raw) & 1023)) & 1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * GW_ROWS, m0 = blockIdx.y * GW_TOK;
  const int ktot = nb / 2;  // K / 64
  const int kbeg = blockIdx.z * kper, kend = kbeg + kper < ktot ? kbeg + kper : ktot;
  const int ksteps = kend > kbeg ? kend - kbeg : 0;
  C += (size_t)blockIdx.z * M * ldc;
  // programmatic dependent launch: the next kernel may start its own weight
  // loads now; this grid reads activations and writes C only after the
  // dependency wait (the producer before its activation loads, the other
  // threads below)
  pb_pdl_trigger();

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(pb_smem_addr(&tmem_base)),
                 "r"(GW_TOK)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int st = 0; st < GW_STAGES; ++st) {
      pb_mbar_init(&full[st], 1);
      pb_mbar_init(&empty[st], 1);
    }
    for (int ab = 0; ab < GW_ABUF; ++ab) {
      pb_mbar_init(&aready[ab], GW_DQ);
      pb_mbar_init(&afree[ab], 1);
    }
    pb_mbar_init(&accf, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_d = tmem_base;

  if (warp == 0) {
    if (lane == 0) {  // producer
      // the Q4_0 payload of step g into stage g % GW_STAGES (weights: final before this grid)
      auto payload = [&](int g) {
        const int st = g % GW_STAGES, ks = kbeg + g;
        unsigned char* sX = ring + GW_ABUF * AB + st * SB;
        if (layout == PB_LAYOUT_TILED8)
          asm volatile(
              "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
              "[%5];" ::"r"(pb_smem_addr(sX + XB)),
              "l"(&map_q), "r"(0), "r"(2 * ks), "r"(n0 >> 3), "r"(pb_smem_addr(&full[st]))
              : "memory");
        else
          pb_tma_load_2d(sX + XB, &map_q, 32 * ks, n0, &full[st]);
      };
      // the activations of step g (written by the previous kernels)
      auto acts = [&](int g) {
        const int st = g % GW_STAGES, ks = kbeg + g;
        unsigned char* sX = ring + GW_ABUF * AB + st * SB;
        const int xk = (ks * GW_K) % xkc, xz = (ks * GW_K) / xkc;
        pb_tma_load_3d(sX, &map_x, TW * xk, m0, xz, &full[st]);
        if (TERMS == 3) pb_tma_load_3d(sX + GW_X_BYTES, &map_x, 2 * xk + 64, m0, xz, &full[st]);
      };
      // the first ring's payloads go out before the dependency wait, their activations after it
      const int first = ksteps < GW_STAGES ? ksteps : GW_STAGES;
      for (int g = 0; g < first; ++g) {
        pb_mbar_arrive_tx(&full[g], SB);
        payload(g);
      }
      pb_pdl_wait();
      for (int g = 0; g < first; ++g) acts(g);
      bool ok = true;
      for (int g = first; g < ksteps && ok; ++g) {
        const int st = g % GW_STAGES;
        if (!(ok = pb_mbar_wait_sleep(&empty[st], ((g / GW_STAGES) - 1) & 1, err))) break;
        pb_mbar_arrive_tx(&full[st], SB);
        payload(g);
        acts(g);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      bool ok = true;
      for (int g = 0; g < ksteps && ok; ++g) {
        const int st = g % GW_STAGES, ab = g % GW_ABUF;
        // the weight tile of step g is written after the payload and activations landed
        if (!(ok = pb_mbar_wait_sleep(&aready[ab], (g / GW_ABUF) & 1, err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        unsigned char* sA = ring + ab * AB;
        unsigned char* sX = ring + GW_ABUF * AB + st * SB;
        const uint64_t da = pb_sw128_desc(pb_smem_addr(sA)), db = pb_sw128_desc(pb_smem_addr(sX));
        const uint64_t dal = pb_sw128_desc(pb_smem_addr(sA + GW_A_BYTES)), dbl = pb_sw128_desc(pb_smem_addr(sX + GW_X_BYTES));
#pragma unroll
        for (int kk = 0; kk < GW_K / 16; ++kk) {
          mma_f16(tmem_d, da + 2 * kk, db + 2 * kk, gm_idesc(GW_TOK), (g > 0 || kk > 0) ? 1u : 0u);
          if (TERMS == 3) {
            mma_f16(tmem_d, da + 2 * kk, dbl + 2 * kk, gm_idesc(GW_TOK), 1u);
            mma_f16(tmem_d, dal + 2 * kk, db + 2 * kk, gm_idesc(GW_TOK), 1u);
          }
        }
        pb_umma_commit(&empty[st]);
        pb_umma_commit(&afree[ab]);
      }
      if (ok && ksteps > 0) pb_umma_commit(&accf);
    }
  } else {
    // dequant: thread t = (block bb = t / 128 of the step, weight row n0 + t % 128); two
    // warps per sub-partition, so one warp's latency hides behind the other's
    const int t = (tid - 64) & (GW_ROWS - 1), bb = (tid - 64) >> 7, row = n0 + t;
    const bool live_row = row < N_pad;
    const uint32_t magic = 0x64086408u;  // f16 1032.0 twice
    // the CTA's payload slice into L2 first (one run per row, or per 8-row tile)
    if (ksteps > 0 && bb == 0) {
      const int b0 = 2 * kbeg, b1 = 2 * kend < nb ? 2 * kend : nb;
      if (layout == PB_LAYOUT_TILED8) {
        const int tile = (n0 >> 3) + t;
        if (t < GW_ROWS / 8 && tile * 8 < N_pad)
          pb_l2_prefetch(qs + ((size_t)tile * nb + b0) * 128, (uint32_t)(b1 - b0) * 128);
      } else if (live_row) {
        pb_l2_prefetch(qs + ((size_t)row * nb + b0) * 16, (uint32_t)(b1 - b0) * 16);
      }
    }
    bool ok = true;
    // the thread's scale of a step, loaded one step ahead (L2-resident after the prefetch)
    auto scales = [&](int ks) -> uint32_t {
      if (!live_row || ks >= kend) return 0u;
      // the reference's scale decode: a zero exponent is +0 (subnormal scales flushed)
      const uint32_t bits = __ldg(dsc + pb_slot(layout, row, 2 * ks + bb, nb));
      return (bits & 0x7C00u) ? bits : 0u;
    };
    uint32_t dnext = scales(kbeg);
    pb_pdl_wait();  // before the epilogue reads or writes C
    for (int g = 0; g < ksteps && ok; ++g) {
      const int st = g % GW_STAGES, ks = kbeg + g;
      const uint32_t d2 = dnext | (dnext << 16);
      dnext = scales(ks + 1);
      const int ab = g % GW_ABUF;
      if (!(ok = pb_mbar_wait_sleep(&full[st], (g / GW_STAGES) & 1, err))) break;
      // the weight buffer is free once the MMAs of step g - GW_ABUF completed
      if (g >= GW_ABUF && !(ok = pb_mbar_wait_sleep(&afree[ab], ((g / GW_ABUF) - 1) & 1, err))) break;
      unsigned char* sA = ring + ab * AB;
      const unsigned char* raw = ring + GW_ABUF * AB + st * SB + XB;
      {
        const uint32_t off =
            layout == PB_LAYOUT_TILED8 ? (uint32_t)((((t >> 3) * 2 + bb) * 8 + (t & 7)) * 16) : (uint32_t)(t * 32 + bb * 16);
        const uint4 q = *reinterpret_cast<const uint4*>(raw + off);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        // f16 pairs (k, k+1): v[0..7] from the low nibbles (k 0..15), v[8..15] the high ones (k 16..31)
        uint32_t v[16], h[16], r[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t a = __byte_perm(w[i], 0u, 0x4140u), b = __byte_perm(w[i], 0u, 0x4342u);
          v[2 * i] = (a & 0x000F000Fu) | 0x64006400u;
          v[2 * i + 1] = (b & 0x000F000Fu) | 0x64006400u;
          v[8 + 2 * i] = ((a >> 4) & 0x000F000Fu) | 0x64006400u;
          v[8 + 2 * i + 1] = ((b >> 4) & 0x000F000Fu) | 0x64006400u;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (TERMS == 3) h2_sub_mul_hl(v[i], magic, d2, h[i], r[i]);
          else h[i] = h2_sub_mul(v[i], magic, d2);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          *reinterpret_cast<uint4*>(sA + pb_sw128(t, 4 * bb + c)) = make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
          if (TERMS == 3)
            *reinterpret_cast<uint4*>(sA + GW_A_BYTES + pb_sw128(t, 4 * bb + c)) =
                make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
        }
      }
      // generic-proxy reads of the payload and writes of the tile -> the async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(pb_smem_addr(&aready[ab])) : "memory");
    }
    // epilogue: TMEM lanes of this warp's quadrant (warp % 4), two warps per quadrant, each
    // 32 of the 64 token columns
    const bool empty_split = ksteps == 0;
    if (ok && !empty_split) ok = pb_mbar_wait_sleep(&accf, 0, err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
      const int q4 = warp & 3, erow = n0 + q4 * 32 + lane, c0 = bb * 32;
      uint32_t v[32];
      pb_tmem_ld32(tmem_d + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, v);
      gemm_emit32(v, empty_split, erow, N, m0 + c0, M, C, ldc, epi);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(GW_TOK) : "memory");
  }
}

// The payload of a resident Q4_0 matrix as a TMA tensor: rows of nb * 16
// bytes (row layout: box 32 B x 128 rows) or 8-row tiles (tiled layout:
// {128 B, nb, N_pad / 8}, box 128 B x 2 blocks x 16 tiles).
static int make_map_q(pb_ctx* ctx, CUtensorMap* map, const pb_qmat* w) {
  auto enc = pb_tensor_map_encoder(ctx);
  if (!enc) return PB_ERR_CUDA;
  CUresult r;
  cuuint32_t estr[3] = {1, 1, 1};
  if (w->layout == PB_LAYOUT_TILED8) {
    cuuint64_t dims[3] = {128, (cuuint64_t)w->nb, (cuuint64_t)(w->N_pad / 8)};
    cuuint64_t strides[2] = {128, (cuuint64_t)w->nb * 128};
    cuuint32_t box[3] = {128, 2, GW_ROWS / 8};
    r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, w->qs, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)w->nb * 16, (cuuint64_t)w->N_pad};
    cuuint64_t strides[1] = {(cuuint64_t)w->nb * 16};
    cuuint32_t box[2] = {32, GW_ROWS};
    r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->qs, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return pb_set_error(ctx, PB_ERR_CUDA, "cuTensorMapEncodeTiled (Q4 payload) failed (%d)", (int)r);
  return PB_OK;
}

bool pb_gemm_uses_ws(const pb_qmat* w, int M) {
  return M <= GW_TOK && w->type == PB_TYPE_Q4_0 && w->K % GW_K == 0;
}

static int launch_gemm_ws(pb_ctx* ctx, const pb_qmat* w, const __half* Xh, int M, float* C, int ldc, float* ws,
                          size_t ws_bytes, const pb_gemm_epi& epi, bool* norm_done) {
  const int ktot = w->K / GW_K;
  dim3 grid(pb_cdiv(w->N, GW_ROWS), 1, 1);
  int splits = 1;
  if (ws) {  // split K while the grid fits one wave of the CTAs an SM holds (shared memory)
    const int plan_n = epi.split_n > 0 ? epi.split_n : w->N;
    static const int per_sm_env = getenv("PB_WS_PER_SM") ? atoi(getenv("PB_WS_PER_SM")) : 0;  // tuning override
    int per_sm = (int)((size_t)227 * 1024 / (gw_smem(epi.terms) + 1024));
    if (per_sm < 1) per_sm = 1;
    if (per_sm_env > 0) per_sm = per_sm_env;
    splits = per_sm * ctx->sm_count / pb_cdiv(plan_n, GW_ROWS);
    const int max_by_k = ktot / 4 > 1 ? ktot / 4 : 1;
    const int max_by_ws = (int)(ws_bytes / ((size_t)M * plan_n * 4));
    const int fit = (int)(ws_bytes / ((size_t)M * w->N * 4));
    splits = splits < max_by_k ? splits : max_by_k;
    splits = splits < max_by_ws ? splits : max_by_ws;
    splits = splits < fit ? splits : fit;
    if (splits < 1) splits = 1;
  }
  const int kper = pb_cdiv(ktot, splits);
  splits = pb_cdiv(ktot, kper);
  grid.z = splits;
  float* dst = splits > 1 ? ws : C;
  const int ldd = splits > 1 ? w->N : ldc;
  pb_gemm_epi kepi = epi;
  if (splits > 1) {
    kepi.mode = PB_GEMM_STORE;
    kepi.h16 = nullptr;
    kepi.h32 = nullptr;
    kepi.xs.world = 0;  // the reduce sends the finished values
  }
  const int xkc = epi.x_chunk ? epi.x_chunk : w->K, tw = epi.terms == 3 ? 2 : 1;
  CUtensorMap mq, mx;
  PB_TRY(make_map_q(ctx, &mq, w));
  PB_TRY(make_map_x(ctx, &mx, Xh, M, w->K * tw, xkc * tw, GW_TOK));
  auto kern = epi.terms == 3 ? k_q4_gemm_ws<3> : k_q4_gemm_ws<1>;
  PB_TRY(pb_launch(ctx, "k_q4_gemm_ws", true, kern, grid, dim3(GW_THREADS), gw_smem(epi.terms), mq, mx,
                   (const uint8_t*)w->qs, (const uint16_t*)w->d, w->layout, w->N, w->N_pad, w->nb, M, xkc, dst, ldd,
                   kper, kepi, ctx->d_err));
  if (splits > 1) PB_TRY(launch_reduce(ctx, ws, splits, M, w->N, C, ldc, epi, norm_done));
  return PB_OK;
}

int pb_setup_gemm_kernels(void) {
  cudaError_t e = cudaSuccess;
  for (auto k : {k_q4_gemm_tc<64, false, 1>, k_q4_gemm_tc<64, true, 1>, k_q4_gemm_tc<128, false, 1>,
                 k_q4_gemm_tc<128, true, 1>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gm_smem(1));
  for (auto k : {k_q4_gemm_tc<64, false, 3>, k_q4_gemm_tc<64, true, 3>, k_q4_gemm_tc<128, false, 3>,
                 k_q4_gemm_tc<128, true, 3>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gm_smem(3));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_q4_gemm_ws<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gw_smem(1));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_q4_gemm_ws<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gw_smem(3));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_gemm_f16_tma<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tg_smem(1));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_gemm_f16_tma<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tg_smem(3));
  return e == cudaSuccess ? PB_OK : PB_ERR_CUDA;
}
