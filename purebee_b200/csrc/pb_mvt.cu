// pb_mvt.cu - the tcgen05 int8 Q4_0 matvec of the fast mode (k_mvt).
//
// y[n] = sum_b d[n][b] * sum_{k in block b} (q[n][k] - 8) * x[k]  (wasm-q4.js
// :118-267 computes the same sum in its own f32 order; this path agrees with
// it within an f32 tolerance, the exact kernels in pb_q4.cu stay the parity
// mode).
//
// The arithmetic is k_mvi's (pb_mvi.cu): the 4-bit codes go to the tensor
// cores as unsigned bytes, x per 32-value block b as three signed byte digits
// (pb_x_digits: x[k] ~= f_b (d0 + d1/254 + d2/254^2)), the integer products
// are exact, and the -8 of the codes is applied through T_b, the sum of each
// digit over the block.  Per (row, block) the three integer sums D0..D2 give
//     v = (D0 - 8 T0) + (D1 - 8 T1) / 254 + (D2 - 8 T2) / 254^2
// and y[row] accumulates v * d[row][b] * f_b in f32, blocks in K order.
//
// Here the products run on the 5th-generation tensor cores:
// tcgen05.mma.kind::i8, M = 128 weight rows, N = 16 (B's rows 0..2 hold the
// three digits of x, the other rows are zero), K = 32 = one Q4_0 block.  A
// block's scale differs per row, so every block gets its own accumulator:
// one MMA per (128-row tile, block) into 16 TMEM columns of its own.  Per
// weight this leaves about a third of an instruction on the SM's pipes (the
// nibble split, a quarter of a logic op, plus the stores); the f32 kernel
// k_mvf spends about four, which bounds it by instruction issue, not HBM.
// Measured on B200, the MMAs bound it instead: a thread issuing these
// M = 128, N = 16, K = 32 MMAs advances one every ~350 cycles (a K step of 4
// took ~1400 cycles whether the payload came by tensor-map boxes or
// contiguous bulk copies, with 2-8 payload stages, 2-4 code tiles, one or two
// commits), so a CTA moves 8 KB per ~1500 cycles and two per SM reach about
// 3 TB/s: gate|up 16384 x 2048 in 11.0 us against 8.4 for k_mvf, the
// vocabulary head in ~48 us against 37.5 for k_mvi.  It is therefore off by
// default (pb_set_mvt); it stays tested against the oracle.
//
// CTA = one 128-row tile and one K chunk (`cb` blocks), 10 warps:
//   warp 0 lane 0: producer - the raw payload of a K step (4 blocks of 128
//     rows, 8 KB) into a 4-stage ring by one bulk copy from the matrix's
//     tile-contiguous copy (tq: a K step of a tile is one contiguous run; a
//     tensor-map box of 128 rows x 64 B, rows 16 nb bytes apart, measured
//     no faster); the weights are final before this grid, so it starts at
//     once;
//   warp 1 lane 0: MMA issuer - per step 4 MMAs (one per block) from the
//     unpacked code tile and the digit tile into one of 4 TMEM accumulator
//     buffers (64 columns each), one commit (it frees the code tile too);
//   warps 2-5: unpack - a 16-byte payload (one row's block) becomes two
//     16-byte code chunks: low nibbles = elements 0..15, high = 16..31, the
//     Q4_0 order (wasm-q4.js:118-267), written to the K-major 128-byte-
//     swizzled code tile; double-buffered;
//   warps 6-9: after the dependency wait, x (RMS-normalised when epi.norm_w
//     is set, with k_mvi's fixed partition, so the same bits) into digits in
//     the swizzled B tile; then the epilogue: thread = row (its TMEM lane),
//     per step 4 x tcgen05.ld of the 3 digit columns, the scales from global
//     memory (two steps ahead), the row's running sum.
// Every wait spins (bounded): suspended waits wake late and measured slower.
// K chunks of one tile (ksplit > 1) form a thread-block cluster; their
// partial sums meet over distributed shared memory and are added in chunk
// order, so the result does not depend on scheduling.  The split is planned
// from the whole matrix's shape, so row slices of a matrix give the same bits
// as one call.  With one chunk the CTA loops over tiles (persistent; the
// vocabulary head).  Every wait is bounded and records PB_DEVERR_WAIT.

#include <cooperative_groups.h>

#include "pb_tc.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int MT_ROWS = 128;                            // weight rows per tile (MMA M)
constexpr int MT_N = 16;                                // MMA N: the 3 digit rows of B, padded with zeros
constexpr int MT_SB = 4;                                // Q4_0 blocks per K step (128 codes: one swizzle row)
constexpr int MT_STAGES = 4;                            // payload ring
constexpr int MT_ABUF = 2;                              // unpacked code tiles
constexpr int MT_ACC = 4;                               // TMEM accumulator buffers
constexpr int MT_ACC_COLS = MT_SB * MT_N;               // 64 columns per buffer
constexpr int MT_TMEM_COLS = MT_ACC * MT_ACC_COLS;      // 256 (a power of two >= 32)
constexpr int MT_THREADS = 320;
constexpr int MT_RW = MT_ROWS / 32;                     // warps of the unpack and of the epilogue role
constexpr int MT_PAY_BYTES = MT_ROWS * MT_SB * 16;      // 8 KB of payload per step
constexpr int MT_A_BYTES = MT_ROWS * MT_SB * 32;        // 16 KB of codes per step
constexpr int MT_B_BYTES = MT_N * MT_SB * 32;           // 2 KB of digits per step
constexpr int MT_MAX_CHUNK = 64;                        // blocks per K chunk (the digits stay in shared memory)
constexpr int MT_MAX_SPLIT = 8;                         // K chunks per tile: a portable cluster
// D s32, A u8, B s8, both K-major, N = 16, M = 128
constexpr uint32_t MT_IDESC =
    (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(MT_N >> 3) << 17) | ((uint32_t)(MT_ROWS >> 4) << 24);
static_assert(MT_THREADS == 64 + 2 * MT_ROWS, "producer, MMA, unpack (a thread per row) and epilogue warps");

__device__ __forceinline__ void mt_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(MT_IDESC), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// Columns c .. c+3 of four accumulator groups (16 columns apart) of this
// warp's 32 TMEM lanes, complete on return (the wait is in the same asm, so
// no use of the registers can be scheduled before it).
__device__ __forceinline__ void mt_ld_step(uint32_t taddr, uint32_t (&v)[MT_SB][4]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%16];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%4, %5, %6, %7}, [%17];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%8, %9, %10, %11}, [%18];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%12, %13, %14, %15}, [%19];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0][0]), "=r"(v[0][1]), "=r"(v[0][2]), "=r"(v[0][3]), "=r"(v[1][0]), "=r"(v[1][1]), "=r"(v[1][2]),
        "=r"(v[1][3]), "=r"(v[2][0]), "=r"(v[2][1]), "=r"(v[2][2]), "=r"(v[2][3]), "=r"(v[3][0]), "=r"(v[3][1]),
        "=r"(v[3][2]), "=r"(v[3][3])
      : "r"(taddr), "r"(taddr + MT_N), "r"(taddr + 2 * MT_N), "r"(taddr + 3 * MT_N)
      : "memory");
}

__device__ __forceinline__ void mt_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(pb_smem_addr(bar)) : "memory");
}

// One arrival for the whole warp: every lane's earlier shared-memory accesses
// are ordered before lane 0's (release) arrival by the warp barrier.
__device__ __forceinline__ void mt_arrive_warp(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mt_arrive(bar);
}

// A bounded spinning wait (a suspended thread wakes late, which the per-step
// hand-offs would pay for).
__device__ __forceinline__ bool mt_wait(uint64_t* bar, uint32_t parity, int* err) {
  return pb_mbar_wait(bar, parity, err);
}

// A bounded wait every lane of the warp takes; false on every lane if any gave up.
__device__ __forceinline__ bool mt_wait_warp(uint64_t* bar, uint32_t parity, int* err) {
  const bool ok = mt_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

}  // namespace

// Shared memory: [A codes: MT_ABUF x 16 KB][payload: MT_STAGES x 8 KB][B digits:
// cb / 4 x 2 KB][tinfo: cb x int4][part: 2 x 128 floats], from a 1024-aligned base.
static size_t mt_smem(int cb) {
  return 1024 + (size_t)MT_ABUF * MT_A_BYTES + (size_t)MT_STAGES * MT_PAY_BYTES + (size_t)(cb / MT_SB) * MT_B_BYTES +
         (size_t)cb * 16 + 2 * MT_ROWS * 4;
}

// grid (ksplit, tile groups); cluster (ksplit, 1, 1) when ksplit > 1 (then one
// tile per CTA).  Tiles are the matrix's 128-row tiles from t_first on; rows in [row_first,
// row_end) are stored.
__global__ void __launch_bounds__(MT_THREADS, 2)
k_mvt(const uint8_t* __restrict__ tq, const uint16_t* __restrict__ dsc, int N, int N_pad, int nb, int cb, int t_first,
      int row_first, int row_end, int ntiles, const float* __restrict__ x, float* __restrict__ y, pb_mv_epi epi,
      int* err) {
  extern __shared__ __align__(1024) unsigned char mt_raw[];
  __shared__ uint64_t full[MT_STAGES], empty[MT_STAGES], aready[MT_ABUF], accfull[MT_ACC],
      accfree[MT_ACC], bready, xred, mdone, tdone[2];
  __shared__ uint32_t tmem_base;
  __shared__ double red[4];
  unsigned char* base = mt_raw + ((1024 - (pb_smem_addr(mt_raw) & 1023)) & 1023);
  unsigned char* sA = base;
  unsigned char* sP = sA + MT_ABUF * MT_A_BYTES;
  unsigned char* sB = sP + MT_STAGES * MT_PAY_BYTES;
  int4* tinfo = reinterpret_cast<int4*>(sB + (size_t)(cb / MT_SB) * MT_B_BYTES);
  float* part = reinterpret_cast<float*>(tinfo + cb);  // [2][128]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ksplit = gridDim.x, chunk = blockIdx.x;
  const int kb0 = chunk * cb, kb1 = kb0 + cb < nb ? kb0 + cb : nb, nblk = kb1 - kb0, nsteps = nblk / MT_SB;
  const int my_tiles = (int)blockIdx.y < ntiles ? (ntiles - 1 - (int)blockIdx.y) / (int)gridDim.y + 1 : 0;
  const int total = my_tiles * nsteps;
  auto tile_of = [&](int i) { return t_first + (int)blockIdx.y + i * (int)gridDim.y; };  // 128-row tile of the matrix
  auto tile_row = [&](int i) { return tile_of(i) * MT_ROWS; };
  const int steps_all = nb / MT_SB;
  // the next kernel may start its own weight loads now; this grid reads x and
  // writes y only after the dependency wait (epilogue warps)
  pb_pdl_trigger();

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(pb_smem_addr(&tmem_base)),
                 "r"(MT_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int st = 0; st < MT_STAGES; ++st) {
      pb_mbar_init(&full[st], 1);
      pb_mbar_init(&empty[st], MT_RW);
    }
    for (int ab = 0; ab < MT_ABUF; ++ab) pb_mbar_init(&aready[ab], MT_RW);
    for (int c = 0; c < MT_ACC; ++c) {
      pb_mbar_init(&accfull[c], 1);
      pb_mbar_init(&accfree[c], MT_RW);
    }
    pb_mbar_init(&bready, MT_RW);
    pb_mbar_init(&xred, MT_RW);
    pb_mbar_init(&mdone, 1);
    pb_mbar_init(&tdone[0], MT_RW);
    pb_mbar_init(&tdone[1], MT_RW);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {  // producer
      const int cta = (int)(blockIdx.y * gridDim.x + blockIdx.x), ncta = (int)(gridDim.x * gridDim.y);
      for (int i = 0; i < PB_MAX_L2_NEXT; ++i) pb_l2_prefetch_share(epi.l2_next[i], epi.l2_next_bytes[i], cta, ncta);
      for (int g = 0; g < total; ++g) {
        const int st = g % MT_STAGES, i = g / nsteps, s = g - i * nsteps;
        if (g >= MT_STAGES && !mt_wait(&empty[st], ((g / MT_STAGES) - 1) & 1, err)) break;
        pb_mbar_arrive_tx(&full[st], MT_PAY_BYTES);
        pb_bulk_g2s(sP + st * MT_PAY_BYTES, tq + ((size_t)tile_of(i) * steps_all + kb0 / MT_SB + s) * MT_PAY_BYTES,
                    (uint32_t)MT_PAY_BYTES, &full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      bool ok = total == 0 || mt_wait(&bready, 0, err);
      int issued = 0;
      for (int g = 0; g < total && ok; ++g) {
        const int ab = g % MT_ABUF, c = g % MT_ACC, s = g % nsteps;
        if (!(ok = mt_wait(&aready[ab], (g / MT_ABUF) & 1, err))) break;
        if (g >= MT_ACC && !(ok = mt_wait(&accfree[c], ((g / MT_ACC) - 1) & 1, err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t da = pb_sw128_desc(pb_smem_addr(sA + ab * MT_A_BYTES));
        const uint64_t db = pb_sw128_desc(pb_smem_addr(sB + s * MT_B_BYTES));
#pragma unroll
        for (int j = 0; j < MT_SB; ++j)  // block j of the step: 32 bytes further along the swizzle row
          mt_mma(tmem + (uint32_t)(c * MT_ACC_COLS + j * MT_N), da + 2 * j, db + 2 * j);
        pb_umma_commit(&accfull[c]);  // the code tile and the accumulator buffer alike
        ++issued;
      }
      if (issued) {  // every MMA has completed before the TMEM is released
        pb_umma_commit(&mdone);
        pb_mbar_wait_sleep(&mdone, 0, err);
      }
    }
  } else if (warp < 6) {  // unpack
    const int u = tid - 64;
    static_assert(MT_ABUF <= MT_ACC, "a code tile is freed by the accumulator commit of its step");
    for (int g = 0; g < total; ++g) {
      const int st = g % MT_STAGES, ab = g % MT_ABUF;
      if (!mt_wait(&full[st], (g / MT_STAGES) & 1, err)) break;
      // the code tile is free once the MMAs of step g - MT_ABUF completed
      if (g >= MT_ABUF && !mt_wait(&accfull[(g - MT_ABUF) % MT_ACC], ((g - MT_ABUF) / MT_ACC) & 1, err)) break;
      // item i = u + 128 m: row i / 4, block i % 4 of the step, at byte 16 i of the stage
      const uint4* P = reinterpret_cast<const uint4*>(sP + st * MT_PAY_BYTES);
      uint4 q[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) q[m] = P[u + MT_ROWS * m];
      unsigned char* A = sA + ab * MT_A_BYTES;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i = u + MT_ROWS * m, r = i >> 2, blk = i & 3;
        const uint4 lo = make_uint4(q[m].x & 0x0F0F0F0Fu, q[m].y & 0x0F0F0F0Fu, q[m].z & 0x0F0F0F0Fu, q[m].w & 0x0F0F0F0Fu);
        const uint4 hi = make_uint4((q[m].x >> 4) & 0x0F0F0F0Fu, (q[m].y >> 4) & 0x0F0F0F0Fu,
                                    (q[m].z >> 4) & 0x0F0F0F0Fu, (q[m].w >> 4) & 0x0F0F0F0Fu);
        *reinterpret_cast<uint4*>(A + pb_sw128(r, 2 * blk)) = lo;      // elements 0..15 of the block
        *reinterpret_cast<uint4*>(A + pb_sw128(r, 2 * blk + 1)) = hi;  // elements 16..31
      }
      // generic-proxy writes of the tile -> the tensor cores' async proxy; and
      // the stage is released only now, after its loads were consumed and
      // fenced against the TMA (async-proxy) write that refills it: released
      // straight after the loads, a refill could overtake a pending load
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mt_arrive(&empty[st]);
        mt_arrive(&aready[ab]);
      }
    }
  } else {  // x staging, then the epilogue
    const int e = tid - 192, ew = e >> 5, q4 = warp & 3, r = q4 * 32 + lane;
    const int K = nb * 32;
    // the first tile's scales do not depend on the previous kernel: into L2 now
    if (my_tiles > 0) {
      const int row = tile_row(0) + r;
      if (row < N_pad) asm volatile("prefetch.global.L2 [%0];" ::"l"(dsc + (size_t)row * nb + kb0));
    }
    pb_pdl_wait();  // x (and the residual) come from the previous kernel
    bool ok = true;
    float inv = 1.0f;
    if (epi.norm_w) {  // k_mvi's partition: chunk c on thread c % 128, batches of 4 loads
      const float4* x4 = reinterpret_cast<const float4*>(x);
      double ss = 0.0;
      for (int c0 = e; c0 < K / 4; c0 += MT_ROWS * 4) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c0 + MT_ROWS * j < K / 4) v[j] = x4[c0 + MT_ROWS * j];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (c0 + MT_ROWS * j < K / 4) {
            ss = __fma_rn((double)v[j].x, (double)v[j].x, ss);
            ss = __fma_rn((double)v[j].y, (double)v[j].y, ss);
            ss = __fma_rn((double)v[j].z, (double)v[j].z, ss);
            ss = __fma_rn((double)v[j].w, (double)v[j].w, ss);
          }
        }
      }
      ss = pb_warp_sum_d(ss);
      if (lane == 0) red[ew] = ss;
      mt_arrive_warp(&xred);
      ok = mt_wait(&xred, 0, err);
      const double s4 = __dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3]));
      inv = (float)(1.0 / __dsqrt_rn(__dadd_rn(__ddiv_rn(s4, (double)K), epi.eps)));
    }
    // B rows 3..15 of every step are zero (bytes 384..2047 of its 2 KB); rows
    // 0..2 are written whole below
    for (int i = e; i < nsteps * 104; i += MT_ROWS) {
      const int s = i / 104, o = i - s * 104;
      *reinterpret_cast<uint4*>(sB + s * MT_B_BYTES + 384 + o * 16) = make_uint4(0, 0, 0, 0);
    }
    const float* w = epi.norm_w;
    for (int b0 = ew; b0 < nblk; b0 += 16) {
      float xv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // four blocks' loads in flight per lane
        const int b = b0 + 4 * u, kx = 32 * (kb0 + b) + lane;
        xv[u] = 0.0f;
        if (b < nblk) {
          xv[u] = x[kx];
          if (w) xv[u] = __fmul_rn(__fmul_rn(xv[u], inv), w[kx]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int b = b0 + 4 * u;
        if (b >= nblk) break;
        int dg[3];
        const float f = pb_x_digits(xv[u], dg[0], dg[1], dg[2]);
        // byte (digit n, K kk) of step b / 4: row n of the swizzled 16 x 128-byte tile
        const int kk = (b & 3) * 32 + lane;
        unsigned char* Bs = sB + (b >> 2) * MT_B_BYTES;
#pragma unroll
        for (int n = 0; n < 3; ++n) Bs[n * 128 + ((((kk >> 4) ^ n)) << 4) + (kk & 15)] = (unsigned char)(int8_t)dg[n];
        const int s0 = __reduce_add_sync(0xffffffffu, dg[0]), s1 = __reduce_add_sync(0xffffffffu, dg[1]),
                  s2 = __reduce_add_sync(0xffffffffu, dg[2]);
        if (lane == 0) tinfo[b] = make_int4(s0, s1, s2, __float_as_int(f));
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mt_arrive_warp(&bready);
    ok = ok && mt_wait(&bready, 0, err);  // every warp's tinfo is visible
    ok = __all_sync(0xffffffffu, ok);
    const uint32_t tq = tmem + ((uint32_t)(q4 * 32) << 16);
    int g = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int row = tile_row(i) + r;
      const bool rl = row < N_pad;
      const uint2* drow = reinterpret_cast<const uint2*>(dsc + (size_t)(rl ? row : 0) * nb + kb0);
      if (i + 1 < my_tiles && tile_row(i + 1) + r < N_pad)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(dsc + (size_t)(tile_row(i + 1) + r) * nb + kb0));
      auto ldsc = [&](int s) { return rl && s < nsteps ? __ldg(drow + s) : make_uint2(0u, 0u); };
      uint2 sc0 = ldsc(0), sc1 = ldsc(1);
      float acc = 0.0f;
      for (int s = 0; s < nsteps; ++s, ++g) {
        const uint2 sc = sc0;
        sc0 = sc1;
        sc1 = ldsc(s + 2);
        const int c = g % MT_ACC;
        if (!(ok = mt_wait_warp(&accfull[c], (g / MT_ACC) & 1, err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint32_t v[MT_SB][4];
        mt_ld_step(tq + (uint32_t)(c * MT_ACC_COLS), v);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mt_arrive_warp(&accfree[c]);
        const uint32_t dw[4] = {sc.x & 0xFFFFu, sc.x >> 16, sc.y & 0xFFFFu, sc.y >> 16};
#pragma unroll
        for (int j = 0; j < MT_SB; ++j) {
          const int4 ti = tinfo[MT_SB * s + j];
          const int e0 = (int)v[j][0] - 8 * ti.x, e1 = (int)v[j][1] - 8 * ti.y, e2 = (int)v[j][2] - 8 * ti.z;
          const float val = __fmaf_rn((float)e2, 1.0f / 64516.0f, __fmaf_rn((float)e1, 1.0f / 254.0f, (float)e0));
          const float scl = __fmul_rn(pb_f16_wasm(dw[j]), __int_as_float(ti.w));
          acc = __fmaf_rn(val, scl, acc);
        }
      }
      if (!ok) break;
      float* pt = part + (i & 1) * MT_ROWS;
      pt[r] = acc;
      if (ksplit == 1) {  // the tile's 16 8-row groups through the matvec epilogue, 4 per warp
        mt_arrive_warp(&tdone[i & 1]);
        if (!(ok = mt_wait_warp(&tdone[i & 1], (i >> 1) & 1, err))) break;
#pragma unroll
        for (int jt = 0; jt < 4; ++jt) {
          const int t8 = ew * 4 + jt;
          pb_mv_epilogue(pt[t8 * 8 + (lane >> 2)], (tile_row(i) >> 3) + t8, N, row_first, row_end, y, epi, err);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (ksplit > 1) {
    // the chunks' partial sums of the tile, added in chunk order: 8-row group
    // t8 on cluster rank t8 % ksplit, warp t8 / ksplit
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    if (my_tiles > 0) {
      for (int t8 = chunk + ksplit * warp; t8 < MT_ROWS / 8; t8 += ksplit * (MT_THREADS / 32)) {
        const int rr = t8 * 8 + (lane >> 2);
        float v = *cl.map_shared_rank(part + rr, 0);
        for (int c = 1; c < ksplit; ++c) v = __fadd_rn(v, *cl.map_shared_rank(part + rr, c));
        pb_mv_epilogue(v, (tile_row(0) >> 3) + t8, N, row_first, row_end, y, epi, err);
      }
    }
    cl.sync();  // no CTA leaves while its partials are read
  }
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(MT_TMEM_COLS) : "memory");
  }
}


// The K split of a matrix (from its whole shape): double the chunks while
// the CTAs still fit one wave of two per SM and each chunk keeps two steps;
// enough chunks for the digits to fit.
static void mt_plan(const pb_qmat* w, int sm_count, int* ksplit, int* cb) {
  const int tiles = pb_cdiv(w->N, MT_ROWS), cap = 2 * sm_count, nb = w->nb;
  int ks = 1;
  while (ks < MT_MAX_SPLIT && tiles * ks * 2 <= cap && nb / (ks * 2) >= 2 * MT_SB) ks *= 2;
  while (pb_cdiv(nb, ks) > MT_MAX_CHUNK) ks *= 2;
  int c = pb_cdiv(pb_cdiv(nb, ks), MT_SB) * MT_SB;
  *cb = c;
  *ksplit = pb_cdiv(nb, c);
}

// The tile-contiguous copy: item (tile T, step s, row r, block j) at byte
// ((T * nb / 4 + s) * 128 + r) * 64 + 16 j; rows past N_pad are zero.
__global__ void k_pack_mvt(const uint8_t* __restrict__ qs, int N_pad, int nb, int64_t items, uint8_t* __restrict__ tq) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= items) return;
  const int j = (int)(i & 3), r = (int)((i >> 2) & (MT_ROWS - 1));
  const int64_t ts = i >> 9;  // T * steps + s
  const int steps = nb / MT_SB, s = (int)(ts % steps), T = (int)(ts / steps);
  const int row = T * MT_ROWS + r, blk = s * MT_SB + j;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (row < N_pad) v = reinterpret_cast<const uint4*>(qs)[(size_t)row * nb + blk];
  reinterpret_cast<uint4*>(tq)[i] = v;
}

// Whether the matrix's shape suits k_mvt (Q4_0 row layout, whole K steps, at
// most MT_MAX_SPLIT chunks of MT_MAX_CHUNK blocks).
static bool mt_shape_ok(const pb_qmat* w) {
  return w && w->type == PB_TYPE_Q4_0 && w->layout == PB_LAYOUT_ROWS && w->nb % MT_SB == 0 &&
         w->nb <= MT_MAX_CHUNK * MT_MAX_SPLIT;
}

int pb_qmat_build_mvt(pb_ctx* ctx, pb_qmat* m) {
  if (!ctx->mvt || !mt_shape_ok(m)) return PB_OK;  // k_mvt off, or it does not take the matrix: no copy
  const int ntiles = pb_cdiv(m->N, MT_ROWS);
  const int64_t items = (int64_t)ntiles * MT_ROWS * m->nb;  // 16-byte pieces
  if (!m->tq && cudaMalloc(&m->tq, (size_t)items * 16) != cudaSuccess) {
    m->tq = nullptr;
    return pb_set_error(ctx, PB_ERR_OOM, "tcgen05 matvec copy");
  }
  k_pack_mvt<<<pb_cdiv(items, 256), 256, 0, ctx->stream>>>(m->qs, m->N_pad, m->nb, items, m->tq);
  PB_LAUNCHED(ctx, "k_pack_mvt");
  return PB_OK;
}

// Dynamic shared memory the kernel may take: all an SM offers a CTA but the
// static part (set by pb_setup_mvt_kernels).
static int mt_smem_limit = 0;

// Whether k_mvt takes the matrix: its shape, and a current tile-contiguous copy.
bool pb_mvt_ok(const pb_qmat* w) { return mt_shape_ok(w) && w->tq && w->mma_ok; }

int pb_launch_mvt(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows, const pb_mv_epi& epi) {
  if (!pb_mvt_ok(w))
    return pb_set_error(ctx, PB_ERR_ARG, "k_mvt: Q4_0 row layout with K %% 128 == 0, K <= 16384, and a current copy");
  int ks = 1, cb = 0;
  mt_plan(w, ctx->sm_count, &ks, &cb);
  const int t_first = row0 / MT_ROWS, ntiles = pb_cdiv(row0 + rows, MT_ROWS) - t_first;
  const size_t smem = mt_smem(cb);
  if (smem > (size_t)mt_smem_limit)
    return pb_set_error(ctx, PB_ERR_ARG, "k_mvt: %zu bytes of shared memory", smem);
  int per_sm = (int)((size_t)227 * 1024 / (smem + 1024));
  per_sm = per_sm < 2 ? (per_sm < 1 ? 1 : per_sm) : 2;
  const int groups = ks > 1 ? ntiles : (ntiles < per_sm * ctx->sm_count ? ntiles : per_sm * ctx->sm_count);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ks, groups);
  cfg.blockDim = dim3(MT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ks > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = ks;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (ctx->pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_mvt, (const uint8_t*)w->tq, (const uint16_t*)w->d, w->N, w->N_pad,
                                     w->nb, cb, t_first, row0, row0 + rows, ntiles, x, y, epi, ctx->d_err);
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, "k_mvt");
  return pb_check_launch(ctx, "k_mvt");
}

int pb_setup_mvt_kernels(void) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, k_mvt) != cudaSuccess) return PB_ERR_CUDA;
  mt_smem_limit = 227 * 1024 - (int)a.sharedSizeBytes;
  return cudaFuncSetAttribute(k_mvt, cudaFuncAttributeMaxDynamicSharedMemorySize, mt_smem_limit) == cudaSuccess
             ? PB_OK
             : PB_ERR_CUDA;
}
