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
  int matvec_mode = PB_MATVEC_FAST;  // resident Q4_0 matvecs (pb_set_matvec_mode)
  size_t l2_bytes = 0;
  cudaStream_t stream = nullptr;
  int timeout_ms = 10000;
  int* d_err = nullptr;         // device error word: 0 = ok
  int64_t launches = 0;
  bool pdl = true;              // launch matvecs with programmatic stream serialization
  int mvi_min_rows = 32768;     // fast mode: matrices of this many rows on take the int8 tensor-core matvec
  bool mvt = false;             // fast mode: the tcgen05 int8 matvec for the matrices it takes (pb_set_mvt)
  bool fuse_attn = false;       // fast mode: decode projection + attention in one kernel (pb_set_fuse_attn)
  std::string err;
  // scratch for one-shot host-buffer calls (grown on demand)
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  // f16 operand copies of the large-batch tensor-core GEMM (grown on demand)
  void* gemm_scratch = nullptr;
  size_t gemm_scratch_bytes = 0;
  // fixed per-device array of pb_attention_noalloc (looked up in pb_init)
  void* noalloc_attn = nullptr;
};

// Device layouts of a quantized matrix (payload and scales split apart, so
// every payload is 16-byte aligned; QB = 16 bytes for Q4, 32 for Q8):
//   PB_LAYOUT_ROWS   (matvec weights): qs [N_pad][nb][QB], d [N_pad][nb] u16
//     (Q4_1: a second array m).  Eight consecutive rows are one contiguous
//     tile, and a warp reading block b..b+31 of one row reads 512 B in a row.
//   PB_LAYOUT_TILED8 (tables read one row per lane: LM head, embedding):
//     qs [N_pad/8][nb][8][QB], d [N_pad/8][nb][8]; block b of 8 consecutive
//     rows is one 128 B (Q4) line.
// N_pad rounds N up to 32; the padding rows hold zeros.
#define PB_LAYOUT_ROWS 0
#define PB_LAYOUT_TILED8 1

struct pb_qmat {
  int type = 0;
  int layout = PB_LAYOUT_ROWS;
  int N = 0, K = 0, N_pad = 0, nb = 0;
  uint8_t* qs = nullptr;
  uint16_t* d = nullptr;
  uint16_t* m = nullptr;  // Q4_1 min
  // A second copy of a Q4_0 matrix for the int8 tensor-core matvec (k_mvi,
  // the fast mode): 16-row tiles, nibbles placed for the mma fragments, the
  // blocks padded to whole spans of 8 (see pb_mvi.cu).  mma_ok: it mirrors
  // the current contents (a writer of qs/d clears it; pb_qmat_build_mma sets it).
  uint8_t* mq = nullptr;
  uint16_t* md = nullptr;
  int nbp = 0;  // blocks per row in the copy (a multiple of 8)
  // The copy the tcgen05 matvec (k_mvt, pb_mvt.cu) streams: the payload in
  // 128-row tiles, each tile's K steps (4 blocks) of 128 rows x 64 B
  // contiguous, so one K step of a tile is one 8 KB run.  Built and
  // invalidated with mq (mma_ok).
  uint8_t* tq = nullptr;
  bool mma_ok = false;
};
int pb_qmat_build_mma(pb_ctx* ctx, pb_qmat* m);  // (re)build the tensor-core copies (mq / md, and tq)
int pb_qmat_build_mvt(pb_ctx* ctx, pb_qmat* m);  // (re)build tq (part of pb_qmat_build_mma)

// ---- host helpers ---------------------------------------------------------

int pb_set_error(pb_ctx* ctx, int code, const char* fmt, ...);
int pb_cuda_error(pb_ctx* ctx, cudaError_t e, const char* what);
int pb_wait(pb_ctx* ctx);  // bounded wait on the context stream
int pb_check_launch(pb_ctx* ctx, const char* what);
int pb_ensure_scratch(pb_ctx* ctx, size_t bytes);
int pb_ensure_gemm_scratch(pb_ctx* ctx, size_t bytes);

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

// Launch a kernel on the context stream, with programmatic dependent launch
// when pdl is set (and not disabled on the context).  A kernel launched this
// way must execute griddepcontrol.wait before it reads anything the previous
// kernel writes, and write nothing before it.
template <typename... KArgs, typename... Args>
static inline int pb_launch(pb_ctx* ctx, const char* what, bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block,
                            size_t smem, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && ctx->pdl) ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, what);
  return pb_check_launch(ctx, what);
}

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

// Index of (row, block) in the tiled layout.
__host__ __device__ __forceinline__ int64_t pb_qslot(int row, int b, int nb) {
  return ((int64_t)(row >> 3) * nb + b) * 8 + (row & 7);
}

// Index of (row, block) in either layout.
__host__ __device__ __forceinline__ int64_t pb_slot(int layout, int row, int b, int nb) {
  return layout == PB_LAYOUT_TILED8 ? pb_qslot(row, b, nb) : (int64_t)row * nb + b;
}

// Fire-and-forget bulk prefetch of [p, p + bytes) into L2 (p and bytes
// multiples of 16).
__device__ __forceinline__ void pb_l2_prefetch(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// CTA share i of n of a region, prefetched into L2 in pieces of at most 64 KB
// (one thread issues them).
__device__ __forceinline__ void pb_l2_prefetch_share(const void* base, size_t bytes, int i, int n) {
  if (!base || !bytes) return;
  const size_t per = ((bytes + n - 1) / n + 15) & ~(size_t)15;
  size_t lo = (size_t)i * per;
  if (lo >= bytes) return;
  size_t hi = lo + per < bytes ? lo + per : bytes;
  hi &= ~(size_t)15;
  for (size_t o = lo; o < hi; o += 65536) {
    const size_t n_ = hi - o < 65536 ? hi - o : 65536;
    pb_l2_prefetch((const char*)base + o, (uint32_t)n_);
  }
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's results.
__device__ __forceinline__ void pb_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pb_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Record the first device-side error; the host reads it with pb_device_error.
__device__ __forceinline__ unsigned long long pb_globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void pb_raise(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Device error codes (also reported as PB_ERR_DEVICE with this detail).
#define PB_DEVERR_BOUNDS 1
#define PB_DEVERR_WAIT 2
#define PB_DEVERR_TOKEN 3

// ---- mbarriers and bulk copies into shared memory -------------------------
__device__ __forceinline__ uint32_t pb_smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void pb_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(pb_smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void pb_mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(pb_smem_addr(bar)), "r"(bytes)
               : "memory");
}
// Wait for the phase of the given parity; gives up after ~2 s of device clock
// (PB_DEVERR_WAIT) and returns false.
__device__ __forceinline__ bool pb_mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = pb_smem_addr(bar);
  const long long t0 = clock64();
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
// As pb_mbar_wait, but each try_wait may suspend the thread (up to 20 us) until
// the phase completes instead of returning at once: for role threads that
// would otherwise spin through many polls.
__device__ __forceinline__ bool pb_mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = pb_smem_addr(bar);
  const long long t0 = clock64();
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(addr), "r"(parity), "r"(20000u)
        : "memory");
    if (ok) return true;
    if ((it & 15) == 15 && clock64() - t0 > 4000000000LL) {
      pb_raise(err, PB_DEVERR_WAIT);
      return false;
    }
  }
}
// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global memory into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void pb_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   pb_smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(pb_smem_addr(bar))
               : "memory");
}

// One 32-value block of x (lane k holds element k) as three signed byte
// digits for the int8 tensor-core matvecs (pb_mvi.cu, pb_mvt.cu):
//   x[k] ~= f * (i0 + i1 / 254 + i2 / 254^2),  f = 2^e / 127,
// e the binary exponent of the block's largest |x| (so 2^-e scales exactly),
// each digit in [-127, 127]; the representation error is about 1e-7 of the
// block's largest |x|.  Returns f, NaN (digits 0) when the block holds an
// inf or NaN.  Every lane of the warp calls it.
__device__ __forceinline__ float pb_x_digits(float xv, int& i0, int& i1, int& i2) {
  // the block maximum of |x| as bits (order-preserving for non-negative floats)
  const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(xv) & 0x7FFFFFFFu);
  const uint32_t E = mb >> 23;  // biased exponent of the maximum
  int e = 0;                    // m = g * 2^e, g in [0.5, 1): |x| * 2^-e < 1
  float v = 0.0f, f = 0.0f;     // v = x * 127 * 2^-e, f = 2^e / 127
  if (mb > 0x7F7FFFFFu) {       // inf or NaN in the block: its rows become NaN
    f = __int_as_float(0x7fc00000);
  } else if (E >= 1 && E <= 252) {
    e = (int)E - 126;
    // 127 * 2^-e is exact, so v is x * 2^-e * 127 rounded once; 2^e * f32(1/127) is f32(2^e / 127)
    v = __fmul_rn(xv, __fmul_rn(__uint_as_float((uint32_t)(127 - e) << 23), 127.0f));
    f = __fmul_rn(__uint_as_float((uint32_t)(127 + e) << 23), 1.0f / 127.0f);
  } else if (mb != 0) {  // a subnormal maximum, or one near the top of the range
    frexpf(__uint_as_float(mb), &e);
    v = __fmul_rn(ldexpf(xv, -e), 127.0f);
    f = __fdiv_rn(ldexpf(1.0f, e), 127.0f);
  }
  i0 = __float2int_rn(v);                                      // |v| <= 127
  const float r1 = __fmul_rn(__fsub_rn(v, (float)i0), 254.0f);  // v - i0 in [-0.5, 0.5], exact
  i1 = __float2int_rn(r1);
  i2 = __float2int_rn(__fmul_rn(__fsub_rn(r1, (float)i1), 254.0f));
  return f;
}

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

// Matvec epilogues (fused into the kernel that produces the rows).
#define PB_EPI_STORE 0     // y[row] = v
#define PB_EPI_RESIDUAL 1  // y[row] = residual[row] + v   (llama-streaming.js:579-580, 601)
#define PB_EPI_ROPE_KV 2   // rows [q | k | v]: RoPE q, k; k, v into the cache at pos (:531-541)
#define PB_EPI_SWIGLU4 3   // tiles [g_4i..g_4i+3 | u_4i..u_4i+3]: h_i = silu(g_i)*u_i (:590-595)
#define PB_EPI_ARGMAX 4    // logits y[row] = v and the greedy key atomicMax (:899-909)

#define PB_MAX_L2_NEXT 4
struct pb_mv_epi {
  int kind = PB_EPI_STORE;
  const float* norm_w = nullptr;  // when set, x is first RMS-normalised with these gains (engine.js:429-449)
  double eps = 1e-5;
  // regions later kernels read, prefetched into L2 by this one
  const void* l2_next[PB_MAX_L2_NEXT] = {};
  size_t l2_next_bytes[PB_MAX_L2_NEXT] = {};
  const float* residual = nullptr;
  const double2* rope_tab = nullptr;
  const int* pos_dev = nullptr;
  int start_pos = 0;
  int q_rows = 0, kv_rows = 0, head_dim = 0, max_len = 0;
  float* kc = nullptr;
  float* vc = nullptr;
  float* h_out = nullptr;
  unsigned long long* amax = nullptr;  // PB_EPI_ARGMAX
};

// The fused epilogue of an 8-row tile of a matvec: every lane of quad r
// (lanes 4r .. 4r + 3) holds row r's value v; the quad's lane 0 stores rows
// in [row_begin, row_end).
__device__ __forceinline__ void pb_mv_epilogue(float v, int tile, int N, int row_begin, int row_end,
                                               float* __restrict__ y, const pb_mv_epi& epi, int* err) {
  const int lane = threadIdx.x & 31, rr = lane >> 2, L = lane & 3;
  const int row = tile * 8 + rr;
  const bool live = L == 0 && row >= row_begin && row < row_end && row < N;
  if (epi.kind == PB_EPI_STORE) {
    if (live) y[row] = v;
  } else if (epi.kind == PB_EPI_RESIDUAL) {
    if (live) y[row] = __fadd_rn(epi.residual[row], v);
  } else if (epi.kind == PB_EPI_ROPE_KV) {
    // rows of a tile are all q, all k or all v (q_rows, kv_rows % 8 == 0)
    const float vp = __shfl_sync(0xffffffffu, v, lane ^ 4);  // partner row rr ^ 1
    const int pos = epi.pos_dev ? *epi.pos_dev : epi.start_pos;
    const bool in_range = pos >= 0 && pos < epi.max_len;
    if (live && !in_range && rr == 0) pb_raise(err, PB_DEVERR_BOUNDS);
    if (live && in_range) {
      const int kvd = epi.kv_rows;
      if (row < epi.q_rows + kvd) {  // q or k: rotate the pair (2i, 2i+1)
        const bool isq = row < epi.q_rows;
        const int rel = isq ? row : row - epi.q_rows;
        const int pr = (rel % epi.head_dim) >> 1;
        const double2 cs = epi.rope_tab[(size_t)pos * (epi.head_dim >> 1) + pr];
        const bool even = (rr & 1) == 0;
        const double x0 = even ? (double)v : (double)vp, x1 = even ? (double)vp : (double)v;
        const float o = even ? (float)__dsub_rn(__dmul_rn(x0, cs.x), __dmul_rn(x1, cs.y))
                             : (float)__dadd_rn(__dmul_rn(x0, cs.y), __dmul_rn(x1, cs.x));
        if (isq) y[row] = o;
        else epi.kc[(size_t)pos * kvd + rel] = o;
      } else {
        epi.vc[(size_t)pos * kvd + (row - epi.q_rows - kvd)] = v;
      }
    }
  } else if (epi.kind == PB_EPI_ARGMAX) {  // logits and the greedy key (llama-streaming.js:899-909)
    if (live) y[row] = v;
    unsigned long long key = live ? pb_argmax_key(v, row) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, key, o);
      key = t > key ? t : key;
    }
    if (lane == 0 && key) atomicMax(epi.amax, key);
  } else {  // PB_EPI_SWIGLU4: rows 0-3 gate, 4-7 up of indices 4*tile .. 4*tile+3
    const float u = __shfl_sync(0xffffffffu, v, (lane + 16) & 31);
    if (L == 0 && rr < 4 && row < N) {
      const double g = v;
      const double silu = __ddiv_rn(g, __dadd_rn(1.0, exp(-g)));
      epi.h_out[tile * 4 + rr] = (float)__dmul_rn(silu, (double)u);
    }
  }
}


// Per-sequence strides (floats) of batched attention launches: blockIdx.z is
// the sequence; its query rows, cache and output rows sit these far apart.
struct pb_seq_geo {
  int64_t q = 0, kv = 0, out = 0;
};

// Epilogues of the tensor-core GEMM (pb_gemm.cu).  The result r[m][n] is
// stored (STORE), added to C (ADD: the residual x += proj, llama-streaming.js
// :579-580), or, for a gate|up matrix in the interleave-4 row order, turned
// into h[m][f] = silu(gate) * up in f32 (SWIGLU) and written as f16 (h16, the
// next GEMM's operand) or f32 (h32), f = 4 * (n / 8) + n % 4.
#define PB_GEMM_STORE 0
#define PB_GEMM_ADD 1
#define PB_GEMM_SWIGLU 2
// The struct also carries the operand layout and the split-K plan:
//   x_chunk > 0: X (f32 or f16) is stored as K / x_chunk column chunks,
//     [K / x_chunk][M][x_chunk] (the all-gathered operand of a row-split
//     model, chunk r written by rank r); x_chunk divides K and is a multiple
//     of 64.  0: row-major X with row stride ldx.
//   split_n > 0: the split-K count is chosen as for a matrix of split_n rows,
//     so a row slice of a matrix sums its K partials in the same order as the
//     whole matrix (and gives the same bits).
// The row split's residual exchange folded into the GEMM that adds into this
// rank's chunk of x (decode steps over peer memory): besides storing the new
// value, the epilogue stores it, two values per 16-byte packet with the
// exchange's epoch twice ({v0, e, v1, e}, the low-latency exchange's format),
// into every peer's slots; the next RMSNorm reads the peers' chunks from its
// own slots (k_rmsnorm_xrecv).  world == 0: off.
struct pb_xsend {
  uint4* slots[8];              // every rank's slot array (PB_MAX_RANKS)
  size_t cap_units = 0;         // packets per (half, sender)
  const unsigned int* epoch = nullptr;  // exchange counter: this exchange is *epoch + 1
  int rank = 0, world = 0;
  int width = 0;                // chunk width: (token m, column c) is unit (m * width + c) / 2
};

// One packet of the fused exchange: columns (c, c + 1) of token m, c even.
__device__ __forceinline__ void pb_xsend_pair(const pb_xsend& xs, int m, int c, float v0, float v1) {
  const unsigned int e = *xs.epoch + 1u;
  const size_t half = e & 1u, u = ((size_t)m * xs.width + c) >> 1;
  for (int q = 0; q < xs.world; ++q) {
    if (q == xs.rank) continue;
    uint4* dst = xs.slots[q] + (half * xs.world + xs.rank) * xs.cap_units + u;
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(__float_as_uint(v0)), "r"(e),
                 "r"(__float_as_uint(v1)), "r"(e)
                 : "memory");
  }
}

struct pb_gemm_epi {
  int mode = PB_GEMM_STORE;
  __half* h16 = nullptr;
  float* h32 = nullptr;
  int x_chunk = 0;
  int split_n = 0;
  // 1: each operand rounded to f16 once; 3: both split into f16 hi + lo and
  // the three products hi*hi + hi*lo + lo*hi summed (f16 operands then come,
  // and h16 goes out, in the hi/lo layout below)
  int terms = 1;
  pb_xsend xs;  // PB_GEMM_ADD: the fused residual exchange (row split, decode steps)
  // The RMSNorm after the GEMM (norm_w set; C row-major with ldc == N, no
  // exchange): each finished row of C, normalised with weights norm_w as
  // k_rmsnorm_t does, into norm_out (f32) or norm_out16 (f16, hi/lo pairs
  // with norm_hl).  A split-K reduce does it in the same kernel; otherwise
  // pb_launch_q4_gemm launches k_rmsnorm_t after the GEMM.  Same bits either way.
  const float* norm_w = nullptr;
  double norm_eps = 1e-5;
  float* norm_out = nullptr;
  __half* norm_out16 = nullptr;
  int norm_hl = 0;
};

// The hi/lo f16 layout of the three-term GEMM operands: a value v is the
// pair hi = f16(v), lo = f16(v - hi) (v - hi is exact in f32, so hi + lo
// carries about 22 bits of v); along K each 64-wide group is stored as its
// 64 hi halves, then its 64 lo halves.  A row of K values takes 2K halves:
// the bytes of the f32 row, so a buffer sized for f32 holds it.
__device__ __forceinline__ size_t pb_hl_index(size_t row_base, int k) {
  return row_base + (size_t)(k >> 6) * 128 + (k & 63);
}
__device__ __forceinline__ void pb_store_hl(__half* p, size_t i, float v) {
  const __half hi = __float2half_rn(v);
  p[i] = hi;
  p[i + 64] = __float2half_rn(__fsub_rn(v, __half2float(hi)));
}
// pdl: launched as a programmatic dependent of the previous kernel (the
// kernel waits for it before reading x)
void pb_launch_rmsnorm(cudaStream_t st, const float* x, int rows, int dim, const float* w, double eps, float* out,
                       __half* out16, int xc, int hl = 0, bool pdl = false);
int pb_launch_q4_gemm(pb_ctx* ctx, const pb_qmat* w, const float* X, int ldx, int M, float* C, int ldc, float* ws,
                      size_t ws_bytes, const pb_gemm_epi* epi = nullptr, const __half* Xh = nullptr);
bool pb_gemm_uses_tma(const pb_qmat* w, int M);  // the f16-operand TMA path (takes Xh)
bool pb_gemm_uses_ws(const pb_qmat* w, int M);   // the decode-size path with f16 activations (Xh)

// pb_comm.cu: in-place all-gather on the communicator's context stream;
// chunk `rank` of base (chunk_bytes each) goes to every rank
int pb_comm_gather_inplace(pb_comm* c, void* base, size_t chunk_bytes);
pb_ctx* pb_comm_ctx(const pb_comm* c);
// Peer memory of the ranks (CUDA IPC): tables of every rank's copy of a buffer
#define PB_MAX_RANKS 8
static_assert(sizeof(pb_xsend::slots) / sizeof(uint4*) == PB_MAX_RANKS, "pb_xsend holds one slot array per rank");
struct pb_peer_bufs {
  char* p[PB_MAX_RANKS];
};
struct pb_peer_sync {
  unsigned long long* flags[PB_MAX_RANKS];  // rank q's arrival epochs, one slot per sender
};
int pb_comm_share(pb_comm* c, void* const* local, int n, void** table);  // table [n][world]
int pb_comm_share_agreed(pb_comm* c, void* const* local, int n, void** table, bool want, bool* agreed);
void pb_comm_unshare(pb_comm* c, void** table, int n);
bool pb_comm_p2p(const pb_comm* c);
int pb_comm_peer_gather(pb_comm* c, void* const* table, size_t chunk_bytes);
// Low-latency exchange slots: s[q] is rank q's slot array [2][world][cap_units]
// (16 bytes = 8 data bytes + two epoch flags each); epoch / done are this
// rank's counters for the exchanges over these slots.
struct pb_ll_slots {
  uint4* s[PB_MAX_RANKS];
};
int pb_comm_ll_gather(pb_comm* c, const pb_ll_slots& slots, size_t cap_units, char* buf, size_t chunk_bytes,
                      unsigned int* epoch, unsigned int* done);

// The receiving end of the fused residual exchange (pb_xsend): this rank's
// slot array and the exchange's counters.
struct pb_xrecv {
  const uint4* mine = nullptr;
  size_t cap_units = 0;
  unsigned int* epoch = nullptr;
  unsigned int* done = nullptr;
  int rank = 0, world = 0;
  unsigned long long limit_ns = 0;  // set by the launcher from the context timeout
  int* err = nullptr;
};
int pb_launch_rmsnorm_xrecv(pb_ctx* ctx, float* x, int rows, int dim, const float* w, double eps, float* out,
                            __half* out16, int xc, int hl, const pb_xrecv& xr);

int pb_launch_matvec(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows,
                     const pb_mv_epi* epi);
int pb_launch_head(pb_ctx* ctx, const pb_qmat* emb, const float* h, float* logits,
                   unsigned long long* argmax_key, int mode);
int pb_launch_head_fast(pb_ctx* ctx, const pb_qmat* t, const float* h, const float* norm_w, double eps, float* logits,
                        unsigned long long* amax);
int pb_launch_head_norm(pb_ctx* ctx, const pb_qmat* emb, const float* h, const float* norm_w, double eps,
                        float* logits, unsigned long long* argmax_key, int mode);
int pb_launch_argmax_finish(pb_ctx* ctx, const unsigned long long* key, int* idx);
int pb_qmat_alloc(pb_ctx* ctx, int type, int layout, int N, int K, pb_qmat** out);
int pb_qmat_pack_from_device(pb_ctx* ctx, pb_qmat* m, const void* gguf_dev);
int pb_setup_q4_kernels(void);
int pb_setup_mvi_kernels(void);
int pb_launch_mvi(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows, const pb_mv_epi& epi);
int pb_setup_mvt_kernels(void);
// The fast-mode kernel choice of a row-layout Q4_0 matrix: true when its
// matvecs run on k_mvf (not on k_mvi or k_mvt).
bool pb_fast_uses_mvf(const pb_ctx* ctx, const pb_qmat* w);
bool pb_mvt_ok(const pb_qmat* w);  // the tcgen05 int8 matvec takes the matrix
int pb_launch_mvt(pb_ctx* ctx, const pb_qmat* w, const float* x, float* y, int row0, int rows, const pb_mv_epi& epi);
int pb_setup_ops_kernels(void);
int pb_setup_gemm_kernels(void);
int pb_setup_sample_kernels(void);
// Top-K sampling (pb_sample.cu): candidate keys needed, and the two launches.
size_t pb_sample_cand_count(int V, int K);
int pb_launch_sample(pb_ctx* ctx, const float* logits, int V, int K, double temperature, uint64_t seed,
                     uint64_t counter, uint64_t* ctr_dev, uint64_t* cand, int* tok_dev, int* pos_dev, int* hist,
                     int hist_len, unsigned long long* key_reset);
int pb_launch_exit_prob(pb_ctx* ctx, const float* logits, int V, uint64_t* cand, double* prob_dev);
int pb_setup_noalloc(pb_ctx* ctx);  // with ctx->device current
