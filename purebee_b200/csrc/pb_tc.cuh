// pb_tc.cuh - shared pieces of the tcgen05 / TMA kernels (pb_gemm.cu, pb_mvt.cu):
// the K-major 128-byte-swizzled shared-memory layout and its UMMA descriptor,
// tensor-map loads, MMA completion, TMEM loads, and the driver's tensor-map
// encoder.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "pb_internal.cuh"

// Byte offset of 16-byte chunk c of row r in a K-major, 128-byte-swizzled
// tile: 8-row groups of 1024 bytes, rows of 128 bytes, chunk index XOR
// (row mod 8).  The tile base is 1024-byte aligned.
__device__ __forceinline__ uint32_t pb_sw128(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024
// bytes apart (stride byte offset), sm100 descriptor version 1.  Adding n to
// the descriptor advances its start by 16 n bytes within the swizzle row.
__device__ __forceinline__ uint64_t pb_sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Arrive on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void pb_umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(pb_smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void pb_tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(pb_smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(pb_smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void pb_tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(pb_smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(pb_smem_addr(bar))
      : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes (one lane per thread),
// complete on return.
__device__ __forceinline__ void pb_tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The driver's cuTensorMapEncodeTiled (looked up once); null with the
// context's error set when the driver has none.
inline PFN_cuTensorMapEncodeTiled_v12000 pb_tensor_map_encoder(pb_ctx* ctx) {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) pb_set_error(ctx, PB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  return fn;
}
