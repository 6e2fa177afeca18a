// pb_comm.cu - NCCL communicators for the row-split batch (one rank per
// process and device), the device-side form of thread-pool.js's workers.
//
// NCCL is opened when the first communicator is made (dlopen of
// libnccl.so.2): a process that already loaded NCCL (torch does) shares that
// copy, and loading this library never chooses the NCCL another library gets.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "pb_internal.cuh"

int pb_comm_share_agreed(pb_comm* c, void* const* local, int n, void** table, bool want, bool* agreed);

struct pb_comm {
  pb_ctx* ctx = nullptr;
  ncclComm_t nc = nullptr;
  int rank = 0, world = 1;
  // peer exchange state (pb_comm_peer_gather): flags[q] is rank q's array of
  // arrival epochs, one slot per sender; epoch counts this rank's exchanges;
  // done counts the exchange kernel's finished CTAs
  bool p2p = false;
  unsigned long long* flags = nullptr;
  pb_peer_sync sync{};
  unsigned long long* epoch = nullptr;
  unsigned int* done = nullptr;
};

namespace {

bool getenv_flag(const char* name) {
  const char* v = getenv(name);
  return v && v[0] == '1';
}

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  std::string why;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      api.why = e ? e : "libnccl.so.2 not found";
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!api.get_unique_id || !api.comm_init_rank || !api.comm_destroy || !api.all_gather || !api.error_string) {
      api = NcclApi();
      api.why = "libnccl.so.2 lacks a required symbol";
    }
  });
  return api;
}

const char* nccl_err(ncclResult_t r) {
  return nccl().error_string ? nccl().error_string(r) : "unknown NCCL error";
}

}  // namespace

// ---------------------------------------------------------------------------
// peer exchange: the in-place all-gather as one kernel over NVLink peer
// memory.  Every rank's buffers are opened in every other rank's address space
// (CUDA IPC); an exchange stores this rank's chunk into each peer's copy of
// the buffer (plain 16-byte stores), and the last CTA to finish raises this
// rank's slot in every peer's flag array to the exchange's epoch, then waits
// (bounded) until every peer has raised its slot in ours.  All ranks run the
// same exchanges in the same order, so the e-th exchange has epoch e on every
// rank, and a rank is at most one exchange ahead of another: between two
// exchanges each rank reads only buffers that the other ranks do not write
// in the next exchange.
// ---------------------------------------------------------------------------

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// chunk_bytes is a multiple of 8 (16 when vec16).
__global__ void __launch_bounds__(256)
k_peer_gather(pb_peer_bufs bufs, size_t chunk_bytes, int rank, int world, pb_peer_sync sync,
              unsigned long long* __restrict__ epoch, unsigned int* __restrict__ done, unsigned long long limit_ns,
              int vec16, int* err) {
  pb_pdl_trigger();
  pb_pdl_wait();  // this rank's chunk (and the epoch) come from the kernels before
  const size_t off = (size_t)rank * chunk_bytes;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec16) {
    const uint4* src = reinterpret_cast<const uint4*>(bufs.p[rank] + off);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunk_bytes / 16; i += stride) {
      const uint4 v = src[i];
      for (int q = 0; q < world; ++q)
        if (q != rank) reinterpret_cast<uint4*>(bufs.p[q] + off)[i] = v;
    }
  } else {
    const uint2* src = reinterpret_cast<const uint2*>(bufs.p[rank] + off);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunk_bytes / 8; i += stride) {
      const uint2 v = src[i];
      for (int q = 0; q < world; ++q)
        if (q != rank) reinterpret_cast<uint2*>(bufs.p[q] + off)[i] = v;
    }
  }
  __syncthreads();  // the CTA's peer stores, ordered before thread 0's system fence
  if (threadIdx.x != 0) return;
  __threadfence_system();
  if (atomicAdd(done, 1u) != gridDim.x - 1) return;
  // the last CTA: every CTA's stores are performed; publish, then wait for the peers
  *done = 0u;
  __threadfence_system();
  const unsigned long long e = *epoch + 1;
  for (int q = 0; q < world; ++q)
    if (q != rank) st_release_sys(sync.flags[q] + rank, e);
  const unsigned long long t0 = globaltimer_ns();
  bool ok = true;
  for (int q = 0; q < world && ok; ++q) {
    if (q == rank) continue;
    for (uint32_t it = 0; ld_acquire_sys(sync.flags[rank] + q) < e; ++it) {
      if ((it & 63) == 63 && globaltimer_ns() - t0 > limit_ns) {
        pb_raise(err, PB_DEVERR_WAIT);
        ok = false;
        break;
      }
    }
  }
  *epoch = e;
  __threadfence_system();
}

static int launch_peer_gather(pb_ctx* ctx, const pb_peer_bufs& bufs, size_t chunk_bytes, int rank, int world,
                              const pb_peer_sync& sync, unsigned long long* epoch, unsigned int* done) {
  if (chunk_bytes % 8) return pb_set_error(ctx, PB_ERR_ARG, "peer exchange chunks are multiples of 8 bytes");
  bool vec16 = chunk_bytes % 16 == 0;
  for (int q = 0; q < world; ++q) vec16 = vec16 && ((uintptr_t)bufs.p[q] % 16 == 0);
  const size_t units = chunk_bytes / (vec16 ? 16 : 8);
  int grid = (int)((units + 256 * 4 - 1) / (256 * 4));
  grid = grid < 1 ? 1 : grid > 2 * ctx->sm_count ? 2 * ctx->sm_count : grid;
  const unsigned long long limit = (unsigned long long)ctx->timeout_ms * 1000000ull;
  return pb_launch(ctx, "k_peer_gather", true, k_peer_gather, dim3(grid), dim3(256), 0, bufs, chunk_bytes, rank, world,
                   sync, epoch, done, limit, vec16 ? 1 : 0, ctx->d_err);
}

// ---------------------------------------------------------------------------
// low-latency exchange for small chunks (the decode step's): no fences.  Each
// 16-byte peer store carries two data words and the exchange's epoch twice
// ({d0, e, d1, e}; an aligned 8-byte half lands whole), into the receiver's
// slot array for this sender; the receiver polls its slots until both flags
// read e and writes the data into its buffer.  Slots alternate between two
// halves by epoch parity: a rank writes half (e & 1) only after finishing
// exchange e - 1, which needs every peer's e - 1 data, which each peer sends
// only after finishing e - 2, the last reader of that half.  All CTAs are
// resident (grid <= SM count), each sends before it polls, and every poll is
// bounded, so the kernel always ends.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256)
k_ll_gather(char* __restrict__ buf, size_t chunk_bytes, int rank, int world, pb_ll_slots slots, size_t cap_units,
            unsigned int* __restrict__ epoch, unsigned int* __restrict__ done, unsigned long long limit_ns, int* err) {
  pb_pdl_trigger();
  pb_pdl_wait();  // this rank's chunk (and the epoch) come from the kernels before
  const unsigned int e = *epoch + 1u;
  const size_t half = e & 1u, n = chunk_bytes / 8;
  const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  const uint2* mine = reinterpret_cast<const uint2*>(buf + (size_t)rank * chunk_bytes);
  for (size_t i = t; i < n; i += stride) {
    const uint2 d = mine[i];
    for (int q = 0; q < world; ++q) {
      if (q == rank) continue;
      uint4* dst = slots.s[q] + (half * world + rank) * cap_units + i;
      asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(d.x), "r"(e), "r"(d.y), "r"(e)
                   : "memory");
    }
  }
  const unsigned long long t0 = globaltimer_ns();
  bool ok = true;
  for (int q = 0; q < world && ok; ++q) {
    if (q == rank) continue;
    const uint4* src = slots.s[rank] + (half * world + q) * cap_units;
    uint2* out = reinterpret_cast<uint2*>(buf + (size_t)q * chunk_bytes);
    for (size_t i = t; i < n && ok; i += stride) {
      uint4 v;
      for (uint32_t it = 0;; ++it) {
        asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(src + i)
                     : "memory");
        if (v.y == e && v.w == e) break;
        if ((it & 63) == 63 && globaltimer_ns() - t0 > limit_ns) {
          pb_raise(err, PB_DEVERR_WAIT);
          ok = false;
          break;
        }
      }
      if (ok) out[i] = make_uint2(v.x, v.z);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(done, 1u) == gridDim.x - 1) {
    *done = 0u;
    *epoch = e;
  }
}

int pb_comm_ll_gather(pb_comm* c, const pb_ll_slots& slots, size_t cap_units, char* buf, size_t chunk_bytes,
                      unsigned int* epoch, unsigned int* done) {
  pb_ctx* ctx = c->ctx;
  if (chunk_bytes % 8 || chunk_bytes / 8 > cap_units)
    return pb_set_error(ctx, PB_ERR_ARG, "low-latency exchange of %zu bytes exceeds its slots", chunk_bytes);
  const size_t n = chunk_bytes / 8;
  int grid = (int)((n + 255) / 256);
  grid = grid < 1 ? 1 : grid > ctx->sm_count ? ctx->sm_count : grid;  // all CTAs resident
  const unsigned long long limit = (unsigned long long)ctx->timeout_ms * 1000000ull;
  return pb_launch(ctx, "k_ll_gather", true, k_ll_gather, dim3(grid), dim3(256), 0, buf, chunk_bytes, c->rank, c->world,
                   slots, cap_units, epoch, done, limit, ctx->d_err);
}

extern "C" int pb_comm_id(void* id_out) {
  if (!id_out) return PB_ERR_ARG;
  static_assert(sizeof(ncclUniqueId) == PB_COMM_ID_BYTES, "NCCL unique id size");
  if (!nccl().get_unique_id) return PB_ERR_CUDA;
  ncclUniqueId id;
  if (nccl().get_unique_id(&id) != ncclSuccess) return PB_ERR_CUDA;
  memcpy(id_out, &id, sizeof(id));
  return PB_OK;
}

extern "C" int pb_comm_init(pb_ctx* ctx, int world, int rank, const void* id, pb_comm** out) {
  if (!ctx || !id || !out || world < 1 || rank < 0 || rank >= world) return PB_ERR_ARG;
  *out = nullptr;
  const NcclApi& api = nccl();
  if (!api.comm_init_rank) return pb_set_error(ctx, PB_ERR_CUDA, "NCCL unavailable: %s", api.why.c_str());
  PB_TRY_CUDA(ctx, cudaSetDevice(ctx->device));
  pb_comm* c = new pb_comm();
  c->ctx = ctx;
  c->rank = rank;
  c->world = world;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  const ncclResult_t r = api.comm_init_rank(&c->nc, world, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return pb_set_error(ctx, PB_ERR_CUDA, "ncclCommInitRank: %s", nccl_err(r));
  }
  // peer exchange: open every rank's flag array; unless every rank can, the
  // exchanges stay NCCL all-gathers
  if (world > 1 && world <= PB_MAX_RANKS) {
    cudaError_t e = cudaMalloc(&c->flags, PB_MAX_RANKS * 8);
    if (e == cudaSuccess) e = cudaMalloc(&c->epoch, 8);
    if (e == cudaSuccess) e = cudaMalloc(&c->done, 4);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->flags, 0, PB_MAX_RANKS * 8, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->epoch, 0, 8, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->done, 0, 4, ctx->stream);
    if (e != cudaSuccess) {
      pb_comm_free(c);
      return pb_cuda_error(ctx, e, "peer exchange state");
    }
    void* table[PB_MAX_RANKS] = {};
    void* local = c->flags;
    int rc = pb_comm_share_agreed(c, &local, 1, table, !getenv_flag("PB_NO_P2P"), &c->p2p);
    if (rc != PB_OK) {
      pb_comm_free(c);
      return rc;
    }
    if (c->p2p)
      for (int q = 0; q < world; ++q) c->sync.flags[q] = static_cast<unsigned long long*>(table[q]);
  }
  *out = c;
  return PB_OK;
}

// Release every batch (its decode graph holds NCCL work and peer mappings) before this.
extern "C" int pb_comm_free(pb_comm* c) {
  if (!c) return PB_OK;
  if (c->ctx) pb_wait(c->ctx);
  if (c->p2p) {
    void* table[PB_MAX_RANKS];
    for (int q = 0; q < PB_MAX_RANKS; ++q) table[q] = c->sync.flags[q];
    pb_comm_unshare(c, table, 1);
  }
  cudaFree(c->flags);
  cudaFree(c->epoch);
  cudaFree(c->done);
  if (c->nc) nccl().comm_destroy(c->nc);
  delete c;
  return PB_OK;
}

// Open every rank's copy of n buffers (local[i] are this rank's, each a whole
// cudaMalloc allocation): table[i * world + q] is rank q's buffer i in this
// process (this rank's own pointer at q == rank).  Collective: the IPC
// handles travel by an NCCL all-gather, which every rank joins even when its
// own handles could not be made.
int pb_comm_share(pb_comm* c, void* const* local, int n, void** table) {
  pb_ctx* ctx = c->ctx;
  const int world = c->world, rank = c->rank;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  std::vector<cudaIpcMemHandle_t> all((size_t)world * n);
  memset(all.data(), 0, all.size() * hb);
  int rc = PB_OK;
  for (int i = 0; i < n && rc == PB_OK; ++i) {
    const cudaError_t e = cudaIpcGetMemHandle(&all[(size_t)rank * n + i], local[i]);
    if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "cudaIpcGetMemHandle");
  }
  char* stage = nullptr;
  PB_TRY_CUDA(ctx, cudaMalloc(&stage, (size_t)world * n * hb));
  cudaError_t e = cudaMemcpyAsync(stage + (size_t)rank * n * hb, &all[(size_t)rank * n], n * hb,
                                  cudaMemcpyHostToDevice, ctx->stream);
  int grc = e != cudaSuccess ? pb_cuda_error(ctx, e, "stage IPC handles") : PB_OK;
  if (grc == PB_OK) grc = pb_comm_allgather(c, stage + (size_t)rank * n * hb, stage, n * hb);
  if (grc == PB_OK) {
    e = cudaMemcpyAsync(all.data(), stage, (size_t)world * n * hb, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) grc = pb_cuda_error(ctx, e, "read IPC handles");
  }
  if (grc == PB_OK) grc = pb_wait(ctx);
  cudaFree(stage);
  for (size_t i = 0; i < (size_t)n * world; ++i) table[i] = nullptr;
  if (rc != PB_OK) return rc;
  if (grc != PB_OK) return grc;
  for (int i = 0; i < n; ++i)
    for (int q = 0; q < world; ++q) {
      void*& slot = table[(size_t)i * world + q];
      if (q == rank) {
        slot = local[i];
        continue;
      }
      e = cudaIpcOpenMemHandle(&slot, all[(size_t)q * n + i], cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        slot = nullptr;
        return pb_cuda_error(ctx, e, "cudaIpcOpenMemHandle");
      }
    }
  return PB_OK;
}

// pb_comm_share, then every rank learns whether every rank opened every
// buffer (and wants peer exchange: `want`); *agreed is the same on all ranks.
// On disagreement the mappings are closed again.  An error return means the
// agreement itself failed (the communicator is unusable).
int pb_comm_share_agreed(pb_comm* c, void* const* local, int n, void** table, bool want, bool* agreed) {
  pb_ctx* ctx = c->ctx;
  *agreed = false;
  const int src = pb_comm_share(c, local, n, table);
  if (src != PB_OK) cudaGetLastError();  // a local failure is voted, not returned
  int* votes = nullptr;
  PB_TRY_CUDA(ctx, cudaMalloc(&votes, (size_t)c->world * sizeof(int)));
  std::vector<int> h(c->world, 0);
  h[c->rank] = (src == PB_OK && want) ? 1 : 0;
  int rc = PB_OK;
  cudaError_t e = cudaMemcpyAsync(votes + c->rank, &h[c->rank], sizeof(int), cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "stage vote");
  if (rc == PB_OK) rc = pb_comm_allgather(c, votes + c->rank, votes, sizeof(int));
  if (rc == PB_OK) {
    e = cudaMemcpyAsync(h.data(), votes, (size_t)c->world * sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "read votes");
  }
  if (rc == PB_OK) rc = pb_wait(ctx);
  cudaFree(votes);
  if (rc != PB_OK) return rc;
  bool all = true;
  for (int v : h) all = all && v == 1;
  if (!all) pb_comm_unshare(c, table, n);
  *agreed = all;
  return PB_OK;
}

// Close the peers' mappings that pb_comm_share opened.
void pb_comm_unshare(pb_comm* c, void** table, int n) {
  for (int i = 0; i < n; ++i)
    for (int q = 0; q < c->world; ++q) {
      void*& slot = table[(size_t)i * c->world + q];
      if (q != c->rank && slot) cudaIpcCloseMemHandle(slot);
      slot = nullptr;
    }
}

bool pb_comm_p2p(const pb_comm* c) { return c && c->p2p; }
extern "C" int pb_comm_peer_access(const pb_comm* c) { return pb_comm_p2p(c) ? 1 : 0; }

// In-place all-gather of a shared buffer (its pb_comm_share table) over peer
// memory.
int pb_comm_peer_gather(pb_comm* c, void* const* table, size_t chunk_bytes) {
  pb_peer_bufs bufs{};
  for (int q = 0; q < c->world; ++q) bufs.p[q] = static_cast<char*>(table[q]);
  return launch_peer_gather(c->ctx, bufs, chunk_bytes, c->rank, c->world, c->sync, c->epoch, c->done);
}

// A buffer registered for in-place all-gathers over peer memory.
struct pb_peerbuf {
  void* table[PB_MAX_RANKS] = {};
  bool p2p = false;
};

extern "C" int pb_comm_register(pb_comm* c, void* buf_dev, pb_peerbuf** out) {
  if (!c || !buf_dev || !out) return PB_ERR_ARG;
  *out = nullptr;
  pb_peerbuf* pb = new pb_peerbuf();
  pb->table[c->rank] = buf_dev;
  if (c->p2p) {
    const int rc = pb_comm_share_agreed(c, &buf_dev, 1, pb->table, true, &pb->p2p);
    if (rc != PB_OK) {
      delete pb;
      return rc;
    }
    if (!pb->p2p) pb->table[c->rank] = buf_dev;
  }
  *out = pb;
  return PB_OK;
}

extern "C" int pb_comm_deregister(pb_comm* c, pb_peerbuf* pb) {
  if (!c || !pb) return PB_ERR_ARG;
  if (pb->p2p) {
    pb_wait(c->ctx);
    pb_comm_unshare(c, pb->table, 1);
  }
  delete pb;
  return PB_OK;
}

extern "C" int pb_comm_allgather_inplace(pb_comm* c, pb_peerbuf* pb, size_t chunk_bytes) {
  if (!c || !pb) return PB_ERR_ARG;
  if (pb->p2p) return pb_comm_peer_gather(c, pb->table, chunk_bytes);
  return pb_comm_gather_inplace(c, pb->table[c->rank], chunk_bytes);
}

// The exchange kernels' bounded waits on one device: two-rank exchanges
// (the bulk kernel, then the low-latency one) whose "peer" is memory on this
// device that never signals.  The copies go to that memory; each wait must
// give up after timeout_ms and raise PB_DEVERR_WAIT, leaving the context
// usable.  *raised is PB_DEVERR_WAIT when both did (the error word is then
// cleared), else the first other code seen (0: a wait did not give up).
extern "C" int pb_comm_selftest_wait(pb_ctx* ctx, int timeout_ms, int* raised) {
  if (!ctx || !raised || timeout_ms <= 0) return PB_ERR_ARG;
  *raised = 0;
  const size_t chunk = 4096, cap = chunk / 8;
  // [2][chunk] buffer of rank 0, [2][chunk] of the fake peer, two flag arrays,
  // epoch + done words, then two slot arrays [2][2][cap] and their counters
  const size_t slot_bytes = 2 * 2 * cap * 16;
  const size_t total = 4 * chunk + 2 * PB_MAX_RANKS * 8 + 32 + 2 * slot_bytes + 16;
  char* mem = nullptr;
  PB_TRY_CUDA(ctx, cudaMalloc(&mem, total));
  char* buf0 = mem;
  char* buf1 = mem + 2 * chunk;
  auto* fl0 = reinterpret_cast<unsigned long long*>(mem + 4 * chunk);
  auto* fl1 = fl0 + PB_MAX_RANKS;
  auto* ep = fl1 + PB_MAX_RANKS;
  auto* dn = reinterpret_cast<unsigned int*>(ep + 2);
  uint4* sl0 = reinterpret_cast<uint4*>(mem + 4 * chunk + 2 * PB_MAX_RANKS * 8 + 32);
  uint4* sl1 = sl0 + 2 * 2 * cap;
  auto* llc = reinterpret_cast<unsigned int*>(sl1 + 2 * 2 * cap);
  int rc = PB_OK;
  cudaError_t e = cudaMemsetAsync(mem, 0, total, ctx->stream);
  if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "selftest memset");
  const int saved = ctx->timeout_ms;
  pb_comm fake;
  fake.ctx = ctx;
  fake.rank = 0;
  fake.world = 2;
  for (int kernel = 0; kernel < 2 && rc == PB_OK; ++kernel) {
    ctx->timeout_ms = timeout_ms;
    if (kernel == 0) {
      pb_peer_bufs bufs{};
      bufs.p[0] = buf0;
      bufs.p[1] = buf1;
      pb_peer_sync sync{};
      sync.flags[0] = fl0;
      sync.flags[1] = fl1;
      rc = launch_peer_gather(ctx, bufs, chunk, 0, 2, sync, ep, dn);
    } else {
      pb_ll_slots slots{};
      slots.s[0] = sl0;
      slots.s[1] = sl1;
      rc = pb_comm_ll_gather(&fake, slots, cap, buf0, chunk, llc, llc + 1);
    }
    ctx->timeout_ms = saved + timeout_ms;  // the host wait outlasts the kernel's
    if (rc == PB_OK) {
      const int wrc = pb_wait(ctx);
      int code = 0;
      e = cudaMemcpy(&code, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) rc = pb_cuda_error(ctx, e, "read device error word");
      else if (code != PB_DEVERR_WAIT) {
        *raised = code;
        rc = wrc;
      } else {
        cudaMemset(ctx->d_err, 0, sizeof(int));
        if (kernel == 1) *raised = PB_DEVERR_WAIT;
      }
    }
  }
  fake.ctx = nullptr;
  ctx->timeout_ms = saved;
  cudaFree(mem);
  return rc;
}

extern "C" int pb_comm_rank(const pb_comm* c) { return c ? c->rank : -1; }
extern "C" int pb_comm_world(const pb_comm* c) { return c ? c->world : 0; }
pb_ctx* pb_comm_ctx(const pb_comm* c) { return c ? c->ctx : nullptr; }

extern "C" int pb_comm_allgather(pb_comm* c, const void* send_dev, void* recv_dev, size_t bytes) {
  if (!c || !send_dev || !recv_dev) return PB_ERR_ARG;
  const ncclResult_t r = nccl().all_gather(send_dev, recv_dev, bytes, ncclUint8, c->nc, c->ctx->stream);
  if (r != ncclSuccess) return pb_set_error(c->ctx, PB_ERR_CUDA, "ncclAllGather: %s", nccl_err(r));
  return PB_OK;
}

int pb_comm_gather_inplace(pb_comm* c, void* base, size_t chunk_bytes) {
  char* p = static_cast<char*>(base);
  return pb_comm_allgather(c, p + (size_t)c->rank * chunk_bytes, p, chunk_bytes);
}
