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

#include "pb_internal.cuh"

struct pb_comm {
  pb_ctx* ctx = nullptr;
  ncclComm_t nc = nullptr;
  int rank = 0, world = 1;
};

namespace {

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
  *out = c;
  return PB_OK;
}

// Release every batch (its decode graph holds NCCL work) before this.
extern "C" int pb_comm_free(pb_comm* c) {
  if (!c) return PB_OK;
  if (c->ctx) pb_wait(c->ctx);
  if (c->nc) nccl().comm_destroy(c->nc);
  delete c;
  return PB_OK;
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
