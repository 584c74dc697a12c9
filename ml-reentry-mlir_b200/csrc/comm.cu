// Collective entry points of the C ABI: one NCCL communicator per context and
// the all-gather a destination-row partition needs (every rank contributes its
// rows of a table and receives everyone's).
//
// NCCL is loaded when first used, not linked: a process that already holds it
// (torch.distributed loads its own copy) reuses that copy, so one process never
// carries two NCCL instances; otherwise libnccl.so.2 is loaded from the library
// search path. The types come from nccl.h; only five functions are called.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool loaded = false;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;

template <typename F>
bool bind(void* lib, const char* name, F& fn) {
  fn = reinterpret_cast<F>(dlsym(lib, name));
  return fn != nullptr;
}

// The NCCL functions, or nullptr with the reason recorded in ctx.
const NcclApi* nccl(gnnc_ctx_t* ctx) {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (g_nccl.loaded) return &g_nccl;
  void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) {
    gnnc::set_error(ctx, GNNC_ERR_NCCL, "libnccl.so.2 not found: %s", dlerror());
    return nullptr;
  }
  NcclApi api;
  if (!bind(lib, "ncclGetUniqueId", api.get_unique_id) ||
      !bind(lib, "ncclCommInitRank", api.comm_init_rank) ||
      !bind(lib, "ncclAllGather", api.all_gather) ||
      !bind(lib, "ncclCommDestroy", api.comm_destroy) ||
      !bind(lib, "ncclGetErrorString", api.error_string)) {
    gnnc::set_error(ctx, GNNC_ERR_NCCL, "libnccl.so.2 lacks a required function");
    return nullptr;
  }
  api.loaded = true;
  g_nccl = api;
  return &g_nccl;
}

int nccl_status(gnnc_ctx_t* ctx, const NcclApi* api, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return GNNC_OK;
  return gnnc::set_error(ctx, GNNC_ERR_NCCL, "%s: %s", what, api->error_string(r));
}

}  // namespace

namespace gnnc {

void comm_release(gnnc_ctx_t* ctx) {
  if (!ctx->comm) return;
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (g_nccl.loaded) g_nccl.comm_destroy(static_cast<ncclComm_t>(ctx->comm));
  ctx->comm = nullptr;
}

}  // namespace gnnc

extern "C" {

int gnnc_comm_unique_id(gnnc_ctx_t* ctx, void* id) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, id != nullptr, "gnnc_comm_unique_id: null id");
  static_assert(sizeof(ncclUniqueId) == GNNC_COMM_ID_BYTES, "NCCL unique id size");
  const NcclApi* api = nccl(ctx);
  if (!api) return GNNC_ERR_NCCL;
  ncclUniqueId uid;
  const int st = nccl_status(ctx, api, api->get_unique_id(&uid), "ncclGetUniqueId");
  if (st == GNNC_OK) std::memcpy(id, &uid, sizeof(uid));
  return st;
}

int gnnc_comm_init(gnnc_ctx_t* ctx, const void* id, int rank, int nranks) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, id != nullptr, "gnnc_comm_init: null id");
  GNNC_CHECK_ARG(ctx, nranks >= 1 && rank >= 0 && rank < nranks, "gnnc_comm_init: bad rank %d of %d",
                 rank, nranks);
  GNNC_CHECK_ARG(ctx, ctx->comm == nullptr, "gnnc_comm_init: the context already has a communicator");
  const NcclApi* api = nccl(ctx);
  if (!api) return GNNC_ERR_NCCL;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  const int st = nccl_status(ctx, api, api->comm_init_rank(&comm, nranks, uid, rank), "ncclCommInitRank");
  if (st == GNNC_OK) {
    ctx->comm = comm;
    ctx->comm_rank = rank;
    ctx->comm_size = nranks;
  }
  return st;
}

int gnnc_allgather(gnnc_ctx_t* ctx, const void* sendbuf, void* recvbuf, size_t count, int dtype) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, ctx->comm != nullptr, "gnnc_allgather: no communicator (gnnc_comm_init)");
  GNNC_CHECK_ARG(ctx, dtype == GNNC_F32 || dtype == GNNC_BF16, "gnnc_allgather: bad dtype %d", dtype);
  GNNC_CHECK_ARG(ctx, count == 0 || (sendbuf && recvbuf), "gnnc_allgather: null buffer");
  if (count == 0) return GNNC_OK;
  const NcclApi* api = nccl(ctx);
  if (!api) return GNNC_ERR_NCCL;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  return nccl_status(ctx, api,
                     api->all_gather(sendbuf, recvbuf, count, dtype == GNNC_F32 ? ncclFloat32 : ncclBfloat16,
                                     static_cast<ncclComm_t>(ctx->comm), ctx->stream),
                     "ncclAllGather");
}

int gnnc_comm_destroy(gnnc_ctx_t* ctx) {
  if (!ctx) return GNNC_ERR_INVALID;
  if (!ctx->comm) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  gnnc::comm_release(ctx);
  return GNNC_OK;
}

}  // extern "C"
