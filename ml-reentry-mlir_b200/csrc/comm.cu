// Collective entry points of the C ABI: one NCCL communicator per context and
// the all-gather a destination-row partition needs (every rank contributes its
// rows of a table and receives everyone's).
//
// NCCL is loaded when first used, not linked: a process that already holds it
// (torch.distributed loads its own copy) reuses that copy, so one process never
// carries two NCCL instances; otherwise libnccl.so.2 is loaded from the library
// search path. The types come from nccl.h.
//
// Deadlines. Communicators are created non-blocking (ncclConfig_t.blocking = 0):
// ncclCommInitRankConfig returns at once and the host polls
// ncclCommGetAsyncError until the communicator is ready, fails, or the
// caller's deadline passes. A peer that never joins therefore cannot hang the
// caller: at the deadline the communicator is aborted (ncclCommAbort) and the
// call returns GNNC_ERR_TIMEOUT. Enqueueing a collective is polled the same
// way, and gnnc_comm_wait bounds the wait for its completion.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int,
                                        ncclConfig_t*) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool loaded = false;
};

// Default deadline of gnnc_comm_init (milliseconds).
constexpr int64_t kDefaultInitTimeoutMs = 120000;

using Clock = std::chrono::steady_clock;

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
      !bind(lib, "ncclCommInitRankConfig", api.comm_init_rank_config) ||
      !bind(lib, "ncclCommGetAsyncError", api.get_async_error) ||
      !bind(lib, "ncclAllGather", api.all_gather) ||
      !bind(lib, "ncclCommDestroy", api.comm_destroy) ||
      !bind(lib, "ncclCommAbort", api.comm_abort) ||
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

// Polls a non-blocking communicator until its pending operation leaves
// ncclInProgress. Returns the final state, or ncclInProgress if the deadline
// passed first.
ncclResult_t poll_until(const NcclApi* api, ncclComm_t comm, Clock::time_point deadline) {
  ncclResult_t state = ncclInProgress;
  for (;;) {
    if (api->get_async_error(comm, &state) != ncclSuccess) return ncclInternalError;
    if (state != ncclInProgress) return state;
    if (Clock::now() >= deadline) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

// Aborts the context's communicator after a failure or a missed deadline; the
// context stays usable and may join a new communicator.
void abort_comm(gnnc_ctx_t* ctx, const NcclApi* api) {
  if (!ctx->comm) return;
  api->comm_abort(static_cast<ncclComm_t>(ctx->comm));
  ctx->comm = nullptr;
  ctx->comm_rank = 0;
  ctx->comm_size = 1;
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

int gnnc_comm_init_timeout(gnnc_ctx_t* ctx, const void* id, int rank, int nranks,
                           int64_t timeout_ms) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, id != nullptr, "gnnc_comm_init: null id");
  GNNC_CHECK_ARG(ctx, nranks >= 1 && rank >= 0 && rank < nranks, "gnnc_comm_init: bad rank %d of %d",
                 rank, nranks);
  GNNC_CHECK_ARG(ctx, timeout_ms > 0, "gnnc_comm_init: timeout must be positive");
  GNNC_CHECK_ARG(ctx, ctx->comm == nullptr, "gnnc_comm_init: the context already has a communicator");
  const NcclApi* api = nccl(ctx);
  if (!api) return GNNC_ERR_NCCL;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = api->comm_init_rank_config(&comm, nranks, uid, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm) api->comm_abort(comm);
    return nccl_status(ctx, api, r, "ncclCommInitRankConfig");
  }
  ctx->comm = comm;
  const ncclResult_t state = poll_until(api, comm, deadline);
  if (state == ncclSuccess) {
    ctx->comm_rank = rank;
    ctx->comm_size = nranks;
    return GNNC_OK;
  }
  abort_comm(ctx, api);
  if (state == ncclInProgress)
    return gnnc::set_error(ctx, GNNC_ERR_TIMEOUT,
                           "gnnc_comm_init: rank %d of %d: not every rank joined within %lld ms; "
                           "the communicator was aborted",
                           rank, nranks, (long long)timeout_ms);
  return nccl_status(ctx, api, state, "ncclCommInitRankConfig");
}

int gnnc_comm_init(gnnc_ctx_t* ctx, const void* id, int rank, int nranks) {
  return gnnc_comm_init_timeout(ctx, id, rank, nranks, kDefaultInitTimeoutMs);
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
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  const ncclResult_t r = api->all_gather(sendbuf, recvbuf, count,
                                         dtype == GNNC_F32 ? ncclFloat32 : ncclBfloat16, comm,
                                         ctx->stream);
  if (r == ncclSuccess) return GNNC_OK;
  if (r != ncclInProgress) return nccl_status(ctx, api, r, "ncclAllGather");
  // non-blocking communicator: the enqueue finishes in the background
  const ncclResult_t state =
      poll_until(api, comm, Clock::now() + std::chrono::milliseconds(kDefaultInitTimeoutMs));
  if (state == ncclSuccess) return GNNC_OK;
  abort_comm(ctx, api);
  if (state == ncclInProgress)
    return gnnc::set_error(ctx, GNNC_ERR_TIMEOUT, "ncclAllGather: enqueue did not finish");
  return nccl_status(ctx, api, state, "ncclAllGather");
}

int gnnc_comm_wait(gnnc_ctx_t* ctx, int64_t timeout_ms) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, timeout_ms > 0, "gnnc_comm_wait: timeout must be positive");
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  const NcclApi* api = ctx->comm ? nccl(ctx) : nullptr;
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(ctx->stream);
    if (q == cudaSuccess) return GNNC_OK;
    if (q != cudaErrorNotReady) return gnnc::cuda_status(ctx, q, "gnnc_comm_wait");
    if (api) {
      ncclResult_t state = ncclSuccess;
      api->get_async_error(static_cast<ncclComm_t>(ctx->comm), &state);
      if (state != ncclSuccess && state != ncclInProgress) {
        abort_comm(ctx, api);
        return nccl_status(ctx, api, state, "gnnc_comm_wait");
      }
    }
    if (Clock::now() >= deadline) {
      if (api) abort_comm(ctx, api);
      return gnnc::set_error(ctx, GNNC_ERR_TIMEOUT,
                             "gnnc_comm_wait: the stream's work did not finish within %lld ms%s",
                             (long long)timeout_ms,
                             api ? "; the communicator was aborted" : "");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
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
