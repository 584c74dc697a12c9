// Peer memory entry points of the C ABI: export a device buffer of this
// process, map another process's buffer (CUDA IPC over NVLink / NVSwitch).
//
// A rank exports the row block it owns; every other rank maps it and its
// kernels read the rows straight from the owner's HBM (plain or TMA loads,
// no multicast). The exporter keeps the buffer alive until every importer has
// closed its mapping.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

std::mutex g_range_mu;
GetAddressRangeFn g_range = nullptr;

GetAddressRangeFn range_fn(gnnc_ctx_t* ctx) {
  std::lock_guard<std::mutex> lock(g_range_mu);
  if (!g_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<GetAddressRangeFn>(fn);
    else
      gnnc::set_error(ctx, GNNC_ERR_CUDA, "cuMemGetAddressRange unavailable");
  }
  return g_range;
}

}  // namespace

extern "C" {

int gnnc_peer_export(gnnc_ctx_t* ctx, const void* ptr, void* handle, uint64_t* offset) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, ptr && handle && offset, "gnnc_peer_export: null argument");
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  GetAddressRangeFn fn = range_fn(ctx);
  if (!fn) return GNNC_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return gnnc::set_error(ctx, GNNC_ERR_INVALID,
                           "gnnc_peer_export: %p is not device memory of this process", ptr);
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess)
    return gnnc::cuda_status(ctx, err,
                             "gnnc_peer_export: cudaIpcGetMemHandle (the buffer must come from "
                             "cudaMalloc, e.g. torch's caching allocator without expandable "
                             "segments)");
  static_assert(sizeof(h) == GNNC_PEER_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = uint64_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return GNNC_OK;
}

int gnnc_peer_open(gnnc_ctx_t* ctx, const void* handle, uint64_t offset, void** ptr) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, handle && ptr, "gnnc_peer_open: null argument");
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return gnnc::cuda_status(ctx, err, "gnnc_peer_open: cudaIpcOpenMemHandle");
  *ptr = static_cast<char*>(base) + offset;
  return GNNC_OK;
}

int gnnc_peer_copy(gnnc_ctx_t* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, (dst && src) || bytes == 0, "gnnc_peer_copy: null pointer");
  if (bytes == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  // device-to-device through unified addressing: a copy-engine transfer over
  // NVLink when one side is a peer mapping; no SM is used
  GNNC_CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, ctx->stream));
  return GNNC_OK;
}

int gnnc_peer_close(gnnc_ctx_t* ctx, void* ptr, uint64_t offset) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, ptr != nullptr, "gnnc_peer_close: null pointer");
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  GNNC_CUDA_TRY(ctx, cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
  return GNNC_OK;
}

}  // extern "C"
