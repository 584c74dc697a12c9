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

// dst[i] = src[idx[i]] for rows of `chunks` 16-byte chunks. A warp copies
// 32 / chunks rows per pass when a row has fewer than 32 chunks (lane ->
// (row slot, chunk), e.g. two 13-chunk rows of 100 bf16 features, 26 lanes
// busy), else one row with its lanes striding over the chunks. An index
// outside [0, n_src) leaves the row alone and raises the context's bad-index
// word (reported by gnnc_synchronize). No lane waits on another.
__global__ void gather_rows_kernel(const char* __restrict__ src, int64_t ld_src,
                                   const int32_t* __restrict__ idx, int64_t n, int64_t n_src,
                                   char* __restrict__ dst, int64_t ld_dst, int64_t chunks,
                                   int* bad) {
  const int lane = threadIdx.x & 31;
  const bool packed = chunks < 32;
  const int rpw = packed ? int(32 / chunks) : 1;
  const int slot = packed ? lane / int(chunks) : 0;
  const int c0 = packed ? lane - slot * int(chunks) : lane;
  const int64_t step = packed ? chunks : 32;
  if (slot >= rpw) return;  // the few lanes past the last whole row
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  for (int64_t i = warp * rpw + slot; i < n; i += warps * rpw) {
    const int32_t r = __ldg(idx + i);
    if (r < 0 || r >= n_src) {
      if (c0 == 0) atomicOr(bad, 1);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(src + int64_t(r) * ld_src);
    uint4* d = reinterpret_cast<uint4*>(dst + i * ld_dst);
    for (int64_t c = c0; c < chunks; c += step) d[c] = __ldg(s + c);
  }
}

}  // namespace

extern "C" {

int gnnc_gather_rows(gnnc_ctx_t* ctx, const void* src, int64_t ld_src, const int32_t* idx,
                     int64_t n, int64_t n_src, void* dst, int64_t ld_dst, int64_t row_bytes) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, n >= 0 && n_src >= 0 && row_bytes > 0, "bad sizes");
  GNNC_CHECK_ARG(ctx, n == 0 || (src && idx && dst), "null argument");
  GNNC_CHECK_ARG(ctx, row_bytes % 16 == 0 && ld_src % 16 == 0 && ld_dst % 16 == 0 &&
                          reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                          reinterpret_cast<uintptr_t>(dst) % 16 == 0,
                 "rows, strides and pointers must be 16-byte aligned");
  GNNC_CHECK_ARG(ctx, ld_src >= row_bytes && ld_dst >= row_bytes, "stride below row size");
  if (n == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  const int64_t chunks = row_bytes / 16;
  const int64_t rows_per_cta = 8 * (chunks < 32 ? 32 / chunks : 1);  // 8 warps
  const int64_t want = (n + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = int64_t(ctx->num_sms) * 8;
  const unsigned grid = unsigned(want < cap ? want : cap);
  gather_rows_kernel<<<grid, 256, 0, ctx->stream>>>(
      static_cast<const char*>(src), ld_src, idx, n, n_src, static_cast<char*>(dst), ld_dst,
      chunks, ctx->dev_words + 2);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}


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
