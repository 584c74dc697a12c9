// Context, stream, workspace and error entry points of the C ABI.
#include <cstring>
#include <new>

#include "common.cuh"

namespace gnnc {

int set_error(gnnc_ctx_t* ctx, int status, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return status;
}

int cuda_status(gnnc_ctx_t* ctx, cudaError_t err, const char* what) {
  if (err == cudaSuccess) return GNNC_OK;
  return set_error(ctx, err == cudaErrorMemoryAllocation ? GNNC_ERR_OOM : GNNC_ERR_CUDA,
                   "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

int ensure_workspace(gnnc_ctx_t* ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return GNNC_OK;
  if (!ctx->ws_owned)
    return set_error(ctx, GNNC_ERR_OOM, "bound workspace holds %zu bytes, %zu needed",
                     ctx->ws_bytes, bytes);
  if (ctx->ws) {
    // The old buffer may still be read by queued work: wait before freeing.
    GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    GNNC_CUDA_TRY(ctx, cudaFree(ctx->ws));
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  size_t want = align_up(bytes, size_t(1) << 20);
  GNNC_CUDA_TRY(ctx, cudaMalloc(&ctx->ws, want));
  ctx->ws_bytes = want;
  return GNNC_OK;
}

}  // namespace gnnc

extern "C" {

int gnnc_abi_version(void) { return GNNC_ABI_VERSION; }

const char* gnnc_status_string(int status) {
  switch (status) {
    case GNNC_OK: return "ok";
    case GNNC_ERR_INVALID: return "invalid argument";
    case GNNC_ERR_UNSUPPORTED: return "unsupported";
    case GNNC_ERR_CUDA: return "cuda error";
    case GNNC_ERR_OOM: return "out of memory";
    case GNNC_ERR_BOUNDS: return "index out of bounds";
    case GNNC_ERR_TIMEOUT: return "timeout";
    case GNNC_ERR_NCCL: return "nccl error";
    default: return "unknown status";
  }
}

int gnnc_init(int device, gnnc_ctx_t** out_ctx) {
  if (!out_ctx) return GNNC_ERR_INVALID;
  *out_ctx = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || device < 0 || device >= count) return GNNC_ERR_CUDA;
  gnnc_ctx_t* ctx = new (std::nothrow) gnnc_ctx_t();
  if (!ctx) return GNNC_ERR_OOM;
  ctx->device = device;
  // The fixed scratch of gnnc_gat_aggregate_noalloc is resolved here, so that
  // the module load and the array's reservation happen at set-up, not inside
  // that entry point.
  if (cudaSetDevice(device) != cudaSuccess ||
      cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device) !=
          cudaSuccess ||
      cudaMalloc(&ctx->dev_words, 64 * sizeof(int)) != cudaSuccess ||
      cudaMemset(ctx->dev_words, 0, 64 * sizeof(int)) != cudaSuccess ||
      gnnc::resolve_static_scratch(ctx) != cudaSuccess) {
    if (ctx->dev_words) cudaFree(ctx->dev_words);
    delete ctx;
    return GNNC_ERR_CUDA;
  }
  *out_ctx = ctx;
  return GNNC_OK;
}

int gnnc_destroy(gnnc_ctx_t* ctx) {
  if (!ctx) return GNNC_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  gnnc::comm_release(ctx);
  if (ctx->ws && ctx->ws_owned) cudaFree(ctx->ws);
  if (ctx->dev_words) cudaFree(ctx->dev_words);
  delete ctx;
  return GNNC_OK;
}

int gnnc_stream_set(gnnc_ctx_t* ctx, void* stream) {
  if (!ctx) return GNNC_ERR_INVALID;
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  return GNNC_OK;
}

int gnnc_last_error(const gnnc_ctx_t* ctx, char* buf, size_t n) {
  if (!ctx || !buf || n == 0) return GNNC_ERR_INVALID;
  size_t len = ctx->last_error.size();
  if (len >= n) len = n - 1;
  memcpy(buf, ctx->last_error.data(), len);
  buf[len] = '\0';
  return GNNC_OK;
}

int gnnc_synchronize(gnnc_ctx_t* ctx) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  // Word 2 is set by the aggregation kernels when they meet a column index
  // outside the feature table (the edge is skipped, never dereferenced).
  // Word 3 is set by a tensor-core projection whose bounded wait gave up.
  int words[2] = {0, 0};
  GNNC_CUDA_TRY(ctx, cudaMemcpy(words, ctx->dev_words + 2, sizeof(words), cudaMemcpyDeviceToHost));
  const int flag = words[0];
  if (words[1]) {
    GNNC_CUDA_TRY(ctx, cudaMemset(ctx->dev_words + 3, 0, sizeof(int)));
    return gnnc::set_error(ctx, GNNC_ERR_TIMEOUT,
                           "a bounded wait on the device gave up (a tensor-core projection "
                           "waiting on its pipeline: its output is incomplete; or "
                           "gnnc_wait_selftest)");
  }
  if (flag) {
    GNNC_CUDA_TRY(ctx, cudaMemset(ctx->dev_words + 2, 0, sizeof(int)));
    return gnnc::set_error(ctx, GNNC_ERR_BOUNDS,
                           "an aggregation met a column index outside [0, n_src); "
                           "those edges were skipped");
  }
  return GNNC_OK;
}

int gnnc_workspace_bind(gnnc_ctx_t* ctx, void* ptr, size_t bytes) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, ptr != nullptr || bytes == 0, "workspace_bind: null pointer");
  GNNC_CHECK_ARG(ctx, (reinterpret_cast<uintptr_t>(ptr) & 255) == 0,
                 "workspace_bind: buffer must be 256-byte aligned");
  if (ctx->ws && ctx->ws_owned) {
    GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    GNNC_CUDA_TRY(ctx, cudaFree(ctx->ws));
  }
  ctx->ws = ptr;
  ctx->ws_bytes = bytes;
  ctx->ws_owned = (ptr == nullptr);
  return GNNC_OK;
}

}  // extern "C"
