// Shared internals of libgnnc_b200: the context and plan objects, error
// plumbing and small device helpers. Nothing here is part of the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "gnnc_b200.h"

struct gnnc_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  std::string last_error;
  // Library-owned scratch, grown on demand (or a caller-bound buffer).
  void* ws = nullptr;
  size_t ws_bytes = 0;
  bool ws_owned = true;
  // Small device area: [0..7] scheduling counters, [8..15] result/error words.
  int* dev_words = nullptr;
  // Device address of the fixed scratch array of gnnc_gat_aggregate_noalloc,
  // looked up by gnnc_init with the device current (aggregate.cu).
  void* static_scratch = nullptr;
  // NCCL communicator (ncclComm_t) of gnnc_comm_init, or null.
  void* comm = nullptr;
  int comm_rank = 0;
  int comm_size = 1;
};

// Row schedule for one CSR (see gnnc_plan_create in gnnc_b200.h).
struct gnnc_plan {
  int64_t n_rows = 0;
  int cta_threshold = 256;
  int split_threshold = 4096;
  int64_t n_warp_rows = 0;     // rows handled by one warp
  int64_t n_cta_rows = 0;      // rows handled by one CTA, written directly
  int64_t n_split_rows = 0;    // rows cut into several CTA segments
  int64_t n_segments = 0;      // partial slots used by split rows
  int64_t n_cta_items = 0;     // CTA work items (cta rows + segments)
  // Rows of up to wide_threshold edges go to the warp path when the rows are
  // wide (a whole warp per edge): their CTA items are the last ones, and
  // launches on wide rows process only the first n_cta_items_wide items.
  int wide_threshold = 256;
  int64_t n_cta_items_wide = 0;
  int64_t n_warp_tasks = 0;    // contiguous row ranges for the warp path
  int max_degree = 0;
  int device = 0;
  int64_t e_begin = 0;  // rowptr[0] and rowptr[n_rows] of the planned CSR; the
  int64_t e_end = 0;    // kernels clamp every edge range to [e_begin, e_end)
  // Device arrays (owned).
  int4* cta_items = nullptr;     // (row, edge_begin, edge_end, slot or -1), largest first
  int4* split_rows = nullptr;    // (row, first_slot, n_slots, 0)
  int32_t* warp_tasks = nullptr; // n_warp_tasks+1 row boundaries
  int64_t n_stream_tasks = 0;
  int2* stream_tasks = nullptr;  // row ranges [x, y) of wide-launch warp rows only
};

namespace gnnc {

int set_error(gnnc_ctx_t* ctx, int status, const char* fmt, ...);

// Destroys the context's communicator, if any (comm.cu).
void comm_release(gnnc_ctx_t* ctx);

// Sets ctx->static_scratch to the device address of the no-alloc entry
// point's fixed array; the device must be current (aggregate.cu).
cudaError_t resolve_static_scratch(gnnc_ctx_t* ctx);

// Returns GNNC_ERR_CUDA with text if err != cudaSuccess.
int cuda_status(gnnc_ctx_t* ctx, cudaError_t err, const char* what);

// Makes sure ctx->ws holds at least `bytes`. GNNC_ERR_OOM when a bound
// (caller-owned) workspace is too small or cudaMalloc fails.
int ensure_workspace(gnnc_ctx_t* ctx, size_t bytes);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace gnnc

#define GNNC_CHECK_ARG(ctx, cond, ...)                                   \
  do {                                                                   \
    if (!(cond)) return gnnc::set_error((ctx), GNNC_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define GNNC_CUDA_TRY(ctx, expr)                                         \
  do {                                                                   \
    cudaError_t _e = (expr);                                             \
    if (_e != cudaSuccess) return gnnc::cuda_status((ctx), _e, #expr);   \
  } while (0)

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void store_val(void* out, int dtype, size_t idx, float v) {
  if (dtype == GNNC_BF16)
    reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(out)[idx] = v;
}
