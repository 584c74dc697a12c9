// tcgen05 (5th-generation tensor core) path of the dense projection.
#pragma once

#include "common.cuh"

namespace gnnc {

// Returned by proj_tc_try when the shapes or alignment do not suit the
// tensor-core kernel; the caller then uses the CUDA-core kernel.
constexpr int kProjTcDeclined = -1;

int proj_tc_try(gnnc_ctx_t* ctx, const void* x, int64_t ldx, const void* w, int64_t ldw,
                int64_t N, int64_t K, int64_t F, const float* att_src, const float* att_dst,
                int64_t H, void* h, int h_dtype, int64_t ldh, float* asrc, float* adst);

}  // namespace gnnc
