// tcgen05 projection (bf16 operands, fp32 accumulation in TMEM).
#include "proj_tc.cuh"

namespace gnnc {

int proj_tc_try(gnnc_ctx_t*, const void*, int64_t, const void*, int64_t, int64_t, int64_t,
                int64_t, const float*, const float*, int64_t, void*, int, int64_t, float*,
                float*) {
  return kProjTcDeclined;
}

}  // namespace gnnc
