// Tensor-core (tcgen05) GEMM path -- placeholder until the sm_100a kernel lands.
#include "gemm.cuh"

namespace fcu {

int gemm_tc(fcu_ctx *ctx, GemmOp op, const float *A, const float *B, float *C, int64_t M,
            int64_t N, int64_t K, int beta) {
  set_error("tensor-core precision mode %d is not built yet", ctx->precision);
  return FCU_ERR_UNSUPPORTED;
}

}  // namespace fcu
