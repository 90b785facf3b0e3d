// Internal GEMM interface shared by gemm.cu (CUDA-core path and dispatch)
// and gemm_tc.cu (tcgen05 tensor-core path).
#pragma once
#include "common.cuh"

namespace fcu {

// The three contractions of matmulT, all computing C[M,N] (+)= ...:
//   kFwd: C = A[M,K] . B[N,K]^T   (Y = X . W^T)
//   kDx : C = A[M,K] . B[K,N]     (dX = dY . W)
//   kDw : C = A[K,M]^T . B[K,N]   (dW = dY^T . X)
enum class GemmOp { kFwd = 0, kDx = 1, kDw = 2 };

int gemm_simt(cudaStream_t st, GemmOp op, const float *A, const float *B, float *C, int64_t M,
              int64_t N, int64_t K, int beta);
int gemm_tc(fcu_ctx *ctx, GemmOp op, const float *A, const float *B, float *C, int64_t M,
            int64_t N, int64_t K, int beta);
int gemm_dispatch(fcu_ctx *ctx, GemmOp op, const float *A, const float *B, float *C, int64_t M,
                  int64_t N, int64_t K, int beta);
// FCU_PREC_FP32_TC: fp32 operands on the tensor cores (three-way bf16 split,
// six products; gemm_tc.cu).
int gemm_split6(fcu_ctx *ctx, GemmOp op, const float *A, const float *B, float *C, int64_t M, int64_t N,
                int64_t K, int beta);

}  // namespace fcu

namespace fcu {
// True when the tensor-core path can take this shape (TMA row strides).
bool gemm_tc_supported(GemmOp op, int64_t M, int64_t N, int64_t K);
// FCU_ERR_TIMEOUT if a tensor-core kernel on this context recorded a bounded
// wait that ran out (synchronises the stream).
int gemm_tc_error(fcu_ctx *ctx);
}  // namespace fcu
