// matmulT forward and backward (src/L2/tensor.js:34-53) and their dispatch.
//
// The three contractions of one matmulT are all "C[m,n] = sum_k A(m,k) B(n,k)"
// with different operand layouts:
//   forward  Y  = X  . W^T : A = X  (k contiguous), B = W (k contiguous)
//   dX       dX = dY . W   : A = dY (k contiguous), B = W^T (n contiguous)
//   dW       dW = dY^T . X : A = dY^T (m contiguous), B = X^T (n contiguous)
// FCU_PREC_FP32 runs them on the CUDA cores (this file); the tensor-core
// modes go to gemm_tc.cu.
#include "common.cuh"
#include "gemm.cuh"

namespace {

// 128x128 output tile, BK = 8, 256 threads, 8x8 outputs per thread.
constexpr int BM = 128, BN = 128, BK = 8, TM = 8, TN = 8, NT = 256;

// A(m,k) = A_KC ? A[m*lda + k] : A[k*lda + m]; likewise B(n,k).
template <bool A_KC, bool B_KC>
__global__ void __launch_bounds__(NT) sgemm_kernel(const float *__restrict__ A, int64_t lda,
                                                   const float *__restrict__ B, int64_t ldb,
                                                   float *__restrict__ C, int64_t ldc, int64_t M,
                                                   int64_t N, int64_t K, int beta) {
  fcu::pdl_trigger();
  __shared__ float As[2][BK][BM + 4];
  __shared__ float Bs[2][BK][BN + 4];
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, each 8 x 8

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.f;

  // Each thread loads 4 elements of the A tile and 4 of the B tile.
  auto load_tile = [&](int buf, int64_t k0) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      int e = tid + r * NT;  // 0 .. 1023 over a BM x BK tile
      int mm, kk;
      if (A_KC) {
        mm = e / BK;
        kk = e % BK;
      } else {
        kk = e / BM;
        mm = e % BM;
      }
      int64_t gm = m0 + mm, gk = k0 + kk;
      float v = 0.f;
      if (gm < M && gk < K) v = A_KC ? A[gm * lda + gk] : A[gk * lda + gm];
      As[buf][kk][mm] = v;
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
      int e = tid + r * NT;
      int nn, kk;
      if (B_KC) {
        nn = e / BK;
        kk = e % BK;
      } else {
        kk = e / BN;
        nn = e % BN;
      }
      int64_t gn = n0 + nn, gk = k0 + kk;
      float v = 0.f;
      if (gn < N && gk < K) v = B_KC ? B[gn * ldb + gk] : B[gk * ldb + gn];
      Bs[buf][kk][nn] = v;
    }
  };

  const int64_t nk = (K + BK - 1) / BK;
  load_tile(0, 0);
  __syncthreads();
  for (int64_t kt = 0; kt < nk; kt++) {
    const int cur = kt & 1;
    if (kt + 1 < nk) load_tile(cur ^ 1, (kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; kk++) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM / 4; i++) {
        float4 v = *reinterpret_cast<const float4 *>(&As[cur][kk][tr * 4 + i * 64]);
        a[i * 4 + 0] = v.x;
        a[i * 4 + 1] = v.y;
        a[i * 4 + 2] = v.z;
        a[i * 4 + 3] = v.w;
      }
#pragma unroll
      for (int j = 0; j < TN / 4; j++) {
        float4 v = *reinterpret_cast<const float4 *>(&Bs[cur][kk][tc * 4 + j * 64]);
        b[j * 4 + 0] = v.x;
        b[j * 4 + 1] = v.y;
        b[j * 4 + 2] = v.z;
        b[j * 4 + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TM; i++) {
    int64_t gm = m0 + tr * 4 + (i / 4) * 64 + (i % 4);
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      int64_t gn = n0 + tc * 4 + (j / 4) * 64 + (j % 4);
      if (gn >= N) continue;
      float *p = C + gm * ldc + gn;
      *p = beta ? *p + acc[i][j] : acc[i][j];
    }
  }
}

template <bool A_KC, bool B_KC>
int launch_sgemm(cudaStream_t st, const float *A, int64_t lda, const float *B, int64_t ldb, float *C,
                 int64_t ldc, int64_t M, int64_t N, int64_t K, int beta) {
  if (M == 0 || N == 0) return FCU_OK;
  FCU_REQUIRE((M + BM - 1) / BM < 65536, "sgemm: M=%lld too large for the grid", (long long)M);
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
  sgemm_kernel<A_KC, B_KC><<<grid, NT, 0, st>>>(A, lda, B, ldb, C, ldc, M, N, K, beta);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // namespace

namespace fcu {

int gemm_simt(cudaStream_t st, GemmOp op, const float *A, const float *B, float *C, int64_t M,
              int64_t N, int64_t K, int beta) {
  switch (op) {
    case GemmOp::kFwd:  // C[M,N] = A[M,K] . B[N,K]^T
      return launch_sgemm<true, true>(st, A, K, B, K, C, N, M, N, K, beta);
    case GemmOp::kDx:  // C[M,N] = A[M,K] . B[K,N]       (A = dY, B = W)
      return launch_sgemm<true, false>(st, A, K, B, N, C, N, M, N, K, beta);
    case GemmOp::kDw:  // C[M,N] = A[K,M]^T . B[K,N]     (A = dY, B = X)
      return launch_sgemm<false, false>(st, A, M, B, N, C, N, M, N, K, beta);
  }
  return FCU_ERR_ARG;
}

int gemm_dispatch(fcu_ctx *ctx, GemmOp op, const float *A, const float *B, float *C, int64_t M,
                  int64_t N, int64_t K, int beta) {
  if (ctx->precision == FCU_PREC_FP32) return gemm_simt(ctx->stream, op, A, B, C, M, N, K, beta);
  if (ctx->precision == FCU_PREC_FP32_TC) return gemm_split6(ctx, op, A, B, C, M, N, K, beta);
  return gemm_tc(ctx, op, A, B, C, M, N, K, beta);
}

}  // namespace fcu

extern "C" {

int fcu_check_device_error(fcu_ctx *ctx) {
  FCU_CTX(ctx);
  return fcu::gemm_tc_error(ctx);
}

int fcu_matmulT_fwd(fcu_ctx *ctx, const float *X, const float *W, float *Y, int64_t M, int64_t K,
                    int64_t N) {
  FCU_CTX(ctx);
  FCU_REQUIRE(M >= 0 && K >= 0 && N >= 0, "fcu_matmulT_fwd: negative size");
  if (M == 0 || N == 0) return FCU_OK;
  FCU_REQUIRE(X && W && Y, "fcu_matmulT_fwd: null pointer");
  if (K == 0) return fcu_memset_zero(ctx, Y, sizeof(float) * (size_t)(M * N));
  return fcu::gemm_dispatch(ctx, fcu::GemmOp::kFwd, X, W, Y, M, N, K, 0);
}

int fcu_matmulT_bwd(fcu_ctx *ctx, const float *dY, const float *X, const float *W, float *dX,
                    int accumulate_dx, float *dW, int accumulate_dw, int64_t M, int64_t K,
                    int64_t N) {
  FCU_CTX(ctx);
  FCU_REQUIRE(M >= 0 && K >= 0 && N >= 0, "fcu_matmulT_bwd: negative size");
  FCU_REQUIRE(dY != nullptr, "fcu_matmulT_bwd: null dY");
  if (dX && M > 0 && K > 0) {
    FCU_REQUIRE(W != nullptr, "fcu_matmulT_bwd: null W");
    int rc;
    if (N == 0)
      rc = accumulate_dx ? FCU_OK : fcu_memset_zero(ctx, dX, sizeof(float) * (size_t)(M * K));
    else
      rc = fcu::gemm_dispatch(ctx, fcu::GemmOp::kDx, dY, W, dX, M, K, N, accumulate_dx);
    if (rc) return rc;
  }
  if (dW && N > 0 && K > 0) {
    FCU_REQUIRE(X != nullptr, "fcu_matmulT_bwd: null X");
    int rc;
    if (M == 0)
      rc = accumulate_dw ? FCU_OK : fcu_memset_zero(ctx, dW, sizeof(float) * (size_t)(N * K));
    else
      rc = fcu::gemm_dispatch(ctx, fcu::GemmOp::kDw, dY, X, dW, N, K, M, accumulate_dw);
    if (rc) return rc;
  }
  return FCU_OK;
}

}  // extern "C"
