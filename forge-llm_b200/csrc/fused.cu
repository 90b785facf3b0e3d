// Row kernels of the fused bf16 training step (FCU_PREC_BF16): the same
// arithmetic as rmsNorm (src/L2/tensor.js:103-128) and swigluRows
// (src/L2/tensor.js:272-290), but reading and writing the bf16 operands the
// tensor-core GEMMs consume, so no separate conversion pass runs.  All are
// single-pass, 16-byte vectorised, HBM-bound kernels.
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"
#include "swiglu_math.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

inline int grid_for(int64_t n, int per_block, int cap) {
  int64_t g = (n + per_block - 1) / per_block;
  return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

// ---------------------------------------------------------------- rmsNorm fwd -> bf16
// One warp per row; out = bf16(x * inv * w), inv[t] = 1/sqrt(mean(x^2) + eps).
// With ADD, x = X + A is formed first and stored to Xout (any D % 4 == 0).
template <bool ADD>
__global__ void rmsnorm_fwd_bf16_kernel(const float *__restrict__ X, const float *__restrict__ w,
                                        int64_t T, int64_t D, float eps,
                                        __nv_bfloat16 *__restrict__ out, float *__restrict__ inv,
                                        const float *__restrict__ A, float *__restrict__ Xout) {
  fcu::pdl_trigger();
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  if (ADD) {
    const float4 *a4 = reinterpret_cast<const float4 *>(A + row * D);
    const float4 *s4 = reinterpret_cast<const float4 *>(X + row * D);
    float4 *d4 = reinterpret_cast<float4 *>(Xout + row * D);
    for (int64_t c = lane; c < (D >> 2); c += 32) {
      float4 v = s4[c];
      const float4 a = a4[c];
      v.x += a.x;
      v.y += a.y;
      v.z += a.z;
      v.w += a.w;
      d4[c] = v;
    }
    __syncwarp();
    X = Xout;
  }
  const float4 *x4 = reinterpret_cast<const float4 *>(X + row * D);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  const int64_t D4 = D >> 2;
  float ss = 0.f;
  for (int64_t c = lane; c < D4; c += 32) {
    const float4 v = x4[c];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  const float iv = rsqrtf(ss / (float)D + eps);
  if (lane == 0) inv[row] = iv;
  uint2 *o2 = reinterpret_cast<uint2 *>(out + row * D);
  for (int64_t c = lane; c < D4; c += 32) {
    const float4 v = x4[c], ww = w4[c];
    uint2 o;
    o.x = pack_bf16(v.x * iv * ww.x, v.y * iv * ww.y);
    o.y = pack_bf16(v.z * iv * ww.z, v.w * iv * ww.w);
    o2[c] = o;
  }
}

// Row cached in registers (D = 128 * NC): one HBM read of x.  With ADD the
// row is x = X + A (the residual add of the branch that produced A), stored
// to Xout before it is normalised.
template <int NC, bool ADD>
__global__ void rmsnorm_fwd_bf16_rc_kernel(const float *__restrict__ X, const float *__restrict__ A,
                                           const float *__restrict__ w, int64_t T, float eps,
                                           float *__restrict__ Xout, __nv_bfloat16 *__restrict__ out,
                                           float *__restrict__ inv) {
  fcu::pdl_trigger();
  constexpr int D = 128 * NC;
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float4 *x4 = reinterpret_cast<const float4 *>(X + row * D);
  float4 v[NC];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NC; i++) {
    v[i] = x4[lane + 32 * i];
    if (ADD) {
      const float4 a = reinterpret_cast<const float4 *>(A + row * D)[lane + 32 * i];
      v[i].x += a.x;
      v[i].y += a.y;
      v[i].z += a.z;
      v[i].w += a.w;
      reinterpret_cast<float4 *>(Xout + row * D)[lane + 32 * i] = v[i];
    }
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  ss = warp_sum(ss);
  const float iv = rsqrtf(ss / (float)D + eps);
  if (lane == 0) inv[row] = iv;
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  uint2 *o2 = reinterpret_cast<uint2 *>(out + row * D);
#pragma unroll
  for (int i = 0; i < NC; i++) {
    const float4 ww = w4[lane + 32 * i];
    uint2 o;
    o.x = pack_bf16(v[i].x * iv * ww.x, v[i].y * iv * ww.y);
    o.y = pack_bf16(v[i].z * iv * ww.z, v[i].w * iv * ww.w);
    o2[lane + 32 * i] = o;
  }
}

template <bool ADD>
int rmsnorm_fwd_rc_launch(cudaStream_t st, const float *X, const float *A, const float *w, int64_t T,
                          int64_t D, float eps, float *Xout, __nv_bfloat16 *out, float *inv) {
  const int blocks = grid_for(T * 32, kThreads, 1 << 30);
  switch (D / 128) {
#define FCU_RMS_CASE(nc)                                                                       \
  case nc:                                                                                     \
    rmsnorm_fwd_bf16_rc_kernel<nc, ADD><<<blocks, kThreads, 0, st>>>(X, A, w, T, eps, Xout, out, inv); \
    break;
    FCU_RMS_CASE(1)
    FCU_RMS_CASE(2)
    FCU_RMS_CASE(3)
    FCU_RMS_CASE(4)
    FCU_RMS_CASE(5)
    FCU_RMS_CASE(6)
    FCU_RMS_CASE(7)
    FCU_RMS_CASE(8)
#undef FCU_RMS_CASE
    default: return FCU_ERR_ARG;
  }
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

// ---------------------------------------------------------------- rmsNorm bwd, fused
// dX (+)= g*w*inv - c*x with c = dot(g*w, x) * inv^3 / D; dXb = bf16(final
// dX) (the next GEMM's operand); per-block dw partials sum g*x*inv over the
// block's rows, accumulated in registers per warp and combined across warps
// in a fixed order (deterministic).  NC = float4 chunks each lane owns.
//
// A float4 of w through the read-only path at each use (an L1 hit): the asm
// keeps the compiler from holding all NC of them in registers for the row.
__device__ __forceinline__ float4 ld_w(const float4 *p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

template <int NC>
__global__ void __launch_bounds__(kThreads, NC <= 6 ? 2 : 1) rmsnorm_bwd_fused_kernel(
    const float *__restrict__ G, const float *__restrict__ X, const float *__restrict__ w,
    const float *__restrict__ inv, int64_t T, int64_t D, int64_t rows_per_block,
    float *__restrict__ dX, int acc_dx, __nv_bfloat16 *__restrict__ dXb, float *__restrict__ part) {
  fcu::pdl_trigger();
  extern __shared__ float sm[];  // [nwarps][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t D4 = D >> 2;
  // w is re-read from L1 per row instead of being held in registers, which
  // leaves room for the prefetched dX at two blocks per SM
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  float4 dw[NC];
#pragma unroll
  for (int k = 0; k < NC; k++) dw[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float invD = 1.f / (float)D;
  const int64_t r0 = blockIdx.x * rows_per_block;
  const int64_t r1 = min(T, r0 + rows_per_block);
  for (int64_t row = r0 + wid; row < r1; row += nw) {
    const float4 *g4 = reinterpret_cast<const float4 *>(G + row * D);
    const float4 *x4 = reinterpret_cast<const float4 *>(X + row * D);
    float4 *d4 = reinterpret_cast<float4 *>(dX + row * D);
    // G, X and (accumulating) the old dX of the row are all requested before
    // the row reduction, so their latencies overlap
    float4 gv[NC], xv[NC], pv[NC];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < NC; k++) {
      const int64_t c = lane + 32 * k;
      if (c < D4) {
        gv[k] = g4[c];
        xv[k] = x4[c];
        pv[k] = acc_dx ? d4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int k = 0; k < NC; k++) {
      const int64_t c = lane + 32 * k;
      if (c < D4) {
        const float4 wv = ld_w(w4 + c);
        dot += gv[k].x * wv.x * xv[k].x + gv[k].y * wv.y * xv[k].y +
               gv[k].z * wv.z * xv[k].z + gv[k].w * wv.w * xv[k].w;
      }
    }
    dot = warp_sum(dot);
    const float iv = inv[row];
    const float cc = dot * iv * iv * iv * invD;
    uint2 *b2 = dXb ? reinterpret_cast<uint2 *>(dXb + row * D) : nullptr;
#pragma unroll
    for (int k = 0; k < NC; k++) {
      const int64_t c = lane + 32 * k;
      if (c < D4) {
        const float4 wv = ld_w(w4 + c);
        float4 o;
        o.x = gv[k].x * wv.x * iv - cc * xv[k].x;
        o.y = gv[k].y * wv.y * iv - cc * xv[k].y;
        o.z = gv[k].z * wv.z * iv - cc * xv[k].z;
        o.w = gv[k].w * wv.w * iv - cc * xv[k].w;
        if (acc_dx) {
          o.x += pv[k].x;
          o.y += pv[k].y;
          o.z += pv[k].z;
          o.w += pv[k].w;
        }
        d4[c] = o;
        if (b2) {
          uint2 u;
          u.x = pack_bf16(o.x, o.y);
          u.y = pack_bf16(o.z, o.w);
          b2[c] = u;
        }
        dw[k].x += gv[k].x * xv[k].x * iv;
        dw[k].y += gv[k].y * xv[k].y * iv;
        dw[k].z += gv[k].z * xv[k].z * iv;
        dw[k].w += gv[k].w * xv[k].w * iv;
      }
    }
  }
  float4 *mine = reinterpret_cast<float4 *>(sm + (int64_t)wid * D);
#pragma unroll
  for (int k = 0; k < NC; k++) {
    const int64_t c = lane + 32 * k;
    if (c < D4) mine[c] = dw[k];
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < nw; k++) s += sm[(int64_t)k * D + i];
    part[(int64_t)blockIdx.x * D + i] = s;
  }
}

// out[c] (+)= sum_b part[b][c]: a (32 x 8) block per 32 columns, each row of
// threads summing every 8th partial, then a fixed-order sum of the 8.
__global__ void colsum_kernel(const float *__restrict__ part, int nblk, int64_t D,
                              float *__restrict__ out, int acc) {
  fcu::pdl_trigger();
  __shared__ float sh[8][33];
  const int64_t c = (int64_t)blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < D)
    for (int b = threadIdx.y; b < nblk; b += 8) s += part[(int64_t)b * D + c];
  sh[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < D) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 8; y++) t += sh[y][threadIdx.x];
    out[c] = acc ? out[c] + t : t;
  }
}

// ---------------------------------------------------------------- swiglu on a [N, 2H] gate|up buffer
// act[t, j] = silu(gu[t, j]) * gu[t, H + j]; 8 units per thread.
__global__ void swiglu_fwd_bf16_kernel(const __nv_bfloat16 *__restrict__ gu, int64_t N, int64_t H,
                                       __nv_bfloat16 *__restrict__ act) {
  fcu::pdl_trigger();
  const int64_t H8 = H >> 3, total = N * H8;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / H8, j = (e - t * H8) * 8;
    const uint4 g4 = *reinterpret_cast<const uint4 *>(gu + t * 2 * H + j);
    const uint4 u4 = *reinterpret_cast<const uint4 *>(gu + t * 2 * H + H + j);
    const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w}, uw[4] = {u4.x, u4.y, u4.z, u4.w};
    uint32_t ow[4];
#pragma unroll
    for (int k = 0; k < 4; k++) ow[k] = fcu::swiglu_fwd_pair(gw[k], uw[k]);
    *reinterpret_cast<uint4 *>(act + t * H + j) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// dgu[t, j] = dact * u * (s + g s (1 - s)),  dgu[t, H + j] = dact * g * s.
__global__ void swiglu_bwd_bf16_kernel(const __nv_bfloat16 *__restrict__ dact,
                                       const __nv_bfloat16 *__restrict__ gu, int64_t N, int64_t H,
                                       __nv_bfloat16 *__restrict__ dgu) {
  fcu::pdl_trigger();
  const int64_t H8 = H >> 3, total = N * H8;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / H8, j = (e - t * H8) * 8;
    const uint4 d4 = *reinterpret_cast<const uint4 *>(dact + t * H + j);
    const uint4 g4 = *reinterpret_cast<const uint4 *>(gu + t * 2 * H + j);
    const uint4 u4 = *reinterpret_cast<const uint4 *>(gu + t * 2 * H + H + j);
    const uint32_t dw[4] = {d4.x, d4.y, d4.z, d4.w}, gw[4] = {g4.x, g4.y, g4.z, g4.w},
                   uw[4] = {u4.x, u4.y, u4.z, u4.w};
    uint32_t og[4], ou[4];
#pragma unroll
    for (int k = 0; k < 4; k++) fcu::swiglu_bwd_pair(dw[k], gw[k], uw[k], og[k], ou[k]);
    *reinterpret_cast<uint4 *>(dgu + t * 2 * H + j) = make_uint4(og[0], og[1], og[2], og[3]);
    *reinterpret_cast<uint4 *>(dgu + t * 2 * H + H + j) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
  }
}

__global__ void to_bf16_kernel(const float *__restrict__ x, int64_t n, __nv_bfloat16 *__restrict__ y) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

__global__ void scale_bf16_dev_kernel(__nv_bfloat16 *__restrict__ y, int64_t n,
                                      const float *__restrict__ alpha) {
  fcu::pdl_trigger();
  const float a = alpha[0];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(__bfloat162float(y[i]) * a);
}

inline bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }

template <int NC>
int rms_bwd_launch(fcu_ctx *ctx, const float *dY, const float *X, const float *w, const float *inv,
                   int64_t T, int64_t D, float *dX, int acc_dx, __nv_bfloat16 *dXb, float *dw,
                   int acc_dw) {
  const int nw = kThreads / 32;
  int64_t nblk = 2 * (int64_t)ctx->num_sms;
  int64_t rpb = (T + nblk - 1) / nblk;
  if (rpb < nw) rpb = nw;
  nblk = (T + rpb - 1) / rpb;
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(float) * (size_t)(nblk * D), &scr);
  if (rc) return rc;
  const size_t smem = sizeof(float) * (size_t)nw * (size_t)D;
  if (smem > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(rmsnorm_bwd_fused_kernel<NC>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rmsnorm_bwd_fused_kernel<NC><<<(int)nblk, kThreads, smem, ctx->stream>>>(
      dY, X, w, inv, T, D, rpb, dX, acc_dx, dXb, (float *)scr);
  FCU_CHECK_LAUNCH();
  colsum_kernel<<<(unsigned)((D + 31) / 32), dim3(32, 8), 0, ctx->stream>>>((float *)scr, (int)nblk,
                                                                            D, dw, acc_dw);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // namespace

extern "C" {

int fcu_rmsnorm_fwd_bf16(fcu_ctx *ctx, const float *X, const float *w, int64_t T, int64_t D,
                         double eps, void *out, float *inv) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && D > 0 && D % 4 == 0, "fcu_rmsnorm_fwd_bf16: D=%lld must be a multiple of 4",
              (long long)D);
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(X && w && out && inv && al16(X) && al16(w) && ((uintptr_t)out & 7) == 0,
              "fcu_rmsnorm_fwd_bf16: null or unaligned pointer");
  if (D % 128 == 0 && D <= 1024)
    return rmsnorm_fwd_rc_launch<false>(ctx->stream, X, nullptr, w, T, D, (float)eps, nullptr,
                                        (__nv_bfloat16 *)out, inv);
  rmsnorm_fwd_bf16_kernel<false><<<grid_for(T * 32, kThreads, 1 << 30), kThreads, 0, ctx->stream>>>(
      X, w, T, D, (float)eps, (__nv_bfloat16 *)out, inv, nullptr, nullptr);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_rmsnorm_fwd_bf16_add(fcu_ctx *ctx, const float *X, const float *A, const float *w, int64_t T,
                             int64_t D, double eps, float *Xout, void *out, float *inv) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && D > 0 && D % 4 == 0,
              "fcu_rmsnorm_fwd_bf16_add: D=%lld must be a multiple of 4", (long long)D);
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(X && A && w && Xout && out && inv && al16(X) && al16(A) && al16(w) && al16(Xout) &&
                  ((uintptr_t)out & 7) == 0,
              "fcu_rmsnorm_fwd_bf16_add: null or unaligned pointer");
  if (D % 128 == 0 && D <= 1024)
    return rmsnorm_fwd_rc_launch<true>(ctx->stream, X, A, w, T, D, (float)eps, Xout,
                                       (__nv_bfloat16 *)out, inv);
  rmsnorm_fwd_bf16_kernel<true><<<grid_for(T * 32, kThreads, 1 << 30), kThreads, 0, ctx->stream>>>(
      X, w, T, D, (float)eps, (__nv_bfloat16 *)out, inv, A, Xout);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_rmsnorm_bwd_fused(fcu_ctx *ctx, const float *dY, const float *X, const float *w,
                          const float *inv, int64_t T, int64_t D, float *dX, int accumulate_dx,
                          void *dX_bf16, float *dw, int accumulate_dw) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && D > 0 && D % 4 == 0 && D <= 2048,
              "fcu_rmsnorm_bwd_fused: D=%lld must be a multiple of 4 and <= 2048", (long long)D);
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(dY && X && w && inv && dX && dw && al16(dY) && al16(X) && al16(w) && al16(dX) &&
                  (dX_bf16 == nullptr || ((uintptr_t)dX_bf16 & 7) == 0),
              "fcu_rmsnorm_bwd_fused: null or unaligned pointer");
  const int64_t nc = (D / 4 + 31) / 32;
  __nv_bfloat16 *b = (__nv_bfloat16 *)dX_bf16;
  if (nc <= 2) return rms_bwd_launch<2>(ctx, dY, X, w, inv, T, D, dX, accumulate_dx, b, dw, accumulate_dw);
  if (nc <= 4) return rms_bwd_launch<4>(ctx, dY, X, w, inv, T, D, dX, accumulate_dx, b, dw, accumulate_dw);
  if (nc <= 6) return rms_bwd_launch<6>(ctx, dY, X, w, inv, T, D, dX, accumulate_dx, b, dw, accumulate_dw);
  if (nc <= 8) return rms_bwd_launch<8>(ctx, dY, X, w, inv, T, D, dX, accumulate_dx, b, dw, accumulate_dw);
  return rms_bwd_launch<16>(ctx, dY, X, w, inv, T, D, dX, accumulate_dx, b, dw, accumulate_dw);
}

int fcu_swiglu_fwd_bf16(fcu_ctx *ctx, const void *gu, int64_t N, int64_t H, void *act) {
  FCU_CTX(ctx);
  FCU_REQUIRE(N >= 0 && H > 0 && H % 8 == 0, "fcu_swiglu_fwd_bf16: H=%lld must be a multiple of 8",
              (long long)H);
  if (N == 0) return FCU_OK;
  FCU_REQUIRE(gu && act && al16(gu) && al16(act), "fcu_swiglu_fwd_bf16: null or unaligned pointer");
  swiglu_fwd_bf16_kernel<<<grid_for(N * H / 8, kThreads, 16 * ctx->num_sms), kThreads, 0, ctx->stream>>>(
      (const __nv_bfloat16 *)gu, N, H, (__nv_bfloat16 *)act);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_swiglu_bwd_bf16(fcu_ctx *ctx, const void *dact, const void *gu, int64_t N, int64_t H,
                        void *dgu) {
  FCU_CTX(ctx);
  FCU_REQUIRE(N >= 0 && H > 0 && H % 8 == 0, "fcu_swiglu_bwd_bf16: H=%lld must be a multiple of 8",
              (long long)H);
  if (N == 0) return FCU_OK;
  FCU_REQUIRE(dact && gu && dgu && al16(dact) && al16(gu) && al16(dgu),
              "fcu_swiglu_bwd_bf16: null or unaligned pointer");
  swiglu_bwd_bf16_kernel<<<grid_for(N * H / 8, kThreads, 16 * ctx->num_sms), kThreads, 0, ctx->stream>>>(
      (const __nv_bfloat16 *)dact, (const __nv_bfloat16 *)gu, N, H, (__nv_bfloat16 *)dgu);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_to_bf16(fcu_ctx *ctx, const float *x, int64_t n, void *y) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && x && y, "fcu_to_bf16: bad args");
  if (n == 0) return FCU_OK;
  to_bf16_kernel<<<grid_for(n, kThreads, 16 * ctx->num_sms), kThreads, 0, ctx->stream>>>(
      x, n, (__nv_bfloat16 *)y);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_scale_bf16_dev(fcu_ctx *ctx, void *y, int64_t n, const float *alpha_dev) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && y && alpha_dev, "fcu_scale_bf16_dev: bad args");
  if (n == 0) return FCU_OK;
  scale_bf16_dev_kernel<<<grid_for(n, kThreads, 16 * ctx->num_sms), kThreads, 0, ctx->stream>>>(
      (__nv_bfloat16 *)y, n, alpha_dev);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // extern "C"
