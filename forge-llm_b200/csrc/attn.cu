// Causal GQA attention, forward and backward, fp32 on the CUDA cores.
//
// Replaces causalAttn (src/L2/tensor.js:191-268) and causalAttnBatch
// (src/L2/tensor.js:299-376).  Instead of the JS's stored P[B,nH,T,T], the
// forward keeps one log-sum-exp per score row and the backward recomputes P
// from it (online softmax; FlashAttention-2 ordering), so memory is O(T).
// The backward is split in two deterministic kernels without atomics:
//   dK/dV: one thread per key row, looping over the group's q heads and
//          every later query (GQA: the group's q heads reduce into one kv head)
//   dQ   : one thread per query row, looping over every earlier key.
#include <math.h>

#include "common.cuh"

namespace {

constexpr int kRows = 64;  // query (or key) rows per CTA, one per thread

// Q [B*T, nH*dH], K/V [B*T, nKV*dH]; row r of sequence b is at (b*T + r).
template <int MAXD>
__global__ void __launch_bounds__(kRows) attn_fwd_kernel(const float *__restrict__ Q,
                                                         const float *__restrict__ K,
                                                         const float *__restrict__ V, int T,
                                                         int nH, int nKV, int dH, float scale,
                                                         float *__restrict__ O,
                                                         float *__restrict__ lse) {
  fcu::pdl_trigger();
  extern __shared__ float smem[];
  float *Ks = smem;                   // [kRows][MAXD]
  float *Vs = smem + kRows * MAXD;    // [kRows][MAXD]
  const int b = blockIdx.z, h = blockIdx.y;
  const int group = nH / nKV, kvh = h / group;
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)nKV * dH;
  const int t0 = blockIdx.x * kRows;
  const int t = t0 + threadIdx.x;
  const bool valid = t < T;
  const int64_t base = (int64_t)b * T;

  float q[MAXD], o[MAXD];
#pragma unroll
  for (int d = 0; d < MAXD; d++) {
    q[d] = (valid && d < dH) ? Q[(base + t) * qD + (int64_t)h * dH + d] * scale : 0.f;
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int last = min(T - 1, t0 + kRows - 1);
  for (int j0 = 0; j0 <= last; j0 += kRows) {
    __syncthreads();
    for (int e = threadIdx.x; e < kRows * MAXD; e += kRows) {
      int jj = e / MAXD, d = e % MAXD;
      int j = j0 + jj;
      float kv = 0.f, vv = 0.f;
      if (j < T && d < dH) {
        int64_t off = (base + j) * kvD + (int64_t)kvh * dH + d;
        kv = K[off];
        vv = V[off];
      }
      Ks[e] = kv;
      Vs[e] = vv;
    }
    __syncthreads();
    if (valid) {
      const int jn = min(kRows, t - j0 + 1);
      for (int jj = 0; jj < jn; jj++) {
        const float4 *k4 = reinterpret_cast<const float4 *>(Ks + jj * MAXD);
        float s = 0.f;
#pragma unroll
        for (int d4 = 0; d4 < MAXD / 4; d4++) {
          float4 kk = k4[d4];
          s = fmaf(q[4 * d4 + 0], kk.x, s);
          s = fmaf(q[4 * d4 + 1], kk.y, s);
          s = fmaf(q[4 * d4 + 2], kk.z, s);
          s = fmaf(q[4 * d4 + 3], kk.w, s);
        }
        if (s > m) {
          float corr = expf(m - s);  // exp(-inf) = 0 on the first key
          l *= corr;
#pragma unroll
          for (int d = 0; d < MAXD; d++) o[d] *= corr;
          m = s;
        }
        float p = expf(s - m);
        l += p;
        const float4 *v4 = reinterpret_cast<const float4 *>(Vs + jj * MAXD);
#pragma unroll
        for (int d4 = 0; d4 < MAXD / 4; d4++) {
          float4 vv = v4[d4];
          o[4 * d4 + 0] = fmaf(p, vv.x, o[4 * d4 + 0]);
          o[4 * d4 + 1] = fmaf(p, vv.y, o[4 * d4 + 1]);
          o[4 * d4 + 2] = fmaf(p, vv.z, o[4 * d4 + 2]);
          o[4 * d4 + 3] = fmaf(p, vv.w, o[4 * d4 + 3]);
        }
      }
    }
  }
  if (valid) {
    const float il = 1.f / l;
#pragma unroll
    for (int d = 0; d < MAXD; d++)
      if (d < dH) O[(base + t) * qD + (int64_t)h * dH + d] = o[d] * il;
    lse[((int64_t)b * nH + h) * T + t] = m + logf(l);
  }
}

// Delta[b,h,t] = sum_d dO[t,h,d] * O[t,h,d]  (the rowsum(P * dP) of the JS).
__global__ void attn_delta_kernel(const float *__restrict__ dO, const float *__restrict__ O,
                                  int B, int T, int nH, int dH, float *__restrict__ delta) {
  fcu::pdl_trigger();
  int64_t rows = (int64_t)B * T * nH;
  int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (w >= rows) return;
  int64_t bt = w / nH;
  int h = (int)(w % nH);
  int b = (int)(bt / T), t = (int)(bt % T);
  const int64_t off = bt * (int64_t)nH * dH + (int64_t)h * dH;
  float s = 0.f;
  for (int d = lane; d < dH; d += 32) s += dO[off + d] * O[off + d];
  s = warp_sum(s);
  if (lane == 0) delta[((int64_t)b * nH + h) * T + t] = s;
}

// dK/dV: thread = key row j of kv head kvh.  K/V rows stay in padded shared
// memory (each thread reads its own row, conflict free); Q/dO tiles are
// broadcast from shared memory.
template <int MAXD>
__global__ void __launch_bounds__(kRows) attn_bwd_dkdv_kernel(
    const float *__restrict__ Q, const float *__restrict__ K, const float *__restrict__ V,
    const float *__restrict__ dO, const float *__restrict__ lse, const float *__restrict__ delta,
    int T, int nH, int nKV, int dH, float scale, float *__restrict__ dK, float *__restrict__ dV,
    int acc) {
  fcu::pdl_trigger();
  extern __shared__ float smem[];
  constexpr int P = MAXD + 1;
  float *Kown = smem;                    // [kRows][P]
  float *Vown = Kown + kRows * P;        // [kRows][P]
  float *Qs = Vown + kRows * P;          // [kRows][MAXD]
  float *dOs = Qs + kRows * MAXD;        // [kRows][MAXD]
  float *Ls = dOs + kRows * MAXD;        // [kRows]
  float *Ds = Ls + kRows;                // [kRows]
  const int b = blockIdx.z, kvh = blockIdx.y;
  const int group = nH / nKV;
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)nKV * dH;
  const int64_t base = (int64_t)b * T;
  const int j0 = blockIdx.x * kRows;
  const int j = j0 + threadIdx.x;
  const bool valid = j < T;

  for (int e = threadIdx.x; e < kRows * MAXD; e += kRows) {
    int jj = e / MAXD, d = e % MAXD;
    float kv = 0.f, vv = 0.f;
    if (j0 + jj < T && d < dH) {
      int64_t off = (base + j0 + jj) * kvD + (int64_t)kvh * dH + d;
      kv = K[off];
      vv = V[off];
    }
    Kown[jj * P + d] = kv;
    Vown[jj * P + d] = vv;
  }
  float dk[MAXD], dv[MAXD];
#pragma unroll
  for (int d = 0; d < MAXD; d++) dk[d] = dv[d] = 0.f;
  const float *kr = Kown + threadIdx.x * P;
  const float *vr = Vown + threadIdx.x * P;

  for (int h = kvh * group; h < (kvh + 1) * group; h++) {
    for (int i0 = j0; i0 < T; i0 += kRows) {
      __syncthreads();
      for (int e = threadIdx.x; e < kRows * MAXD; e += kRows) {
        int ii = e / MAXD, d = e % MAXD;
        float qv = 0.f, gv = 0.f;
        if (i0 + ii < T && d < dH) {
          int64_t off = (base + i0 + ii) * qD + (int64_t)h * dH + d;
          qv = Q[off];
          gv = dO[off];
        }
        Qs[e] = qv;
        dOs[e] = gv;
      }
      if (threadIdx.x < kRows) {
        int i = i0 + threadIdx.x;
        Ls[threadIdx.x] = i < T ? lse[((int64_t)b * nH + h) * T + i] : 0.f;
        Ds[threadIdx.x] = i < T ? delta[((int64_t)b * nH + h) * T + i] : 0.f;
      }
      __syncthreads();
      if (!valid) continue;
      const int in = min(kRows, T - i0);
      for (int ii = max(0, j - i0); ii < in; ii++) {  // causal: query i >= key j
        const float4 *q4 = reinterpret_cast<const float4 *>(Qs + ii * MAXD);
        const float4 *g4 = reinterpret_cast<const float4 *>(dOs + ii * MAXD);
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int d4 = 0; d4 < MAXD / 4; d4++) {
          float4 qq = q4[d4], gg = g4[d4];
          s = fmaf(qq.x, kr[4 * d4 + 0], s);
          s = fmaf(qq.y, kr[4 * d4 + 1], s);
          s = fmaf(qq.z, kr[4 * d4 + 2], s);
          s = fmaf(qq.w, kr[4 * d4 + 3], s);
          dp = fmaf(gg.x, vr[4 * d4 + 0], dp);
          dp = fmaf(gg.y, vr[4 * d4 + 1], dp);
          dp = fmaf(gg.z, vr[4 * d4 + 2], dp);
          dp = fmaf(gg.w, vr[4 * d4 + 3], dp);
        }
        const float p = expf(s * scale - Ls[ii]);
        const float ds = p * (dp - Ds[ii]) * scale;
#pragma unroll
        for (int d4 = 0; d4 < MAXD / 4; d4++) {
          float4 qq = q4[d4], gg = g4[d4];
          dv[4 * d4 + 0] = fmaf(p, gg.x, dv[4 * d4 + 0]);
          dv[4 * d4 + 1] = fmaf(p, gg.y, dv[4 * d4 + 1]);
          dv[4 * d4 + 2] = fmaf(p, gg.z, dv[4 * d4 + 2]);
          dv[4 * d4 + 3] = fmaf(p, gg.w, dv[4 * d4 + 3]);
          dk[4 * d4 + 0] = fmaf(ds, qq.x, dk[4 * d4 + 0]);
          dk[4 * d4 + 1] = fmaf(ds, qq.y, dk[4 * d4 + 1]);
          dk[4 * d4 + 2] = fmaf(ds, qq.z, dk[4 * d4 + 2]);
          dk[4 * d4 + 3] = fmaf(ds, qq.w, dk[4 * d4 + 3]);
        }
      }
    }
  }
  if (valid) {
    const int64_t off = (base + j) * kvD + (int64_t)kvh * dH;
#pragma unroll
    for (int d = 0; d < MAXD; d++) {
      if (d < dH) {
        dK[off + d] = acc ? dK[off + d] + dk[d] : dk[d];
        dV[off + d] = acc ? dV[off + d] + dv[d] : dv[d];
      }
    }
  }
}

// dQ: thread = query row t of head h; K/V tiles broadcast from shared memory,
// the thread's dO row in padded shared memory.
template <int MAXD>
__global__ void __launch_bounds__(kRows) attn_bwd_dq_kernel(
    const float *__restrict__ Q, const float *__restrict__ K, const float *__restrict__ V,
    const float *__restrict__ dO, const float *__restrict__ lse, const float *__restrict__ delta,
    int T, int nH, int nKV, int dH, float scale, float *__restrict__ dQ, int acc) {
  fcu::pdl_trigger();
  extern __shared__ float smem[];
  constexpr int P = MAXD + 1;
  float *Ks = smem;                  // [kRows][MAXD]
  float *Vs = Ks + kRows * MAXD;     // [kRows][MAXD]
  float *Gown = Vs + kRows * MAXD;   // [kRows][P]
  const int b = blockIdx.z, h = blockIdx.y;
  const int group = nH / nKV, kvh = h / group;
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)nKV * dH;
  const int64_t base = (int64_t)b * T;
  const int t0 = blockIdx.x * kRows;
  const int t = t0 + threadIdx.x;
  const bool valid = t < T;

  for (int e = threadIdx.x; e < kRows * MAXD; e += kRows) {
    int ii = e / MAXD, d = e % MAXD;
    Gown[ii * P + d] = (t0 + ii < T && d < dH) ? dO[(base + t0 + ii) * qD + (int64_t)h * dH + d] : 0.f;
  }
  float q[MAXD], dq[MAXD];
#pragma unroll
  for (int d = 0; d < MAXD; d++) {
    q[d] = (valid && d < dH) ? Q[(base + t) * qD + (int64_t)h * dH + d] : 0.f;
    dq[d] = 0.f;
  }
  const float L = valid ? lse[((int64_t)b * nH + h) * T + t] : 0.f;
  const float Dl = valid ? delta[((int64_t)b * nH + h) * T + t] : 0.f;
  const float *gr = Gown + threadIdx.x * P;
  const int last = min(T - 1, t0 + kRows - 1);
  for (int j0 = 0; j0 <= last; j0 += kRows) {
    __syncthreads();
    for (int e = threadIdx.x; e < kRows * MAXD; e += kRows) {
      int jj = e / MAXD, d = e % MAXD;
      float kv = 0.f, vv = 0.f;
      if (j0 + jj < T && d < dH) {
        int64_t off = (base + j0 + jj) * kvD + (int64_t)kvh * dH + d;
        kv = K[off];
        vv = V[off];
      }
      Ks[e] = kv;
      Vs[e] = vv;
    }
    __syncthreads();
    if (!valid) continue;
    const int jn = min(kRows, t - j0 + 1);
    for (int jj = 0; jj < jn; jj++) {
      const float4 *k4 = reinterpret_cast<const float4 *>(Ks + jj * MAXD);
      const float4 *v4 = reinterpret_cast<const float4 *>(Vs + jj * MAXD);
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d4 = 0; d4 < MAXD / 4; d4++) {
        float4 kk = k4[d4], vv = v4[d4];
        s = fmaf(q[4 * d4 + 0], kk.x, s);
        s = fmaf(q[4 * d4 + 1], kk.y, s);
        s = fmaf(q[4 * d4 + 2], kk.z, s);
        s = fmaf(q[4 * d4 + 3], kk.w, s);
        dp = fmaf(gr[4 * d4 + 0], vv.x, dp);
        dp = fmaf(gr[4 * d4 + 1], vv.y, dp);
        dp = fmaf(gr[4 * d4 + 2], vv.z, dp);
        dp = fmaf(gr[4 * d4 + 3], vv.w, dp);
      }
      const float p = expf(s * scale - L);
      const float ds = p * (dp - Dl) * scale;
#pragma unroll
      for (int d4 = 0; d4 < MAXD / 4; d4++) {
        float4 kk = k4[d4];
        dq[4 * d4 + 0] = fmaf(ds, kk.x, dq[4 * d4 + 0]);
        dq[4 * d4 + 1] = fmaf(ds, kk.y, dq[4 * d4 + 1]);
        dq[4 * d4 + 2] = fmaf(ds, kk.z, dq[4 * d4 + 2]);
        dq[4 * d4 + 3] = fmaf(ds, kk.w, dq[4 * d4 + 3]);
      }
    }
  }
  if (valid) {
    const int64_t off = (base + t) * qD + (int64_t)h * dH;
#pragma unroll
    for (int d = 0; d < MAXD; d++)
      if (d < dH) dQ[off + d] = acc ? dQ[off + d] + dq[d] : dq[d];
  }
}

template <int MAXD>
int attn_fwd_launch(cudaStream_t st, const float *Q, const float *K, const float *V, int B, int T,
                    int nH, int nKV, int dH, float *O, float *lse) {
  size_t smem = sizeof(float) * 2 * kRows * MAXD;
  if (smem > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_kernel<MAXD>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(fcu::div_up(T, kRows), nH, B);
  attn_fwd_kernel<MAXD><<<grid, kRows, smem, st>>>(Q, K, V, T, nH, nKV, dH,
                                                   (float)(1.0 / sqrt((double)dH)), O, lse);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

template <int MAXD>
int attn_bwd_launch(cudaStream_t st, const float *dO, const float *Q, const float *K,
                    const float *V, const float *lse, const float *delta, int B, int T, int nH,
                    int nKV, int dH, float *dQ, float *dK, float *dV, int acc) {
  const float scale = (float)(1.0 / sqrt((double)dH));
  size_t smem_kv = sizeof(float) * (2 * kRows * (MAXD + 1) + 2 * kRows * MAXD + 2 * kRows);
  if (smem_kv > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_kernel<MAXD>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_kv));
  dim3 gkv(fcu::div_up(T, kRows), nKV, B);
  attn_bwd_dkdv_kernel<MAXD><<<gkv, kRows, smem_kv, st>>>(Q, K, V, dO, lse, delta, T, nH, nKV, dH,
                                                          scale, dK, dV, acc);
  FCU_CHECK_LAUNCH();
  size_t smem_q = sizeof(float) * (2 * kRows * MAXD + kRows * (MAXD + 1));
  if (smem_q > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dq_kernel<MAXD>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_q));
  dim3 gq(fcu::div_up(T, kRows), nH, B);
  attn_bwd_dq_kernel<MAXD><<<gq, kRows, smem_q, st>>>(Q, K, V, dO, lse, delta, T, nH, nKV, dH,
                                                       scale, dQ, acc);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int check_attn_args(int B, int T, int nH, int nKV, int dH) {
  FCU_REQUIRE(B > 0 && T > 0 && nH > 0 && nKV > 0 && dH > 0,
              "fcu_attn: bad shape B=%d T=%d nH=%d nKV=%d dH=%d", B, T, nH, nKV, dH);
  FCU_REQUIRE(nH % nKV == 0, "fcu_attn: nH (%d) must be a multiple of nKV (%d)", nH, nKV);
  FCU_REQUIRE(dH <= 128, "fcu_attn: dH=%d above the supported 128", dH);
  FCU_REQUIRE(nH <= 65535 && B <= 65535, "fcu_attn: grid limits");
  return FCU_OK;
}

}  // namespace

extern "C" {

int fcu_attn_fwd(fcu_ctx *ctx, const float *Q, const float *K, const float *V, int B, int T,
                 int nH, int nKV, int dH, float *O, float *lse) {
  FCU_CTX(ctx);
  int rc = check_attn_args(B, T, nH, nKV, dH);
  if (rc) return rc;
  FCU_REQUIRE(Q && K && V && O && lse, "fcu_attn_fwd: null pointer");
  cudaStream_t st = ctx->stream;
  if (ctx->precision == FCU_PREC_BF16 && fcu::attn_tmem_op_supported(dH, Q, K, V, O))
    return fcu::attn_fwd_op_tmem(ctx, Q, K, V, B, T, nH, nKV, dH, O, lse);
  if (ctx->precision == FCU_PREC_BF16 && fcu::attn_tc_supported(dH, Q, K, V))
    return fcu::attn_fwd_tc(st, Q, K, V, B, T, nH, nKV, dH, O, lse);
  if (dH <= 16) return attn_fwd_launch<16>(st, Q, K, V, B, T, nH, nKV, dH, O, lse);
  if (dH <= 32) return attn_fwd_launch<32>(st, Q, K, V, B, T, nH, nKV, dH, O, lse);
  if (dH <= 64) return attn_fwd_launch<64>(st, Q, K, V, B, T, nH, nKV, dH, O, lse);
  return attn_fwd_launch<128>(st, Q, K, V, B, T, nH, nKV, dH, O, lse);
}

int fcu_attn_bwd(fcu_ctx *ctx, const float *dO, const float *Q, const float *K, const float *V,
                 const float *O, const float *lse, int B, int T, int nH, int nKV, int dH, float *dQ,
                 float *dK, float *dV, int accumulate) {
  FCU_CTX(ctx);
  int rc = check_attn_args(B, T, nH, nKV, dH);
  if (rc) return rc;
  FCU_REQUIRE(dO && Q && K && V && O && lse && dQ && dK && dV, "fcu_attn_bwd: null pointer");
  if (ctx->precision == FCU_PREC_BF16 && fcu::attn_tmem_op_supported(dH, Q, K, V, O) &&
      fcu::attn_tmem_op_supported(dH, dO, dQ, dK, dV))
    return fcu::attn_bwd_op_tmem(ctx, dO, Q, K, V, O, lse, B, T, nH, nKV, dH, dQ, dK, dV, accumulate);
  void *scr = nullptr;
  rc = fcu::ctx_scratch(ctx, sizeof(float) * (size_t)B * nH * T, &scr);
  if (rc) return rc;
  float *delta = (float *)scr;
  int64_t rows = (int64_t)B * T * nH;
  attn_delta_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, ctx->stream>>>(dO, O, B, T, nH, dH,
                                                                                  delta);
  FCU_CHECK_LAUNCH();
  cudaStream_t st = ctx->stream;
  if (ctx->precision == FCU_PREC_BF16 && fcu::attn_tc_supported(dH, Q, K, V) &&
      (((uintptr_t)dO | (uintptr_t)dQ | (uintptr_t)dK | (uintptr_t)dV) & 15) == 0)
    return fcu::attn_bwd_tc(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dH, dQ, dK, dV, accumulate);
  if (dH <= 16)
    return attn_bwd_launch<16>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dH, dQ, dK, dV, accumulate);
  if (dH <= 32)
    return attn_bwd_launch<32>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dH, dQ, dK, dV, accumulate);
  if (dH <= 64)
    return attn_bwd_launch<64>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dH, dQ, dK, dV, accumulate);
  return attn_bwd_launch<128>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dH, dQ, dK, dV, accumulate);
}

}  // extern "C"
