// Causal GQA flash attention on the tensor cores (bf16 operands, fp32
// softmax and accumulation), used in FCU_PREC_BF16 mode.
//
// Same contract as attn.cu (causalAttn / causalAttnBatch, src/L2/tensor.js:
// 191-268 and 299-376): fp32 Q/K/V/O in HBM, lse per score row kept for the
// backward.  Operands are rounded to bf16 as they are staged in shared
// memory; scores, the online softmax, P.V and all gradients accumulate in
// fp32 registers through m16n8k16 tensor-core MMAs (FlashAttention-2 tiling:
// 4 warps x 16 query rows, 64-key tiles; P and dS are re-used from the
// accumulator registers as the A operand of the next product).
//
// Backward is two deterministic kernels (no atomics):
//   dK/dV: a CTA owns 64 keys of one kv head and sweeps the group's q heads
//          and every later query tile, computing S^T, P^T, dP^T, dS^T with
//          keys as rows; dV += P^T dO, dK += dS^T Q.
//   dQ   : a CTA owns 64 queries and sweeps every earlier key tile; dQ += dS K.
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"

namespace fcu {
namespace {

constexpr int kTile = 64;       // query rows and key rows per tile
constexpr int kWarps = 4;       // 16 rows per warp
constexpr int kThreads = kWarps * 32;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Smem {
  static constexpr int LD = D + 8;  // bf16 row stride: +16 B keeps ldmatrix conflict free
  static constexpr int TILE = kTile * LD;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// D[16x8] += A[16x16] . B[16x8], bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3},"
      " {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// Stage rows [r0, r0+64) of one head (columns [col0, col0+D)) of an fp32
// matrix with row stride ld into a bf16 tile; rows >= nrows are zero.
template <int D>
__device__ __forceinline__ void stage_tile(__nv_bfloat16 *dst, const float *__restrict__ src,
                                           int64_t row_base, int r0, int nrows, int64_t ld,
                                           int64_t col0) {
  constexpr int LD = Smem<D>::LD;
  constexpr int V4 = D / 4;
  for (int e = threadIdx.x; e < kTile * V4; e += kThreads) {
    const int r = e / V4, c = (e % V4) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < nrows)
      v = *reinterpret_cast<const float4 *>(src + (row_base + r0 + r) * ld + col0 + c);
    uint2 o;
    o.x = pack_bf16(v.x, v.y);
    o.y = pack_bf16(v.z, v.w);
    *reinterpret_cast<uint2 *>(dst + r * LD + c) = o;
  }
}

// A fragments (16 rows x D) of rows [row0, row0+16) of a staged tile.
template <int D>
__device__ __forceinline__ void load_a_frags(uint32_t (&f)[D / 16][4], const __nv_bfloat16 *tile,
                                             int row0, int lane) {
  constexpr int LD = Smem<D>::LD;
#pragma unroll
  for (int kb = 0; kb < D / 16; kb++)
    ldsm_x4(f[kb], tile + (row0 + (lane & 15)) * LD + kb * 16 + (lane >> 4) * 8);
}

// acc[16 x 64] = A[16 x D] . T^T where T is a staged [64 x D] tile (rows of T
// are the 64 output columns): the S = Q K^T / dP = dO V^T pattern.
template <int D>
__device__ __forceinline__ void mm_abt(float (&acc)[8][4], const uint32_t (&a)[D / 16][4],
                                       const __nv_bfloat16 *tile, int lane) {
  constexpr int LD = Smem<D>::LD;
#pragma unroll
  for (int j = 0; j < 8; j++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[j][i] = 0.f;
#pragma unroll
  for (int kb = 0; kb < D / 16; kb++) {
#pragma unroll
    for (int np = 0; np < 4; np++) {  // pairs of 8-column blocks
      uint32_t b[4];
      ldsm_x4(b, tile + (np * 16 + (lane >> 4) * 8 + (lane & 7)) * LD + kb * 16 +
                     ((lane >> 3) & 1) * 8);
      mma16816(acc[2 * np], a[kb], b[0], b[1]);
      mma16816(acc[2 * np + 1], a[kb], b[2], b[3]);
    }
  }
}

// acc[16 x D] += P[16 x 64] . T where T is a staged [64 x D] tile (rows of T
// are the contraction index): the O += P V / dV += P^T dO pattern.  P comes
// from accumulator registers (8 column blocks of 16 x 8).
template <int D>
__device__ __forceinline__ void mm_pt(float (&acc)[D / 8][4], const float (&p)[8][4],
                                      const __nv_bfloat16 *tile, int lane) {
  constexpr int LD = Smem<D>::LD;
#pragma unroll
  for (int kb = 0; kb < 4; kb++) {  // 16 contraction rows per step
    uint32_t a[4];
    a[0] = pack_bf16(p[2 * kb][0], p[2 * kb][1]);
    a[1] = pack_bf16(p[2 * kb][2], p[2 * kb][3]);
    a[2] = pack_bf16(p[2 * kb + 1][0], p[2 * kb + 1][1]);
    a[3] = pack_bf16(p[2 * kb + 1][2], p[2 * kb + 1][3]);
#pragma unroll
    for (int np = 0; np < D / 16; np++) {
      uint32_t b[4];
      ldsm_x4_t(b, tile + (kb * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + np * 16 +
                       (lane >> 4) * 8);
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// ------------------------------------------------------------------ forward
template <int D>
__global__ void __launch_bounds__(kThreads) attn_fwd_tc_kernel(
    const float *__restrict__ Q, const float *__restrict__ K, const float *__restrict__ V, int T,
    int nH, int nKV, float scale, float *__restrict__ O, float *__restrict__ lse) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sK = sQ + Smem<D>::TILE;
  __nv_bfloat16 *sV = sK + Smem<D>::TILE;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (nH / nKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t qD = (int64_t)nH * D, kvD = (int64_t)nKV * D, base = (int64_t)b * T;
  const int q0 = qt * kTile;
  const float c = scale * kLog2e;

  stage_tile<D>(sQ, Q, base, q0, T, qD, (int64_t)h * D);
  __syncthreads();
  uint32_t qf[D / 16][4];
  load_a_frags<D>(qf, sQ, warp * 16, lane);

  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; j++)
#pragma unroll
    for (int i = 0; i < 4; i++) o[j][i] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int row[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};

  for (int kt = 0; kt <= qt; kt++) {
    const int k0 = kt * kTile;
    __syncthreads();
    stage_tile<D>(sK, K, base, k0, T, kvD, (int64_t)kvh * D);
    stage_tile<D>(sV, V, base, k0, T, kvD, (int64_t)kvh * D);
    __syncthreads();
    float s[8][4];
    mm_abt<D>(s, qf, sK, lane);
    float mx[2] = {m[0], m[1]};
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int key = k0 + j * 8 + 2 * t4 + (i & 1);
        const int r = i >> 1;
        float v = s[j][i] * c;
        if (key > row[r] || key >= T) v = -INFINITY;
        s[j][i] = v;
        mx[r] = fmaxf(mx[r], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; r++) corr[r] = (mx[r] == -INFINITY) ? 1.f : exp2f(m[r] - mx[r]);
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int r = i >> 1;
        float p = (mx[r] == -INFINITY) ? 0.f : exp2f(s[j][i] - mx[r]);
        s[j][i] = p;
        rs[r] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l[r] = l[r] * corr[r] + rs[r];
      m[r] = mx[r];
    }
#pragma unroll
    for (int j = 0; j < D / 8; j++) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    mm_pt<D>(o, s, sV, lane);
  }
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if (row[r] >= T) continue;
    const float il = 1.f / l[r];
    float *orow = O + (base + row[r]) * qD + (int64_t)h * D;
#pragma unroll
    for (int j = 0; j < D / 8; j++) {
      float2 v = make_float2(o[j][2 * r] * il, o[j][2 * r + 1] * il);
      *reinterpret_cast<float2 *>(orow + j * 8 + 2 * t4) = v;
    }
    if (t4 == 0) lse[((int64_t)b * nH + h) * T + row[r]] = (m[r] + log2f(l[r])) / kLog2e;
  }
}

// ------------------------------------------------------------------ backward dK dV
template <int D>
__global__ void __launch_bounds__(kThreads) attn_bwd_dkdv_tc_kernel(
    const float *__restrict__ Q, const float *__restrict__ K, const float *__restrict__ V,
    const float *__restrict__ dO, const float *__restrict__ lse, const float *__restrict__ delta,
    int T, int nH, int nKV, float scale, float *__restrict__ dK, float *__restrict__ dV, int acc) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16 *sK = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sV = sK + Smem<D>::TILE;
  __nv_bfloat16 *sQ = sV + Smem<D>::TILE;
  __nv_bfloat16 *sG = sQ + Smem<D>::TILE;
  float *sL = reinterpret_cast<float *>(sG + Smem<D>::TILE);
  float *sD = sL + kTile;
  const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = nH / nKV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t qD = (int64_t)nH * D, kvD = (int64_t)nKV * D, base = (int64_t)b * T;
  const int k0 = kt * kTile;
  const float c = scale * kLog2e;

  stage_tile<D>(sK, K, base, k0, T, kvD, (int64_t)kvh * D);
  stage_tile<D>(sV, V, base, k0, T, kvD, (int64_t)kvh * D);
  __syncthreads();
  uint32_t kf[D / 16][4], vf[D / 16][4];
  load_a_frags<D>(kf, sK, warp * 16, lane);
  load_a_frags<D>(vf, sV, warp * 16, lane);
  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; j++)
#pragma unroll
    for (int i = 0; i < 4; i++) dk[j][i] = dv[j][i] = 0.f;
  const int key[2] = {k0 + warp * 16 + g, k0 + warp * 16 + g + 8};
  const int ntiles = (T + kTile - 1) / kTile;

  for (int h = kvh * group; h < (kvh + 1) * group; h++) {
    for (int qt = kt; qt < ntiles; qt++) {
      const int q0 = qt * kTile;
      __syncthreads();
      stage_tile<D>(sQ, Q, base, q0, T, qD, (int64_t)h * D);
      stage_tile<D>(sG, dO, base, q0, T, qD, (int64_t)h * D);
      for (int i = threadIdx.x; i < kTile; i += kThreads) {
        const int q = q0 + i;
        sL[i] = q < T ? lse[((int64_t)b * nH + h) * T + q] * kLog2e : 0.f;
        sD[i] = q < T ? delta[((int64_t)b * nH + h) * T + q] : 0.f;
      }
      __syncthreads();
      float st[8][4], dpt[8][4];
      mm_abt<D>(st, kf, sQ, lane);   // S^T: keys x queries
      mm_abt<D>(dpt, vf, sG, lane);  // dP^T = V dO^T
#pragma unroll
      for (int j = 0; j < 8; j++) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int qi = j * 8 + 2 * t4 + (i & 1);
          const int q = q0 + qi;
          const int r = i >> 1;
          float p = 0.f;
          if (q < T && q >= key[r]) p = exp2f(st[j][i] * c - sL[qi]);
          st[j][i] = p;
          dpt[j][i] = p * (dpt[j][i] - sD[qi]);
        }
      }
      mm_pt<D>(dv, st, sG, lane);   // dV += P^T dO
      mm_pt<D>(dk, dpt, sQ, lane);  // dK += dS^T Q
    }
  }
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if (key[r] >= T) continue;
    const int64_t off = (base + key[r]) * kvD + (int64_t)kvh * D;
#pragma unroll
    for (int j = 0; j < D / 8; j++) {
      float2 *pk = reinterpret_cast<float2 *>(dK + off + j * 8 + 2 * t4);
      float2 *pv = reinterpret_cast<float2 *>(dV + off + j * 8 + 2 * t4);
      float2 vk = make_float2(dk[j][2 * r] * scale, dk[j][2 * r + 1] * scale);
      float2 vv = make_float2(dv[j][2 * r], dv[j][2 * r + 1]);
      if (acc) {
        float2 ok = *pk, ov = *pv;
        vk.x += ok.x;
        vk.y += ok.y;
        vv.x += ov.x;
        vv.y += ov.y;
      }
      *pk = vk;
      *pv = vv;
    }
  }
}

// ------------------------------------------------------------------ backward dQ
template <int D>
__global__ void __launch_bounds__(kThreads) attn_bwd_dq_tc_kernel(
    const float *__restrict__ Q, const float *__restrict__ K, const float *__restrict__ V,
    const float *__restrict__ dO, const float *__restrict__ lse, const float *__restrict__ delta,
    int T, int nH, int nKV, float scale, float *__restrict__ dQ, int acc) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sG = sQ + Smem<D>::TILE;
  __nv_bfloat16 *sK = sG + Smem<D>::TILE;
  __nv_bfloat16 *sV = sK + Smem<D>::TILE;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (nH / nKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t qD = (int64_t)nH * D, kvD = (int64_t)nKV * D, base = (int64_t)b * T;
  const int q0 = qt * kTile;
  const float c = scale * kLog2e;

  stage_tile<D>(sQ, Q, base, q0, T, qD, (int64_t)h * D);
  stage_tile<D>(sG, dO, base, q0, T, qD, (int64_t)h * D);
  __syncthreads();
  uint32_t qf[D / 16][4], gf[D / 16][4];
  load_a_frags<D>(qf, sQ, warp * 16, lane);
  load_a_frags<D>(gf, sG, warp * 16, lane);
  const int row[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};
  float L[2], Dl[2];
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const bool ok = row[r] < T;
    L[r] = ok ? lse[((int64_t)b * nH + h) * T + row[r]] * kLog2e : 0.f;
    Dl[r] = ok ? delta[((int64_t)b * nH + h) * T + row[r]] : 0.f;
  }
  float dq[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; j++)
#pragma unroll
    for (int i = 0; i < 4; i++) dq[j][i] = 0.f;

  for (int kt = 0; kt <= qt; kt++) {
    const int k0 = kt * kTile;
    __syncthreads();
    stage_tile<D>(sK, K, base, k0, T, kvD, (int64_t)kvh * D);
    stage_tile<D>(sV, V, base, k0, T, kvD, (int64_t)kvh * D);
    __syncthreads();
    float s[8][4], dp[8][4];
    mm_abt<D>(s, qf, sK, lane);
    mm_abt<D>(dp, gf, sV, lane);
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int key = k0 + j * 8 + 2 * t4 + (i & 1);
        const int r = i >> 1;
        float p = 0.f;
        if (row[r] < T && key <= row[r]) p = exp2f(s[j][i] * c - L[r]);
        dp[j][i] = p * (dp[j][i] - Dl[r]);
      }
    }
    mm_pt<D>(dq, dp, sK, lane);  // dQ += dS K
  }
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if (row[r] >= T) continue;
    float *qrow = dQ + (base + row[r]) * qD + (int64_t)h * D;
#pragma unroll
    for (int j = 0; j < D / 8; j++) {
      float2 *p = reinterpret_cast<float2 *>(qrow + j * 8 + 2 * t4);
      float2 v = make_float2(dq[j][2 * r] * scale, dq[j][2 * r + 1] * scale);
      if (acc) {
        float2 o = *p;
        v.x += o.x;
        v.y += o.y;
      }
      *p = v;
    }
  }
}

template <int D>
int fwd_launch(cudaStream_t st, const float *Q, const float *K, const float *V, int B, int T,
               int nH, int nKV, float *O, float *lse) {
  const size_t smem = 3 * sizeof(__nv_bfloat16) * Smem<D>::TILE;
  if (smem > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel<D>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(div_up(T, kTile), nH, B);
  attn_fwd_tc_kernel<D><<<grid, kThreads, smem, st>>>(Q, K, V, T, nH, nKV,
                                                      (float)(1.0 / sqrt((double)D)), O, lse);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

template <int D>
int bwd_launch(cudaStream_t st, const float *dO, const float *Q, const float *K, const float *V,
               const float *lse, const float *delta, int B, int T, int nH, int nKV, float *dQ,
               float *dK, float *dV, int acc) {
  const float scale = (float)(1.0 / sqrt((double)D));
  const size_t smem_kv = 4 * sizeof(__nv_bfloat16) * Smem<D>::TILE + 2 * kTile * sizeof(float);
  const size_t smem_q = 4 * sizeof(__nv_bfloat16) * Smem<D>::TILE;
  if (smem_kv > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel<D>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_kv));
  if (smem_q > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<D>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_q));
  dim3 gkv(div_up(T, kTile), nKV, B);
  attn_bwd_dkdv_tc_kernel<D><<<gkv, kThreads, smem_kv, st>>>(Q, K, V, dO, lse, delta, T, nH, nKV,
                                                              scale, dK, dV, acc);
  FCU_CHECK_LAUNCH();
  dim3 gq(div_up(T, kTile), nH, B);
  attn_bwd_dq_tc_kernel<D><<<gq, kThreads, smem_q, st>>>(Q, K, V, dO, lse, delta, T, nH, nKV, scale,
                                                          dQ, acc);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // namespace

bool attn_tc_supported(int dH, const void *Q, const void *K, const void *V) {
  if (dH != 16 && dH != 32 && dH != 64 && dH != 128) return false;
  return (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V) & 15) == 0;
}

int attn_fwd_tc(cudaStream_t st, const float *Q, const float *K, const float *V, int B, int T,
                int nH, int nKV, int dH, float *O, float *lse) {
  switch (dH) {
    case 16: return fwd_launch<16>(st, Q, K, V, B, T, nH, nKV, O, lse);
    case 32: return fwd_launch<32>(st, Q, K, V, B, T, nH, nKV, O, lse);
    case 64: return fwd_launch<64>(st, Q, K, V, B, T, nH, nKV, O, lse);
    case 128: return fwd_launch<128>(st, Q, K, V, B, T, nH, nKV, O, lse);
  }
  set_error("attn_fwd_tc: unsupported head dim %d", dH);
  return FCU_ERR_ARG;
}

int attn_bwd_tc(cudaStream_t st, const float *dO, const float *Q, const float *K, const float *V,
                const float *lse, const float *delta, int B, int T, int nH, int nKV, int dH,
                float *dQ, float *dK, float *dV, int acc) {
  switch (dH) {
    case 16: return bwd_launch<16>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dQ, dK, dV, acc);
    case 32: return bwd_launch<32>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dQ, dK, dV, acc);
    case 64: return bwd_launch<64>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dQ, dK, dV, acc);
    case 128: return bwd_launch<128>(st, dO, Q, K, V, lse, delta, B, T, nH, nKV, dQ, dK, dV, acc);
  }
  set_error("attn_bwd_tc: unsupported head dim %d", dH);
  return FCU_ERR_ARG;
}

}  // namespace fcu
