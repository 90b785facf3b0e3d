// Causal GQA flash attention on the tensor cores (bf16 operands, fp32
// softmax and accumulation).
//
// Same contract as attn.cu (causalAttn / causalAttnBatch, src/L2/tensor.js:
// 191-268 and 299-376): lse per score row is kept for the backward instead of
// the JS's P.  Operands are bf16 in shared memory; scores, the online softmax,
// P.V and all gradients accumulate in fp32 registers through m16n8k16
// tensor-core MMAs (FlashAttention-2 tiling: 4 warps x 16 rows, 64-key tiles;
// P and dS are re-used from the accumulator registers as the A operand of the
// next product).
//
// These mma.sync kernels serve the op-level API (fp32 tensors, rounded to
// bf16 while staged) when its operands cannot take the tcgen05 path of
// attn_tmem.cu (a tensor that is not 16-byte aligned).  The fused model
// path's bf16 entries at the end of this file validate their operands and
// always run the tcgen05 kernels.  The templates also take bf16 tensors read
// straight out of one [N, (nH+2nKV)*dH] qkv buffer by row stride and column
// offset (O and dQ/dK/dV written in bf16, the RoPE backward R^T,
// src/L2/tensor.js:150-165, applied to dQ and dK on the way out); no entry
// instantiates that flavour now.
//
// Backward is two deterministic kernels (no atomics):
//   dK/dV: a CTA owns 64 keys of one kv head and sweeps the group's q heads
//          and every later query tile (S^T, P^T, dP^T, dS^T with keys as
//          rows); dV += P^T dO, dK += dS^T Q.
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

// A [rows, heads*D] tensor inside a wider row-major buffer: element
// (row r, head h, dim d) lives at p[r*ld + col + h*D + d].
template <typename T>
struct View {
  T *p;
  int64_t ld;
  int64_t col;
};

struct Args {
  View<const void> q, k, v, o_in, dO;   // inputs (o_in: the forward output, for delta)
  View<void> o, dq, dk, dv;             // outputs
  float *lse;
  const float *delta;
  const float2 *rope;                   // (cos, sin) [T][D/2] for the RoPE backward, or null
  int T, nH, nKV;
  float scale;
  int acc;                              // fp32 outputs: accumulate
  // dK/dV with one CTA per (key tile, q head) instead of per (key tile, kv
  // head): each writes fp32 partials pk/pv [group][B*T][nKV*D] that
  // attn_kv_reduce_kernel sums over the group in order (small grids only).
  int split_heads;
  float *pk, *pv;
  int64_t rows;                         // B*T
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

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Stage rows [r0, r0+64) of head `h` of view `src` (rows of sequence base
// `row_base`; rows >= nrows are zero) into a bf16 tile.  fp32 sources are
// converted through registers; bf16 sources are copied with cp.async (the
// caller commits and waits).
template <int D, typename TI>
__device__ __forceinline__ void stage(__nv_bfloat16 *dst, View<const void> src, int64_t row_base,
                                      int r0, int nrows, int h) {
  constexpr int LD = Smem<D>::LD;
  if constexpr (sizeof(TI) == 4) {
    const float *s = reinterpret_cast<const float *>(src.p);
    constexpr int V4 = D / 4;
    for (int e = threadIdx.x; e < kTile * V4; e += kThreads) {
      const int r = e / V4, c = (e % V4) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r0 + r < nrows)
        v = *reinterpret_cast<const float4 *>(s + (row_base + r0 + r) * src.ld + src.col + (int64_t)h * D + c);
      uint2 o;
      o.x = pack_bf16(v.x, v.y);
      o.y = pack_bf16(v.z, v.w);
      *reinterpret_cast<uint2 *>(dst + r * LD + c) = o;
    }
  } else {
    const __nv_bfloat16 *s = reinterpret_cast<const __nv_bfloat16 *>(src.p);
    constexpr int C8 = D / 8;
    for (int e = threadIdx.x; e < kTile * C8; e += kThreads) {
      const int r = e / C8, c = (e % C8) * 8;
      const bool ok = r0 + r < nrows;
      const __nv_bfloat16 *g = ok ? s + (row_base + r0 + r) * src.ld + src.col + (int64_t)h * D + c : s;
      cp_async16(dst + r * LD + c, g, ok);
    }
  }
}

template <typename TI>
__device__ __forceinline__ void stage_done() {
  if constexpr (sizeof(TI) == 2) {
    cp_async_commit();
    cp_async_wait_all();
  }
  __syncthreads();
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

// Store one accumulator row fragment (16 rows x D, this thread's two rows)
// of head h: fp32 (optionally accumulating) or bf16, optionally rotated back
// by R^T (pairs (2i, 2i+1) of the head, position row % T).
template <int D, typename TO>
__device__ __forceinline__ void store_rows(View<void> dst, const float (&a)[D / 8][4],
                                           const int (&row)[2], int64_t base, int h, int T,
                                           float mul, int acc, const float2 *rope, int t4) {
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if (row[r] >= T) continue;
    const int64_t off = (base + row[r]) * dst.ld + dst.col + (int64_t)h * D;
#pragma unroll
    for (int j = 0; j < D / 8; j++) {
      float x = a[j][2 * r] * mul, y = a[j][2 * r + 1] * mul;
      if (rope) {
        const float2 cs = rope[(int64_t)row[r] * (D / 2) + j * 4 + t4];
        const float u = x * cs.x + y * cs.y, w = -x * cs.y + y * cs.x;
        x = u;
        y = w;
      }
      const int64_t e = off + j * 8 + 2 * t4;
      if constexpr (sizeof(TO) == 4) {
        float2 *p = reinterpret_cast<float2 *>(reinterpret_cast<float *>(dst.p) + e);
        float2 v = make_float2(x, y);
        if (acc) {
          const float2 o = *p;
          v.x += o.x;
          v.y += o.y;
        }
        *p = v;
      } else {
        *reinterpret_cast<uint32_t *>(reinterpret_cast<__nv_bfloat16 *>(dst.p) + e) = pack_bf16(x, y);
      }
    }
  }
}

// ------------------------------------------------------------------ forward
template <int D, typename TI, typename TO>
__global__ void __launch_bounds__(kThreads) attn_fwd_tc_kernel(Args A) {
  fcu::pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  constexpr bool kAsync = sizeof(TI) == 2;
  __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sK[2] = {sQ + Smem<D>::TILE, sQ + 3 * Smem<D>::TILE};
  __nv_bfloat16 *sV[2] = {sQ + 2 * Smem<D>::TILE, sQ + 4 * Smem<D>::TILE};
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = A.T, kvh = h / (A.nH / A.nKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t base = (int64_t)b * T;
  const int q0 = qt * kTile;
  const float c = A.scale * kLog2e;

  stage<D, TI>(sQ, A.q, base, q0, T, h);
  stage<D, TI>(sK[0], A.k, base, 0, T, kvh);
  stage<D, TI>(sV[0], A.v, base, 0, T, kvh);
  stage_done<TI>();
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
    const int buf = kAsync ? (kt & 1) : 0;
    if (kt > 0 && !kAsync) {
      __syncthreads();
      stage<D, TI>(sK[0], A.k, base, kt * kTile, T, kvh);
      stage<D, TI>(sV[0], A.v, base, kt * kTile, T, kvh);
      __syncthreads();
    }
    if (kAsync && kt < qt) {  // prefetch the next tile into the other buffer
      stage<D, TI>(sK[buf ^ 1], A.k, base, (kt + 1) * kTile, T, kvh);
      stage<D, TI>(sV[buf ^ 1], A.v, base, (kt + 1) * kTile, T, kvh);
      cp_async_commit();
    }
    const int k0 = kt * kTile;
    float s[8][4];
    mm_abt<D>(s, qf, sK[buf], lane);
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
    mm_pt<D>(o, s, sV[buf], lane);
    if (kAsync) {
      cp_async_wait_all();
      __syncthreads();  // next tile landed; everyone is done with this one
    }
  }
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const float il = 1.f / l[r];
#pragma unroll
    for (int j = 0; j < D / 8; j++) {
      o[j][2 * r] *= il;
      o[j][2 * r + 1] *= il;
    }
    if (row[r] < T && t4 == 0)
      A.lse[((int64_t)b * A.nH + h) * T + row[r]] = (m[r] + log2f(l[r])) / kLog2e;
  }
  store_rows<D, TO>(A.o, o, row, base, h, T, 1.f, 0, nullptr, t4);
}

// ------------------------------------------------------------------ backward dK dV
template <int D, typename TI, typename TO>
__global__ void __launch_bounds__(kThreads) attn_bwd_dkdv_tc_kernel(Args A) {
  fcu::pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  constexpr bool kAsync = sizeof(TI) == 2;
  __nv_bfloat16 *sK = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sV = sK + Smem<D>::TILE;
  __nv_bfloat16 *sQ[2] = {sV + Smem<D>::TILE, sV + 3 * Smem<D>::TILE};
  __nv_bfloat16 *sG[2] = {sV + 2 * Smem<D>::TILE, sV + 4 * Smem<D>::TILE};
  float *sL = reinterpret_cast<float *>(sV + 5 * Smem<D>::TILE);  // [2][kTile]
  float *sD = sL + 2 * kTile;                                     // [2][kTile]
  const int kt = blockIdx.x, b = blockIdx.z;
  const int T = A.T, nH = A.nH, group = nH / A.nKV;
  const int kvh = A.split_heads ? (int)blockIdx.y / group : (int)blockIdx.y;
  const int h_begin = A.split_heads ? (int)blockIdx.y : kvh * group;
  const int n_heads = A.split_heads ? 1 : group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t base = (int64_t)b * T;
  const int k0 = kt * kTile;
  const float c = A.scale * kLog2e;
  const int ntiles = (T + kTile - 1) / kTile;
  const int per_head = ntiles - kt;          // query tiles at or after this key tile
  const int n_iter = n_heads * per_head;

  auto load_q = [&](int it, int bi) {        // stage query tile `it` into buffer bi
    const int h = h_begin + it / per_head;
    const int q0 = (kt + it % per_head) * kTile;
    stage<D, TI>(sQ[bi], A.q, base, q0, T, h);
    stage<D, TI>(sG[bi], A.dO, base, q0, T, h);
    for (int i = threadIdx.x; i < kTile; i += kThreads) {
      const int q = q0 + i;
      sL[bi * kTile + i] = q < T ? A.lse[((int64_t)b * nH + h) * T + q] * kLog2e : 0.f;
      sD[bi * kTile + i] = q < T ? A.delta[((int64_t)b * nH + h) * T + q] : 0.f;
    }
  };

  stage<D, TI>(sK, A.k, base, k0, T, kvh);
  stage<D, TI>(sV, A.v, base, k0, T, kvh);
  load_q(0, 0);
  stage_done<TI>();
  uint32_t kf[D / 16][4], vf[D / 16][4];
  load_a_frags<D>(kf, sK, warp * 16, lane);
  load_a_frags<D>(vf, sV, warp * 16, lane);
  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; j++)
#pragma unroll
    for (int i = 0; i < 4; i++) dk[j][i] = dv[j][i] = 0.f;
  const int key[2] = {k0 + warp * 16 + g, k0 + warp * 16 + g + 8};

  for (int it = 0; it < n_iter; it++) {
    const int buf = kAsync ? (it & 1) : 0;
    if (it > 0 && !kAsync) {
      __syncthreads();
      load_q(it, 0);
      __syncthreads();
    }
    if (kAsync && it + 1 < n_iter) {
      load_q(it + 1, buf ^ 1);
      cp_async_commit();
    }
    const int q0 = (kt + it % per_head) * kTile;
    const float *L = sL + buf * kTile;
    const float *Dd = sD + buf * kTile;
    float st[8][4], dpt[8][4];
    mm_abt<D>(st, kf, sQ[buf], lane);   // S^T: keys x queries
    mm_abt<D>(dpt, vf, sG[buf], lane);  // dP^T = V dO^T
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int qi = j * 8 + 2 * t4 + (i & 1);
        const int q = q0 + qi;
        const int r = i >> 1;
        float p = 0.f;
        if (q < T && q >= key[r]) p = exp2f(st[j][i] * c - L[qi]);
        st[j][i] = p;
        dpt[j][i] = p * (dpt[j][i] - Dd[qi]);
      }
    }
    mm_pt<D>(dv, st, sG[buf], lane);   // dV += P^T dO
    mm_pt<D>(dk, dpt, sQ[buf], lane);  // dK += dS^T Q
    if (kAsync) {
      cp_async_wait_all();
      __syncthreads();
    }
  }
  if (A.split_heads) {
    const int64_t kvD = (int64_t)A.nKV * D;
    const int g = h_begin - kvh * group;
    View<void> pk{A.pk + (int64_t)g * A.rows * kvD, kvD, 0};
    View<void> pv{A.pv + (int64_t)g * A.rows * kvD, kvD, 0};
    store_rows<D, float>(pk, dk, key, base, kvh, T, A.scale, 0, nullptr, t4);
    store_rows<D, float>(pv, dv, key, base, kvh, T, 1.f, 0, nullptr, t4);
    return;
  }
  store_rows<D, TO>(A.dk, dk, key, base, kvh, T, A.scale, A.acc, A.rope, t4);
  store_rows<D, TO>(A.dv, dv, key, base, kvh, T, 1.f, A.acc, nullptr, t4);
}

// dK/dV of the head-split backward: sum the group's fp32 partials in order,
// rotate dK back (R^T) and store bf16 into the dqkv buffer.  One thread per
// (row, kv head, element pair).
template <int D>
__global__ void attn_kv_reduce_kernel(Args A, int group) {
  fcu::pdl_trigger();
  const int64_t kvD = (int64_t)A.nKV * D;
  const int64_t pairs = A.rows * (kvD / 2);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < pairs;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / (kvD / 2);
    const int64_t c = (e - row * (kvD / 2)) * 2;   // column within [0, kvD)
    float k0 = 0.f, k1 = 0.f, v0 = 0.f, v1 = 0.f;
    for (int g = 0; g < group; g++) {
      const int64_t o = (int64_t)g * A.rows * kvD + row * kvD + c;
      const float2 pk = *reinterpret_cast<const float2 *>(A.pk + o);
      const float2 pv = *reinterpret_cast<const float2 *>(A.pv + o);
      k0 += pk.x;
      k1 += pk.y;
      v0 += pv.x;
      v1 += pv.y;
    }
    if (A.rope) {
      const float2 cs = A.rope[(row % A.T) * (D / 2) + (c % D) / 2];
      const float u = k0 * cs.x + k1 * cs.y, w = -k0 * cs.y + k1 * cs.x;
      k0 = u;
      k1 = w;
    }
    __nv_bfloat16 *dk = reinterpret_cast<__nv_bfloat16 *>(A.dk.p) + row * A.dk.ld + A.dk.col + c;
    __nv_bfloat16 *dv = reinterpret_cast<__nv_bfloat16 *>(A.dv.p) + row * A.dv.ld + A.dv.col + c;
    *reinterpret_cast<uint32_t *>(dk) = pack_bf16(k0, k1);
    *reinterpret_cast<uint32_t *>(dv) = pack_bf16(v0, v1);
  }
}

// ------------------------------------------------------------------ backward dQ
template <int D, typename TI, typename TO>
__global__ void __launch_bounds__(kThreads) attn_bwd_dq_tc_kernel(Args A) {
  fcu::pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  constexpr bool kAsync = sizeof(TI) == 2;
  __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sG = sQ + Smem<D>::TILE;
  __nv_bfloat16 *sK[2] = {sG + Smem<D>::TILE, sG + 3 * Smem<D>::TILE};
  __nv_bfloat16 *sV[2] = {sG + 2 * Smem<D>::TILE, sG + 4 * Smem<D>::TILE};
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = A.T, nH = A.nH, kvh = h / (nH / A.nKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t base = (int64_t)b * T;
  const int q0 = qt * kTile;
  const float c = A.scale * kLog2e;

  stage<D, TI>(sQ, A.q, base, q0, T, h);
  stage<D, TI>(sG, A.dO, base, q0, T, h);
  stage<D, TI>(sK[0], A.k, base, 0, T, kvh);
  stage<D, TI>(sV[0], A.v, base, 0, T, kvh);
  stage_done<TI>();
  uint32_t qf[D / 16][4], gf[D / 16][4];
  load_a_frags<D>(qf, sQ, warp * 16, lane);
  load_a_frags<D>(gf, sG, warp * 16, lane);
  const int row[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};
  float L[2], Dl[2];
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const bool ok = row[r] < T;
    L[r] = ok ? A.lse[((int64_t)b * nH + h) * T + row[r]] * kLog2e : 0.f;
    Dl[r] = ok ? A.delta[((int64_t)b * nH + h) * T + row[r]] : 0.f;
  }
  float dq[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; j++)
#pragma unroll
    for (int i = 0; i < 4; i++) dq[j][i] = 0.f;

  for (int kt = 0; kt <= qt; kt++) {
    const int buf = kAsync ? (kt & 1) : 0;
    if (kt > 0 && !kAsync) {
      __syncthreads();
      stage<D, TI>(sK[0], A.k, base, kt * kTile, T, kvh);
      stage<D, TI>(sV[0], A.v, base, kt * kTile, T, kvh);
      __syncthreads();
    }
    if (kAsync && kt < qt) {
      stage<D, TI>(sK[buf ^ 1], A.k, base, (kt + 1) * kTile, T, kvh);
      stage<D, TI>(sV[buf ^ 1], A.v, base, (kt + 1) * kTile, T, kvh);
      cp_async_commit();
    }
    const int k0 = kt * kTile;
    float s[8][4], dp[8][4];
    mm_abt<D>(s, qf, sK[buf], lane);
    mm_abt<D>(dp, gf, sV[buf], lane);
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
    mm_pt<D>(dq, dp, sK[buf], lane);  // dQ += dS K
    if (kAsync) {
      cp_async_wait_all();
      __syncthreads();
    }
  }
  store_rows<D, TO>(A.dq, dq, row, base, h, T, A.scale, A.acc, A.rope, t4);
}

// delta[b,h,t] = sum_d dO[t,h,d] * O[t,h,d] (the rowsum(P * dP) of the JS), one warp per row.
template <typename TI>
__global__ void attn_delta_tc_kernel(Args A, int B, int D) {
  fcu::pdl_trigger();
  const int64_t rows = (int64_t)B * A.T * A.nH;
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const int64_t bt = w / A.nH;
  const int h = (int)(w % A.nH);
  const TI *g = reinterpret_cast<const TI *>(A.dO.p) + bt * A.dO.ld + A.dO.col + (int64_t)h * D;
  const TI *o = reinterpret_cast<const TI *>(A.o_in.p) + bt * A.o_in.ld + A.o_in.col + (int64_t)h * D;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s += (float)g[d] * (float)o[d];
  s = warp_sum(s);
  if (lane == 0) {
    const int b = (int)(bt / A.T), t = (int)(bt % A.T);
    ((float *)A.delta)[((int64_t)b * A.nH + h) * A.T + t] = s;
  }
}

template <int D, typename TI, typename TO>
int fwd_launch(cudaStream_t st, const Args &a, int B) {
  const size_t smem = 5 * sizeof(__nv_bfloat16) * Smem<D>::TILE;
  if (smem > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel<D, TI, TO>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(div_up(a.T, kTile), a.nH, B);
  attn_fwd_tc_kernel<D, TI, TO><<<grid, kThreads, smem, st>>>(a);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

template <int D, typename TI, typename TO>
int bwd_launch(cudaStream_t st, const Args &a, int B) {
  const size_t smem_kv = 6 * sizeof(__nv_bfloat16) * Smem<D>::TILE + 4 * kTile * sizeof(float);
  const size_t smem_q = 6 * sizeof(__nv_bfloat16) * Smem<D>::TILE;
  if (smem_kv > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel<D, TI, TO>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_kv));
  if (smem_q > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<D, TI, TO>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_q));
  dim3 gkv(div_up(a.T, kTile), a.split_heads ? a.nH : a.nKV, B);
  attn_bwd_dkdv_tc_kernel<D, TI, TO><<<gkv, kThreads, smem_kv, st>>>(a);
  FCU_CHECK_LAUNCH();
  if (a.split_heads) {
    const int64_t pairs = a.rows * ((int64_t)a.nKV * D / 2);
    int blocks = (int)((pairs + 255) / 256);
    if (blocks > 65535) blocks = 65535;
    attn_kv_reduce_kernel<D><<<blocks, 256, 0, st>>>(a, a.nH / a.nKV);
    FCU_CHECK_LAUNCH();
  }
  dim3 gq(div_up(a.T, kTile), a.nH, B);
  attn_bwd_dq_tc_kernel<D, TI, TO><<<gq, kThreads, smem_q, st>>>(a);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

template <typename TI, typename TO>
int fwd_dispatch(cudaStream_t st, const Args &a, int B, int dH) {
  switch (dH) {
    case 16: return fwd_launch<16, TI, TO>(st, a, B);
    case 32: return fwd_launch<32, TI, TO>(st, a, B);
    case 64: return fwd_launch<64, TI, TO>(st, a, B);
    case 128: return fwd_launch<128, TI, TO>(st, a, B);
  }
  set_error("tensor-core attention: unsupported head dim %d", dH);
  return FCU_ERR_ARG;
}

template <typename TI, typename TO>
int bwd_dispatch(cudaStream_t st, const Args &a, int B, int dH) {
  switch (dH) {
    case 16: return bwd_launch<16, TI, TO>(st, a, B);
    case 32: return bwd_launch<32, TI, TO>(st, a, B);
    case 64: return bwd_launch<64, TI, TO>(st, a, B);
    case 128: return bwd_launch<128, TI, TO>(st, a, B);
  }
  set_error("tensor-core attention: unsupported head dim %d", dH);
  return FCU_ERR_ARG;
}

Args fp32_args(const float *Q, const float *K, const float *V, int T, int nH, int nKV, int dH) {
  Args a{};
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)nKV * dH;
  a.q = {Q, qD, 0};
  a.k = {K, kvD, 0};
  a.v = {V, kvD, 0};
  a.T = T;
  a.nH = nH;
  a.nKV = nKV;
  a.scale = (float)(1.0 / sqrt((double)dH));
  return a;
}

}  // namespace

bool attn_tc_supported(int dH, const void *Q, const void *K, const void *V) {
  if (dH != 16 && dH != 32 && dH != 64 && dH != 128) return false;
  return (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V) & 15) == 0;
}

int attn_fwd_tc(cudaStream_t st, const float *Q, const float *K, const float *V, int B, int T,
                int nH, int nKV, int dH, float *O, float *lse) {
  Args a = fp32_args(Q, K, V, T, nH, nKV, dH);
  a.o = {O, (int64_t)nH * dH, 0};
  a.lse = lse;
  return fwd_dispatch<float, float>(st, a, B, dH);
}

int attn_bwd_tc(cudaStream_t st, const float *dO, const float *Q, const float *K, const float *V,
                const float *lse, const float *delta, int B, int T, int nH, int nKV, int dH,
                float *dQ, float *dK, float *dV, int acc) {
  Args a = fp32_args(Q, K, V, T, nH, nKV, dH);
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)nKV * dH;
  a.dO = {dO, qD, 0};
  a.dq = {dQ, qD, 0};
  a.dk = {dK, kvD, 0};
  a.dv = {dV, kvD, 0};
  a.lse = const_cast<float *>(lse);
  a.delta = delta;
  a.acc = acc;
  return bwd_dispatch<float, float>(st, a, B, dH);
}


}  // namespace fcu

extern "C" {

int fcu_attn_fwd_bf16(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV,
                      int dH, void *O, float *lse) {
  using namespace fcu;
  FCU_CTX(ctx);
  FCU_REQUIRE(B > 0 && T > 0 && nH > 0 && nKV > 0 && nH % nKV == 0,
              "fcu_attn_fwd_bf16: bad shape B=%d T=%d nH=%d nKV=%d", B, T, nH, nKV);
  FCU_REQUIRE(dH == 16 || dH == 32 || dH == 64 || dH == 128, "fcu_attn_fwd_bf16: dH=%d", dH);
  FCU_REQUIRE(ld_qkv >= (int64_t)(nH + 2 * nKV) * dH && ld_qkv % 8 == 0,
              "fcu_attn_fwd_bf16: qkv row stride %lld", (long long)ld_qkv);
  FCU_REQUIRE(qkv && O && lse && (((uintptr_t)qkv | (uintptr_t)O) & 15) == 0,
              "fcu_attn_fwd_bf16: null or unaligned pointer");
  if (attn_tmem_fwd_supported(dH)) return attn_fwd_tmem(ctx, qkv, ld_qkv, B, T, nH, nKV, O, lse, dH);
  // dH is 16 or 32 here: zero-padded to 64-column heads
  return attn_fwd_tmem_padded(ctx, qkv, ld_qkv, B, T, nH, nKV, dH, O, lse);
}

int fcu_attn_bwd_bf16(fcu_ctx *ctx, const void *dO, const void *qkv, int64_t ld_qkv, const void *O,
                      const float *lse, int B, int T, int nH, int nKV, int dH, double rope_theta,
                      void *dqkv) {
  using namespace fcu;
  FCU_CTX(ctx);
  FCU_REQUIRE(B > 0 && T > 0 && nH > 0 && nKV > 0 && nH % nKV == 0,
              "fcu_attn_bwd_bf16: bad shape B=%d T=%d nH=%d nKV=%d", B, T, nH, nKV);
  FCU_REQUIRE(dH == 16 || dH == 32 || dH == 64 || dH == 128, "fcu_attn_bwd_bf16: dH=%d", dH);
  FCU_REQUIRE(ld_qkv >= (int64_t)(nH + 2 * nKV) * dH && ld_qkv % 8 == 0,
              "fcu_attn_bwd_bf16: qkv row stride %lld", (long long)ld_qkv);
  FCU_REQUIRE(dO && qkv && O && lse && dqkv &&
                  (((uintptr_t)dO | (uintptr_t)qkv | (uintptr_t)O | (uintptr_t)dqkv) & 15) == 0,
              "fcu_attn_bwd_bf16: null or unaligned pointer");
  const int64_t kvD = (int64_t)nKV * dH;
  if (attn_tmem_supported(dH)) {
    // tcgen05 kernels, one CTA per SM: split dK/dV per q head when one CTA
    // per kv head would leave the GPU with fewer than 4 CTAs per SM.
    const int64_t ctas = (int64_t)div_up(T, 128) * nKV * B;
    const int split = (nH > nKV && ctas < 4 * (int64_t)ctx->num_sms) ? 1 : 0;
    const size_t delta_bytes = (sizeof(float) * (size_t)B * nH * T + 255) & ~(size_t)255;
    const size_t part_bytes = split ? sizeof(float) * (size_t)(nH / nKV) * B * T * kvD : 0;
    void *scr = nullptr;
    int rc = ctx_scratch(ctx, delta_bytes + 2 * part_bytes, &scr);
    if (rc) return rc;
    const float2 *rope = nullptr;
    if (rope_theta > 0) {
      rc = rope_table_f32(ctx, T, dH, rope_theta, &rope);
      if (rc) return rc;
    }
    float *pk = split ? (float *)((uint8_t *)scr + delta_bytes) : nullptr;
    float *pv = split ? (float *)((uint8_t *)scr + delta_bytes + part_bytes) : nullptr;
    return attn_bwd_tmem(ctx, dO, qkv, ld_qkv, O, lse, (float *)scr, B, T, nH, nKV, rope, dqkv, split,
                         pk, pv, dH);
  }
  // dH is 16 or 32 here: zero-padded to 64-column heads
  return attn_bwd_tmem_padded(ctx, dO, qkv, ld_qkv, O, lse, B, T, nH, nKV, dH, rope_theta, dqkv);
}

}  // extern "C"
