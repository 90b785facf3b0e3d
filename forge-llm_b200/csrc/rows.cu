// Row-wise and elementwise kernels of the training hot path: embedding,
// rmsNorm, ropeRows, sliceCols, swiglu, residual add, fused cross-entropy and
// small helpers.  All are single-pass, coalesced, HBM-bound kernels.
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t n, int per_block, int cap) {
  int64_t g = (n + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (int)g;
}

// ---------------------------------------------------------------- embedding
// out[t, :] = W[ids[t], :]; an id outside [0, V) yields NaN, as the JS read
// of an out-of-range typed-array slot does (undefined -> NaN on store).
__global__ void embed_fwd_kernel(const float *__restrict__ W, const int32_t *__restrict__ ids,
                                 int64_t T, int64_t V, int64_t D, float *__restrict__ out) {
  fcu::pdl_trigger();
  int64_t total = T * D;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = e / D, d = e - t * D;
    int32_t id = ids[t];
    out[e] = (id >= 0 && id < V) ? W[(int64_t)id * D + d] : __int_as_float(0x7fc00000);
  }
}

// Keys (id << 32 | t) are unique, so sorting them orders tokens by id and,
// within an id, by ascending t -- the order the JS loop adds them in.
__global__ void embed_keys_kernel(const int32_t *__restrict__ ids, int64_t T, int64_t P,
                                  unsigned long long *__restrict__ keys) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < P;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i < T) {
      uint32_t id = (uint32_t)ids[i];
      keys[i] = ((unsigned long long)id << 32) | (unsigned long long)(uint32_t)i;
    } else {
      keys[i] = ~0ull;  // padding sorts last
    }
  }
}

constexpr int kSortSpan = 2048;  // elements sorted per CTA in shared memory

// Bitonic stages k in [k_lo, k_hi] (powers of two) restricted to strides
// j < kSortSpan, on chunks of kSortSpan elements.
__global__ void bitonic_smem_kernel(unsigned long long *__restrict__ a, int64_t k_lo, int64_t k_hi) {
  fcu::pdl_trigger();
  __shared__ unsigned long long s[kSortSpan];
  const int64_t base = (int64_t)blockIdx.x * kSortSpan;
  for (int i = threadIdx.x; i < kSortSpan; i += blockDim.x) s[i] = a[base + i];
  __syncthreads();
  for (int64_t k = k_lo; k <= k_hi; k <<= 1) {
    for (int64_t j = (k >> 1) < (kSortSpan >> 1) ? (k >> 1) : (kSortSpan >> 1); j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < kSortSpan; i += blockDim.x) {
        int ixj = i ^ (int)j;
        if (ixj > i) {
          int64_t gi = base + i;
          bool asc = (gi & k) == 0;
          unsigned long long x = s[i], y = s[ixj];
          if (asc ? (x > y) : (x < y)) {
            s[i] = y;
            s[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < kSortSpan; i += blockDim.x) a[base + i] = s[i];
}

__global__ void bitonic_global_kernel(unsigned long long *__restrict__ a, int64_t P, int64_t j,
                                      int64_t k) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < P;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t ixj = i ^ j;
    if (ixj > i) {
      bool asc = (i & k) == 0;
      unsigned long long x = a[i], y = a[ixj];
      if (asc ? (x > y) : (x < y)) {
        a[i] = y;
        a[ixj] = x;
      }
    }
  }
}

// One warp per sorted position; the first position of each id walks its
// tokens in ascending t and adds their rows into dW[id].
__global__ void embed_segsum_kernel(const unsigned long long *__restrict__ keys, int64_t T,
                                    int64_t V, int64_t D, const float *__restrict__ dX,
                                    float *__restrict__ dW) {
  fcu::pdl_trigger();
  int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (i >= T) return;
  uint32_t id = (uint32_t)(keys[i] >> 32);
  if (i > 0 && (uint32_t)(keys[i - 1] >> 32) == id) return;
  if ((int32_t)id < 0 || (int64_t)(int32_t)id >= V) return;  // JS: out-of-range store is a no-op
  int64_t end = i + 1;
  while (end < T && (uint32_t)(keys[end] >> 32) == id) end++;
  float *row = dW + (int64_t)id * D;
  for (int64_t c = lane; c < D; c += 32) {
    float acc = row[c];
    for (int64_t s = i; s < end; s++) {
      int64_t t = (int64_t)(uint32_t)(keys[s] & 0xffffffffull);
      acc += dX[t * D + c];
    }
    row[c] = acc;
  }
}

// The same for D = 128 * NC: each lane keeps NC float4 of the row in
// registers and every token row is one round of independent 16-byte loads.
// Per element the order is unchanged: the existing dW value, then the tokens
// in ascending t.
template <int NC>
__global__ void embed_segsum4_kernel(const unsigned long long *__restrict__ keys, int64_t T, int64_t V,
                                     const float *__restrict__ dX, float *__restrict__ dW) {
  fcu::pdl_trigger();
  constexpr int D = 128 * NC;
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= T) return;
  const uint32_t id = (uint32_t)(keys[i] >> 32);
  if (i > 0 && (uint32_t)(keys[i - 1] >> 32) == id) return;
  if ((int32_t)id < 0 || (int64_t)(int32_t)id >= V) return;  // JS: out-of-range store is a no-op
  float4 *row = reinterpret_cast<float4 *>(dW + (int64_t)id * D);
  float4 acc[NC];
#pragma unroll
  for (int k = 0; k < NC; k++) acc[k] = row[lane + 32 * k];
  for (int64_t s = i; s < T; s++) {
    const unsigned long long key = keys[s];
    if ((uint32_t)(key >> 32) != id) break;
    const float4 *x = reinterpret_cast<const float4 *>(dX + (int64_t)(uint32_t)(key & 0xffffffffull) * D);
#pragma unroll
    for (int k = 0; k < NC; k++) {
      const float4 v = x[lane + 32 * k];
      acc[k].x += v.x;
      acc[k].y += v.y;
      acc[k].z += v.z;
      acc[k].w += v.w;
    }
  }
#pragma unroll
  for (int k = 0; k < NC; k++) row[lane + 32 * k] = acc[k];
}

// ---------------------------------------------------------------- rmsNorm
// One warp per row.  inv[t] = 1/sqrt(sum(x^2)/D + eps) (double reduction,
// stored fp32 as the JS Float32Array does); out = x * inv * w.
__global__ void rmsnorm_fwd_kernel(const float *__restrict__ X, const float *__restrict__ w,
                                   int64_t T, int64_t D, double eps, float *__restrict__ out,
                                   float *__restrict__ inv) {
  fcu::pdl_trigger();
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float *x = X + row * D;
  double ss = 0;
  for (int64_t i = lane; i < D; i += 32) {
    double v = x[i];
    ss += v * v;
  }
  ss = warp_sum_d(ss);
  float iv = (float)(1.0 / sqrt(ss / (double)D + eps));
  if (lane == 0 && inv) inv[row] = iv;
  float *o = out + row * D;
  for (int64_t i = lane; i < D; i += 32) o[i] = x[i] * iv * w[i];
}

// dX = g*w*inv - c*x, c = dot(g*w, x)/(D r^3), r = 1/inv.  Each CTA also
// leaves its partial dw[D] = sum over its rows of g*x*inv in `part`; warps
// accumulate into private shared rows, summed in fixed order (deterministic).
__global__ void rmsnorm_bwd_kernel(const float *__restrict__ G, const float *__restrict__ X,
                                   const float *__restrict__ w, const float *__restrict__ inv,
                                   int64_t T, int64_t D, int64_t rows_per_block,
                                   float *__restrict__ dX, int acc_dx, float *__restrict__ part) {
  fcu::pdl_trigger();
  extern __shared__ float sm[];  // [nwarps][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float *mine = sm + (int64_t)wid * D;
  for (int64_t i = lane; i < D; i += 32) mine[i] = 0.f;
  const int64_t r0 = blockIdx.x * rows_per_block;
  int64_t r1 = r0 + rows_per_block;
  if (r1 > T) r1 = T;
  for (int64_t row = r0 + wid; row < r1; row += nw) {
    const float *g = G + row * D, *x = X + row * D;
    double iv = inv[row];
    double r = 1.0 / iv;
    double dot = 0;
    for (int64_t i = lane; i < D; i += 32) dot += (double)g[i] * (double)w[i] * (double)x[i];
    dot = warp_sum_d(dot);
    float c = (float)(dot / ((double)D * r * r * r));
    float ivf = (float)iv;
    float *dx = dX + row * D;
    for (int64_t i = lane; i < D; i += 32) {
      float gi = g[i], xi = x[i];
      float v = gi * w[i] * ivf - c * xi;
      dx[i] = acc_dx ? dx[i] + v : v;
      mine[i] += gi * xi * ivf;
    }
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

// ---------------------------------------------------------------- ropeRows
// tab[pos][i] = (cos, sin)(pos / theta^(2i/dHead)), in double as the JS.
__global__ void rope_table_kernel(double2 *tab, int npos, int half, int dHead, double theta) {
  fcu::pdl_trigger();
  int64_t n = (int64_t)npos * half;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t p = e / half, i = e - p * half;
    double freq = 1.0 / pow(theta, (double)(2 * i) / (double)dHead);
    double ang = (double)p * freq;
    double s, c;
    sincos(ang, &s, &c);
    tab[e] = make_double2(c, s);
  }
}

template <bool BWD>
__global__ void rope_kernel(const float *__restrict__ X, int64_t T, int nHead, int dHead, int pos0,
                            int posStride, const double2 *__restrict__ tab,
                            float *__restrict__ out, int acc) {
  fcu::pdl_trigger();
  const int half = dHead >> 1;
  const int64_t D = (int64_t)nHead * dHead;
  const int64_t npairs = T * nHead * half;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < npairs;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = e / ((int64_t)nHead * half);
    int64_t rem = e - t * nHead * half;
    int h = (int)(rem / half), i = (int)(rem - (int64_t)h * half);
    int64_t pos = pos0 + (posStride > 0 ? t % posStride : t);
    double2 cs = tab[pos * half + i];
    int64_t o = t * D + (int64_t)h * dHead + 2 * i;
    double a = X[o], b = X[o + 1];
    float ra, rb;
    if (!BWD) {
      ra = (float)(a * cs.x - b * cs.y);
      rb = (float)(a * cs.y + b * cs.x);
    } else {
      ra = (float)(a * cs.x + b * cs.y);
      rb = (float)(-a * cs.y + b * cs.x);
    }
    if (acc) {
      out[o] += ra;
      out[o + 1] += rb;
    } else {
      out[o] = ra;
      out[o + 1] = rb;
    }
  }
}

// ---------------------------------------------------------------- sliceCols
template <bool BWD>
__global__ void slicecols_kernel(const float *__restrict__ src, int64_t M, int64_t K, int64_t off,
                                 int64_t len, float *__restrict__ dst, int acc) {
  fcu::pdl_trigger();
  int64_t n = M * len;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t m = e / len, i = e - m * len;
    if (!BWD) {
      dst[e] = src[m * K + off + i];
    } else {
      float v = src[e];
      float *p = dst + m * K + off + i;
      *p = acc ? *p + v : v;
    }
  }
}

// ---------------------------------------------------------------- swiglu
__global__ void swiglu_fwd_kernel(const float *__restrict__ G, const float *__restrict__ U,
                                  int64_t n, float *__restrict__ out) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float g = G[i];
    float s = 1.f / (1.f + expf(-g));
    out[i] = g * s * U[i];
  }
}

__global__ void swiglu_bwd_kernel(const float *__restrict__ dO, const float *__restrict__ G,
                                  const float *__restrict__ U, int64_t n, float *__restrict__ dG,
                                  float *__restrict__ dU, int acc) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float g = G[i], d = dO[i];
    float s = 1.f / (1.f + expf(-g));
    float vg = d * U[i] * (s + g * s * (1.f - s));
    float vu = d * (g * s);
    if (acc) {
      dG[i] += vg;
      dU[i] += vu;
    } else {
      dG[i] = vg;
      dU[i] = vu;
    }
  }
}

// ---------------------------------------------------------------- add
__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b, int64_t n,
                           float *__restrict__ out) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = a[i] + b[i];
}

__global__ void add_bwd_kernel(const float *__restrict__ g, int64_t n, float *__restrict__ da,
                               int acc_a, float *__restrict__ db, int acc_b) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = g[i];
    if (da) da[i] = acc_a ? da[i] + v : v;
    if (db) db[i] = acc_b ? db[i] + v : v;
  }
}

// ---------------------------------------------------------------- cross entropy
// One CTA per row.  Pass 1: online (max, sum exp) over the row; pass 2 writes
// (exp(l - lse) - onehot)/T.
constexpr int kCeThreads = 1024;

__device__ __forceinline__ void ce_merge(float &m, float &s, float m2, float s2) {
  float mn = fmaxf(m, m2);
  if (mn == -INFINITY) {
    s = 0.f;
  } else {
    s = s * expf(m - mn) + s2 * expf(m2 - mn);
  }
  m = mn;
}

__device__ __forceinline__ void ce_block_reduce(float &m, float &s, float *shm, float *shs) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    ce_merge(m, s, m2, s2);
  }
  if (lane == 0) {
    shm[wid] = m;
    shs[wid] = s;
  }
  __syncthreads();
  m = lane < nw ? shm[lane] : -INFINITY;
  s = lane < nw ? shs[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    ce_merge(m, s, m2, s2);
  }
}

__device__ __forceinline__ void ce_store1(float *p, float v) { *p = v; }
__device__ __forceinline__ void ce_store1(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// CE for rows that the vectorised ce2_kernel cannot read (a logits or
// gradient pointer not 16-byte aligned, or V not a multiple of 4): scalar
// loads, two passes over the row.  TO = float: the op-level gradient; TO =
// bf16: the fused path, where the gradient is the next GEMM's operand.
template <typename TO = float>
__global__ void __launch_bounds__(kCeThreads) ce_fwd_kernel(const float *logits,
                                                            const int32_t *__restrict__ targets,
                                                            int64_t T, int64_t V,
                                                            float *row_loss, TO *dunit) {
  fcu::pdl_trigger();
  __shared__ float shm[32], shs[32];
  const int64_t row = blockIdx.x;
  const float *l = logits + row * V;
  TO *du = dunit + row * V;
  const float invT = (float)(1.0 / (double)T);
  const int32_t tgt = targets[row];
  float m = -INFINITY, s = 0.f;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    float v = l[i];
    if (v > m) {
      s = (m == -INFINITY) ? 0.f : s * expf(m - v);
      m = v;
    }
    s += expf(v - m);
  }
  ce_block_reduce(m, s, shm, shs);
  const float lse = m + logf(s);
  const float lt = (tgt >= 0 && tgt < V) ? l[tgt] : __int_as_float(0x7fc00000);
  __syncthreads();  // every thread has read l[tgt] before any in-place write
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    float v = l[i];
    ce_store1(du + i, (expf(v - lse) - (i == tgt ? 1.f : 0.f)) * invT);
  }
  if (threadIdx.x == 0) row_loss[row] = lse - lt;
}

// CE with the gradient as bf16 (the fused path) or fp32 (the operator), loss
// per row.  Online max / sum in the
// log2 domain (one FMA + one ex2 per logit), one block reduction, then a
// second pass that re-reads the row (from L2: two 512-thread CTAs per SM keep
// ~300 rows, under 40 MB, in flight) and writes (softmax - onehot) / T.
__device__ __forceinline__ float ex2_approx(float x) {   // 2^x on the MUFU unit (ftz)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

constexpr int kCe2Threads = 512;
constexpr int kCe2Unroll = 4;

__device__ __forceinline__ void ce2_store4(__nv_bfloat16 *du, int64_t i4, float a, float b, float c, float d) {
  reinterpret_cast<uint2 *>(du)[i4] = make_uint2(pack_bf16(a, b), pack_bf16(c, d));
}
__device__ __forceinline__ void ce2_store4(float *du, int64_t i4, float a, float b, float c, float d) {
  reinterpret_cast<float4 *>(du)[i4] = make_float4(a, b, c, d);
}

template <typename TO>
__global__ void __launch_bounds__(kCe2Threads, 2)
    ce2_kernel(const float *__restrict__ logits, const int32_t *__restrict__ targets, int64_t T,
               int64_t V, float *__restrict__ row_loss, TO *__restrict__ du) {
  fcu::pdl_trigger();
  __shared__ float shm[32], shs[32];
  constexpr float kL2e = 1.4426950408889634f;
  const int64_t row = blockIdx.x;
  const float4 *l4 = reinterpret_cast<const float4 *>(logits + row * V);
  const int64_t V4 = V >> 2;
  const int32_t tgt = targets[row];
  float lt = 0.f;
  if (threadIdx.x == 0) lt = (tgt >= 0 && tgt < V) ? logits[row * V + tgt] : __int_as_float(0x7fc00000);
  float m = -INFINITY, s = 0.f;                 // log2 domain: m = max(x log2e), s = sum 2^(x log2e - m)
  for (int64_t base = threadIdx.x; base < V4; base += (int64_t)kCe2Threads * kCe2Unroll) {
    float4 v[kCe2Unroll];
#pragma unroll
    for (int u = 0; u < kCe2Unroll; u++) {
      const int64_t i4 = base + (int64_t)u * kCe2Threads;
      v[u] = i4 < V4 ? l4[i4] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
#pragma unroll
    for (int u = 0; u < kCe2Unroll; u++) {
      const float mx = fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w)) * kL2e;
      if (mx > m) {
        s *= ex2_approx(m - mx);                // 0 while m is -inf
        m = mx;
      }
      if (mx != -INFINITY)
        s += ex2_approx(fmaf(v[u].x, kL2e, -m)) + ex2_approx(fmaf(v[u].y, kL2e, -m)) +
             ex2_approx(fmaf(v[u].z, kL2e, -m)) + ex2_approx(fmaf(v[u].w, kL2e, -m));
    }
  }
  // combine (m, s) over the block
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * ex2_approx(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * ex2_approx(m2 - mm));
    m = mm;
  }
  if (lane == 0) {
    shm[wid] = m;
    shs[wid] = s;
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kCe2Threads / 32; w++) M = fmaxf(M, shm[w]);
  float S = 0.f;
  for (int w = 0; w < kCe2Threads / 32; w++) S += shm[w] == -INFINITY ? 0.f : shs[w] * ex2_approx(shm[w] - M);
  const float lse2 = M + __log2f(S);            // log2-domain log-sum-exp
  const float invT = (float)(1.0 / (double)T);
  TO *drow = du + row * V;
  for (int64_t base = threadIdx.x; base < V4; base += (int64_t)kCe2Threads * kCe2Unroll) {
    float4 v[kCe2Unroll];
#pragma unroll
    for (int u = 0; u < kCe2Unroll; u++) {
      const int64_t i4 = base + (int64_t)u * kCe2Threads;
      if (i4 < V4) v[u] = l4[i4];
    }
#pragma unroll
    for (int u = 0; u < kCe2Unroll; u++) {
      const int64_t i4 = base + (int64_t)u * kCe2Threads;
      if (i4 >= V4) continue;
      const int64_t i = i4 * 4;
      const float o0 = (ex2_approx(fmaf(v[u].x, kL2e, -lse2)) - (i + 0 == tgt ? 1.f : 0.f)) * invT;
      const float o1 = (ex2_approx(fmaf(v[u].y, kL2e, -lse2)) - (i + 1 == tgt ? 1.f : 0.f)) * invT;
      const float o2 = (ex2_approx(fmaf(v[u].z, kL2e, -lse2)) - (i + 2 == tgt ? 1.f : 0.f)) * invT;
      const float o3 = (ex2_approx(fmaf(v[u].w, kL2e, -lse2)) - (i + 3 == tgt ? 1.f : 0.f)) * invT;
      ce2_store4(drow, i4, o0, o1, o2, o3);
    }
  }
  if (threadIdx.x == 0) row_loss[row] = lse2 * 0.6931471805599453f - lt;
}

// Training windows (train.js:258-262): out[b][i] = data[s_b + i], or the last
// token of the stream where the window runs past its end.
__global__ void gather_windows_kernel(const int32_t *__restrict__ data, int64_t n,
                                      const int32_t *__restrict__ starts, int B, int T1,
                                      int32_t *__restrict__ out) {
  fcu::pdl_trigger();
  const int64_t total = (int64_t)B * T1;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(e / T1), i = (int)(e - (int64_t)b * T1);
    const int64_t k = (int64_t)starts[b] + i;
    out[e] = (k >= 0 && k < n) ? data[k] : data[n - 1];
  }
}

// loss = sum(row_loss) / T, summed in double in row order by one CTA.
__global__ void mean_kernel(const float *__restrict__ v, int64_t n, float *__restrict__ out) {
  fcu::pdl_trigger();
  __shared__ double sh[32];
  double s = 0;
  // fixed assignment: thread i takes rows i, i+blockDim, ... then a fixed tree
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += (double)v[i];
  s = block_sum(s, sh);
  if (threadIdx.x == 0) out[0] = (float)(s / (double)n);
}

__global__ void wsum_kernel(const float *__restrict__ Y, const float *__restrict__ t, int64_t n,
                            float *__restrict__ out) {
  fcu::pdl_trigger();
  __shared__ double sh[32];
  double s = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += (double)Y[i] * (double)t[i];
  s = block_sum(s, sh);
  if (threadIdx.x == 0) out[0] = (float)s;
}

__global__ void axpy_dev_kernel(const float *__restrict__ alpha, const float *__restrict__ x,
                                int64_t n, float *__restrict__ y, int acc) {
  fcu::pdl_trigger();
  const float a = alpha[0];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = acc ? y[i] + a * x[i] : a * x[i];
}

__global__ void scale_kernel(float *__restrict__ y, int64_t n, float a) {
  fcu::pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] *= a;
}

int ensure_rope_table(fcu_ctx *ctx, int npos, int dHead, double theta) {
  int half = dHead >> 1;
  if (ctx->rope_tab && ctx->rope_half == half && ctx->rope_theta == theta && ctx->rope_pos >= npos)
    return FCU_OK;
  int want = npos < 4096 ? 4096 : npos;
  if (ctx->rope_tab) {
    FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
    FCU_CHECK_CUDA(cudaFree(ctx->rope_tab));
    ctx->rope_tab = nullptr;
  }
  FCU_CHECK_CUDA(cudaMalloc(&ctx->rope_tab, sizeof(double2) * (size_t)want * (half > 0 ? half : 1)));
  int64_t n = (int64_t)want * half;
  if (n > 0) {
    rope_table_kernel<<<grid_for(n, kThreads, 4096), kThreads, 0, ctx->stream>>>(
        ctx->rope_tab, want, half, dHead, theta);
    FCU_CHECK_LAUNCH();
  }
  ctx->rope_pos = want;
  ctx->rope_half = half;
  ctx->rope_theta = theta;
  return FCU_OK;
}

}  // namespace

// ======================================================================== C-ABI
extern "C" {

int fcu_embed_fwd(fcu_ctx *ctx, const float *W, const int32_t *ids, int64_t T, int64_t V,
                  int64_t D, float *out) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && V > 0 && D > 0, "fcu_embed_fwd: bad shape T=%lld V=%lld D=%lld",
              (long long)T, (long long)V, (long long)D);
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(W && ids && out, "fcu_embed_fwd: null pointer");
  embed_fwd_kernel<<<grid_for(T * D, kThreads, 65535), kThreads, 0, ctx->stream>>>(W, ids, T, V, D,
                                                                                    out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_embed_bwd(fcu_ctx *ctx, const float *dX, const int32_t *ids, int64_t T, int64_t V,
                  int64_t D, float *dW) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && V > 0 && D > 0 && T < (1ll << 31), "fcu_embed_bwd: bad shape");
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(dX && ids && dW, "fcu_embed_bwd: null pointer");
  int64_t P = kSortSpan;
  while (P < T) P <<= 1;
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(unsigned long long) * (size_t)P, &scr);
  if (rc) return rc;
  unsigned long long *keys = (unsigned long long *)scr;
  embed_keys_kernel<<<grid_for(P, kThreads, 65535), kThreads, 0, ctx->stream>>>(ids, T, P, keys);
  FCU_CHECK_LAUNCH();
  const int nchunks = (int)(P / kSortSpan);
  bitonic_smem_kernel<<<nchunks, 1024, 0, ctx->stream>>>(keys, 2, kSortSpan);
  FCU_CHECK_LAUNCH();
  for (int64_t k = 2 * kSortSpan; k <= P; k <<= 1) {
    for (int64_t j = k >> 1; j >= kSortSpan; j >>= 1) {
      bitonic_global_kernel<<<grid_for(P, kThreads, 65535), kThreads, 0, ctx->stream>>>(keys, P, j,
                                                                                        k);
      FCU_CHECK_LAUNCH();
    }
    bitonic_smem_kernel<<<nchunks, 1024, 0, ctx->stream>>>(keys, k, k);
    FCU_CHECK_LAUNCH();
  }
  const int blocks = grid_for(T * 32, kThreads, 1 << 30);
  const bool vec = D % 128 == 0 && D <= 1024 && (((uintptr_t)dX | (uintptr_t)dW) & 15) == 0;
  switch (vec ? D / 128 : 0) {
#define FCU_SEGSUM_CASE(nc) \
  case nc: embed_segsum4_kernel<nc><<<blocks, kThreads, 0, ctx->stream>>>(keys, T, V, dX, dW); break;
    FCU_SEGSUM_CASE(1)
    FCU_SEGSUM_CASE(2)
    FCU_SEGSUM_CASE(3)
    FCU_SEGSUM_CASE(4)
    FCU_SEGSUM_CASE(5)
    FCU_SEGSUM_CASE(6)
    FCU_SEGSUM_CASE(7)
    FCU_SEGSUM_CASE(8)
#undef FCU_SEGSUM_CASE
    default: embed_segsum_kernel<<<blocks, kThreads, 0, ctx->stream>>>(keys, T, V, D, dX, dW);
  }
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_rmsnorm_fwd(fcu_ctx *ctx, const float *X, const float *w, int64_t T, int64_t D, double eps,
                    float *out, float *inv) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && D > 0, "fcu_rmsnorm_fwd: bad shape");
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(X && w && out, "fcu_rmsnorm_fwd: null pointer");
  rmsnorm_fwd_kernel<<<grid_for(T * 32, kThreads, 1 << 30), kThreads, 0, ctx->stream>>>(X, w, T, D,
                                                                                         eps, out, inv);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_rmsnorm_bwd(fcu_ctx *ctx, const float *dY, const float *X, const float *w,
                    const float *inv, int64_t T, int64_t D, float *dX, int accumulate_dx, float *dw,
                    int accumulate_dw) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && D > 0, "fcu_rmsnorm_bwd: bad shape");
  FCU_REQUIRE(D <= 6144, "fcu_rmsnorm_bwd: D=%lld above the supported 6144", (long long)D);
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(dY && X && w && inv && dX && dw, "fcu_rmsnorm_bwd: null pointer");
  const int threads = 256, nw = threads / 32;
  int64_t nblk = 2 * (int64_t)ctx->num_sms;
  int64_t rpb = (T + nblk - 1) / nblk;
  if (rpb < nw) rpb = nw;
  nblk = (T + rpb - 1) / rpb;
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(float) * (size_t)(nblk * D), &scr);
  if (rc) return rc;
  size_t smem = sizeof(float) * (size_t)nw * (size_t)D;
  if (smem > 48 * 1024)
    FCU_CHECK_CUDA(cudaFuncSetAttribute(rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
  rmsnorm_bwd_kernel<<<(int)nblk, threads, smem, ctx->stream>>>(dY, X, w, inv, T, D, rpb, dX,
                                                                 accumulate_dx, (float *)scr);
  FCU_CHECK_LAUNCH();
  colsum_kernel<<<(unsigned)((D + 31) / 32), dim3(32, 8), 0, ctx->stream>>>((float *)scr, (int)nblk, D,
                                                                            dw, accumulate_dw);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

static int rope_common(fcu_ctx *ctx, const float *X, int64_t T, int nHead, int dHead, int pos0,
                       double theta, int posStride, float *out, int acc, bool bwd) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T >= 0 && nHead > 0 && dHead > 0 && (dHead % 2) == 0 && pos0 >= 0 && posStride >= 0,
              "fcu_rope: bad shape (dHead must be even)");
  if (T == 0) return FCU_OK;
  FCU_REQUIRE(X && out, "fcu_rope: null pointer");
  int64_t span = posStride > 0 ? (posStride < T ? posStride : T) : T;
  FCU_REQUIRE((int64_t)pos0 + span <= (1 << 24), "fcu_rope: positions beyond 2^24");
  int rc = ensure_rope_table(ctx, (int)(pos0 + span), dHead, theta);
  if (rc) return rc;
  int64_t npairs = T * nHead * (dHead / 2);
  if (bwd)
    rope_kernel<true><<<grid_for(npairs, kThreads, 65535), kThreads, 0, ctx->stream>>>(
        X, T, nHead, dHead, pos0, posStride, ctx->rope_tab, out, acc);
  else
    rope_kernel<false><<<grid_for(npairs, kThreads, 65535), kThreads, 0, ctx->stream>>>(
        X, T, nHead, dHead, pos0, posStride, ctx->rope_tab, out, 0);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_rope_fwd(fcu_ctx *ctx, const float *X, int64_t T, int nHead, int dHead, int pos0,
                 double theta, int posStride, float *out) {
  return rope_common(ctx, X, T, nHead, dHead, pos0, theta, posStride, out, 0, false);
}

int fcu_rope_bwd(fcu_ctx *ctx, const float *dY, int64_t T, int nHead, int dHead, int pos0,
                 double theta, int posStride, float *dX, int accumulate) {
  return rope_common(ctx, dY, T, nHead, dHead, pos0, theta, posStride, dX, accumulate, true);
}

int fcu_slicecols_fwd(fcu_ctx *ctx, const float *X, int64_t M, int64_t K, int64_t off, int64_t len,
                      float *out) {
  FCU_CTX(ctx);
  FCU_REQUIRE(M >= 0 && K > 0 && off >= 0 && len >= 0 && off + len <= K, "fcu_slicecols: bad range");
  if (M == 0 || len == 0) return FCU_OK;
  slicecols_kernel<false><<<grid_for(M * len, kThreads, 65535), kThreads, 0, ctx->stream>>>(
      X, M, K, off, len, out, 0);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_slicecols_bwd(fcu_ctx *ctx, const float *dY, int64_t M, int64_t K, int64_t off,
                      int64_t len, float *dX, int accumulate) {
  FCU_CTX(ctx);
  FCU_REQUIRE(M >= 0 && K > 0 && off >= 0 && len >= 0 && off + len <= K, "fcu_slicecols: bad range");
  if (M == 0 || len == 0) return FCU_OK;
  slicecols_kernel<true><<<grid_for(M * len, kThreads, 65535), kThreads, 0, ctx->stream>>>(
      dY, M, K, off, len, dX, accumulate);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_swiglu_fwd(fcu_ctx *ctx, const float *G, const float *U, int64_t n, float *out) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0, "fcu_swiglu_fwd: bad n");
  if (n == 0) return FCU_OK;
  swiglu_fwd_kernel<<<grid_for(n, kThreads, 65535), kThreads, 0, ctx->stream>>>(G, U, n, out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_swiglu_bwd(fcu_ctx *ctx, const float *dO, const float *G, const float *U, int64_t n,
                   float *dG, float *dU, int accumulate) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0, "fcu_swiglu_bwd: bad n");
  if (n == 0) return FCU_OK;
  swiglu_bwd_kernel<<<grid_for(n, kThreads, 65535), kThreads, 0, ctx->stream>>>(dO, G, U, n, dG, dU,
                                                                                accumulate);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_add_fwd(fcu_ctx *ctx, const float *a, const float *b, int64_t n, float *out) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0, "fcu_add_fwd: bad n");
  if (n == 0) return FCU_OK;
  add_kernel<<<grid_for(n, kThreads, 65535), kThreads, 0, ctx->stream>>>(a, b, n, out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_add_bwd(fcu_ctx *ctx, const float *g, int64_t n, float *da, int accumulate_a, float *db,
                int accumulate_b) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0, "fcu_add_bwd: bad n");
  if (n == 0) return FCU_OK;
  add_bwd_kernel<<<grid_for(n, kThreads, 65535), kThreads, 0, ctx->stream>>>(g, n, da, accumulate_a,
                                                                             db, accumulate_b);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_ce_fwd(fcu_ctx *ctx, const float *logits, const int32_t *targets, int64_t T, int64_t V,
               float *loss_out, float *dunit) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T > 0 && V > 0 && T < (1ll << 31), "fcu_ce_fwd: bad shape");
  FCU_REQUIRE(logits && targets && loss_out && dunit, "fcu_ce_fwd: null pointer");
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(float) * (size_t)T, &scr);
  if (rc) return rc;
  float *row_loss = (float *)scr;
  bool aligned = ((uintptr_t)logits % 16 == 0) && ((uintptr_t)dunit % 16 == 0);
  if (aligned && V % 4 == 0)
    ce2_kernel<float><<<(int)T, kCe2Threads, 0, ctx->stream>>>(logits, targets, T, V, row_loss, dunit);
  else
    ce_fwd_kernel<float><<<(int)T, kCeThreads, 0, ctx->stream>>>(logits, targets, T, V, row_loss, dunit);
  FCU_CHECK_LAUNCH();
  mean_kernel<<<1, 1024, 0, ctx->stream>>>(row_loss, T, loss_out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_gather_windows(fcu_ctx *ctx, const int32_t *data, int64_t n, const int32_t *starts, int B,
                       int T1, int32_t *out) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n > 0 && B >= 0 && T1 > 0 && data && starts && out, "fcu_gather_windows: bad args");
  if (B == 0) return FCU_OK;
  const int64_t total = (int64_t)B * T1;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 4 * ctx->num_sms) blocks = 4 * ctx->num_sms;
  gather_windows_kernel<<<blocks, 256, 0, ctx->stream>>>(data, n, starts, B, T1, out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_ce_fwd_bf16grad(fcu_ctx *ctx, const float *logits, const int32_t *targets, int64_t T,
                        int64_t V, float *loss_out, void *dlogits_bf16) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T > 0 && V > 0 && T < (1ll << 31), "fcu_ce_fwd_bf16grad: bad shape");
  FCU_REQUIRE(logits && targets && loss_out && dlogits_bf16, "fcu_ce_fwd_bf16grad: null pointer");
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(float) * (size_t)T, &scr);
  if (rc) return rc;
  float *row_loss = (float *)scr;
  __nv_bfloat16 *du = (__nv_bfloat16 *)dlogits_bf16;
  bool aligned = ((uintptr_t)logits % 16 == 0) && ((uintptr_t)du % 8 == 0);
  if (aligned && V % 4 == 0)
    ce2_kernel<__nv_bfloat16><<<(int)T, kCe2Threads, 0, ctx->stream>>>(logits, targets, T, V, row_loss, du);
  else
    ce_fwd_kernel<__nv_bfloat16><<<(int)T, kCeThreads, 0, ctx->stream>>>(logits, targets, T, V,
                                                                                row_loss, du);
  FCU_CHECK_LAUNCH();
  mean_kernel<<<1, 1024, 0, ctx->stream>>>(row_loss, T, loss_out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- no-allocation CE
// Scratch of fcu_ce_fwd_static: one float per logits row, in a fixed device
// array instead of memory the context allocates.  It lives in every GPU that
// loads this library, for the life of the process.
namespace {

constexpr int64_t kCeStaticMaxRows = 65536;  // 256 KiB per device
static __device__ __align__(256) float g_ce_static_rows[kCeStaticMaxRows];

std::mutex g_ce_static_mu;
float *g_ce_static_ptr[64] = {nullptr};  // device address of the array, per device ordinal

// The host-side name g_ce_static_rows is only a stand-in for the device
// array, so its device address is looked up once per device, with that
// device current, and cached.
int ce_static_rows(int device, float **out) {
  FCU_REQUIRE(device >= 0 && device < 64, "fcu_ce_fwd_static: device ordinal %d out of range", device);
  std::lock_guard<std::mutex> lock(g_ce_static_mu);
  if (!g_ce_static_ptr[device]) {
    int cur = -1;
    FCU_CHECK_CUDA(cudaGetDevice(&cur));
    if (cur != device) FCU_CHECK_CUDA(cudaSetDevice(device));
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ce_static_rows);
    if (cur != device) {
      cudaError_t e2 = cudaSetDevice(cur);
      if (e == cudaSuccess) e = e2;
    }
    FCU_CHECK_CUDA(e);
    g_ce_static_ptr[device] = (float *)p;
  }
  *out = g_ce_static_ptr[device];
  return FCU_OK;
}

}  // namespace

extern "C" {

int fcu_ce_fwd_static(fcu_ctx *ctx, const float *logits, const int32_t *targets, int64_t T,
                      int64_t V, float *loss_out, float *dunit) {
  FCU_CTX(ctx);
  FCU_REQUIRE(T > 0 && V > 0, "fcu_ce_fwd_static: bad shape T=%lld V=%lld", (long long)T,
              (long long)V);
  FCU_REQUIRE(T <= kCeStaticMaxRows,
              "fcu_ce_fwd_static: T=%lld rows exceeds the fixed scratch of %lld rows; split the "
              "rows across calls or use fcu_ce_fwd",
              (long long)T, (long long)kCeStaticMaxRows);
  FCU_REQUIRE(logits && targets && loss_out && dunit, "fcu_ce_fwd_static: null pointer");
  float *row_loss = nullptr;
  int rc = ce_static_rows(ctx->device, &row_loss);
  if (rc) return rc;
  // Every row writes its own slot before mean_kernel reads it, so nothing
  // left over from an earlier call is ever read.
  bool aligned = ((uintptr_t)logits % 16 == 0) && ((uintptr_t)dunit % 16 == 0);
  if (aligned && V % 4 == 0)
    ce2_kernel<float><<<(int)T, kCe2Threads, 0, ctx->stream>>>(logits, targets, T, V, row_loss, dunit);
  else
    ce_fwd_kernel<float><<<(int)T, kCeThreads, 0, ctx->stream>>>(logits, targets, T, V, row_loss, dunit);
  FCU_CHECK_LAUNCH();
  mean_kernel<<<1, 1024, 0, ctx->stream>>>(row_loss, T, loss_out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_axpy_dev(fcu_ctx *ctx, const float *alpha_dev, const float *x, int64_t n, float *y,
                 int accumulate) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && alpha_dev && x && y, "fcu_axpy_dev: bad args");
  if (n == 0) return FCU_OK;
  axpy_dev_kernel<<<grid_for(n, kThreads, 65535), kThreads, 0, ctx->stream>>>(alpha_dev, x, n, y,
                                                                              accumulate);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_wsum_fwd(fcu_ctx *ctx, const float *Y, const float *t, int64_t n, float *out) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && Y && t && out, "fcu_wsum_fwd: bad args");
  wsum_kernel<<<1, 1024, 0, ctx->stream>>>(Y, t, n, out);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_scale(fcu_ctx *ctx, float *y, int64_t n, float alpha) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && y, "fcu_scale: bad args");
  if (n == 0) return FCU_OK;
  scale_kernel<<<grid_for(n, kThreads, 65535), kThreads, 0, ctx->stream>>>(y, n, alpha);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // extern "C"
