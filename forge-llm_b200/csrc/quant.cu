// Inference-side weight kernels: GGUF (GGML) block formats read on the GPU.
//
//   fcu_quant_matvec     QuantLinear.forward (src/L4/nn.js:27-32) for M input
//                        vectors at once: Y[m, n] = sum_k W[n, k] X[m, k], W a
//                        GGML byte stream (src/L3/quant.js: dotQ :215-310,
//                        matvec src/L0/numeric.js:85-100 for F32)
//   fcu_dequantize_rows  dequantize (src/L3/quant.js:109-209) of whole rows,
//                        optionally gathered by row id (the quantized
//                        embedding lookup, src/L6/transformer.js:122-132)
//
// The matvec reads each weight byte once (the bound is HBM).  Rows are
// contiguous in a GGML tensor, so a CTA takes a chunk of whole rows as one
// byte range and stages it in shared memory with one untiled bulk copy
// (cp.async.bulk, completing on an mbarrier; the range is widened to 16-byte
// boundaries and the last < 16 bytes of the tensor are read with plain loads).
// Three chunks are in flight per CTA.  Every format is then decoded from
// shared memory, whatever its block alignment (Q6_K blocks are 210 bytes).
// The input vectors live in shared memory for the whole kernel; each warp
// takes a row, each lane 8 elements of every 256-element unit, and the
// dequantized weight is used for all M vectors.  Formats and the arithmetic
// of each element follow quant.js (the dequantized weights are bit-identical
// to dequantize's); the dot products accumulate in fp32 instead of the JS's
// double, so results agree to fp32 rounding (relL2 ~1e-7).
#include <cuda_fp16.h>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace fcu {
namespace {

using namespace tc;

enum : int { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ5_0 = 6, kQ8_0 = 8, kQ4K = 12, kQ5K = 13, kQ6K = 14 };

// Elements and bytes per block (TYPE_INFO, src/L3/quant.js:42-55).
__host__ __device__ constexpr int fmt_bs(int t) {
  return t == kF32 || t == kF16 ? 1 : (t == kQ4K || t == kQ5K || t == kQ6K) ? 256 : 32;
}
__host__ __device__ constexpr int fmt_bb(int t) {
  return t == kF32 ? 4 : t == kF16 ? 2 : t == kQ4_0 ? 18 : t == kQ5_0 ? 22 : t == kQ8_0 ? 34
       : t == kQ4K ? 144 : t == kQ5K ? 176 : 210;
}
bool fmt_known(int t) {
  return t == kF32 || t == kF16 || t == kQ4_0 || t == kQ5_0 || t == kQ8_0 || t == kQ4K || t == kQ5K ||
         t == kQ6K;
}

// Every block size is even and tensors start 16-byte aligned, so 16-bit loads
// of block fields are aligned.
__device__ __forceinline__ uint32_t ld16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }
__device__ __forceinline__ uint32_t ld32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ float h2f(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }
// v (< 2^23) as a float without the int -> float conversion unit.
__device__ __forceinline__ float small_u2f(uint32_t v) {
  return __int_as_float(0x4B000000u | v) - 8388608.0f;
}

// getScaleMinK4Into (quant.js:98-106): 6-bit scale and min of sub-block j.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *q, float &sc, float &mn) {
  uint32_t s, m;
  if (j < 4) {
    s = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    s = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
  sc = small_u2f(s);
  mn = small_u2f(m);
}

// Element e of the block at b, as dequantize writes it.
template <int T>
__device__ __forceinline__ float deq_elem(const uint8_t *b, int e) {
  if (T == kF32) return __int_as_float((int)ld32(b));
  if (T == kF16) return h2f(ld16(b));
  if (T == kQ8_0) return h2f(ld16(b)) * (float)(int8_t)b[2 + e];
  if (T == kQ4_0 || T == kQ5_0) {
    const uint32_t u = b[2 + (e >> 1)];
    const int q = (int)((e & 1) ? (u >> 4) : (u & 0xF));
    return (float)(T == kQ4_0 ? q - 8 : q) * h2f(ld16(b));
  }
  if (T == kQ4K || T == kQ5K) {
    const int j = e >> 6, h = (e >> 5) & 1, l = e & 31, sub = 2 * j + h;
    float sc, mn;
    scale_min_k4(sub, b + 4, sc, mn);
    const float d1 = h2f(ld16(b)) * sc, n1 = h2f(ld16(b + 2)) * mn;
    const uint32_t byte = b[(T == kQ4K ? 16 : 48) + j * 32 + l];
    uint32_t q = h ? (byte >> 4) : (byte & 0xF);
    if (T == kQ5K) q += ((b[16 + l] >> sub) & 1) ? 16 : 0;
    return fmaf(d1, (float)q, -n1);
  }
  // Q6_K: ql[128], qh[64], scales[16], d at the end of the block
  const int n2 = e & ~127, r = e & 127, qd = r >> 5, l = r & 31;
  const uint32_t ql = b[(n2 >> 1) + l + (qd & 1) * 32];
  const uint32_t nib = qd < 2 ? (ql & 0xF) : (ql >> 4);
  const uint32_t qh = (b[128 + (n2 >> 2) + l] >> (2 * qd)) & 3;
  const int q = (int)(nib | (qh << 4)) - 32;
  const int sc = (int8_t)b[192 + (n2 >> 4) + (l >> 4) + 2 * qd];
  return h2f(ld16(b + 208)) * (float)sc * (float)q;
}

template <int T>
__global__ void __launch_bounds__(256) dequant_rows_kernel(const uint8_t *__restrict__ W, int64_t N, int64_t K,
                                                           int64_t row_bytes, const int32_t *__restrict__ rows,
                                                           int64_t nrows, float *__restrict__ out) {
  const int64_t total = nrows * K;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / K, k = idx - r * K;
    const int64_t src = rows ? rows[r] : r;
    float v;
    if (src < 0 || src >= N) {
      v = __int_as_float(0x7fc00000);   // a row that is not there reads as NaN
    } else {
      constexpr int bs = fmt_bs(T), bb = fmt_bb(T);
      v = deq_elem<T>(W + src * row_bytes + (k / bs) * bb, (int)(k % bs));
    }
    out[idx] = v;
  }
}

// ---------------------------------------------------------------- matvec
constexpr int kQmvThreads = 256;
constexpr int kQmvWarps = kQmvThreads / 32;
constexpr int kQmvStages = 3;
constexpr int kQmvChunk = 16384;               // bytes of rows per stage (3 CTAs per SM fit)
constexpr int kQmvChunkMax = 24576;            // a stage grown to hold 8 rows
constexpr int kQmvPad = 32;                    // room for the 16-byte widening
// Shared-memory header: mbarriers, abort flag, counters, the barrier path's
// row partials at 128, the free-run partials [stages][8][MB] at 512.
__host__ __device__ constexpr int qmv_header(int mb) { return (512 + kQmvStages * 8 * mb * 4 + 127) & ~127; }

struct QmvArgs {
  const uint8_t *W;
  int64_t N, K, row_bytes, total_bytes;
  const float *X;   // [M, K]
  float *Y;         // [M, N]
  int M, rows_per_chunk;
  int64_t n_chunks;
  int *err;
  int stage_bytes;  // bytes of rows per stage (a multiple of 16); stages are stage_bytes + 32 apart
  int free_run;     // 1: every chunk holds whole warps' rows (or is the last) and no tail bytes:
                    // warps run through the chunks independently (no CTA barrier per chunk)
};

// acc[m] += w * x[m][k] for the MB vectors (m < M).
template <int MB>
__device__ __forceinline__ void fma_x(float (&acc)[MB], float w, const float *xs, int64_t K, int M, int64_t k) {
#pragma unroll
  for (int m = 0; m < MB; m++)
    if (m < M) acc[m] = fmaf(w, xs[m * K + k], acc[m]);
}
template <int MB>
__device__ __forceinline__ void fma_x4(float (&acc)[MB], const float (&w)[4], const float *xs, int64_t K, int M,
                                       int64_t k) {
#pragma unroll
  for (int m = 0; m < MB; m++)
    if (m < M) {
      const float4 x = *reinterpret_cast<const float4 *>(xs + m * K + k);
      acc[m] = fmaf(w[0], x.x, acc[m]);
      acc[m] = fmaf(w[1], x.y, acc[m]);
      acc[m] = fmaf(w[2], x.z, acc[m]);
      acc[m] = fmaf(w[3], x.w, acc[m]);
    }
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// Where x[k] sits in shared memory.  For Q4_K / Q5_K the float4 index bits
// (2-3) are XORed with the 64-element group bits (6-7), for Q8_0 bit 2 with
// the block parity (bit 5): the 8 lanes of a quarter-warp then read 8
// different bank quads.  Linear for the others.
template <int T>
__device__ __forceinline__ int64_t xs_swz(int64_t k) {
  if (T == kQ4K || T == kQ5K) return k ^ (((k >> 6) & 3) << 2);
  if (T == kQ8_0) return k ^ (((k >> 5) & 1) << 2);   // odd blocks' halves swapped
  return k;
}
template <int T>
__host__ __device__ constexpr bool uses_xsum() { return T == kQ4K || T == kQ5K; }

// 6-bit scale / min of K-quant sub-block j from the block header words
// hy = scales[0..3], hz = scales[4..7], hw = scales[8..11] (getScaleMinK4Into).
__device__ __forceinline__ void scale_min_hdr(int j, uint32_t hy, uint32_t hz, uint32_t hw, float &sc, float &mn) {
  uint32_t s, m;
  if (j < 4) {
    s = byte_of(hy, j) & 63;
    m = byte_of(hz, j) & 63;
  } else {
    s = (byte_of(hw, j - 4) & 0xF) | ((byte_of(hy, j - 4) >> 6) << 4);
    m = (byte_of(hw, j - 4) >> 4) | ((byte_of(hz, j - 4) >> 6) << 4);
  }
  sc = small_u2f(s);
  mn = small_u2f(m);
}

// One row (in shared memory) against the MB vectors: this lane's share of
// the row's 256-element units u0, u0 + ustep, ... (a K-quant super-block, 8
// blocks of 32, or 256 F32 / F16 elements; lane l takes 8 of the 256).
template <int T, int MB>
__device__ __forceinline__ void row_dot(const uint8_t *row, const float *xs, int64_t K, int M, int lane,
                                        float (&acc)[MB], int u0, int ustep) {
  if (T == kQ4K || T == kQ5K) {
    // lane = (super-block sbl of 4, 64-element group j, half h): 16 quant
    // bytes = the 16 low-nibble elements j*64 + 16h + i (sub-block 2j) and
    // the 16 high-nibble ones 32 further on (sub-block 2j + 1).  Each
    // sub-block's scale is factored out: d*sc*sum(q x) - dmin*m*sum(x), with
    // the sums of x over 16 elements precomputed (xsum); x is read through
    // the swizzle of xs_index.
    const int sbl = lane >> 3, j = (lane >> 1) & 3, h = lane & 1;
    const int nsb = (int)(K >> 8);
    const float *xsum = xs + (int64_t)M * K;     // [M][K / 16]
    // The loop runs warp-uniformly (the scale shuffles need every lane); a
    // lane group past the row's last super-block reads super-block 0 and
    // skips the sums.
#pragma unroll 1
    for (int base = u0 * 4; base < nsb; base += ustep * 4) {
      const int sb = base + sbl;
      const bool act = sb < nsb;
      const uint8_t *b = row + (int64_t)(act ? sb : 0) * fmt_bb(T);
      const uint4 hd = *reinterpret_cast<const uint4 *>(b);   // d, dmin, scales[12]
      const uint4 qv = *reinterpret_cast<const uint4 *>(b + (T == kQ4K ? 16 : 48) + j * 32 + 16 * h);
      uint4 qhv = make_uint4(0, 0, 0, 0);
      if (T == kQ5K) qhv = *reinterpret_cast<const uint4 *>(b + 16 + 16 * h);
      const float d = h2f(hd.x & 0xFFFFu), dmin = h2f(hd.x >> 16);
      // the 8 lanes of a super-block decode one sub-block's scale / min each
      // (lane (j, h): sub-block 2j + h) and fetch their pair's by shuffle
      float scm, mnm;
      scale_min_hdr(2 * j + h, hd.y, hd.z, hd.w, scm, mnm);
      const float sc0 = __shfl_sync(0xffffffffu, scm, lane & ~1), sc1 = __shfl_sync(0xffffffffu, scm, lane | 1);
      const float mn0 = __shfl_sync(0xffffffffu, mnm, lane & ~1), mn1 = __shfl_sync(0xffffffffu, mnm, lane | 1);
      if (!act) continue;
      const int64_t klo = (int64_t)sb * 256 + j * 64 + 16 * h;
      if constexpr (MB <= 4) {
      // packed f32x2 sums: (even, odd) elements of the even / odd float4s,
      // four short FMA chains per half
      float2 slo[MB][2], shi[MB][2];
#pragma unroll
      for (int m = 0; m < MB; m++)
        slo[m][0] = slo[m][1] = shi[m][0] = shi[m][1] = make_float2(0.f, 0.f);
      const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
      const uint32_t hw[4] = {qhv.x, qhv.y, qhv.z, qhv.w};
      const float2 bias = make_float2(-8388608.0f, -8388608.0f);
#pragma unroll
      for (int f = 0; f < 4; f++) {
        uint32_t lo = qw[f] & 0x0F0F0F0Fu, hi = (qw[f] >> 4) & 0x0F0F0F0Fu;
        if (T == kQ5K) {   // bit 2j (low) / 2j+1 (high) of each qh byte is the 5th bit
          lo |= ((hw[f] >> (2 * j)) & 0x01010101u) << 4;
          hi |= ((hw[f] >> (2 * j + 1)) & 0x01010101u) << 4;
        }
        // the bytes as 2^23 + q, the 2^23 removed two at a time
        float2 ql[2], qh[2];
#pragma unroll
        for (int e = 0; e < 2; e++) {
          ql[e] = add2(make_float2(__int_as_float((int)__byte_perm(lo, 0x4B000000u, 0x7650u | (2 * e))),
                                   __int_as_float((int)__byte_perm(lo, 0x4B000000u, 0x7650u | (2 * e + 1)))),
                       bias);
          qh[e] = add2(make_float2(__int_as_float((int)__byte_perm(hi, 0x4B000000u, 0x7650u | (2 * e))),
                                   __int_as_float((int)__byte_perm(hi, 0x4B000000u, 0x7650u | (2 * e + 1)))),
                       bias);
        }
#pragma unroll
        for (int m = 0; m < MB; m++)
          if (m < M) {
            const float4 xl = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(klo + 4 * f));
            const float4 xh = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(klo + 32 + 4 * f));
            float2 &sl = slo[m][f & 1], &sh = shi[m][f & 1];
            sl = fma2(ql[0], make_float2(xl.x, xl.y), sl);
            sl = fma2(ql[1], make_float2(xl.z, xl.w), sl);
            sh = fma2(qh[0], make_float2(xh.x, xh.y), sh);
            sh = fma2(qh[1], make_float2(xh.z, xh.w), sh);
          }
      }
      const float d1 = d * sc0, n1 = dmin * mn0, d2 = d * sc1, n2 = dmin * mn1;
#pragma unroll
      for (int m = 0; m < MB; m++)
        if (m < M) {
          const float xl = xsum[m * (K >> 4) + (klo >> 4)], xh = xsum[m * (K >> 4) + (klo >> 4) + 2];
          const float2 l2 = add2(slo[m][0], slo[m][1]), h2 = add2(shi[m][0], shi[m][1]);
          acc[m] = fmaf(d1, l2.x + l2.y, acc[m]);
          acc[m] = fmaf(-n1, xl, acc[m]);
          acc[m] = fmaf(d2, h2.x + h2.y, acc[m]);
          acc[m] = fmaf(-n2, xh, acc[m]);
        }
      } else {   // 8 vectors: scalar sums (the packed ones would spill)
      // two partial sums per half (even / odd float4) keep the FMA chains short
      float slo[MB][2], shi[MB][2];
#pragma unroll
      for (int m = 0; m < MB; m++) slo[m][0] = slo[m][1] = shi[m][0] = shi[m][1] = 0.f;
      const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
      const uint32_t hw[4] = {qhv.x, qhv.y, qhv.z, qhv.w};
#pragma unroll
      for (int f = 0; f < 4; f++) {
        uint32_t lo = qw[f] & 0x0F0F0F0Fu, hi = (qw[f] >> 4) & 0x0F0F0F0Fu;
        if (T == kQ5K) {   // bit 2j (low) / 2j+1 (high) of each qh byte is the 5th bit
          lo |= ((hw[f] >> (2 * j)) & 0x01010101u) << 4;
          hi |= ((hw[f] >> (2 * j + 1)) & 0x01010101u) << 4;
        }
        float ql[4], qh[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          ql[e] = __int_as_float((int)__byte_perm(lo, 0x4B000000u, 0x7650u | e)) - 8388608.0f;
          qh[e] = __int_as_float((int)__byte_perm(hi, 0x4B000000u, 0x7650u | e)) - 8388608.0f;
        }
#pragma unroll
        for (int m = 0; m < MB; m++)
          if (m < M) {
            const float4 xl = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(klo + 4 * f));
            const float4 xh = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(klo + 32 + 4 * f));
            float &sl = slo[m][f & 1], &sh = shi[m][f & 1];
            sl = fmaf(ql[0], xl.x, sl);
            sl = fmaf(ql[1], xl.y, sl);
            sl = fmaf(ql[2], xl.z, sl);
            sl = fmaf(ql[3], xl.w, sl);
            sh = fmaf(qh[0], xh.x, sh);
            sh = fmaf(qh[1], xh.y, sh);
            sh = fmaf(qh[2], xh.z, sh);
            sh = fmaf(qh[3], xh.w, sh);
          }
      }
      const float d1 = d * sc0, n1 = dmin * mn0, d2 = d * sc1, n2 = dmin * mn1;
#pragma unroll
      for (int m = 0; m < MB; m++)
        if (m < M) {
          const float xl = xsum[m * (K >> 4) + (klo >> 4)], xh = xsum[m * (K >> 4) + (klo >> 4) + 2];
          acc[m] = fmaf(d1, slo[m][0] + slo[m][1], acc[m]);
          acc[m] = fmaf(-n1, xl, acc[m]);
          acc[m] = fmaf(d2, shi[m][0] + shi[m][1], acc[m]);
          acc[m] = fmaf(-n2, xh, acc[m]);
        }
      }
    }
  } else if (T == kQ6K && MB <= 4) {
    // 16 lanes per super-block (two super-blocks per warp step): lane (sub,
    // half, l0) takes elements half*128 + qd*32 + l0 .. +3 for qd = 0..3.
    // The 4 low-nibble bytes and the 4 high-bit bytes of those elements are
    // combined 4 at a time in 32-bit words, each byte becomes 2^23 + q by one
    // permute, and the 2^23 + 32 offset goes in one packed add; the 16-element
    // group's scale multiplies the group's sum.  (Blocks are 210 bytes, so
    // the words are read as 16-bit halves.)
    const int sub = lane >> 4, half = (lane >> 3) & 1, l0 = (lane & 7) * 4, is = l0 >> 4;
    const int nsb = (int)(K >> 8);
    const float2 bias = make_float2(-8388640.0f, -8388640.0f);   // -(2^23 + 32)
#pragma unroll 2
    for (int sb = 2 * u0 + sub; sb < nsb; sb += 2 * ustep) {
      const uint8_t *b = row + (int64_t)sb * 210;
      const float d = h2f(ld16(b + 208));
      const uint8_t *qlp = b + half * 64 + l0, *qhp = b + 128 + half * 32 + l0;
      const uint32_t qa = ld16(qlp) | (ld16(qlp + 2) << 16);          // qd 0 (low nibbles), 2 (high)
      const uint32_t qb = ld16(qlp + 32) | (ld16(qlp + 34) << 16);    // qd 1, 3
      const uint32_t qh = ld16(qhp) | (ld16(qhp + 2) << 16);
      const int64_t k0 = (int64_t)sb * 256 + half * 128 + l0;
#pragma unroll
      for (int qd = 0; qd < 4; qd++) {
        const uint32_t src = (qd & 1) ? qb : qa;
        const uint32_t q4 = ((qd < 2 ? src : (src >> 4)) & 0x0F0F0F0Fu) | (((qh >> (2 * qd)) & 0x03030303u) << 4);
        const float dq = d * (float)(int8_t)b[192 + half * 8 + is + 2 * qd];
        const float2 w01 = add2(make_float2(__int_as_float((int)__byte_perm(q4, 0x4B000000u, 0x7650u)),
                                            __int_as_float((int)__byte_perm(q4, 0x4B000000u, 0x7651u))),
                                bias);
        const float2 w23 = add2(make_float2(__int_as_float((int)__byte_perm(q4, 0x4B000000u, 0x7652u)),
                                            __int_as_float((int)__byte_perm(q4, 0x4B000000u, 0x7653u))),
                                bias);
#pragma unroll
        for (int m = 0; m < MB; m++)
          if (m < M) {
            const float4 x = *reinterpret_cast<const float4 *>(xs + m * K + k0 + qd * 32);
            const float2 t = fma2(w23, make_float2(x.z, x.w), mul2(w01, make_float2(x.x, x.y)));
            acc[m] = fmaf(dq, t.x + t.y, acc[m]);
          }
      }
    }
  } else if (T == kQ6K) {   // 8 vectors: a lane per 2 elements of 4 groups (fewer live registers)
    const int half = lane >> 4, l0 = (lane & 15) * 2, is = l0 >> 4;
    const int nsb = (int)(K >> 8);
#pragma unroll 2
    for (int sb = u0; sb < nsb; sb += ustep) {
      const uint8_t *b = row + (int64_t)sb * 210;
      const float d = h2f(ld16(b + 208));
      const uint32_t qa = ld16(b + half * 64 + l0), qb = ld16(b + half * 64 + 32 + l0);
      const uint32_t qh = ld16(b + 128 + half * 32 + l0);
#pragma unroll
      for (int qd = 0; qd < 4; qd++) {
        const float dq = d * (float)(int8_t)b[192 + half * 8 + is + 2 * qd];
        const uint32_t ql = (qd & 1) ? qb : qa;
        float w[2];
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const uint32_t byte = (ql >> (8 * e)) & 0xFF;
          const uint32_t nib = qd < 2 ? (byte & 0xF) : (byte >> 4);
          const uint32_t hb = (qh >> (8 * e + 2 * qd)) & 3;
          w[e] = dq * (small_u2f(nib | (hb << 4)) - 32.0f);
        }
        const int64_t k = (int64_t)sb * 256 + half * 128 + qd * 32 + l0;
#pragma unroll
        for (int m = 0; m < MB; m++)
          if (m < M) {
            const float2 x = *reinterpret_cast<const float2 *>(xs + m * K + k);
            acc[m] = fmaf(w[0], x.x, acc[m]);
            acc[m] = fmaf(w[1], x.y, acc[m]);
          }
      }
    }
  } else if (T == kQ8_0 || T == kQ4_0 || T == kQ5_0) {
    const int64_t nblk = K >> 5;
    const int nunit = (int)((nblk + 7) >> 3);
    const int o = (lane & 3) * 8;
#pragma unroll 2
    for (int u = u0; u < nunit; u += ustep) {
      const int64_t blk = (int64_t)u * 8 + (lane >> 2);
      if (blk >= nblk) continue;
      const uint8_t *b = row + blk * fmt_bb(T);
      const float d = h2f(ld16(b));
      if constexpr (T == kQ8_0) {
        // d * sum(q x): int8 q as a float by one byte permute into 2^23's
        // exponent (q + 128 after the sign flip), then the bias removed
        if constexpr (MB <= 4) {
        float2 q[4];
        const float2 bias = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const uint32_t v = ld16(b + 2 + o + e);
          q[e / 2] = add2(make_float2(__int_as_float((int)(__byte_perm(v, 0x4B000000u, 0x7650u) ^ 0x80u)),
                                      __int_as_float((int)(__byte_perm(v, 0x4B000000u, 0x7651u) ^ 0x80u))),
                          bias);
        }
        const int64_t k = blk * 32 + o;
#pragma unroll
        for (int m = 0; m < MB; m++)
          if (m < M) {
            const float4 x0 = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(k));
            const float4 x1 = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(k + 4));
            float2 sa = mul2(q[0], make_float2(x0.x, x0.y)), sb = mul2(q[2], make_float2(x1.x, x1.y));
            sa = fma2(q[1], make_float2(x0.z, x0.w), sa);
            sb = fma2(q[3], make_float2(x1.z, x1.w), sb);
            const float2 t = add2(sa, sb);
            acc[m] = fmaf(d, t.x + t.y, acc[m]);
          }
        } else {
        float q[8];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const uint32_t v = ld16(b + 2 + o + e);
          q[e] = __int_as_float((int)(__byte_perm(v, 0x4B000000u, 0x7650u) ^ 0x80u)) - 8388736.0f;
          q[e + 1] = __int_as_float((int)(__byte_perm(v, 0x4B000000u, 0x7651u) ^ 0x80u)) - 8388736.0f;
        }
        const int64_t k = blk * 32 + o;
#pragma unroll
        for (int m = 0; m < MB; m++)
          if (m < M) {
            const float4 x0 = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(k));
            const float4 x1 = *reinterpret_cast<const float4 *>(xs + m * K + xs_swz<T>(k + 4));
            float sa = q[0] * x0.x, sb = q[4] * x1.x;
            sa = fmaf(q[1], x0.y, sa);
            sb = fmaf(q[5], x1.y, sb);
            sa = fmaf(q[2], x0.z, sa);
            sb = fmaf(q[6], x1.z, sb);
            sa = fmaf(q[3], x0.w, sa);
            sb = fmaf(q[7], x1.w, sb);
            acc[m] = fmaf(d, sa + sb, acc[m]);
          }
        }
      } else {
        // byte 2 + j/2, nibble j&1 (the reference's reading of these blocks)
        float w[8];
#pragma unroll
        for (int e = 0; e < 8; e += 4) {
          const uint32_t v = ld16(b + 2 + (o >> 1) + (e >> 1));
#pragma unroll
          for (int t = 0; t < 4; t++) {
            const uint32_t q = (v >> (4 * t)) & 0xF;
            w[e + t] = (small_u2f(q) - (T == kQ4_0 ? 8.0f : 0.0f)) * d;
          }
        }
        const int64_t k = blk * 32 + o;
        const float w0[4] = {w[0], w[1], w[2], w[3]}, w1[4] = {w[4], w[5], w[6], w[7]};
        fma_x4<MB>(acc, w0, xs, K, M, k);
        fma_x4<MB>(acc, w1, xs, K, M, k + 4);
      }
    }
  } else {   // F32 / F16: element k of the row at byte k * (4 | 2)
    const int nunit = (int)((K + 255) >> 8);
    for (int u = u0; u < nunit; u += ustep) {
#pragma unroll
      for (int t = 0; t < 8; t++) {
        const int64_t k = (int64_t)u * 256 + t * 32 + lane;
        if (k < K) {
          const float w = T == kF32 ? __int_as_float((int)ld32(row + 4 * k)) : h2f(ld16(row + 2 * k));
          fma_x<MB>(acc, w, xs, K, M, k);
        }
      }
    }
  }
}

template <int T, int MB>
__global__ void __launch_bounds__(kQmvThreads, 3) quant_matvec_kernel(QmvArgs a) {
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 64);
  float *part = reinterpret_cast<float *>(smem + 128);   // [8 warps][MB]: split rows' partials
  unsigned *done_cnt = reinterpret_cast<unsigned *>(smem + 384);   // [stages]: warps done with the stage
  unsigned *n_iss = reinterpret_cast<unsigned *>(smem + 400);      // [stages]: copies issued into it
  unsigned *row_cnt = reinterpret_cast<unsigned *>(smem + 448);    // [stages][8]: warps done with a row
  float *fpart = reinterpret_cast<float *>(smem + 512);            // [stages][8][MB]: free-run partials
  const int buf_stride = a.stage_bytes + kQmvPad;
  uint8_t *bufs = smem + qmv_header(MB);
  float *xs = reinterpret_cast<float *>(bufs + kQmvStages * buf_stride);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < kQmvStages; s++) {
      mbar_init(&full[s], 1);
      done_cnt[s] = 0;
      n_iss[s] = 0;
      for (int r = 0; r < kQmvWarps; r++) row_cnt[s * kQmvWarps + r] = 0;
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();
  const int64_t my_chunks =
      blockIdx.x < a.n_chunks ? (a.n_chunks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t tma_limit = a.total_bytes & ~(int64_t)15;   // bulk copies stay below this

  // chunk i of this CTA: rows, byte range, 16-byte-aligned copy start
  auto chunk_rows = [&](int64_t i, int64_t &r0, int64_t &r1) {
    const int64_t c = blockIdx.x + i * gridDim.x;
    r0 = c * a.rows_per_chunk;
    r1 = r0 + a.rows_per_chunk < a.N ? r0 + a.rows_per_chunk : a.N;
  };
  auto issue = [&](int64_t i) {
    int64_t r0, r1;
    chunk_rows(i, r0, r1);
    const int64_t s0 = r0 * a.row_bytes, e0 = r1 * a.row_bytes;
    const int64_t a0 = s0 & ~(int64_t)15;
    int64_t a1 = (e0 + 15) & ~(int64_t)15;
    if (a1 > tma_limit) a1 = tma_limit;
    const int st = (int)(i % kQmvStages);
    const uint32_t bytes = a1 > a0 ? (uint32_t)(a1 - a0) : 0u;
    n_iss[st]++;
    mbar_expect_tx(&full[st], bytes);
    if (bytes) bulk_load_1d(bufs + st * buf_stride, a.W + a0, bytes, &full[st]);
  };

  if (tid == 0)
    for (int64_t i = 0; i < my_chunks && i < kQmvStages; i++) issue(i);
  // the input vectors, for the whole kernel (and, for the K-quants, their
  // sums over each 16 elements, in element order)
  for (int64_t i = tid; i < (int64_t)a.M * a.K; i += kQmvThreads) {
    const int64_t m = i / a.K, k = i - m * a.K;
    xs[m * a.K + xs_swz<T>(k)] = a.X[i];
  }
  if (uses_xsum<T>()) {
    float *xsum = xs + (int64_t)a.M * a.K;
    for (int64_t g = tid; g < (int64_t)a.M * (a.K >> 4); g += kQmvThreads) {
      const float *src = a.X + g * 16;
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < 16; i++) v += src[i];
      xsum[g] = v;
    }
  }
  __syncthreads();

  if (a.free_run) {
    // Each warp takes its rows of every chunk as soon as the chunk has
    // landed (rows warp, warp + 8, ... of a chunk of 8k rows; a chunk of 1, 2
    // or 4 rows gives each row 8, 4 or 2 warps, whose partial sums the warp
    // that finishes the row last adds in warp order).  The warp that finishes
    // a stage last (a shared-memory counter) refills it with the chunk
    // kQmvStages further on.
    bool ok = true;
    for (int64_t i = 0; i < my_chunks; i++) {
      const int st = (int)(i % kQmvStages);
      if (!warp_wait(&full[st], (uint32_t)((i / kQmvStages) & 1), abort_flag)) {
        ok = false;
        break;
      }
      int64_t r0, r1;
      chunk_rows(i, r0, r1);
      const int64_t s0 = r0 * a.row_bytes;
      const uint8_t *rows = bufs + st * buf_stride + (s0 & 15);
      const int rc = (int)(r1 - r0);
      int wpr = 1;
      while (wpr * 2 * rc <= kQmvWarps) wpr *= 2;
      const int groups = kQmvWarps / wpr, gi = warp / wpr, wi = warp - gi * wpr;
      for (int lr = gi; lr < rc; lr += groups) {
        float acc[MB];
#pragma unroll
        for (int m = 0; m < MB; m++) acc[m] = 0.f;
        if (wpr == 1)   // the common case, with the unit loop's start and step known
          row_dot<T, MB>(rows + (int64_t)lr * a.row_bytes, xs, a.K, a.M, lane, acc, 0, 1);
        else
          row_dot<T, MB>(rows + (int64_t)lr * a.row_bytes, xs, a.K, a.M, lane, acc, wi, wpr);
        float v[MB];
#pragma unroll
        for (int m = 0; m < MB; m++) v[m] = warp_sum(acc[m]);
        if (lane == 0) {
          if (wpr == 1) {
#pragma unroll
            for (int m = 0; m < MB; m++)
              if (m < a.M) a.Y[m * a.N + r0 + lr] = v[m];
          } else {
            float *pr = fpart + (st * kQmvWarps + lr * wpr) * MB;   // this row's wpr slots
#pragma unroll
            for (int m = 0; m < MB; m++) pr[wi * MB + m] = v[m];
            __threadfence_block();
            if (atomicAdd(&row_cnt[st * kQmvWarps + lr], 1u) == (unsigned)(wpr - 1)) {
              row_cnt[st * kQmvWarps + lr] = 0;
              __threadfence_block();
              for (int m = 0; m < a.M && m < MB; m++) {
                float t = 0.f;
                for (int w = 0; w < wpr; w++) t += ((volatile float *)pr)[w * MB + m];
                a.Y[m * a.N + r0 + lr] = t;
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();   // this warp's reads of the stage come before its count
        if (atomicAdd(&done_cnt[st], 1u) == (unsigned)(kQmvWarps - 1)) {
          done_cnt[st] = 0;
          __threadfence_block();
          if (i + kQmvStages < my_chunks) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // before the copy rewrites it
            issue(i + kQmvStages);
          }
        }
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicExch(a.err, 40);
    }
    __syncthreads();
    // every copy issued has landed before the CTA exits (at once on the normal path)
    if (tid == 0)
      for (int s = 0; s < kQmvStages; s++)
        if (n_iss[s]) mbar_wait_drain(&full[s], (n_iss[s] - 1) & 1u);
    return;
  }

  for (int64_t i = 0; i < my_chunks; i++) {
    const int st = (int)(i % kQmvStages);
    const uint32_t ph = (uint32_t)((i / kQmvStages) & 1);
    bool ok = mbar_wait(&full[st], ph, abort_flag);
    if (!__syncthreads_and(ok)) {
      if (tid == 0) {
        *abort_flag = 1;
        atomicExch(a.err, 40);
        // drain the copies still in flight before the CTA exits
        for (int64_t j = i; j < my_chunks && j < i + kQmvStages; j++)
          mbar_wait_drain(&full[j % kQmvStages], (uint32_t)((j / kQmvStages) & 1));
      }
      return;
    }
    int64_t r0, r1;
    chunk_rows(i, r0, r1);
    const int64_t s0 = r0 * a.row_bytes, e0 = r1 * a.row_bytes;
    const int64_t a0 = s0 & ~(int64_t)15;
    uint8_t *buf = bufs + st * buf_stride;
    // the tensor's last < 16 bytes, which no bulk copy covers
    const int64_t tail0 = tma_limit > a0 ? tma_limit : a0;
    if (e0 > tail0) {
      for (int64_t t = tail0 + tid; t < e0; t += kQmvThreads) buf[t - a0] = a.W[t];
      __syncthreads();
    }
    const uint8_t *rows = buf + (s0 - a0);
    // rows of the chunk over the warps; a chunk of fewer than 8 rows gives
    // each row wpr warps, which take its units in turn and leave partial sums
    // that are added in warp order below (deterministic)
    const int rc = (int)(r1 - r0);
    int wpr = 1;
    while (wpr * 2 * rc <= kQmvWarps) wpr *= 2;
    const int groups = kQmvWarps / wpr, gi = warp / wpr, wi = warp - gi * wpr;
    for (int lr = gi; lr < rc; lr += groups) {
      float acc[MB];
#pragma unroll
      for (int m = 0; m < MB; m++) acc[m] = 0.f;
      row_dot<T, MB>(rows + (int64_t)lr * a.row_bytes, xs, a.K, a.M, lane, acc, wi, wpr);
#pragma unroll
      for (int m = 0; m < MB; m++) {
        const float v = warp_sum(acc[m]);
        if (lane == 0 && m < a.M) {
          if (wpr == 1) a.Y[m * a.N + r0 + lr] = v;
          else part[(lr * wpr + wi) * MB + m] = v;
        }
      }
    }
    __syncthreads();   // every warp is done with this stage before it is refilled
    if (wpr > 1)
      for (int t = tid; t < rc * a.M; t += kQmvThreads) {
        const int r = t / a.M, m = t - r * a.M;
        float v = 0.f;
        for (int w = 0; w < wpr; w++) v += part[(r * wpr + w) * MB + m];
        a.Y[m * a.N + r0 + r] = v;
      }
    if (tid == 0 && i + kQmvStages < my_chunks) issue(i + kQmvStages);
  }
}

template <int T>
int launch_matvec_t(fcu_ctx *ctx, const QmvArgs &a, int MB, int grid, size_t smem) {
  cudaError_t e;
  switch (MB) {
#define FCU_QMV_CASE(mb)                                                                           \
  case mb: {                                                                                       \
    static bool set[64] = {false};                                                                 \
    if (!set[ctx->device & 63]) {                                                                  \
      FCU_CHECK_CUDA(cudaFuncSetAttribute(quant_matvec_kernel<T, mb>,                              \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)); \
      set[ctx->device & 63] = true;                                                                \
    }                                                                                              \
    e = launch_pdl(quant_matvec_kernel<T, mb>, dim3(grid), dim3(kQmvThreads), smem, ctx->stream, a); \
    break;                                                                                         \
  }
    FCU_QMV_CASE(1)
    FCU_QMV_CASE(2)
    FCU_QMV_CASE(4)
    FCU_QMV_CASE(8)
#undef FCU_QMV_CASE
    default:
      return FCU_ERR_ARG;
  }
  FCU_CHECK_CUDA(e);
  note_launch();
  return FCU_OK;
}

int launch_matvec(fcu_ctx *ctx, int type, const QmvArgs &a, int MB, int grid, size_t smem) {
  switch (type) {
    case kF32: return launch_matvec_t<kF32>(ctx, a, MB, grid, smem);
    case kF16: return launch_matvec_t<kF16>(ctx, a, MB, grid, smem);
    case kQ4_0: return launch_matvec_t<kQ4_0>(ctx, a, MB, grid, smem);
    case kQ5_0: return launch_matvec_t<kQ5_0>(ctx, a, MB, grid, smem);
    case kQ8_0: return launch_matvec_t<kQ8_0>(ctx, a, MB, grid, smem);
    case kQ4K: return launch_matvec_t<kQ4K>(ctx, a, MB, grid, smem);
    case kQ5K: return launch_matvec_t<kQ5K>(ctx, a, MB, grid, smem);
    case kQ6K: return launch_matvec_t<kQ6K>(ctx, a, MB, grid, smem);
  }
  return FCU_ERR_ARG;
}

template <int T>
int matvec_occupancy_t(int mb, size_t smem, int *out) {
  auto query = [&](auto kernel) -> int {
    FCU_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    FCU_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(out, kernel, kQmvThreads, smem));
    return FCU_OK;
  };
  switch (mb) {
    case 1: return query(quant_matvec_kernel<T, 1>);
    case 2: return query(quant_matvec_kernel<T, 2>);
    case 4: return query(quant_matvec_kernel<T, 4>);
    case 8: return query(quant_matvec_kernel<T, 8>);
  }
  return FCU_ERR_ARG;
}

int matvec_occupancy_uncached(int type, int mb, size_t smem, int *out) {
  switch (type) {
    case kF32: return matvec_occupancy_t<kF32>(mb, smem, out);
    case kF16: return matvec_occupancy_t<kF16>(mb, smem, out);
    case kQ4_0: return matvec_occupancy_t<kQ4_0>(mb, smem, out);
    case kQ5_0: return matvec_occupancy_t<kQ5_0>(mb, smem, out);
    case kQ8_0: return matvec_occupancy_t<kQ8_0>(mb, smem, out);
    case kQ4K: return matvec_occupancy_t<kQ4K>(mb, smem, out);
    case kQ5K: return matvec_occupancy_t<kQ5K>(mb, smem, out);
    case kQ6K: return matvec_occupancy_t<kQ6K>(mb, smem, out);
  }
  return FCU_ERR_ARG;
}

// Cached per (device, format, vectors, shared memory): the decode step calls
// the matvec with a handful of shapes, many times.
int matvec_occupancy(int type, int mb, size_t smem, int *out) {
  struct Entry {
    int dev = -1, type = -1, mb = 0;
    size_t smem = 0;
    int per_sm = 0;
  };
  static thread_local Entry cache[32];
  static thread_local int next = 0;
  int dev = 0;
  FCU_CHECK_CUDA(cudaGetDevice(&dev));
  for (const Entry &e : cache)
    if (e.dev == dev && e.type == type && e.mb == mb && e.smem == smem) {
      *out = e.per_sm;
      return FCU_OK;
    }
  int rc = matvec_occupancy_uncached(type, mb, smem, out);
  if (rc) return rc;
  cache[next] = Entry{dev, type, mb, smem, *out};
  next = (next + 1) % 32;
  return FCU_OK;
}

template <int T>
void launch_dequant_t(cudaStream_t st, int grid, const uint8_t *W, int64_t N, int64_t K, int64_t rb,
                      const int32_t *rows, int64_t nrows, float *out) {
  dequant_rows_kernel<T><<<grid, 256, 0, st>>>(W, N, K, rb, rows, nrows, out);
}

}  // namespace
}  // namespace fcu

extern "C" {

int64_t fcu_ggml_row_bytes(int type, int64_t n) {
  if (!fcu::fmt_known(type) || n < 0) return -1;
  const int bs = fcu::fmt_bs(type);
  return (n + bs - 1) / bs * fcu::fmt_bb(type);
}

int fcu_quant_matvec(fcu_ctx *ctx, int type, const void *W, int64_t N, int64_t K, const float *X, int64_t M,
                     float *Y) {
  using namespace fcu;
  FCU_CTX(ctx);
  FCU_REQUIRE(fmt_known(type), "fcu_quant_matvec: GGML type %d is not supported", type);
  FCU_REQUIRE(N >= 0 && K > 0 && M >= 0, "fcu_quant_matvec: bad shape N=%lld K=%lld M=%lld", (long long)N,
              (long long)K, (long long)M);
  if (N == 0 || M == 0) return FCU_OK;
  FCU_REQUIRE(W && X && Y, "fcu_quant_matvec: null pointer");
  FCU_REQUIRE(K % fmt_bs(type) == 0, "fcu_quant_matvec: K=%lld is not a multiple of the %d-element block",
              (long long)K, fmt_bs(type));
  FCU_REQUIRE((uintptr_t)W % 16 == 0, "fcu_quant_matvec: W must be 16-byte aligned");
  FCU_REQUIRE((uintptr_t)X % 16 == 0, "fcu_quant_matvec: X must be 16-byte aligned");
  const int64_t rb = fcu_ggml_row_bytes(type, K);
  FCU_REQUIRE(rb <= kQmvChunk, "fcu_quant_matvec: a row of %lld bytes exceeds the %d-byte stage",
              (long long)rb, kQmvChunk);
  // a stage holds 8 rows (one per warp), else 4 (two warps per row), where
  // that fits in kQmvChunkMax
  int64_t stage = kQmvChunk;
  for (int rows = kQmvWarps; rows >= 4; rows /= 2)
    if (rb * rows <= kQmvChunkMax) {
      if (rb * rows > stage) stage = (rb * rows + 15) & ~(int64_t)15;
      break;
    }
  FCU_REQUIRE(K <= 24576, "fcu_quant_matvec: K=%lld exceeds 24576", (long long)K);
  int *err = nullptr;
  int rc = tc_error_word(ctx, &err);
  if (rc) return rc;
  // vectors per launch: as many as fit beside the stages (<= 8)
  const int64_t x_budget = 227 * 1024 - qmv_header(8) - kQmvStages * (stage + kQmvPad);
  int MB = 8;
  while (MB > 1 && (int64_t)MB * (K + K / 16) * 4 > x_budget) MB >>= 1;
  // rows per chunk: whole warps' worth (a multiple of 8) where rows are
  // narrow, fewer (each split over several warps) where they are wide or the
  // tensor is small, so that every SM gets chunks
  const int64_t rows_max = stage / rb;
  int64_t R = (N + 4 * ctx->num_sms - 1) / (4 * ctx->num_sms);
  if (R < 1) R = 1;
  if (R > rows_max) R = rows_max;
  if (R >= kQmvWarps) R -= R % kQmvWarps;
  else if (R > 4) R = 4;          // 1, 2 or 4 rows: whole warps per row
  else if (R == 3) R = 2;
  QmvArgs a{};
  a.W = (const uint8_t *)W;
  a.N = N;
  a.K = K;
  a.row_bytes = rb;
  a.total_bytes = N * rb;
  a.rows_per_chunk = (int)R;
  a.n_chunks = (N + R - 1) / R;
  a.err = err;
  a.stage_bytes = (int)stage;
  a.free_run = (a.total_bytes & 15) == 0;
  for (int64_t m0 = 0; m0 < M; m0 += MB) {
    const int mg = (int)(M - m0 < MB ? M - m0 : MB);
    int mb = 1;
    while (mb < mg) mb <<= 1;
    a.X = X + m0 * K;
    a.Y = Y + m0 * N;
    a.M = mg;
    const size_t smem = qmv_header(mb) + kQmvStages * (size_t)(stage + kQmvPad) + (size_t)mb * K * 4 +
                        (size_t)mb * (K / 16) * 4;
    int per_sm = 0;   // CTAs that are resident together on an SM (the persistent grid)
    rc = matvec_occupancy(type, mb, smem, &per_sm);
    if (rc) return rc;
    if (per_sm < 1) per_sm = 1;
    int64_t grid = a.n_chunks < (int64_t)per_sm * ctx->num_sms ? a.n_chunks : (int64_t)per_sm * ctx->num_sms;
    rc = launch_matvec(ctx, type, a, mb, (int)grid, smem);
    if (rc) return rc;
  }
  return FCU_OK;
}

int fcu_dequantize_rows(fcu_ctx *ctx, int type, const void *W, int64_t N, int64_t K, const int32_t *rows,
                        int64_t nrows, float *out) {
  using namespace fcu;
  FCU_CTX(ctx);
  FCU_REQUIRE(fmt_known(type), "fcu_dequantize_rows: GGML type %d is not supported", type);
  FCU_REQUIRE(N >= 0 && K > 0 && nrows >= 0, "fcu_dequantize_rows: bad shape");
  if (nrows == 0) return FCU_OK;
  FCU_REQUIRE(W && out, "fcu_dequantize_rows: null pointer");
  FCU_REQUIRE(K % fmt_bs(type) == 0, "fcu_dequantize_rows: K=%lld is not a multiple of the %d-element block",
              (long long)K, fmt_bs(type));
  FCU_REQUIRE((uintptr_t)W % 4 == 0, "fcu_dequantize_rows: W must be 4-byte aligned");
  FCU_REQUIRE(rows != nullptr || nrows <= N, "fcu_dequantize_rows: %lld rows of a %lld-row tensor",
              (long long)nrows, (long long)N);
  const int64_t rb = fcu_ggml_row_bytes(type, K);
  const int64_t total = nrows * K;
  int grid = (int)((total + 255) / 256);
  if (grid > 8 * ctx->num_sms) grid = 8 * ctx->num_sms;
  const uint8_t *w = (const uint8_t *)W;
  switch (type) {
    case kF32: launch_dequant_t<kF32>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
    case kF16: launch_dequant_t<kF16>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
    case kQ4_0: launch_dequant_t<kQ4_0>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
    case kQ5_0: launch_dequant_t<kQ5_0>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
    case kQ8_0: launch_dequant_t<kQ8_0>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
    case kQ4K: launch_dequant_t<kQ4K>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
    case kQ5K: launch_dequant_t<kQ5K>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
    case kQ6K: launch_dequant_t<kQ6K>(ctx->stream, grid, w, N, K, rb, rows, nrows, out); break;
  }
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // extern "C"
