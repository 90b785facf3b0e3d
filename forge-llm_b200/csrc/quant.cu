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
constexpr int kQmvChunk = 24576;               // bytes of rows per stage
constexpr int kQmvBuf = kQmvChunk + 32;        // + room for the 16-byte widening
constexpr int kQmvHeader = 128;                // mbarriers + abort flag

struct QmvArgs {
  const uint8_t *W;
  int64_t N, K, row_bytes, total_bytes;
  const float *X;   // [M, K]
  float *Y;         // [M, N]
  int M, rows_per_chunk;
  int64_t n_chunks;
  int *err;
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

// One row (in shared memory) against the MB vectors: this lane's share.
template <int T, int MB>
__device__ __forceinline__ void row_dot(const uint8_t *row, const float *xs, int64_t K, int M, int lane,
                                        float (&acc)[MB]) {
  if (T == kQ4K || T == kQ5K) {
    const int j = lane >> 3, p = (lane & 7) * 4;
    const int64_t nsb = K >> 8;
    for (int64_t sb = 0; sb < nsb; sb++) {
      const uint8_t *b = row + sb * fmt_bb(T);
      const float d = h2f(ld16(b)), dmin = h2f(ld16(b + 2));
      float sc0, mn0, sc1, mn1;
      scale_min_k4(2 * j, b + 4, sc0, mn0);
      scale_min_k4(2 * j + 1, b + 4, sc1, mn1);
      const float d1 = d * sc0, n1 = dmin * mn0, d2 = d * sc1, n2 = dmin * mn1;
      const uint32_t q = ld32(b + (T == kQ4K ? 16 : 48) + j * 32 + p);
      uint32_t qh = 0;
      if (T == kQ5K) qh = ld32(b + 16 + p);
      float wl[4], wh[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        uint32_t lo = (q >> (8 * e)) & 0xF, hi = (q >> (8 * e + 4)) & 0xF;
        if (T == kQ5K) {
          lo |= ((qh >> (8 * e + 2 * j)) & 1) << 4;
          hi |= ((qh >> (8 * e + 2 * j + 1)) & 1) << 4;
        }
        wl[e] = fmaf(d1, small_u2f(lo), -n1);
        wh[e] = fmaf(d2, small_u2f(hi), -n2);
      }
      const int64_t kb = sb * 256 + j * 64 + p;
      fma_x4<MB>(acc, wl, xs, K, M, kb);
      fma_x4<MB>(acc, wh, xs, K, M, kb + 32);
    }
  } else if (T == kQ6K) {
    const int half = lane >> 4, l0 = (lane & 15) * 2, is = l0 >> 4;
    const int64_t nsb = K >> 8;
    for (int64_t sb = 0; sb < nsb; sb++) {
      const uint8_t *b = row + sb * 210;
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
        const int64_t k = sb * 256 + half * 128 + qd * 32 + l0;
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
    const int o = (lane & 3) * 8;
    for (int64_t blk = lane >> 2; blk < nblk; blk += 8) {
      const uint8_t *b = row + blk * fmt_bb(T);
      const float d = h2f(ld16(b));
      float w[8];
      if (T == kQ8_0) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const uint32_t v = ld16(b + 2 + o + e);
          w[e] = d * (small_u2f((v & 0xFF) ^ 0x80) - 128.0f);
          w[e + 1] = d * (small_u2f(((v >> 8) & 0xFF) ^ 0x80) - 128.0f);
        }
      } else {
        // byte 2 + j/2, nibble j&1 (the reference's reading of these blocks)
#pragma unroll
        for (int e = 0; e < 8; e += 4) {
          const uint32_t v = ld16(b + 2 + (o >> 1) + (e >> 1));
#pragma unroll
          for (int t = 0; t < 4; t++) {
            const uint32_t q = (v >> (4 * t)) & 0xF;
            w[e + t] = (small_u2f(q) - (T == kQ4_0 ? 8.0f : 0.0f)) * d;
          }
        }
      }
      const int64_t k = blk * 32 + o;
      const float w0[4] = {w[0], w[1], w[2], w[3]}, w1[4] = {w[4], w[5], w[6], w[7]};
      fma_x4<MB>(acc, w0, xs, K, M, k);
      fma_x4<MB>(acc, w1, xs, K, M, k + 4);
    }
  } else {   // F32 / F16: element k of the row at byte k * (4 | 2)
    for (int64_t k = lane; k < K; k += 32) {
      const float w = T == kF32 ? __int_as_float((int)ld32(row + 4 * k)) : h2f(ld16(row + 2 * k));
      fma_x<MB>(acc, w, xs, K, M, k);
    }
  }
}

template <int T, int MB>
__global__ void __launch_bounds__(kQmvThreads) quant_matvec_kernel(QmvArgs a) {
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 64);
  uint8_t *bufs = smem + kQmvHeader;
  float *xs = reinterpret_cast<float *>(bufs + kQmvStages * kQmvBuf);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < kQmvStages; s++) mbar_init(&full[s], 1);
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
    mbar_expect_tx(&full[st], bytes);
    if (bytes) bulk_load_1d(bufs + st * kQmvBuf, a.W + a0, bytes, &full[st]);
  };

  if (tid == 0)
    for (int64_t i = 0; i < my_chunks && i < kQmvStages; i++) issue(i);
  // the input vectors, for the whole kernel
  for (int64_t i = tid; i < (int64_t)a.M * a.K; i += kQmvThreads) xs[i] = a.X[i];
  __syncthreads();

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
    uint8_t *buf = bufs + st * kQmvBuf;
    // the tensor's last < 16 bytes, which no bulk copy covers
    const int64_t tail0 = tma_limit > a0 ? tma_limit : a0;
    if (e0 > tail0) {
      for (int64_t t = tail0 + tid; t < e0; t += kQmvThreads) buf[t - a0] = a.W[t];
      __syncthreads();
    }
    const uint8_t *rows = buf + (s0 - a0);
    for (int64_t lr = warp; lr < r1 - r0; lr += kQmvWarps) {
      float acc[MB];
#pragma unroll
      for (int m = 0; m < MB; m++) acc[m] = 0.f;
      row_dot<T, MB>(rows + lr * a.row_bytes, xs, a.K, a.M, lane, acc);
#pragma unroll
      for (int m = 0; m < MB; m++) {
        const float v = warp_sum(acc[m]);
        if (lane == 0 && m < a.M) a.Y[m * a.N + r0 + lr] = v;
      }
    }
    __syncthreads();   // every warp is done with this stage before it is refilled
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
  FCU_REQUIRE(K <= 24576, "fcu_quant_matvec: K=%lld exceeds 24576", (long long)K);
  int *err = nullptr;
  int rc = tc_error_word(ctx, &err);
  if (rc) return rc;
  // vectors per launch: as many as fit beside the stages (<= 8)
  const int64_t x_budget = 227 * 1024 - kQmvHeader - kQmvStages * kQmvBuf;
  int MB = 8;
  while (MB > 1 && (int64_t)MB * K * 4 > x_budget) MB >>= 1;
  const int64_t rows_max = kQmvChunk / rb;
  int64_t R = (N + 4 * ctx->num_sms - 1) / (4 * ctx->num_sms);
  if (R < 1) R = 1;
  if (R > rows_max) R = rows_max;
  QmvArgs a{};
  a.W = (const uint8_t *)W;
  a.N = N;
  a.K = K;
  a.row_bytes = rb;
  a.total_bytes = N * rb;
  a.rows_per_chunk = (int)R;
  a.n_chunks = (N + R - 1) / R;
  a.err = err;
  for (int64_t m0 = 0; m0 < M; m0 += MB) {
    const int mg = (int)(M - m0 < MB ? M - m0 : MB);
    int mb = 1;
    while (mb < mg) mb <<= 1;
    a.X = X + m0 * K;
    a.Y = Y + m0 * N;
    a.M = mg;
    const size_t smem = kQmvHeader + kQmvStages * kQmvBuf + (size_t)mb * K * 4;
    const int per_sm = smem <= 113 * 1024 ? 2 : 1;
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
