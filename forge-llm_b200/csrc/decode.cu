// Decode-side attention kernels: one new token per sequence against its KV
// cache (src/L6/transformer.js:149-176 with attentionDecode,
// src/L5/attention.js:31-57, and the caches of attention.js:128-187).
//
//   fcu_decode_rope_kv  applyRopeHead (transformer.js:56-64, table of
//                       ropeTable, src/L1/special.js:116-127) on the q and k
//                       heads of each sequence's qkv row, in place, and
//                       KVCache.put / PagedKVCache.put of k and v at the
//                       sequence's position
//   fcu_attn_decode     causal GQA attention of that token over positions
//                       [0, n) of its cache
//
// Cache layout: position p of sequence b lives in row
//   block_table[b * max_blocks + p / block_size] * block_size + p % block_size
// (block_table NULL: block b * max_blocks + p / block_size, i.e. sequence b
// owns max_blocks * block_size contiguous rows), each row holding all kv
// heads (row_stride floats apart).  KVCache is block_size = maxSeq with one
// block per sequence; PagedKVCache's linear block numbering is the NULL table.
//
// fcu_attn_decode splits each sequence's positions into chunks of kChunk; a
// CTA takes one (sequence, kv head, chunk), reads each K and V row of the
// chunk once for all the q heads of that kv head's group, computes the
// scores, their maximum, exp and the weighted V sum, and writes either the
// final output (a one-chunk sequence) or (o, max, sum) partials that
// attn_decode_combine merges.  The bound is reading the cache (HBM).
#include "common.cuh"

namespace fcu {
namespace {

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kChunk = 256;         // positions per CTA
constexpr int kMaxGroup = 16;       // q heads per kv head
constexpr int kMaxDh = 256;
constexpr int kMaxAcc = 64;         // group x elements per lane held in registers

struct DecArgs {
  const float *q;
  int64_t ld_q;
  const float *kc, *vc;
  int64_t row_stride;
  const int32_t *table;
  int max_blocks, block_size;
  const int32_t *seq_lens;
  int64_t cap;      // positions a sequence can hold: max_blocks * block_size
  int B, nH, nKV, dH, splits;
  float scale;
  float *part_o;    // [B, nH, splits, dH]
  float *part_ml;   // [B, nH, splits, 2]
  float *out;       // [B, nH * dH]
};

__device__ __forceinline__ int64_t cache_row(const int32_t *table, int max_blocks, int block_size, int b,
                                             int64_t p) {
  const int64_t blk = p / block_size;
  const int64_t phys = table ? (int64_t)table[(int64_t)b * max_blocks + blk] : (int64_t)b * max_blocks + blk;
  return phys * block_size + p % block_size;
}

// Dynamic shared memory of one CTA: q [g][dH], scores [g][kChunk], the
// warps' partial outputs [kDecWarps][g * EPL * 32], max and sum [2][g].
__host__ __device__ inline size_t decode_smem_bytes(int g, int dH, int epl) {
  return sizeof(float) * ((size_t)g * dH + (size_t)g * kChunk + (size_t)kDecWarps * g * epl * 32 + 2 * g);
}

template <int EPL, int GMAX>   // EPL = ceil(dH / 32) elements per lane; g <= GMAX
__global__ void __launch_bounds__(kDecThreads) attn_decode_kernel(DecArgs a) {
  pdl_trigger();
  extern __shared__ __align__(16) float dsm[];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = a.nH / a.nKV, dH = a.dH;
  float *q_s = dsm;                                  // [g][dH]
  float *s_s = q_s + g * dH;                         // [g][kChunk]
  float *o_s = s_s + g * kChunk;                     // [kDecWarps][g * EPL * 32]
  float *m_s = o_s + kDecWarps * g * EPL * 32;       // [g]
  float *l_s = m_s + g;                              // [g]
  pdl_wait();
  int64_t n = a.seq_lens[b];
  if (n < 0) n = 0;
  if (n > a.cap) n = a.cap;                          // never past the sequence's own rows
  const int64_t p0 = (int64_t)split * kChunk;
  if (p0 >= n && !(split == 0 && n == 0)) return;
  const int64_t p1 = p0 + kChunk < n ? p0 + kChunk : n;
  const int np = (int)(p1 > p0 ? p1 - p0 : 0);
  const int nsplit = (int)((n + kChunk - 1) / kChunk);
  for (int i = threadIdx.x; i < g * dH; i += kDecThreads) {
    const int hg = i / dH, e = i - hg * dH;
    q_s[i] = a.q[(int64_t)b * a.ld_q + (int64_t)(kvh * g + hg) * dH + e];
  }
  __syncthreads();
  // scores: a warp per position, lanes across the head dimension
  for (int j = warp; j < np; j += kDecWarps) {
    const float *kr = a.kc + cache_row(a.table, a.max_blocks, a.block_size, b, p0 + j) * a.row_stride +
                      (int64_t)kvh * dH;
    float kv[EPL];
#pragma unroll
    for (int t = 0; t < EPL; t++) {
      const int e = lane + 32 * t;
      kv[t] = e < dH ? kr[e] : 0.f;
    }
#pragma unroll
    for (int hg = 0; hg < GMAX; hg++) {
      if (hg < g) {
        float s = 0.f;
#pragma unroll
        for (int t = 0; t < EPL; t++) {
          const int e = lane + 32 * t;
          if (e < dH) s = fmaf(q_s[hg * dH + e], kv[t], s);
        }
        s = warp_sum(s);
        if (lane == 0) s_s[hg * kChunk + j] = s * a.scale;
      }
    }
  }
  __syncthreads();
  // per head: the chunk's maximum, then p = exp(s - max) in place and its sum
  for (int hg = warp; hg < g; hg += kDecWarps) {
    float m = -INFINITY;
    for (int j = lane; j < np; j += 32) m = fmaxf(m, s_s[hg * kChunk + j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < np; j += 32) {
      const float p = expf(s_s[hg * kChunk + j] - m);
      s_s[hg * kChunk + j] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      m_s[hg] = m;
      l_s[hg] = l;
    }
  }
  __syncthreads();
  // o[hg][e] = sum_j p[hg][j] v[j][e]: a warp per position, lanes across e
  float acc[GMAX][EPL];
#pragma unroll
  for (int hg = 0; hg < GMAX; hg++)
#pragma unroll
    for (int t = 0; t < EPL; t++) acc[hg][t] = 0.f;
  for (int j = warp; j < np; j += kDecWarps) {
    const float *vr = a.vc + cache_row(a.table, a.max_blocks, a.block_size, b, p0 + j) * a.row_stride +
                      (int64_t)kvh * dH;
    float vv[EPL];
#pragma unroll
    for (int t = 0; t < EPL; t++) {
      const int e = lane + 32 * t;
      vv[t] = e < dH ? vr[e] : 0.f;
    }
#pragma unroll
    for (int hg = 0; hg < GMAX; hg++) {
      if (hg < g) {
        const float p = s_s[hg * kChunk + j];
#pragma unroll
        for (int t = 0; t < EPL; t++) acc[hg][t] = fmaf(p, vv[t], acc[hg][t]);
      }
    }
  }
#pragma unroll
  for (int hg = 0; hg < GMAX; hg++)
    if (hg < g)
#pragma unroll
      for (int t = 0; t < EPL; t++) o_s[(warp * g + hg) * EPL * 32 + t * 32 + lane] = acc[hg][t];
  __syncthreads();
  for (int i = threadIdx.x; i < g * dH; i += kDecThreads) {
    const int hg = i / dH, e = i - hg * dH, t = e >> 5, ln = e & 31;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; w++) o += o_s[(w * g + hg) * EPL * 32 + t * 32 + ln];
    const int h = kvh * g + hg;
    if (nsplit <= 1) {
      // the whole sequence in this CTA (n == 0 gives the JS's zero output)
      a.out[(int64_t)b * a.nH * dH + (int64_t)h * dH + e] = np > 0 ? o * (1.0f / l_s[hg]) : 0.f;
    } else {
      a.part_o[(((int64_t)b * a.nH + h) * a.splits + split) * dH + e] = o;
      if (e == 0) {
        float *ml = a.part_ml + (((int64_t)b * a.nH + h) * a.splits + split) * 2;
        ml[0] = m_s[hg];
        ml[1] = l_s[hg];
      }
    }
  }
}

// The same for head dims that are a multiple of 32 (dH = 32 * E4) on 16-byte
// aligned caches, with more rows in flight and fewer shuffles: 8 lanes share
// a cache row (lane li holds the float4 chunks at elements c * 32 + 4 * li,
// so each load instruction reads 128 contiguous bytes of a row), a warp
// covers 4 rows per step and loads two steps (8 rows) before using them.  A
// score is the lane's 4 * E4 products summed, then over its 8 lanes.  In the
// weighted V sum each lane accumulates its chunks for its rows; the 4 row
// groups of a warp are summed at the end.  Scores, softmax and the merge are
// those of attn_decode_kernel.
template <int E4, int GMAX>   // E4 = dH / 32; g <= GMAX, GMAX * E4 <= 16
__global__ void __launch_bounds__(kDecThreads) attn_decode8_kernel(DecArgs a) {
  pdl_trigger();
  extern __shared__ __align__(16) float dsm[];
  constexpr int dH = 32 * E4;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane >> 3, li = lane & 7;
  const int g = a.nH / a.nKV;
  float *q_s = dsm;                                  // [g][dH]
  float *s_s = q_s + g * dH;                         // [g][kChunk]
  float *o_s = s_s + g * kChunk;                     // [kDecWarps][g][dH]
  float *m_s = o_s + kDecWarps * g * dH;             // [g]
  float *l_s = m_s + g;                              // [g]
  pdl_wait();
  int64_t n = a.seq_lens[b];
  if (n < 0) n = 0;
  if (n > a.cap) n = a.cap;                          // never past the sequence's own rows
  const int64_t p0 = (int64_t)split * kChunk;
  if (p0 >= n && !(split == 0 && n == 0)) return;
  const int64_t p1 = p0 + kChunk < n ? p0 + kChunk : n;
  const int np = (int)(p1 > p0 ? p1 - p0 : 0);
  const int nsplit = (int)((n + kChunk - 1) / kChunk);
  for (int i = threadIdx.x; i < g * dH; i += kDecThreads) {
    const int hg = i / dH, e = i - hg * dH;
    q_s[i] = a.q[(int64_t)b * a.ld_q + (int64_t)(kvh * g + hg) * dH + e];
  }
  __syncthreads();
  // rows j0 + sub (r = 0) and j0 + 4 + sub (r = 1) of this warp's step
  auto load_rows = [&](const float *cache, int j0, float4 (&v)[2][E4]) {
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int j = j0 + 4 * r + sub;
      if (j < np) {
        const float4 *row = reinterpret_cast<const float4 *>(
            cache + cache_row(a.table, a.max_blocks, a.block_size, b, p0 + j) * a.row_stride + (int64_t)kvh * dH);
#pragma unroll
        for (int c = 0; c < E4; c++) v[r][c] = row[c * 8 + li];
      } else {
#pragma unroll
        for (int c = 0; c < E4; c++) v[r][c] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  for (int j0 = warp * 8; j0 < np; j0 += kDecWarps * 8) {
    float4 kv[2][E4];
    load_rows(a.kc, j0, kv);
#pragma unroll
    for (int hg = 0; hg < GMAX; hg++) {
      if (hg < g) {
        const float4 *qv = reinterpret_cast<const float4 *>(q_s + hg * dH);
        float s[2] = {0.f, 0.f};
#pragma unroll
        for (int c = 0; c < E4; c++) {
          const float4 qq = qv[c * 8 + li];
#pragma unroll
          for (int r = 0; r < 2; r++) {
            s[r] = fmaf(qq.x, kv[r][c].x, s[r]);
            s[r] = fmaf(qq.y, kv[r][c].y, s[r]);
            s[r] = fmaf(qq.z, kv[r][c].z, s[r]);
            s[r] = fmaf(qq.w, kv[r][c].w, s[r]);
          }
        }
#pragma unroll
        for (int r = 0; r < 2; r++) {
          s[r] += __shfl_xor_sync(0xffffffffu, s[r], 1);
          s[r] += __shfl_xor_sync(0xffffffffu, s[r], 2);
          s[r] += __shfl_xor_sync(0xffffffffu, s[r], 4);
          const int j = j0 + 4 * r + sub;
          if (li == 0 && j < np) s_s[hg * kChunk + j] = s[r] * a.scale;
        }
      }
    }
  }
  __syncthreads();
  // per head: the chunk's maximum, then p = exp(s - max) in place and its sum
  for (int hg = warp; hg < g; hg += kDecWarps) {
    float m = -INFINITY;
    for (int j = lane; j < np; j += 32) m = fmaxf(m, s_s[hg * kChunk + j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < np; j += 32) {
      const float p = expf(s_s[hg * kChunk + j] - m);
      s_s[hg * kChunk + j] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      m_s[hg] = m;
      l_s[hg] = l;
    }
  }
  __syncthreads();
  float4 acc[GMAX][E4];
#pragma unroll
  for (int hg = 0; hg < GMAX; hg++)
#pragma unroll
    for (int c = 0; c < E4; c++) acc[hg][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j0 = warp * 8; j0 < np; j0 += kDecWarps * 8) {
    float4 vv[2][E4];
    load_rows(a.vc, j0, vv);
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int j = j0 + 4 * r + sub;
#pragma unroll
      for (int hg = 0; hg < GMAX; hg++) {
        if (hg < g) {
          const float p = j < np ? s_s[hg * kChunk + j] : 0.f;
#pragma unroll
          for (int c = 0; c < E4; c++) {
            acc[hg][c].x = fmaf(p, vv[r][c].x, acc[hg][c].x);
            acc[hg][c].y = fmaf(p, vv[r][c].y, acc[hg][c].y);
            acc[hg][c].z = fmaf(p, vv[r][c].z, acc[hg][c].z);
            acc[hg][c].w = fmaf(p, vv[r][c].w, acc[hg][c].w);
          }
        }
      }
    }
  }
  // the warp's 4 row groups summed (lanes li, li + 8, li + 16, li + 24)
#pragma unroll
  for (int hg = 0; hg < GMAX; hg++) {
    if (hg < g) {
#pragma unroll
      for (int c = 0; c < E4; c++) {
        float4 v = acc[hg][c];
#pragma unroll
        for (int x = 8; x <= 16; x <<= 1) {
          v.x += __shfl_xor_sync(0xffffffffu, v.x, x);
          v.y += __shfl_xor_sync(0xffffffffu, v.y, x);
          v.z += __shfl_xor_sync(0xffffffffu, v.z, x);
          v.w += __shfl_xor_sync(0xffffffffu, v.w, x);
        }
        if (sub == 0) *reinterpret_cast<float4 *>(o_s + (warp * g + hg) * dH + c * 32 + 4 * li) = v;
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < g * dH; i += kDecThreads) {
    const int hg = i / dH, e = i - hg * dH;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; w++) o += o_s[(w * g + hg) * dH + e];
    const int h = kvh * g + hg;
    if (nsplit <= 1) {
      a.out[(int64_t)b * a.nH * dH + (int64_t)h * dH + e] = np > 0 ? o * (1.0f / l_s[hg]) : 0.f;
    } else {
      a.part_o[(((int64_t)b * a.nH + h) * a.splits + split) * dH + e] = o;
      if (e == 0) {
        float *ml = a.part_ml + (((int64_t)b * a.nH + h) * a.splits + split) * 2;
        ml[0] = m_s[hg];
        ml[1] = l_s[hg];
      }
    }
  }
}

// Merges the chunks of every sequence longer than one chunk:
// out = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M).
__global__ void __launch_bounds__(128) attn_decode_combine(DecArgs a) {
  pdl_trigger();
  const int h = blockIdx.x, b = blockIdx.y;
  pdl_wait();
  int64_t n = a.seq_lens[b];
  if (n > a.cap) n = a.cap;
  const int nsplit = (int)((n + kChunk - 1) / kChunk);
  if (nsplit <= 1) return;
  const float *ml = a.part_ml + ((int64_t)b * a.nH + h) * a.splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; s++) M = fmaxf(M, ml[2 * s]);
  float L = 0.f;
  for (int s = 0; s < nsplit; s++) L += ml[2 * s + 1] * expf(ml[2 * s] - M);
  const float inv = 1.0f / L;
  for (int e = threadIdx.x; e < a.dH; e += blockDim.x) {
    float o = 0.f;
    for (int s = 0; s < nsplit; s++)
      o += a.part_o[(((int64_t)b * a.nH + h) * a.splits + s) * a.dH + e] * expf(ml[2 * s] - M);
    a.out[(int64_t)b * a.nH * a.dH + (int64_t)h * a.dH + e] = o * inv;
  }
}

// applyRopeHead on q and k heads of row b at position pos_b (cos / sin rounded
// to fp32 as the Float32Array table holds them; the rotation in double as the
// JS computes it), then k and v into the cache row of that position.
__global__ void __launch_bounds__(256) decode_rope_kv_kernel(float *qkv, int64_t ld, int nH, int nKV, int dH,
                                                             double theta, const int32_t *pos, float *kc,
                                                             float *vc, int64_t row_stride, const int32_t *table,
                                                             int max_blocks, int block_size) {
  pdl_trigger();
  const int b = blockIdx.x;
  pdl_wait();
  const int64_t p = pos[b];
  // a position outside the sequence's cache rows changes nothing
  if (p < 0 || p >= (int64_t)max_blocks * block_size) return;
  float *x = qkv + (int64_t)b * ld;
  const int half = dH / 2;
  const int pairs = (nH + nKV) * half;
  const int64_t row = cache_row(table, max_blocks, block_size, b, p);
  for (int t = threadIdx.x; t < pairs; t += blockDim.x) {
    const int head = t / half, i = t - head * half;
    const double freq = 1.0 / pow(theta, (double)(2 * i) / dH);
    const double ang = (double)p * freq;
    const double c = (double)(float)cos(ang), s = (double)(float)sin(ang);
    const int64_t e = (int64_t)head * dH + 2 * i;
    const double u = x[e], v = x[e + 1];
    const float r0 = (float)(u * c - v * s), r1 = (float)(u * s + v * c);
    x[e] = r0;
    x[e + 1] = r1;
    if (head >= nH) {
      float *kr = kc + row * row_stride + (int64_t)(head - nH) * dH + 2 * i;
      kr[0] = r0;
      kr[1] = r1;
    }
  }
  const int kvd = nKV * dH;
  for (int e = threadIdx.x; e < kvd; e += blockDim.x)
    vc[row * row_stride + e] = x[(int64_t)(nH + nKV) * dH + e];
}

}  // namespace
}  // namespace fcu

extern "C" {

int fcu_decode_rope_kv(fcu_ctx *ctx, float *qkv, int64_t ld_qkv, int B, int nH, int nKV, int dH, double theta,
                       const int32_t *positions, float *k_cache, float *v_cache, int64_t row_stride,
                       const int32_t *block_table, int max_blocks, int block_size) {
  FCU_CTX(ctx);
  FCU_REQUIRE(B >= 0 && nH > 0 && nKV > 0 && nH % nKV == 0 && dH > 0 && dH % 2 == 0,
              "fcu_decode_rope_kv: bad heads nH=%d nKV=%d dH=%d", nH, nKV, dH);
  FCU_REQUIRE(ld_qkv >= (int64_t)(nH + 2 * nKV) * dH && row_stride >= (int64_t)nKV * dH,
              "fcu_decode_rope_kv: row strides too small");
  FCU_REQUIRE(max_blocks > 0 && block_size > 0, "fcu_decode_rope_kv: bad cache geometry");
  if (B == 0) return FCU_OK;
  FCU_REQUIRE(qkv && positions && k_cache && v_cache, "fcu_decode_rope_kv: null pointer");
  cudaError_t e = fcu::launch_pdl(fcu::decode_rope_kv_kernel, dim3(B), dim3(256), 0, ctx->stream, qkv,
                                  ld_qkv, nH, nKV, dH, theta, positions, k_cache, v_cache, row_stride,
                                  block_table, max_blocks, block_size);
  FCU_CHECK_CUDA(e);
  fcu::note_launch();
  return FCU_OK;
}

int fcu_attn_decode(fcu_ctx *ctx, const float *q, int64_t ld_q, const float *k_cache, const float *v_cache,
                    int64_t row_stride, const int32_t *block_table, int max_blocks, int block_size,
                    const int32_t *seq_lens, int B, int nH, int nKV, int dH, double scale, float *out) {
  using namespace fcu;
  FCU_CTX(ctx);
  FCU_REQUIRE(B >= 0 && nH > 0 && nKV > 0 && nH % nKV == 0, "fcu_attn_decode: bad heads nH=%d nKV=%d", nH,
              nKV);
  FCU_REQUIRE(nH / nKV <= kMaxGroup, "fcu_attn_decode: %d q heads per kv head (max %d)", nH / nKV, kMaxGroup);
  FCU_REQUIRE(dH > 0 && dH <= kMaxDh, "fcu_attn_decode: head dim %d (1..%d)", dH, kMaxDh);
  FCU_REQUIRE(ld_q >= (int64_t)nH * dH && row_stride >= (int64_t)nKV * dH, "fcu_attn_decode: strides too small");
  FCU_REQUIRE(max_blocks > 0 && block_size > 0, "fcu_attn_decode: bad cache geometry");
  if (B == 0) return FCU_OK;
  FCU_REQUIRE(q && k_cache && v_cache && seq_lens && out, "fcu_attn_decode: null pointer");
  const int64_t cap = (int64_t)max_blocks * block_size;
  const int splits = (int)((cap + kChunk - 1) / kChunk);
  FCU_REQUIRE(splits <= 65535, "fcu_attn_decode: a cache of %lld positions per sequence is too long",
              (long long)cap);
  DecArgs a{};
  a.q = q;
  a.ld_q = ld_q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.row_stride = row_stride;
  a.table = block_table;
  a.max_blocks = max_blocks;
  a.block_size = block_size;
  a.seq_lens = seq_lens;
  a.B = B;
  a.nH = nH;
  a.nKV = nKV;
  a.dH = dH;
  a.splits = splits;
  a.cap = cap;
  a.scale = (float)scale;
  a.out = out;
  if (splits > 1) {
    void *scr = nullptr;
    const size_t per = (size_t)B * nH * splits;
    int rc = ctx_scratch(ctx, per * (dH + 2) * sizeof(float), &scr);
    if (rc) return rc;
    a.part_o = (float *)scr;
    a.part_ml = a.part_o + per * dH;
  }
  dim3 grid(splits, nKV, B);
  const int g = nH / nKV, epl = (dH + 31) / 32;
  cudaError_t e = cudaErrorInvalidValue;
  // head dims 32 / 64 / 128 / 256 on 16-byte aligned caches: 8 lanes per row
  int g2 = 1;
  while (g2 < g) g2 <<= 1;
  const int e4 = dH / 32;
  const bool rows8 = dH % 32 == 0 && (e4 == 1 || e4 == 2 || e4 == 4 || e4 == 8) && g2 * e4 <= 16 &&
                     row_stride % 4 == 0 && (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15) == 0;
  if (rows8) {
    const size_t smem8 = decode_smem_bytes(g, dH, e4);
#define FCU_DEC8_CASE(E, G)                                                                         \
  if (e4 == E && g2 == G) {                                                                         \
    static bool set[64] = {false};                                                                  \
    if (!set[ctx->device & 63]) {                                                                   \
      FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_decode8_kernel<E, G>,                                \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)); \
      set[ctx->device & 63] = true;                                                                 \
    }                                                                                               \
    e = launch_pdl(attn_decode8_kernel<E, G>, grid, dim3(kDecThreads), smem8, ctx->stream, a);      \
  }
    FCU_DEC8_CASE(1, 1) FCU_DEC8_CASE(1, 2) FCU_DEC8_CASE(1, 4) FCU_DEC8_CASE(1, 8) FCU_DEC8_CASE(1, 16)
    FCU_DEC8_CASE(2, 1) FCU_DEC8_CASE(2, 2) FCU_DEC8_CASE(2, 4) FCU_DEC8_CASE(2, 8)
    FCU_DEC8_CASE(4, 1) FCU_DEC8_CASE(4, 2) FCU_DEC8_CASE(4, 4)
    FCU_DEC8_CASE(8, 1) FCU_DEC8_CASE(8, 2)
#undef FCU_DEC8_CASE
    FCU_CHECK_CUDA(e);
    note_launch();
    if (splits > 1) {
      e = launch_pdl(attn_decode_combine, dim3(nH, B), dim3(128), 0, ctx->stream, a);
      FCU_CHECK_CUDA(e);
      note_launch();
    }
    return FCU_OK;
  }
  int gmax = 1;
  while (gmax < g) gmax <<= 1;
  int eplp = 1;
  while (eplp < epl) eplp <<= 1;
  FCU_REQUIRE(gmax * eplp <= kMaxAcc, "fcu_attn_decode: %d q heads per kv head at head dim %d is too wide",
              g, dH);
  const size_t smem = decode_smem_bytes(g, dH, eplp);
#define FCU_DEC_CASE(E, G)                                                                          \
  if (eplp == E && gmax == G) {                                                                     \
    static bool set[64] = {false};                                                                  \
    if (!set[ctx->device & 63]) {                                                                   \
      FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_decode_kernel<E, G>,                                 \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)); \
      set[ctx->device & 63] = true;                                                                 \
    }                                                                                               \
    e = launch_pdl(attn_decode_kernel<E, G>, grid, dim3(kDecThreads), smem, ctx->stream, a);        \
  }
  FCU_DEC_CASE(1, 1) FCU_DEC_CASE(1, 2) FCU_DEC_CASE(1, 4) FCU_DEC_CASE(1, 8) FCU_DEC_CASE(1, 16)
  FCU_DEC_CASE(2, 1) FCU_DEC_CASE(2, 2) FCU_DEC_CASE(2, 4) FCU_DEC_CASE(2, 8) FCU_DEC_CASE(2, 16)
  FCU_DEC_CASE(4, 1) FCU_DEC_CASE(4, 2) FCU_DEC_CASE(4, 4) FCU_DEC_CASE(4, 8) FCU_DEC_CASE(4, 16)
  FCU_DEC_CASE(8, 1) FCU_DEC_CASE(8, 2) FCU_DEC_CASE(8, 4) FCU_DEC_CASE(8, 8)
#undef FCU_DEC_CASE
  FCU_CHECK_CUDA(e);
  note_launch();
  if (splits > 1) {
    e = launch_pdl(attn_decode_combine, dim3(nH, B), dim3(128), 0, ctx->stream, a);
    FCU_CHECK_CUDA(e);
    note_launch();
  }
  return FCU_OK;
}

}  // extern "C"
