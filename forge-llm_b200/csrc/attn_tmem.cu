// Causal GQA flash attention on the sm_100a tensor cores: tcgen05.mma with
// the score and output accumulators in TMEM, Q/K/V tiles staged by TMA from
// the bf16 [tokens, (nH + 2 nKV) * 64] qkv buffer (RoPE already applied).
//
// Forward, per CTA: one 128-row query tile of one head, looping over the
// 128-key blocks at or before its diagonal.
//   warp 0      TMA: Q once, then a 3-deep ring of (K, V) blocks
//   warp 1      TMEM owner + MMA issuer (warp-wide, elect.sync picks the lane):
//                 S_j = Q K_j^T        128x128x64  -> TMEM cols [0, 128)
//                 O  += P_j V_j        128x64x128  -> TMEM cols [128, 192)
//               issued in the order S_0, S_1, PV_0, S_2, PV_1, ... so the next
//               score tile is computed while the softmax works on this one
//   warps 2..5  softmax: thread = query row = TMEM lane.  Reads its S row,
//               applies the causal mask, keeps the running max / sum, writes
//               P = exp2(S*scale*log2e - m) as bf16 pairs into TMEM (cols
//               [192, 256)), where the PV MMA reads it as its A operand, and
//               at the end normalises O and stores it with the log-sum-exp.
// The running max used for P is only moved when the block max exceeds it by
// more than 2^8: P then stays <= 256, and O (in TMEM) and the row sum are
// rescaled rarely, by the same factor, so O / l is unchanged.
// Two CTAs share an SM (112 KB shared memory, 256 TMEM columns each), so one
// CTA's MMAs overlap the other's softmax.
//
// Every wait is bounded: on timeout a CTA records an error code in the
// device error word, drains what it issued, frees TMEM and returns.
#include "common.cuh"
#include "tc_ptx.cuh"

namespace fcu {
namespace {

using namespace tc;

constexpr int kBM = 128;                       // query rows per CTA
constexpr int kBN = 128;                       // keys per block
constexpr int kD = 64;                         // head dim
constexpr int kTile = kBM * kD * 2;            // one [128][64] bf16 tile: 16 KB
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;            // S [0,128), O [128,192), P [192,256) (bf16 pairs)
constexpr int kFwdStages = 3;                  // K/V ring depth
constexpr float kRescaleLog2 = 8.f;
#ifndef FCU_POLY_BWD
#define FCU_POLY_BWD 4
#endif
// In the backward element loops one exponential pair in kPolyEvery is
// computed on the FMA pipe (exp2_poly2) instead of the MUFU unit (0: MUFU
// only).  Measured at config 4: dK/dV 461 -> 440 us and dQ 385 -> 377 us with
// one pair in 4; one in 2 is slower.  The forward softmax, whose issue slots
// are scarcer, takes one pair in 8 (247 -> 236 us; one in 4: 260 us).
constexpr int kPolyEvery = FCU_POLY_BWD;
constexpr int kPolyEveryFwd = 8;
template <int kEvery>
__device__ __forceinline__ float2 exp2_pair(float2 x, int pair) {
  if constexpr (kEvery > 0)
    if (pair % kEvery == kEvery - 1) return exp2_poly2(x);
  return make_float2(ex2_ftz(x.x), ex2_ftz(x.y));
}
constexpr float kLog2e = 1.4426950408889634f;

// The forward at head dim D (64 or 128).  A [128][D] bf16 tile is D / 64
// TMA boxes of [128 rows][64 columns] (16 KB, 1024-byte aligned for the
// swizzle), one after the other.  D = 64: a 3-deep K/V ring and 256 TMEM
// columns (S [0,128), O [128,192), P [192,256)), two CTAs per SM.  D = 128:
// a 2-deep ring (the shared memory of three would exceed 227 KB) and 512
// columns (O [128,256), P [256,320)), one CTA per SM.
template <int D>
struct FwdCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileQ = kBM * D * 2;
  static constexpr int kTileKV = kBN * D * 2;
  static constexpr int kStages = D == 64 ? kFwdStages : 2;
  static constexpr uint32_t kCols = D == 64 ? 256u : 512u;
  static constexpr int kMinBlocks = D == 64 ? 2 : 1;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileQ;             // kStages tiles
  static constexpr int kOffV = kOffK + kStages * kTileKV;
  static constexpr int kOffBar = kOffV + kStages * kTileKV;
  static constexpr int kSmemBytes = kOffBar + (6 + 4 * kStages) * 8 + 16;
};

struct FwdParams {
  int B, T, nH, nKV, n_qt;
  float scale_log2;          // softmax scale * log2(e)
  __nv_bfloat16 *O;          // [B*T, nH*D]
  float *lse;                // [B][nH][T], natural log
  int *err;
};

template <int D>
__global__ void __launch_bounds__(kThreads, FwdCfg<D>::kMinBlocks)
    attn_fwd_tmem_kernel(const __grid_constant__ CUtensorMap tm, FwdParams p) {
  fcu::pdl_trigger();
  using Cfg = FwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *sQ = smem + Cfg::kOffQ, *sK = smem + Cfg::kOffK, *sV = smem + Cfg::kOffV;
  uint64_t *bars = (uint64_t *)(smem + Cfg::kOffBar);
  constexpr int S = Cfg::kStages;
  constexpr int kBoxBytes = kBM * 64 * 2;        // one [128][64] box: 16 KB
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1, *k_empty = bars + 1 + S;         // [S] each
  uint64_t *v_full = bars + 1 + 2 * S, *v_empty = bars + 1 + 3 * S;
  uint64_t *s_full = bars + 1 + 4 * S, *s_free = s_full + 1;
  uint64_t *p_full = s_full + 2, *o_done = s_full + 3, *mma_done = s_full + 4;
  uint32_t *tmem_slot = (uint32_t *)(s_full + 5);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work item: the latest (most expensive) query tiles go first.
  const int per = p.nH * p.B;
  const int qt = p.n_qt - 1 - (int)(blockIdx.x / per);
  const int rest = (int)(blockIdx.x % per);
  const int h = rest % p.nH, b = rest / p.nH;
  const int kvh = h / (p.nH / p.nKV);
  const int q0 = qt * kBM;
  const int nkv = qt + 1;                       // key blocks 0..qt (kBN == kBM)
  const int row0 = b * p.T;                     // first token row of this sequence
  const bool aligned = (smem_u32(smem) & 1023u) == 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S; s++) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    if (!aligned) atomicExch(p.err, 10);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128, tP = tmem + 128 + D;
  pdl_wait();   // the previous kernel's outputs are complete from here on

  if (!aligned) {
    // nothing issued; fall through to the dealloc
  } else if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    int nk = 0, nv = 0;
    bool ok = true;
    mbar_expect_tx(q_full, Cfg::kTileQ);
#pragma unroll
    for (int a = 0; a < Cfg::kBoxes; a++) tma_load_2d(sQ + a * kBoxBytes, &tm, h * D + 64 * a, row0 + q0, q_full);
    for (int j = 0; j < nkv; j++) {
      const int s = j % S;
      const uint32_t ph = (uint32_t)(j / S) & 1u;
      if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
      mbar_expect_tx(&k_full[s], Cfg::kTileKV);
#pragma unroll
      for (int a = 0; a < Cfg::kBoxes; a++)
        tma_load_2d(sK + s * Cfg::kTileKV + a * kBoxBytes, &tm, (p.nH + kvh) * D + 64 * a, row0 + j * kBN,
                    &k_full[s]);
      nk++;
      if (!mbar_wait(&v_empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
      mbar_expect_tx(&v_full[s], Cfg::kTileKV);
#pragma unroll
      for (int a = 0; a < Cfg::kBoxes; a++)
        tma_load_2d(sV + s * Cfg::kTileKV + a * kBoxBytes, &tm, (p.nH + p.nKV + kvh) * D + 64 * a,
                    row0 + j * kBN, &v_full[s]);
      nv++;
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 11);
    }
    // Every copy issued has landed before the CTA exits.
    mbar_wait_drain(q_full, 0);
    for (int i = nk - S < 0 ? 0 : nk - S; i < nk; i++) mbar_wait_drain(&k_full[i % S], (uint32_t)(i / S) & 1u);
    for (int i = nv - S < 0 ? 0 : nv - S; i < nv; i++) mbar_wait_drain(&v_full[i % S], (uint32_t)(i / S) & 1u);
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp; elect.sync picks the issuing lane)
    const uint32_t id_s = instr_desc_bf16(0, 0, kBM, kBN);   // Q, K both K-major
    const uint32_t id_o = instr_desc_bf16(0, 1, kBM, D);     // P K-major, V MN-major
    bool ok = warp_wait(q_full, 0, abort_flag);
    const uint64_t dQ = desc_k(smem_u32(sQ));
    // V's D / 64 boxes are its MN-major atoms, kBN rows (16 KB) apart
    const uint64_t dK0 = desc_k(smem_u32(sK)), dV0 = desc_mn(smem_u32(sV), kBN);
    constexpr uint64_t kTileStep = Cfg::kTileKV >> 4, kBoxStep = kBoxBytes >> 4;
    for (int j = 0; j <= nkv && ok; j++) {
      if (j < nkv) {
        const int s = j % S;
        if (!warp_wait(&k_full[s], (uint32_t)(j / S) & 1u, abort_flag)) { ok = false; break; }
        if (j > 0 && !warp_wait(s_free, (uint32_t)(j - 1) & 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint64_t dK = dK0 + (uint64_t)s * kTileStep;
        // K = D: 4 slices of 16 per 64-column box
#pragma unroll
        for (int k = 0; k < D / 16; k++)
          umma_bf16_w(tS, dQ + (k >> 2) * kBoxStep + (k & 3) * kDescKStep,
                      dK + (k >> 2) * kBoxStep + (k & 3) * kDescKStep, id_s, k > 0 ? 1u : 0u);
        umma_commit_w(s_full);
        umma_commit_w(&k_empty[s]);
      }
      if (j > 0) {
        const int i = j - 1, s = i % S;
        if (!warp_wait(&v_full[s], (uint32_t)(i / S) & 1u, abort_flag) ||
            !warp_wait(p_full, (uint32_t)i & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t dV = dV0 + (uint64_t)s * kTileStep;
#pragma unroll
        for (int k = 0; k < kBN / 16; k++)
          umma_bf16_ts_w(tO, tP + (uint32_t)(8 * k), dV + k * kDescMNStep, id_o, (i > 0 || k > 0) ? 1u : 0u);
        umma_commit_w(o_done);
        umma_commit_w(&v_empty[s]);
      }
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 12);
    }
    umma_commit_w(mma_done);
    mbar_wait_drain(mma_done, 0);
  } else if (warp >= 2) {
    // ---------------- softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;          // tile row == TMEM lane
    const int q = q0 + r;                       // query position in the sequence
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; j++) {
      if (!warp_wait(s_full, (uint32_t)j & 1u, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[kBN];
      tmem_ld128(tS + lane_addr, s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      if (j == nkv - 1) {                       // diagonal block: keys after q are masked
        const int lim = q - j * kBN;
#pragma unroll
        for (int c = 0; c < kBN; c++)
          if (c > lim) s[c] = -INFINITY;
      }
      // Row max and sum over 8 independent chains (short dependency chains).
      float mx8[8];
#pragma unroll
      for (int u = 0; u < 8; u++) mx8[u] = s[u];
#pragma unroll
      for (int c = 8; c < kBN; c++) mx8[c & 7] = fmaxf(mx8[c & 7], s[c]);
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      mx *= p.scale_log2;
      float alpha = 1.f;
      bool rescale_o = false;
      if (mx > m + kRescaleLog2) {
        alpha = ex2_ftz(m - mx);                // 0 on the first block
        rescale_o = j > 0;
        m = mx;
      }
      const float neg_m = -m;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[kBN / 2];                     // P as bf16 pairs
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float2 e = exp2_pair<kPolyEveryFwd>(fma2(make_float2(s[c], s[c + 1]), make_float2(p.scale_log2, p.scale_log2),
                                        make_float2(neg_m, neg_m)), c / 2);
        rs4[(c >> 1) & 3] += e.x + e.y;
        pk[c / 2] = pack2_bf16(e.x, e.y);
      }
      const float rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      l = l * alpha + rs;
      // PV_{j-1} must be done with P and O before P is overwritten / O rescaled.
      if (j > 0 && !warp_wait(o_done, (uint32_t)(j - 1) & 1u, abort_flag)) { ok = false; break; }
      tmem_st32(tP + lane_addr, pk);
      tmem_st32(tP + lane_addr + 32, pk + 32);
      if (__any_sync(0xffffffffu, rescale_o)) {   // warp-collective: alpha = 1 on other rows
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < D / 32; half++) {
          uint32_t o[32];
          tmem_ld32(tO + lane_addr + half * 32, o);
#pragma unroll
          for (int c = 0; c < 32; c++) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(tO + lane_addr + half * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && warp_wait(o_done, (uint32_t)(nkv - 1) & 1u, abort_flag)) {
      tc_fence_after();
      const float inv = 1.f / l;
#pragma unroll
      for (int a = 0; a < D / 64; a++) {        // 64 columns of O at a time
        float o[64];
        tmem_ld64(tO + lane_addr + (uint32_t)(64 * a), o);
        if (q < p.T) {
          uint4 *dst = reinterpret_cast<uint4 *>(p.O + ((int64_t)(row0 + q) * p.nH + h) * D + 64 * a);
#pragma unroll
          for (int c8 = 0; c8 < 8; c8++) {
            uint4 v;
            v.x = pack2_bf16(o[8 * c8 + 0] * inv, o[8 * c8 + 1] * inv);
            v.y = pack2_bf16(o[8 * c8 + 2] * inv, o[8 * c8 + 3] * inv);
            v.z = pack2_bf16(o[8 * c8 + 4] * inv, o[8 * c8 + 5] * inv);
            v.w = pack2_bf16(o[8 * c8 + 6] * inv, o[8 * c8 + 7] * inv);
            dst[c8] = v;
          }
        }
      }
      if (q < p.T) p.lse[((int64_t)b * p.nH + h) * p.T + q] = (m + log2f(l)) / kLog2e;
    } else {
      ok = false;
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 13);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Cfg::kCols);
}

// ------------------------------------------------------------------ backward
//
// Two kernels, both deterministic (every gradient element is summed by one
// CTA in a fixed order), with the softmax probabilities recomputed from the
// forward's log-sum-exp:
//
// dK/dV, per CTA one 128-key tile of one kv head (or, head-split, of one q
// head), looping over the query tiles at or after it of every q head of the
// GQA group:
//   warp 0      TMA: K, V once; a 4-deep ring of (Q, dO) tiles plus the
//               tile's log-sum-exp and delta = rowsum(dO * O) rows
//   warp 1      MMA (warp-wide, elect.sync):  S^T = K Q^T, dP^T = V dO^T (128x128x64,
//               TMEM cols [0,128), [128,256)), then for the previous tile
//               dV += P^T dO, dK += dS^T Q (128x64x128, cols [256,320),
//               [320,384))
//   warps 2..9  thread = key row, two warps per TMEM lane quarter splitting
//               the 128 query columns: P^T = exp2(S^T c - L), dS^T =
//               P^T (dP^T - delta), both into TMEM as bf16 pairs (cols
//               [384,448), [448,512)), the A operands of the dV / dK MMAs;
//               at the end dV, and dK * scale rotated back by RoPE.
// dQ, per CTA one 128-row query tile of one q head, looping over the key
// tiles at or before it: S = Q K^T, dP = dO V^T, dS = P (dP - delta) (into
// TMEM cols [320,384) as the A operand), dQ += dS K; at the end dQ * scale
// rotated back by RoPE.
constexpr int kBwdThreads = 320;
constexpr uint32_t kBwdTmemCols = 512;

struct BwdParams {
  int B, T, nH, nKV, n_t, group, split;
  float scale, scale_log2;
  const float *lse, *delta;         // [B][nH][T]
  const float2 *rope;               // (cos, sin) [T][32], or null: no RoPE backward
  __nv_bfloat16 *dqkv;              // dq | dk | dv columns, row stride ld
  int64_t ld;
  float *pk, *pv;                   // head-split: fp32 partials [group][B*T][nKV*64]
  int *err;
};

// The dQ element loop: dS = exp2(S c - L) (dP - delta) for this warp's 64 key
// columns as bf16 pairs, instantiated with and without the diagonal mask
// (column valid iff column <= lim).  Only the last key tile of a query tile
// needs the mask, and the loop is issue-bound, so the other tiles skip its
// compares and selects.
template <bool kMasked>
__device__ __forceinline__ void dq_elements(const BwdParams &p, const float (&sv)[64], const float (&dp)[64],
                                            float L, float Dq, int lim, uint32_t (&dd)[32]) {
  const float2 sc = make_float2(p.scale_log2, p.scale_log2), nl = make_float2(-L, -L);
  const float2 nd = make_float2(-Dq, -Dq);
#pragma unroll
  for (int c = 0; c < 32; c++) {
    const float2 t = fma2(make_float2(sv[2 * c], sv[2 * c + 1]), sc, nl);   // s c - L
    const float2 e = exp2_pair<kPolyEvery>(t, c);
    float p0 = e.x, p1 = e.y;
    if (kMasked) {
      if (2 * c > lim) p0 = 0.f;
      if (2 * c + 1 > lim) p1 = 0.f;
    }
    const float2 g = mul2(make_float2(p0, p1), add2(make_float2(dp[2 * c], dp[2 * c + 1]), nd));
    dd[c] = pack2_bf16(g.x, g.y);
  }
}

// The dK/dV element loop for this warp's 64 query columns: P^T = exp2(S^T c
// - L) and dS^T = P^T (dP^T - delta) as bf16 pairs (packed f32x2 FMA / add /
// mul), with -L and -delta of the columns read from shared memory four at a
// time.  The compiler barrier at the end of each step keeps the loads from
// being hoisted to the top, where their 128 registers would spill.
__device__ __forceinline__ void dkdv_elements(float scale_log2, const float (&sv)[64], const float (&dp)[64],
                                              const float4 *nL4, const float4 *nD4, uint32_t (&pp)[32],
                                              uint32_t (&dd)[32]) {
#pragma unroll
  for (int c4 = 0; c4 < 16; c4++) {
    const float4 l4 = nL4[c4], d4 = nD4[c4];
    const int c = 4 * c4;
    const float2 sc = make_float2(scale_log2, scale_log2);
    const float2 e0 = exp2_pair<kPolyEvery>(fma2(make_float2(sv[c], sv[c + 1]), sc, make_float2(l4.x, l4.y)), 2 * c4);
    const float2 e1 = exp2_pair<kPolyEvery>(fma2(make_float2(sv[c + 2], sv[c + 3]), sc, make_float2(l4.z, l4.w)), 2 * c4 + 1);
    const float p0 = e0.x, p1 = e0.y, p2 = e1.x, p3 = e1.y;
    pp[2 * c4] = pack2_bf16(p0, p1);
    pp[2 * c4 + 1] = pack2_bf16(p2, p3);
    dd[2 * c4] = pack2_bf16(p0 * (dp[c] + d4.x), p1 * (dp[c + 1] + d4.y));
    dd[2 * c4 + 1] = pack2_bf16(p2 * (dp[c + 2] + d4.z), p3 * (dp[c + 3] + d4.w));
    asm volatile("" ::: "memory");
  }
}

// Masked columns (column c valid iff lo <= c < hi: queries before the key on
// the diagonal tile, past the sequence end on a ragged one) get P = dS = +0
// by clearing their bf16 halves; run only on the tiles that need it, after
// the element loop, when its inputs are no longer live.
__device__ __forceinline__ void dkdv_mask(int lo, int hi, uint32_t (&pp)[32], uint32_t (&dd)[32]) {
#pragma unroll
  for (int w = 0; w < 32; w++) {
    const int c = 2 * w;
    const uint32_t k = (c >= lo && c < hi ? 0x0000ffffu : 0u) | (c + 1 >= lo && c + 1 < hi ? 0xffff0000u : 0u);
    pp[w] &= k;
    dd[w] &= k;
  }
}

// dK/dV kernel shared memory at head dim D: K / V per item (double-buffered
// at D = 64, single at D = 128), a (Q, dO, lse, delta) ring across items (4
// deep at D = 64, 2 at D = 128).  The TMEM columns (S^T, dP^T, one 64-column
// slice of dV and of dK, bf16 P^T and dS^T) are those of D = 64: at D = 128
// each work item accumulates one 64-column half of dV and dK, its S^T / dP^T
// contracting over all 128 columns (two 64-column boxes).
template <int D>
struct KvCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileT = kBM * D * 2;
  static constexpr int kKV = D == 64 ? 2 : 1;          // K / V buffers
  static constexpr int kStages = D == 64 ? 4 : 2;
  static constexpr int K = 0;                          // [kKV] tiles
  static constexpr int V = K + kKV * kTileT;           // [kKV] tiles
  static constexpr int Q = V + kKV * kTileT;           // kStages tiles
  static constexpr int G = Q + kStages * kTileT;       // kStages tiles (dO)
  static constexpr int L = G + kStages * kTileT;       // [kStages][128] f32
  static constexpr int Dl = L + kStages * 128 * 4;     // [kStages][128] f32
  static constexpr int Bar = Dl + kStages * 128 * 4;
  static constexpr int Smem = Bar + (13 + 2 * kStages) * 8 + 16;
  static_assert(Smem <= 232448, "dK/dV shared memory");
};

// dQ kernel shared memory at head dim D: Q / dO tiles per item (double-
// buffered at D = 64, single at D = 128), a K/V ring (4 deep at D = 64, 2 at
// D = 128: [128][128] tiles are 32 KB), and TMEM S [0,128), dP [128,256),
// dS [256,320), dQ accumulators from 320 (two of 64 columns at D = 64, one of
// 128 at D = 128).  A [128][D] tile is D / 64 boxes of [128][64], 16 KB each.
template <int D>
struct DqCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileT = kBM * D * 2;
  static constexpr int kQG = D == 64 ? 2 : 1;          // Q / dO buffers
  static constexpr int kStages = D == 64 ? 4 : 2;      // K / V ring
  static constexpr int kNAcc = D == 64 ? 2 : 1;        // dQ accumulators
  static constexpr int Q = 0;
  static constexpr int G = Q + kQG * kTileT;
  static constexpr int K = G + kQG * kTileT;
  static constexpr int V = K + kStages * kTileT;
  static constexpr int Bar = V + kStages * kTileT;
  static constexpr int Smem = Bar + (13 + 2 * kStages) * 8 + 16;
  static_assert(Smem <= 232448 && 320 + kNAcc * D <= 512, "dQ shared memory / TMEM");
};

// Rotates interleaved pairs back by R^T: (x, y) -> (x c + y s, -x s + y c).
__device__ __forceinline__ void rope_back(float &x, float &y, float2 cs) {
  const float u = x * cs.x + y * cs.y, w = -x * cs.y + y * cs.x;
  x = u;
  y = w;
}

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_dkdv_tmem_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                              const __grid_constant__ CUtensorMap tm_do, BwdParams p) {
  fcu::pdl_trigger();
  using Cfg = KvCfg<D>;
  constexpr int kKStages = Cfg::kStages, kKV = Cfg::kKV, kTileT = Cfg::kTileT, kHalves = D / 64;
  constexpr uint64_t kBoxStep = kTile >> 4;            // next 64-column box of a tile
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *sK = smem + Cfg::K, *sV = smem + Cfg::V, *sQ = smem + Cfg::Q, *sG = smem + Cfg::G;
  float *sL = (float *)(smem + Cfg::L), *sDl = (float *)(smem + Cfg::Dl);
  uint64_t *bars = (uint64_t *)(smem + Cfg::Bar);
  uint64_t *kv_full = bars, *kv_empty = bars + 2;                        // [2]
  uint64_t *q_full = bars + 4, *q_empty = bars + 4 + kKStages;           // [kKStages]
  uint64_t *st_full = bars + 4 + 2 * kKStages, *st_free = st_full + 1;
  uint64_t *pds_full = st_full + 2, *pds_free = st_full + 3;
  uint64_t *acc_full = st_full + 4, *acc_free = st_full + 5, *mma_done = st_full + 6;
  uint32_t *tmem_slot = (uint32_t *)(st_full + 7);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work items (key tile, head, sequence, 64-column half of dV / dK), early
  // key tiles (most query tiles after them) first, strided over the
  // persistent grid.
  const int heads_cta = p.split ? p.nH : p.nKV;
  const int per = heads_cta * p.B * kHalves;
  const int n_items = p.n_t * per;
  const int n_heads = p.split ? 1 : p.group;
  const bool aligned = (smem_u32(smem) & 1023u) == 0;
  struct Item {
    int kt, kvh, h_begin, b, per_head, n_iter, dh;
  };
  auto item = [&](int idx) {
    Item w;
    w.kt = idx / per;
    const int rest0 = idx % per;
    w.dh = rest0 % kHalves;
    const int rest = rest0 / kHalves, hx = rest % heads_cta;
    w.b = rest / heads_cta;
    w.kvh = p.split ? hx / p.group : hx;
    w.h_begin = p.split ? hx : w.kvh * p.group;
    w.per_head = p.n_t - w.kt;                  // query tiles kt..n_t-1
    w.n_iter = n_heads * w.per_head;
    return w;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKV; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int s = 0; s < kKStages; s++) {
      mbar_init(&q_full[s], 2);               // TMA bytes + lse / delta staged
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_free, 8);
    mbar_init(pds_full, 8);
    mbar_init(pds_free, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_free, 8);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    if (!aligned) atomicExch(p.err, 20);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, kBwdTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 320;
  const uint32_t tPt = tmem + 384, tDt = tmem + 448;   // P^T, dS^T as bf16 pairs
  pdl_wait();   // the previous kernel's outputs are complete from here on

  if (!aligned) {
  } else if (warp == 0) {
    // ---------------- producer (lane 0 issues TMA; the warp stages lse / delta)
    bool ok = true;
    int u = 0, nk = 0;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
      const Item w = item(idx);
      const int row0 = w.b * p.T, kb = nk % kKV;
      if (!warp_wait(&kv_empty[kb], ((uint32_t)(nk / kKV) & 1u) ^ 1u, abort_flag)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        mbar_expect_tx(&kv_full[kb], 2 * kTileT);
#pragma unroll
        for (int bx = 0; bx < Cfg::kBoxes; bx++) {
          tma_load_2d(sK + kb * kTileT + bx * kTile, &tm_qkv, (p.nH + w.kvh) * D + bx * 64, row0 + w.kt * kBN,
                      &kv_full[kb]);
          tma_load_2d(sV + kb * kTileT + bx * kTile, &tm_qkv, (p.nH + p.nKV + w.kvh) * D + bx * 64,
                      row0 + w.kt * kBN, &kv_full[kb]);
        }
      }
      nk++;
      for (int it = 0; it < w.n_iter; it++, u++) {
        const int s = u % kKStages;
        if (!warp_wait(&q_empty[s], ((uint32_t)(u / kKStages) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const int h = w.h_begin + it / w.per_head;
        const int q0 = (w.kt + it % w.per_head) * kBM;
        if (lane == 0) {                      // copies first: their latency overlaps the loads below
          mbar_expect_tx(&q_full[s], 2 * kTileT);
#pragma unroll
          for (int bx = 0; bx < Cfg::kBoxes; bx++) {
            tma_load_2d(sQ + s * kTileT + bx * kTile, &tm_qkv, h * D + bx * 64, row0 + q0, &q_full[s]);
            tma_load_2d(sG + s * kTileT + bx * kTile, &tm_do, h * D + bx * 64, row0 + q0, &q_full[s]);
          }
        }
        const int64_t lrow = ((int64_t)w.b * p.nH + h) * p.T;
#pragma unroll
        for (int e = lane; e < kBM; e += 32) {
          const int q = q0 + e;
          sL[s * kBM + e] = q < p.T ? -(p.lse[lrow + q] * kLog2e) : 0.f;   // negated: the FMA adds them
          sDl[s * kBM + e] = q < p.T ? -p.delta[lrow + q] : 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[s]);
      }
    }
    if (lane == 0) {
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.err, 21);
      }
      for (int i = nk - kKV < 0 ? 0 : nk - kKV; i < nk; i++)
        mbar_wait_drain(&kv_full[i % kKV], (uint32_t)(i / kKV) & 1u);
      for (int i = u - kKStages < 0 ? 0 : u - kKStages; i < u; i++)
        mbar_wait_drain(&q_full[i % kKStages], (uint32_t)(i / kKStages) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp; elect.sync picks the issuing lane)
    {
      const uint32_t id_n128 = instr_desc_bf16(0, 0, kBM, kBN);
      const uint32_t id_n64 = instr_desc_bf16(0, 1, kBM, 64);
      constexpr uint64_t kTileStep = kTileT >> 4;
      const uint64_t dK0 = desc_k(smem_u32(sK)), dV0 = desc_k(smem_u32(sV));
      const uint64_t dQk0 = desc_k(smem_u32(sQ)), dGk0 = desc_k(smem_u32(sG));
      const uint64_t dQm0 = desc_mn(smem_u32(sQ), kBM), dGm0 = desc_mn(smem_u32(sG), kBM);
      bool ok = true, have_prev = false, prev_first = false, prev_last = false;
      int u = 0, ii = 0, prev_u = 0, prev_s = 0, prev_kb = 0, prev_ii = 0, prev_dh = 0;
      // dV += P^T dO, dK += dS^T Q for the previous unit (one unit behind its
      // S / dP MMAs), over the item's 64-column box of dO and Q
      auto issue_dvdk = [&]() -> bool {
        if (!warp_wait(pds_full, (uint32_t)prev_u & 1u, abort_flag)) return false;
        if (prev_first && !warp_wait(acc_free, ((uint32_t)prev_ii & 1u) ^ 1u, abort_flag)) return false;
        tc_fence_after();
        const uint64_t bq = dQm0 + (uint64_t)prev_s * kTileStep + (uint64_t)prev_dh * kBoxStep;
        const uint64_t bg = dGm0 + (uint64_t)prev_s * kTileStep + (uint64_t)prev_dh * kBoxStep;
#pragma unroll
        for (int k = 0; k < kBM / 16; k++)
          umma_bf16_ts_w(tdV, tPt + (uint32_t)(8 * k), bg + k * kDescMNStep, id_n64, (!prev_first || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < kBM / 16; k++)
          umma_bf16_ts_w(tdK, tDt + (uint32_t)(8 * k), bq + k * kDescMNStep, id_n64, (!prev_first || k > 0) ? 1u : 0u);
        umma_commit_w(pds_free);
        umma_commit_w(&q_empty[prev_s]);
        if (prev_last) {
          umma_commit_w(acc_full);
          umma_commit_w(&kv_empty[prev_kb]);
        }
        return true;
      };
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ii++) {
        const Item w = item(idx);
        const int kb = ii % kKV;
        // With one K/V buffer (D = 128) the producer refills it once the
        // previous item's last dV / dK MMAs have committed: issue them now
        // rather than after this item's first S^T / dP^T.
        if (kKV == 1 && have_prev) {
          if (!issue_dvdk()) {
            ok = false;
            break;
          }
          have_prev = false;
        }
        if (!warp_wait(&kv_full[kb], (uint32_t)(ii / kKV) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        const uint64_t ak = dK0 + (uint64_t)kb * kTileStep, av = dV0 + (uint64_t)kb * kTileStep;
        for (int it = 0; it < w.n_iter; it++, u++) {
          const int s = u % kKStages;
          if (!warp_wait(&q_full[s], (uint32_t)(u / kKStages) & 1u, abort_flag) ||
              (u > 0 && !warp_wait(st_free, (uint32_t)(u - 1) & 1u, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bq = dQk0 + (uint64_t)s * kTileStep, bg = dGk0 + (uint64_t)s * kTileStep;
#pragma unroll
          for (int k = 0; k < D / 16; k++)
            umma_bf16_w(tS, ak + (k >> 2) * kBoxStep + (k & 3) * kDescKStep, bq + (k >> 2) * kBoxStep + (k & 3) * kDescKStep,
                        id_n128, k > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < D / 16; k++)
            umma_bf16_w(tdP, av + (k >> 2) * kBoxStep + (k & 3) * kDescKStep, bg + (k >> 2) * kBoxStep + (k & 3) * kDescKStep,
                        id_n128, k > 0 ? 1u : 0u);
          umma_commit_w(st_full);
          if (have_prev && !issue_dvdk()) {
            ok = false;
            break;
          }
          have_prev = true;
          prev_u = u;
          prev_s = s;
          prev_kb = kb;
          prev_ii = ii;
          prev_dh = w.dh;
          prev_first = it == 0;
          prev_last = it == w.n_iter - 1;
        }
      }
      if (ok && have_prev && !issue_dvdk()) ok = false;
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.err, 22);
      }
      umma_commit_w(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
  } else {
    // ---------------- P^T / dS^T and the dK / dV epilogue (warps 2..9)
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;          // key row == TMEM lane
    const uint32_t la = (uint32_t)(quarter * 32) << 16;
    const int cb = half * 64;                   // this warp's 64 query columns
    bool ok = true;
    int u = 0, ii = 0;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ii++) {
      const Item w = item(idx);
      const int key = w.kt * kBN + r;
      for (int it = 0; it < w.n_iter; it++, u++) {
        const int s = u % kKStages;
        const int q0 = (w.kt + it % w.per_head) * kBM;
        if (!warp_wait(&q_full[s], (uint32_t)(u / kKStages) & 1u, abort_flag) ||
            !warp_wait(st_full, (uint32_t)u & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[64], dp[64];
        tmem_ld64x2(tS + la + cb, tdP + la + cb, sv, dp);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(st_free);
        const float4 *L4 = reinterpret_cast<const float4 *>(sL + s * kBM + cb);
        const float4 *D4 = reinterpret_cast<const float4 *>(sDl + s * kBM + cb);
        const int qc = q0 + cb;                 // first query of these columns
        uint32_t pp[32], dd[32];
        // queries before the key (diagonal tile) or past the sequence end are masked
        dkdv_elements(p.scale_log2, sv, dp, L4, D4, pp, dd);
        if (qc < key || qc + 64 > p.T) dkdv_mask(key - qc, p.T - qc, pp, dd);
        // dV/dK of the previous unit must be done reading P^T / dS^T.
        if (u > 0 && !warp_wait(pds_free, (uint32_t)(u - 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tmem_st32(tPt + la + (uint32_t)(32 * half), pp);
        tmem_st32(tDt + la + (uint32_t)(32 * half), dd);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pds_full);
      }
      if (!ok || !warp_wait(acc_full, (uint32_t)ii & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[64];
      tmem_ld64((half ? tdK : tdV) + la, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_free);
      if (key < p.T) {
        const int row0 = w.b * p.T;
        const float mul = half ? p.scale : 1.f;
        if (p.split) {
          const int g = w.h_begin - w.kvh * p.group;
          float *dst = (half ? p.pk : p.pv) +
                       ((int64_t)g * p.B * p.T + row0 + key) * ((int64_t)p.nKV * D) + w.kvh * D + w.dh * 64;
#pragma unroll
          for (int c4 = 0; c4 < 16; c4++)
            reinterpret_cast<float4 *>(dst)[c4] =
                make_float4(v[4 * c4] * mul, v[4 * c4 + 1] * mul, v[4 * c4 + 2] * mul, v[4 * c4 + 3] * mul);
        } else {
#pragma unroll
          for (int c = 0; c < 64; c++) v[c] *= mul;
          if (half && p.rope) {
#pragma unroll
            for (int i = 0; i < 32; i++)
              rope_back(v[2 * i], v[2 * i + 1], p.rope[(int64_t)key * (D / 2) + w.dh * 32 + i]);
          }
          uint4 *dst = reinterpret_cast<uint4 *>(p.dqkv + (int64_t)(row0 + key) * p.ld +
                                                 (int64_t)(p.nH + (half ? 0 : p.nKV) + w.kvh) * D + w.dh * 64);
#pragma unroll
          for (int c8 = 0; c8 < 8; c8++)
            dst[c8] = make_uint4(pack2_bf16(v[8 * c8], v[8 * c8 + 1]), pack2_bf16(v[8 * c8 + 2], v[8 * c8 + 3]),
                                 pack2_bf16(v[8 * c8 + 4], v[8 * c8 + 5]), pack2_bf16(v[8 * c8 + 6], v[8 * c8 + 7]));
        }
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicExch(p.err, 23);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kBwdTmemCols);
}

// dQ, persistent: one CTA per SM walks the (query tile, head) items, latest
// query tiles first, strided over the grid.  Per item it loops over the key
// tiles at or before its query tile: S = Q K^T, dP = dO V^T, dS = P (dP -
// delta) into TMEM cols [256,320) as the A operand, dQ += dS K into one of
// two TMEM accumulators (cols [320,384), [384,448)), so one item's epilogue
// (dQ * scale rotated back by RoPE) overlaps the next item's first MMAs.
// Q/dO tiles are double-buffered per item; the K/V ring runs across items.
template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_dq_tmem_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                            const __grid_constant__ CUtensorMap tm_do, BwdParams p) {
  fcu::pdl_trigger();
  using Cfg = DqCfg<D>;
  constexpr int kQStages = Cfg::kStages, kQG = Cfg::kQG, kNAcc = Cfg::kNAcc, kTileT = Cfg::kTileT;
  constexpr uint64_t kBoxStep = kTile >> 4;            // next 64-column box of a tile
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *sQ = smem + Cfg::Q, *sG = smem + Cfg::G, *sK = smem + Cfg::K, *sV = smem + Cfg::V;
  uint64_t *bars = (uint64_t *)(smem + Cfg::Bar);
  uint64_t *qg_full = bars, *qg_empty = bars + 2;                       // [2]
  uint64_t *kv_full = bars + 4, *kv_empty = bars + 4 + kQStages;        // [kQStages]
  uint64_t *sp_full = bars + 4 + 2 * kQStages, *sp_free = sp_full + 1;
  uint64_t *ds_full = sp_full + 2, *ds_free = sp_full + 3;
  uint64_t *acc_full = sp_full + 4, *acc_free = sp_full + 6;            // [2]
  uint64_t *mma_done = sp_full + 8;
  uint32_t *tmem_slot = (uint32_t *)(mma_done + 1);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = p.nH * p.B;
  const int n_items = p.n_t * per;
  const bool aligned = (smem_u32(smem) & 1023u) == 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&qg_full[i], 1);
      mbar_init(&qg_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_free[i], 8);
    }
    for (int s = 0; s < kQStages; s++) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(sp_free, 8);
    mbar_init(ds_full, 8);
    mbar_init(ds_free, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    if (!aligned) atomicExch(p.err, 30);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, kBwdTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdS = tmem + 256, tdQ0 = tmem + 320;
  pdl_wait();   // the previous kernel's outputs are complete from here on

  if (!aligned) {
  } else if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      bool ok = true;
      int u = 0, nq = 0;
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
        const int qt = p.n_t - 1 - idx / per, rest = idx % per;
        const int h = rest % p.nH, b = rest / p.nH, kvh = h / p.group;
        const int row0 = b * p.T, qb = nq % kQG;
        if (!mbar_wait(&qg_empty[qb], ((uint32_t)(nq / kQG) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&qg_full[qb], 2 * kTileT);
#pragma unroll
        for (int bx = 0; bx < Cfg::kBoxes; bx++) {
          tma_load_2d(sQ + qb * kTileT + bx * kTile, &tm_qkv, h * D + bx * 64, row0 + qt * kBM, &qg_full[qb]);
          tma_load_2d(sG + qb * kTileT + bx * kTile, &tm_do, h * D + bx * 64, row0 + qt * kBM, &qg_full[qb]);
        }
        nq++;
        for (int j = 0; j <= qt; j++, u++) {
          const int s = u % kQStages;
          if (!mbar_wait(&kv_empty[s], ((uint32_t)(u / kQStages) & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&kv_full[s], 2 * kTileT);
#pragma unroll
          for (int bx = 0; bx < Cfg::kBoxes; bx++) {
            tma_load_2d(sK + s * kTileT + bx * kTile, &tm_qkv, (p.nH + kvh) * D + bx * 64, row0 + j * kBN, &kv_full[s]);
            tma_load_2d(sV + s * kTileT + bx * kTile, &tm_qkv, (p.nH + p.nKV + kvh) * D + bx * 64, row0 + j * kBN,
                        &kv_full[s]);
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.err, 31);
      }
      for (int i = nq - kQG < 0 ? 0 : nq - kQG; i < nq; i++)
        mbar_wait_drain(&qg_full[i % kQG], (uint32_t)(i / kQG) & 1u);
      for (int i = u - kQStages < 0 ? 0 : u - kQStages; i < u; i++)
        mbar_wait_drain(&kv_full[i % kQStages], (uint32_t)(i / kQStages) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp; elect.sync picks the issuing lane)
    {
      const uint32_t id_n128 = instr_desc_bf16(0, 0, kBM, kBN);
      const uint32_t id_nD = instr_desc_bf16(0, 1, kBM, D);
      const uint64_t dQ0 = desc_k(smem_u32(sQ)), dG0 = desc_k(smem_u32(sG));
      const uint64_t dKk0 = desc_k(smem_u32(sK)), dVk0 = desc_k(smem_u32(sV));
      const uint64_t dKm0 = desc_mn(smem_u32(sK), kBN);   // K as B of dS K: D / 64 atoms 16 KB apart
      constexpr uint64_t kTileStep = kTileT >> 4;
      bool ok = true, have_prev = false, prev_first = false, prev_last = false;
      int u = 0, ii = 0, prev_u = 0, prev_s = 0, prev_ab = 0, prev_ii = 0;
      // dQ += dS K for the previous unit (one unit behind its S / dP MMAs).
      // An item's first dQ MMA waits for the epilogue that last read its
      // accumulator; with one accumulator (D = 128) that is the previous
      // item's, whose own last dQ MMA has been issued by then.
      auto issue_dq = [&]() -> bool {
        if (!warp_wait(ds_full, (uint32_t)prev_u & 1u, abort_flag)) return false;
        if (prev_first && !warp_wait(&acc_free[prev_ab], ((uint32_t)(prev_ii / kNAcc) & 1u) ^ 1u, abort_flag))
          return false;
        tc_fence_after();
        const uint64_t bk = dKm0 + (uint64_t)prev_s * kTileStep;
        const uint32_t acc = tdQ0 + (uint32_t)(prev_ab * D);
#pragma unroll
        for (int k = 0; k < kBN / 16; k++)
          umma_bf16_ts_w(acc, tdS + (uint32_t)(8 * k), bk + k * kDescMNStep, id_nD, (!prev_first || k > 0) ? 1u : 0u);
        umma_commit_w(ds_free);
        umma_commit_w(&kv_empty[prev_s]);
        if (prev_last) umma_commit_w(&acc_full[prev_ab]);
        return true;
      };
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ii++) {
        const int qt = p.n_t - 1 - idx / per;
        const int qb = ii % kQG, ab = ii % kNAcc;
        if (!warp_wait(&qg_full[qb], (uint32_t)(ii / kQG) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        const uint64_t aq = dQ0 + (uint64_t)qb * kTileStep, ag = dG0 + (uint64_t)qb * kTileStep;
        for (int j = 0; j <= qt; j++, u++) {
          const int s = u % kQStages;
          if (!warp_wait(&kv_full[s], (uint32_t)(u / kQStages) & 1u, abort_flag) ||
              (u > 0 && !warp_wait(sp_free, (uint32_t)(u - 1) & 1u, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bk = dKk0 + (uint64_t)s * kTileStep, bv = dVk0 + (uint64_t)s * kTileStep;
#pragma unroll
          for (int k = 0; k < D / 16; k++)
            umma_bf16_w(tS, aq + (k >> 2) * kBoxStep + (k & 3) * kDescKStep, bk + (k >> 2) * kBoxStep + (k & 3) * kDescKStep,
                        id_n128, k > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < D / 16; k++)
            umma_bf16_w(tdP, ag + (k >> 2) * kBoxStep + (k & 3) * kDescKStep, bv + (k >> 2) * kBoxStep + (k & 3) * kDescKStep,
                        id_n128, k > 0 ? 1u : 0u);
          umma_commit_w(sp_full);
          if (j == qt) umma_commit_w(&qg_empty[qb]);   // this item's Q / dO are read
          if (have_prev && !issue_dq()) {
            ok = false;
            break;
          }
          have_prev = true;
          prev_u = u;
          prev_s = s;
          prev_ab = ab;
          prev_ii = ii;
          prev_first = j == 0;
          prev_last = j == qt;
        }
      }
      if (ok && have_prev && !issue_dq()) ok = false;
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.err, 32);
      }
      umma_commit_w(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
  } else {
    // ---------------- dS and the dQ epilogue (warps 2..9)
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;          // query row == TMEM lane
    const uint32_t la = (uint32_t)(quarter * 32) << 16;
    const int cb = half * 64;                   // this warp's 64 key columns
    bool ok = true;
    int u = 0, ii = 0;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ii++) {
      const int qt = p.n_t - 1 - idx / per, rest = idx % per;
      const int h = rest % p.nH, b = rest / p.nH;
      const int q = qt * kBM + r, ab = ii % kNAcc;
      const int64_t li = ((int64_t)b * p.nH + h) * p.T + q;
      const float L = q < p.T ? p.lse[li] * kLog2e : 0.f;
      const float Dq = q < p.T ? p.delta[li] : 0.f;
      for (int j = 0; j <= qt; j++, u++) {
        if (!warp_wait(sp_full, (uint32_t)u & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[64], dp[64];
        tmem_ld64x2(tS + la + cb, tdP + la + cb, sv, dp);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sp_free);
        const int lim = r - cb;                 // diagonal tile: key column c valid if c <= lim
        uint32_t dd[32];
        if (j == qt)                            // only the diagonal key tile needs the mask
          dq_elements<true>(p, sv, dp, L, Dq, lim, dd);
        else
          dq_elements<false>(p, sv, dp, L, Dq, lim, dd);
        if (u > 0 && !warp_wait(ds_free, (uint32_t)(u - 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tmem_st32(tdS + la + (uint32_t)(32 * half), dd);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
      }
      if (!ok || !warp_wait(&acc_full[ab], (uint32_t)(ii / kNAcc) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // this warp's D / 2 columns of dQ
      constexpr int kHalf = D / 2;
      float v[kHalf];
      const uint32_t tq = tdQ0 + (uint32_t)(ab * D) + la + (uint32_t)(half * kHalf);
      if constexpr (kHalf == 32) {
        uint32_t uq[32];
        tmem_ld32(tq, uq);
#pragma unroll
        for (int c = 0; c < 32; c++) v[c] = __uint_as_float(uq[c]);
      } else {
        tmem_ld64(tq, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[ab]);
      if (q < p.T) {
#pragma unroll
        for (int c = 0; c < kHalf; c++) v[c] *= p.scale;
        if (p.rope) {
#pragma unroll
          for (int i = 0; i < kHalf / 2; i++)
            rope_back(v[2 * i], v[2 * i + 1], p.rope[(int64_t)q * (D / 2) + half * (kHalf / 2) + i]);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(p.dqkv + (int64_t)(b * p.T + q) * p.ld + (int64_t)h * D + half * kHalf);
#pragma unroll
        for (int c8 = 0; c8 < kHalf / 8; c8++)
          dst[c8] = make_uint4(pack2_bf16(v[8 * c8], v[8 * c8 + 1]), pack2_bf16(v[8 * c8 + 2], v[8 * c8 + 3]),
                               pack2_bf16(v[8 * c8 + 4], v[8 * c8 + 5]), pack2_bf16(v[8 * c8 + 6], v[8 * c8 + 7]));
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicExch(p.err, 33);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kBwdTmemCols);
}

// delta[b][h][t] = sum_d dO[bt, h*D + d] * O[bt, h*D + d]; D / 8 threads
// per (token, head), one 16-byte load of each operand per thread.
template <int D>
__global__ void attn_delta_kernel(const __nv_bfloat16 *__restrict__ dO,
                                  const __nv_bfloat16 *__restrict__ O, int64_t units, int nH, int T,
                                  float *__restrict__ delta) {
  fcu::pdl_trigger();
  constexpr int kLanes = D / 8;
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t unit = t / kLanes;              // token row * nH + head
  float s = 0.f;
  if (unit < units) {
    const uint4 g = reinterpret_cast<const uint4 *>(dO)[t];
    const uint4 o = reinterpret_cast<const uint4 *>(O)[t];
    const __nv_bfloat162 *g2 = reinterpret_cast<const __nv_bfloat162 *>(&g);
    const __nv_bfloat162 *o2 = reinterpret_cast<const __nv_bfloat162 *>(&o);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 a = __bfloat1622float2(g2[i]), c = __bfloat1622float2(o2[i]);
      s = fmaf(a.x, c.x, s);
      s = fmaf(a.y, c.y, s);
    }
  }
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (unit < units && (t % kLanes) == 0) {
    const int64_t row = unit / nH;
    const int h = (int)(unit - row * nH);
    const int64_t b = row / T, tt = row - b * T;
    delta[(b * nH + h) * T + tt] = s;
  }
}

// Head-split dK/dV: sums the group's fp32 partials in order, rotates dK back
// and stores both as bf16 into the dqkv buffer.  One thread per 4 columns.
template <int D>
__global__ void attn_kv_reduce_kernel(const float *__restrict__ pk, const float *__restrict__ pv,
                                      int group, int64_t rows, int nH, int nKV, int T,
                                      const float2 *__restrict__ rope, __nv_bfloat16 *dqkv, int64_t ld) {
  fcu::pdl_trigger();
  const int64_t kvD = (int64_t)nKV * D, q4 = kvD / 4, n = rows * q4;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / q4;
    const int64_t c = (e - row * q4) * 4;
    float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
    for (int g = 0; g < group; g++) {
      const int64_t o = ((int64_t)g * rows + row) * kvD + c;
      const float4 a = *reinterpret_cast<const float4 *>(pk + o);
      const float4 d = *reinterpret_cast<const float4 *>(pv + o);
      k.x += a.x; k.y += a.y; k.z += a.z; k.w += a.w;
      v.x += d.x; v.y += d.y; v.z += d.z; v.w += d.w;
    }
    if (rope) {
      const float2 *cs = rope + (row % T) * (D / 2) + (c % D) / 2;
      rope_back(k.x, k.y, cs[0]);
      rope_back(k.z, k.w, cs[1]);
    }
    __nv_bfloat16 *dk = dqkv + row * ld + (int64_t)nH * D + c;
    __nv_bfloat16 *dv = dk + kvD;
    *reinterpret_cast<uint2 *>(dk) = make_uint2(pack2_bf16(k.x, k.y), pack2_bf16(k.z, k.w));
    *reinterpret_cast<uint2 *>(dv) = make_uint2(pack2_bf16(v.x, v.y), pack2_bf16(v.z, v.w));
  }
}

}  // namespace

bool attn_tmem_supported(int dH) { return dH == kD || dH == 128; }

// O [B*T, nH*D] bf16 and lse [B][nH][T] from the bf16 qkv buffer (row stride
// ld_qkv elements: q heads, then k heads, then v heads, D columns each; D =
// 128 when dh is 128, else 64 with heads of dh < 64 zero-padded).
template <int D>
int attn_fwd_tmem_d(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV, void *O,
                    float *lse, int dh) {
  using Cfg = FwdCfg<D>;
  int rc = tc_get_encode();
  if (rc) return rc;
  int *err = nullptr;
  rc = tc_error_word(ctx, &err);
  if (rc) return rc;
  CUtensorMap map;
  rc = tc_make_map(&map, qkv, (uint64_t)B * T, (uint64_t)(nH + 2 * nKV) * D, (uint64_t)ld_qkv, 64, kBM);
  if (rc) return rc;
  FwdParams p{};
  p.B = B;
  p.T = T;
  p.nH = nH;
  p.nKV = nKV;
  p.n_qt = div_up(T, kBM);
  p.scale_log2 = (float)(1.0 / sqrt((double)dh)) * kLog2e;
  p.O = (__nv_bfloat16 *)O;
  p.lse = lse;
  p.err = err;
  static bool attr_set[64] = {false};
  if (!attr_set[ctx->device & 63]) {
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_tmem_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Cfg::kSmemBytes));
    attr_set[ctx->device & 63] = true;
  }
  const int64_t grid = (int64_t)p.n_qt * nH * B;
  FCU_REQUIRE(grid <= INT32_MAX, "attention: grid too large");
  FCU_CHECK_CUDA(launch_pdl(attn_fwd_tmem_kernel<D>, dim3((unsigned)grid), dim3(kThreads), Cfg::kSmemBytes,
                            ctx->stream, map, p));
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int attn_fwd_tmem(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV,
                  void *O, float *lse, int dh) {
  if (dh == 128) return attn_fwd_tmem_d<128>(ctx, qkv, ld_qkv, B, T, nH, nKV, O, lse, dh);
  return attn_fwd_tmem_d<64>(ctx, qkv, ld_qkv, B, T, nH, nKV, O, lse, dh);
}

namespace {

// Backward at head width D (64: heads of dh <= 64, zero-padded below 64; 128).
template <int D>
int attn_bwd_tmem_d(fcu_ctx *ctx, const void *dO, const void *qkv, int64_t ld_qkv, const void *O,
                    const float *lse, float *delta, int B, int T, int nH, int nKV, const float2 *rope,
                    void *dqkv, int split, float *pk, float *pv, int dh) {
  int rc = tc_get_encode();
  if (rc) return rc;
  int *err = nullptr;
  rc = tc_error_word(ctx, &err);
  if (rc) return rc;
  CUtensorMap map_qkv, map_do;
  rc = tc_make_map(&map_qkv, qkv, (uint64_t)B * T, (uint64_t)(nH + 2 * nKV) * D, (uint64_t)ld_qkv, 64,
                   kBM);
  if (!rc) rc = tc_make_map(&map_do, dO, (uint64_t)B * T, (uint64_t)nH * D, (uint64_t)nH * D, 64, kBM);
  if (rc) return rc;
  const int64_t units = (int64_t)B * T * nH;
  attn_delta_kernel<D><<<(unsigned)((units * (D / 8) + 255) / 256), 256, 0, ctx->stream>>>(
      (const __nv_bfloat16 *)dO, (const __nv_bfloat16 *)O, units, nH, T, delta);
  FCU_CHECK_LAUNCH();
  BwdParams p{};
  p.B = B;
  p.T = T;
  p.nH = nH;
  p.nKV = nKV;
  p.n_t = div_up(T, kBM);
  p.group = nH / nKV;
  p.split = split;
  p.scale = (float)(1.0 / sqrt((double)dh));
  p.scale_log2 = p.scale * kLog2e;
  p.lse = lse;
  p.delta = delta;
  p.rope = rope;
  p.dqkv = (__nv_bfloat16 *)dqkv;
  p.ld = ld_qkv;
  p.pk = pk;
  p.pv = pv;
  p.err = err;
  static bool attr_set[64] = {false};
  if (!attr_set[ctx->device & 63]) {
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_tmem_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        KvCfg<D>::Smem));
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tmem_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        DqCfg<D>::Smem));
    attr_set[ctx->device & 63] = true;
  }
  const int64_t items_kv = (int64_t)p.n_t * (split ? nH : nKV) * B * (D / 64);
  const int64_t grid_kv = items_kv < ctx->num_sms ? items_kv : ctx->num_sms;   // persistent
  const int64_t items_q = (int64_t)p.n_t * nH * B;
  const int64_t grid_q = items_q < ctx->num_sms ? items_q : ctx->num_sms;   // persistent
  FCU_REQUIRE(items_q <= INT32_MAX && items_kv <= INT32_MAX, "attention backward: grid too large");
  FCU_CHECK_CUDA(launch_pdl(attn_bwd_dkdv_tmem_kernel<D>, dim3((unsigned)grid_kv), dim3(kBwdThreads),
                            KvCfg<D>::Smem, ctx->stream, map_qkv, map_do, p));
  FCU_CHECK_LAUNCH();
  if (split) {
    const int64_t n = (int64_t)B * T * nKV * D / 4;
    int blocks = (int)((n + 255) / 256);
    if (blocks > 16 * ctx->num_sms) blocks = 16 * ctx->num_sms;
    attn_kv_reduce_kernel<D><<<blocks, 256, 0, ctx->stream>>>(pk, pv, p.group, (int64_t)B * T, nH, nKV, T, rope,
                                                              (__nv_bfloat16 *)dqkv, ld_qkv);
    FCU_CHECK_LAUNCH();
  }
  FCU_CHECK_CUDA(launch_pdl(attn_bwd_dq_tmem_kernel<D>, dim3((unsigned)grid_q), dim3(kBwdThreads), DqCfg<D>::Smem,
                            ctx->stream, map_qkv, map_do, p));
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // namespace

// Backward from the bf16 qkv buffer, dO and O ([B*T, nH*W] bf16, W = 128 when
// dh is 128, else 64) and the forward's lse: dq | dk | dv (RoPE rotated back
// when `rope` is given) into the bf16 dqkv buffer (same layout and row stride
// as qkv).  `delta` is scratch of B*nH*T floats; `pk`, `pv` are the head-split
// partial buffers (group * B*T * nKV*W floats each), used when `split` is set.
int attn_bwd_tmem(fcu_ctx *ctx, const void *dO, const void *qkv, int64_t ld_qkv, const void *O,
                  const float *lse, float *delta, int B, int T, int nH, int nKV, const float2 *rope,
                  void *dqkv, int split, float *pk, float *pv, int dh) {
  if (dh == 128)
    return attn_bwd_tmem_d<128>(ctx, dO, qkv, ld_qkv, O, lse, delta, B, T, nH, nKV, rope, dqkv, split, pk, pv, dh);
  return attn_bwd_tmem_d<64>(ctx, dO, qkv, ld_qkv, O, lse, delta, B, T, nH, nKV, rope, dqkv, split, pk, pv, dh);
}

// ------------------------------------------------------------------ operator entries
// causalAttn / causalAttnBatch on fp32 operands (fcu_attn_fwd / fcu_attn_bwd
// in FCU_PREC_BF16 mode, head dim 64) on the same tcgen05 kernels: the fp32
// Q / K / V (and dO, O) are packed into the bf16 qkv layout the kernels read,
// and the bf16 outputs are widened back to fp32 (adding into the gradients
// when accumulating, the JS `grad +=`).  The packed copies live in a buffer
// of their own (grown on demand, one per device), so the kernels' scratch
// (delta, head-split partials) is untouched.
namespace {

int op_buffer(fcu_ctx *ctx, size_t bytes, void **out) {
  struct Buf {
    void *p = nullptr;
    size_t n = 0;
  };
  static thread_local Buf bufs[64];
  Buf &b = bufs[ctx->device & 63];
  if (bytes > b.n) {
    if (b.p) {
      FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
      FCU_CHECK_CUDA(cudaFree(b.p));
      b.p = nullptr;
      b.n = 0;
    }
    FCU_CHECK_CUDA(cudaMalloc(&b.p, bytes));
    b.n = bytes;
  }
  *out = b.p;
  return FCU_OK;
}

// Head-padded layouts.  The kernels read 64 columns per head; a head of dh
// < 64 columns (dh % 4 == 0) is carried as its dh values followed by 64 - dh
// zeros.  Zero columns add nothing to q.k, and the O / dq / dk / dv columns
// they produce are zero and dropped, so the padded problem is the original
// one (the softmax scale stays 1/sqrt(dh)).

// dst[r, col0 + h*hw + c] = bf16(src[r, h*dh + c]) for c < dh, 0 for dh <= c < hw
__global__ void pack_bf16_kernel(const float *__restrict__ src, int64_t rows, int heads, int dh, int hw,
                                 __nv_bfloat16 *dst, int64_t ld, int col0) {
  const int64_t n = rows * heads * (hw / 4);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rh = i / (hw / 4);
    const int c = (int)(i - rh * (hw / 4)) * 4;
    const int64_t r = rh / heads;
    const int h = (int)(rh - r * heads);
    uint2 u = make_uint2(0u, 0u);
    if (c < dh) {
      const float4 v = *reinterpret_cast<const float4 *>(src + (r * heads + h) * dh + c);
      __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
      u.x = *reinterpret_cast<uint32_t *>(&a);
      u.y = *reinterpret_cast<uint32_t *>(&b);
    }
    *reinterpret_cast<uint2 *>(dst + r * ld + col0 + h * hw + c) = u;
  }
}

// dst[r, h*dh + c] (+)= float(src[r, col0 + h*hw + c]) for c < dh
__global__ void unpack_bf16_kernel(const __nv_bfloat16 *__restrict__ src, int64_t ld, int col0, int64_t rows,
                                   int heads, int dh, int hw, float *dst, int accumulate) {
  const int c4 = dh / 4;
  const int64_t n = rows * heads * c4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rh = i / c4;
    const int c = (int)(i - rh * c4) * 4;
    const int64_t r = rh / heads;
    const int h = (int)(rh - r * heads);
    const uint2 u = *reinterpret_cast<const uint2 *>(src + r * ld + col0 + h * hw + c);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
    float4 v = make_float4(a.x, a.y, b.x, b.y);
    float4 *d = reinterpret_cast<float4 *>(dst + rh * dh + c);
    if (accumulate) {
      const float4 o = *d;
      v.x += o.x;
      v.y += o.y;
      v.z += o.z;
      v.w += o.w;
    }
    *d = v;
  }
}

// bf16 rows of dh-column heads <-> rows of 64-column heads (to_pad: zero
// fill of columns [dh, 64); otherwise those columns are dropped).
__global__ void repad_bf16_kernel(const __nv_bfloat16 *__restrict__ src, int64_t lds, __nv_bfloat16 *dst,
                                  int64_t ldd, int64_t rows, int heads, int dh, int to_pad) {
  const int c4 = (to_pad ? kD : dh) / 4;
  const int64_t n = rows * heads * c4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rh = i / c4;
    const int c = (int)(i - rh * c4) * 4;
    const int64_t r = rh / heads;
    const int h = (int)(rh - r * heads);
    if (to_pad) {
      uint2 u = make_uint2(0u, 0u);
      if (c < dh) u = *reinterpret_cast<const uint2 *>(src + r * lds + h * dh + c);
      *reinterpret_cast<uint2 *>(dst + r * ldd + h * kD + c) = u;
    } else {
      *reinterpret_cast<uint2 *>(dst + r * ldd + h * dh + c) =
          *reinterpret_cast<const uint2 *>(src + r * lds + h * kD + c);
    }
  }
}

int grid_for(fcu_ctx *ctx, int64_t n) {
  return (int)((n + 255) / 256 < 16 * ctx->num_sms ? (n + 255) / 256 : 16 * ctx->num_sms);
}

// hw: the head width of the bf16 layout (64, or 128 for heads of 128)
int pack(fcu_ctx *ctx, const float *src, int64_t rows, int heads, int dh, __nv_bfloat16 *dst, int64_t ld,
         int col0, int hw = kD) {
  pack_bf16_kernel<<<grid_for(ctx, rows * heads * (hw / 4)), 256, 0, ctx->stream>>>(src, rows, heads, dh, hw,
                                                                                     dst, ld, col0);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int unpack(fcu_ctx *ctx, const __nv_bfloat16 *src, int64_t ld, int col0, int64_t rows, int heads, int dh,
           float *dst, int accumulate, int hw = kD) {
  unpack_bf16_kernel<<<grid_for(ctx, rows * heads * (dh / 4)), 256, 0, ctx->stream>>>(
      src, ld, col0, rows, heads, dh, hw, dst, accumulate);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int repad(fcu_ctx *ctx, const void *src, int64_t lds, void *dst, int64_t ldd, int64_t rows, int heads, int dh,
          int to_pad) {
  repad_bf16_kernel<<<grid_for(ctx, rows * heads * ((to_pad ? kD : dh) / 4)), 256, 0, ctx->stream>>>(
      (const __nv_bfloat16 *)src, lds, (__nv_bfloat16 *)dst, ldd, rows, heads, dh, to_pad);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

bool op_aligned(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

bool attn_tmem_padded(int dH) { return dH > 0 && dH <= kD && dH % 4 == 0; }

bool attn_tmem_op_supported(int dH, const void *a, const void *b, const void *c, const void *d) {
  return (attn_tmem_padded(dH) || dH == 128) && op_aligned(a) && op_aligned(b) && op_aligned(c) && op_aligned(d);
}

int attn_fwd_op_tmem(fcu_ctx *ctx, const float *Q, const float *K, const float *V, int B, int T, int nH,
                     int nKV, int dH, float *O, float *lse) {
  const int hw = dH == 128 ? 128 : kD;   // head width of the bf16 layout
  const int64_t rows = (int64_t)B * T, W = (int64_t)(nH + 2 * nKV) * hw, qD = (int64_t)nH * hw,
                kvD = (int64_t)nKV * hw;
  void *buf = nullptr;
  int rc = op_buffer(ctx, (size_t)rows * (W + qD) * sizeof(__nv_bfloat16), &buf);
  if (rc) return rc;
  __nv_bfloat16 *qkv = (__nv_bfloat16 *)buf, *Ob = qkv + rows * W;
  if ((rc = pack(ctx, Q, rows, nH, dH, qkv, W, 0, hw)) || (rc = pack(ctx, K, rows, nKV, dH, qkv, W, (int)qD, hw)) ||
      (rc = pack(ctx, V, rows, nKV, dH, qkv, W, (int)(qD + kvD), hw)))
    return rc;
  rc = attn_fwd_tmem(ctx, qkv, W, B, T, nH, nKV, Ob, lse, dH);
  if (rc) return rc;
  return unpack(ctx, Ob, qD, 0, rows, nH, dH, O, 0, hw);
}

bool attn_tmem_fwd_supported(int dH) { return dH == kD || dH == 128; }

namespace {

// delta, and the head-split dK / dV partials (kv columns padded to 64 per
// head) on small grids, from the context scratch.
int bwd_scratch(fcu_ctx *ctx, int B, int T, int nH, int nKV, int *split, float **delta, float **pk,
                float **pv, int hw = kD) {
  const int64_t ctas = (int64_t)div_up(T, kBM) * nKV * B;
  *split = (nH > nKV && ctas < 4 * (int64_t)ctx->num_sms) ? 1 : 0;
  const size_t delta_bytes = (sizeof(float) * (size_t)B * nH * T + 255) & ~(size_t)255;
  const size_t part_bytes = *split ? sizeof(float) * (size_t)(nH / nKV) * B * T * nKV * hw : 0;
  void *scr = nullptr;
  int rc = ctx_scratch(ctx, delta_bytes + 2 * part_bytes, &scr);
  if (rc) return rc;
  *delta = (float *)scr;
  *pk = *split ? (float *)((uint8_t *)scr + delta_bytes) : nullptr;
  *pv = *split ? (float *)((uint8_t *)scr + delta_bytes + part_bytes) : nullptr;
  return FCU_OK;
}

}  // namespace

int attn_bwd_op_tmem(fcu_ctx *ctx, const float *dO, const float *Q, const float *K, const float *V,
                     const float *O, const float *lse, int B, int T, int nH, int nKV, int dH, float *dQ,
                     float *dK, float *dV, int accumulate) {
  const int hw = dH == 128 ? 128 : kD;   // head width of the bf16 layout
  const int64_t rows = (int64_t)B * T, W = (int64_t)(nH + 2 * nKV) * hw, qD = (int64_t)nH * hw,
                kvD = (int64_t)nKV * hw;
  void *buf = nullptr;
  // qkv and dqkv [rows, W], dO and O [rows, qD], all bf16
  int rc = op_buffer(ctx, (size_t)rows * (2 * W + 2 * qD) * sizeof(__nv_bfloat16), &buf);
  if (rc) return rc;
  __nv_bfloat16 *qkv = (__nv_bfloat16 *)buf, *dqkv = qkv + rows * W, *dOb = dqkv + rows * W,
                *Ob = dOb + rows * qD;
  if ((rc = pack(ctx, Q, rows, nH, dH, qkv, W, 0, hw)) || (rc = pack(ctx, K, rows, nKV, dH, qkv, W, (int)qD, hw)) ||
      (rc = pack(ctx, V, rows, nKV, dH, qkv, W, (int)(qD + kvD), hw)) ||
      (rc = pack(ctx, dO, rows, nH, dH, dOb, qD, 0, hw)) || (rc = pack(ctx, O, rows, nH, dH, Ob, qD, 0, hw)))
    return rc;
  int split = 0;
  float *delta = nullptr, *pk = nullptr, *pv = nullptr;
  if ((rc = bwd_scratch(ctx, B, T, nH, nKV, &split, &delta, &pk, &pv, hw))) return rc;
  rc = attn_bwd_tmem(ctx, dOb, qkv, W, Ob, lse, delta, B, T, nH, nKV, nullptr, dqkv, split, pk, pv, dH);
  if (rc) return rc;
  if ((rc = unpack(ctx, dqkv, W, 0, rows, nH, dH, dQ, accumulate, hw)) ||
      (rc = unpack(ctx, dqkv, W, (int)qD, rows, nKV, dH, dK, accumulate, hw)))
    return rc;
  return unpack(ctx, dqkv, W, (int)(qD + kvD), rows, nKV, dH, dV, accumulate, hw);
}

// The fused path's bf16 entries at head dims below 64: qkv (and dO, O) are
// re-laid out with 64-column heads in the operator buffer, and the results
// copied back to dh-column heads.  RoPE's backward runs inside the kernels
// on a [T][32] table whose pairs past dh/2 are the identity.
int attn_fwd_tmem_padded(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV, int dH,
                         void *O, float *lse) {
  const int64_t rows = (int64_t)B * T, W = (int64_t)(nH + 2 * nKV) * kD, qD = (int64_t)nH * kD;
  void *buf = nullptr;
  int rc = op_buffer(ctx, (size_t)rows * (W + qD) * sizeof(__nv_bfloat16), &buf);
  if (rc) return rc;
  __nv_bfloat16 *qkvp = (__nv_bfloat16 *)buf, *Op = qkvp + rows * W;
  if ((rc = repad(ctx, qkv, ld_qkv, qkvp, W, rows, nH + 2 * nKV, dH, 1))) return rc;
  if ((rc = attn_fwd_tmem(ctx, qkvp, W, B, T, nH, nKV, Op, lse, dH))) return rc;
  return repad(ctx, Op, qD, O, (int64_t)nH * dH, rows, nH, dH, 0);
}

int attn_bwd_tmem_padded(fcu_ctx *ctx, const void *dO, const void *qkv, int64_t ld_qkv, const void *O,
                         const float *lse, int B, int T, int nH, int nKV, int dH, double rope_theta, void *dqkv) {
  const int64_t rows = (int64_t)B * T, W = (int64_t)(nH + 2 * nKV) * kD, qD = (int64_t)nH * kD;
  void *buf = nullptr;
  int rc = op_buffer(ctx, (size_t)rows * (2 * W + 2 * qD) * sizeof(__nv_bfloat16), &buf);
  if (rc) return rc;
  __nv_bfloat16 *qkvp = (__nv_bfloat16 *)buf, *dqkvp = qkvp + rows * W, *dOp = dqkvp + rows * W,
                *Op = dOp + rows * qD;
  const int64_t ldo = (int64_t)nH * dH;
  if ((rc = repad(ctx, qkv, ld_qkv, qkvp, W, rows, nH + 2 * nKV, dH, 1)) ||
      (rc = repad(ctx, dO, ldo, dOp, qD, rows, nH, dH, 1)) || (rc = repad(ctx, O, ldo, Op, qD, rows, nH, dH, 1)))
    return rc;
  const float2 *rope = nullptr;
  if (rope_theta > 0 && (rc = rope_table_f32(ctx, T, dH, rope_theta, &rope, kD / 2))) return rc;
  int split = 0;
  float *delta = nullptr, *pk = nullptr, *pv = nullptr;
  if ((rc = bwd_scratch(ctx, B, T, nH, nKV, &split, &delta, &pk, &pv))) return rc;
  rc = attn_bwd_tmem(ctx, dOp, qkvp, W, Op, lse, delta, B, T, nH, nKV, rope, dqkvp, split, pk, pv, dH);
  if (rc) return rc;
  return repad(ctx, dqkvp, W, dqkv, ld_qkv, rows, nH + 2 * nKV, dH, 0);
}

}  // namespace fcu
