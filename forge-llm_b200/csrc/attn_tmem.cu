// Causal GQA flash attention on the sm_100a tensor cores: tcgen05.mma with
// the score and output accumulators in TMEM, Q/K/V tiles staged by TMA from
// the bf16 [tokens, (nH + 2 nKV) * 64] qkv buffer (RoPE already applied).
//
// Forward, per CTA: one 128-row query tile of one head, looping over the
// 128-key blocks at or before its diagonal.
//   warp 0      TMA: Q once, then a 2-deep ring of (K, V) blocks
//   warp 1      TMEM owner + MMA issuer (one thread):
//                 S_j = Q K_j^T        128x128x64  -> TMEM cols [0, 128)
//                 O  += P_j V_j        128x64x128  -> TMEM cols [128, 192)
//               issued in the order S_0, S_1, PV_0, S_2, PV_1, ... so the next
//               score tile is computed while the softmax works on this one
//   warps 2..5  softmax: thread = query row = TMEM lane.  Reads its S row,
//               applies the causal mask, keeps the running max / sum, writes
//               P = exp2(S*scale*log2e - m) as bf16 into shared memory in the
//               128B-swizzled K-major layout the PV MMA reads, and at the end
//               normalises O and stores it with the log-sum-exp.
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
constexpr uint32_t kTmemCols = 256;            // S [0,128), O [128,192)
constexpr float kRescaleLog2 = 8.f;
constexpr float kLog2e = 1.4426950408889634f;

// Shared memory map (byte offsets; tiles 1024-byte aligned for the swizzle).
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;           // 2 stages
constexpr int kOffV = kOffK + 2 * kTile;       // 2 stages
constexpr int kOffP = kOffV + 2 * kTile;       // 2 halves (keys 0-63, 64-127)
constexpr int kOffBar = kOffP + 2 * kTile;
constexpr int kSmemBytes = kOffBar + 16 * 8 + 16;

struct FwdParams {
  int B, T, nH, nKV, n_qt;
  float scale_log2;          // softmax scale * log2(e)
  __nv_bfloat16 *O;          // [B*T, nH*64]
  float *lse;                // [B][nH][T], natural log
  int *err;
};

__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_tmem_kernel(const __grid_constant__ CUtensorMap tm, FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *sQ = smem + kOffQ, *sK = smem + kOffK, *sV = smem + kOffV, *sP = smem + kOffP;
  uint64_t *bars = (uint64_t *)(smem + kOffBar);
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1, *k_empty = bars + 3;   // [2] each
  uint64_t *v_full = bars + 5, *v_empty = bars + 7;   // [2] each
  uint64_t *s_full = bars + 9, *s_free = bars + 10;
  uint64_t *p_full = bars + 11, *o_done = bars + 12, *mma_done = bars + 13;
  uint32_t *tmem_slot = (uint32_t *)(bars + 14);
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
    for (int s = 0; s < 2; s++) {
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
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (!aligned) {
    // nothing issued; fall through to the dealloc
  } else if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    int nk = 0, nv = 0;
    bool ok = true;
    mbar_expect_tx(q_full, kTile);
    tma_load_2d(sQ, &tm, h * kD, row0 + q0, q_full);
    for (int j = 0; j < nkv; j++) {
      const int s = j & 1;
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
      mbar_expect_tx(&k_full[s], kTile);
      tma_load_2d(sK + s * kTile, &tm, (p.nH + kvh) * kD, row0 + j * kBN, &k_full[s]);
      nk++;
      if (!mbar_wait(&v_empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
      mbar_expect_tx(&v_full[s], kTile);
      tma_load_2d(sV + s * kTile, &tm, (p.nH + p.nKV + kvh) * kD, row0 + j * kBN, &v_full[s]);
      nv++;
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 11);
    }
    // Every copy issued has landed before the CTA exits.
    mbar_wait_drain(q_full, 0);
    for (int i = nk - 2 < 0 ? 0 : nk - 2; i < nk; i++) mbar_wait_drain(&k_full[i & 1], (uint32_t)(i >> 1) & 1u);
    for (int i = nv - 2 < 0 ? 0 : nv - 2; i < nv; i++) mbar_wait_drain(&v_full[i & 1], (uint32_t)(i >> 1) & 1u);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    const uint32_t id_s = instr_desc_bf16(0, 0, kBM, kBN);   // Q, K both K-major
    const uint32_t id_o = instr_desc_bf16(0, 1, kBM, kD);    // P K-major, V MN-major
    bool ok = mbar_wait(q_full, 0, abort_flag);
    const uint32_t aq = smem_u32(sQ), ap = smem_u32(sP);
    for (int j = 0; j <= nkv && ok; j++) {
      if (j < nkv) {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (uint32_t)(j >> 1) & 1u, abort_flag)) { ok = false; break; }
        if (j > 0 && !mbar_wait(s_free, (uint32_t)(j - 1) & 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t bk = smem_u32(sK + s * kTile);
#pragma unroll
        for (int k = 0; k < kD / 16; k++)
          umma_bf16(tS, operand_desc(aq, k, 0, kD), operand_desc(bk, k, 0, kD), id_s, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        umma_commit(&k_empty[s]);
      }
      if (j > 0) {
        const int i = j - 1, s = i & 1;
        if (!mbar_wait(&v_full[s], (uint32_t)(i >> 1) & 1u, abort_flag) ||
            !mbar_wait(p_full, (uint32_t)i & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t bv = smem_u32(sV + s * kTile);
#pragma unroll
        for (int k = 0; k < kBN / 16; k++)
          umma_bf16(tO, operand_desc(ap + (uint32_t)(k >> 2) * kTile, k & 3, 0, kD),
                    operand_desc(bv, k, 1, kBN), id_o, (i > 0 || k > 0) ? 1u : 0u);
        umma_commit(o_done);
        umma_commit(&v_empty[s]);
      }
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 12);
    }
    umma_commit(mma_done);
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
      tmem_ld64(tS + lane_addr, s);
      tmem_ld64(tS + lane_addr + 64, s + 64);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      if (j == nkv - 1) {                       // diagonal block: keys after q are masked
        const int lim = q - j * kBN;
#pragma unroll
        for (int c = 0; c < kBN; c++)
          if (c > lim) s[c] = -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int c = 1; c < kBN; c++) mx = fmaxf(mx, s[c]);
      mx *= p.scale_log2;
      float alpha = 1.f;
      bool rescale_o = false;
      if (mx > m + kRescaleLog2) {
        alpha = exp2f(m - mx);                  // 0 on the first block
        rescale_o = j > 0;
        m = mx;
      }
      const float neg_m = -m;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kBN; c++) {
        const float e = exp2f(fmaf(s[c], p.scale_log2, neg_m));
        s[c] = e;
        rs += e;
      }
      l = l * alpha + rs;
      // PV_{j-1} must be done with P and O before P is overwritten / O rescaled.
      if (j > 0 && !warp_wait(o_done, (uint32_t)(j - 1) & 1u, abort_flag)) { ok = false; break; }
#pragma unroll
      for (int c8 = 0; c8 < kBN / 8; c8++) {
        uint4 v;
        v.x = pack2_bf16(s[8 * c8 + 0], s[8 * c8 + 1]);
        v.y = pack2_bf16(s[8 * c8 + 2], s[8 * c8 + 3]);
        v.z = pack2_bf16(s[8 * c8 + 4], s[8 * c8 + 5]);
        v.w = pack2_bf16(s[8 * c8 + 6], s[8 * c8 + 7]);
        *reinterpret_cast<uint4 *>(sP + (c8 >> 3) * kTile + sw128_offset(r, c8 & 7)) = v;
      }
      if (__any_sync(0xffffffffu, rescale_o)) {   // warp-collective: alpha = 1 on other rows
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; half++) {
          uint32_t o[32];
          tmem_ld32(tO + lane_addr + half * 32, o);
#pragma unroll
          for (int c = 0; c < 32; c++) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(tO + lane_addr + half * 32, o);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && warp_wait(o_done, (uint32_t)(nkv - 1) & 1u, abort_flag)) {
      tc_fence_after();
      float o[kD];
      tmem_ld64(tO + lane_addr, o);
      if (q < p.T) {
        const float inv = 1.f / l;
        uint4 *dst = reinterpret_cast<uint4 *>(p.O + ((int64_t)(row0 + q) * p.nH + h) * kD);
#pragma unroll
        for (int c8 = 0; c8 < kD / 8; c8++) {
          uint4 v;
          v.x = pack2_bf16(o[8 * c8 + 0] * inv, o[8 * c8 + 1] * inv);
          v.y = pack2_bf16(o[8 * c8 + 2] * inv, o[8 * c8 + 3] * inv);
          v.z = pack2_bf16(o[8 * c8 + 4] * inv, o[8 * c8 + 5] * inv);
          v.w = pack2_bf16(o[8 * c8 + 6] * inv, o[8 * c8 + 7] * inv);
          dst[c8] = v;
        }
        p.lse[((int64_t)b * p.nH + h) * p.T + q] = (m + log2f(l)) / kLog2e;
      }
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
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

bool attn_tmem_supported(int dH) { return dH == kD; }

// O [B*T, nH*64] bf16 and lse [B][nH][T] from the bf16 qkv buffer (row stride
// ld_qkv elements: q heads, then k heads, then v heads, 64 columns each).
int attn_fwd_tmem(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV,
                  void *O, float *lse) {
  int rc = tc_get_encode();
  if (rc) return rc;
  int *err = nullptr;
  rc = tc_error_word(ctx, &err);
  if (rc) return rc;
  CUtensorMap map;
  rc = tc_make_map(&map, qkv, (uint64_t)B * T, (uint64_t)(nH + 2 * nKV) * kD, (uint64_t)ld_qkv, 64,
                   kBM);
  if (rc) return rc;
  FwdParams p{};
  p.B = B;
  p.T = T;
  p.nH = nH;
  p.nKV = nKV;
  p.n_qt = div_up(T, kBM);
  p.scale_log2 = (float)(1.0 / sqrt((double)kD)) * kLog2e;
  p.O = (__nv_bfloat16 *)O;
  p.lse = lse;
  p.err = err;
  static bool attr_set[64] = {false};
  if (!attr_set[ctx->device & 63]) {
    FCU_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_tmem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kSmemBytes));
    attr_set[ctx->device & 63] = true;
  }
  const int64_t grid = (int64_t)p.n_qt * nH * B;
  FCU_REQUIRE(grid <= INT32_MAX, "attention: grid too large");
  attn_fwd_tmem_kernel<<<(unsigned)grid, kThreads, kSmemBytes, ctx->stream>>>(map, p);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // namespace fcu
