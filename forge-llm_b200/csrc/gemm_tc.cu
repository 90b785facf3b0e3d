// Tensor-core GEMM for sm_100a: tcgen05.mma with TMEM accumulators, operands
// staged in shared memory by TMA, persistent warp-specialised CTAs.
//
//   C[M,N] (+)= sum_k A(m,k) B(n,k)      (bf16 operands, fp32 accumulate)
//
// A and B are each either K-major (k contiguous: the forward's X and W, the
// dX contraction's dY) or MN-major (m/n contiguous: W in dX = dY.W, both
// operands of dW = dY^T.X).  tcgen05 reads both majors straight from the
// 128-byte-swizzled tiles TMA writes, so no operand is ever transposed.
//
// CTA = 6 warps, one CTA per SM, looping over output tiles:
//   warp 0      TMA producer: STAGES-deep ring of (A,B) k-blocks
//   warp 1      TMEM owner + MMA issuer (warp-wide, elect.sync picks the
//               lane): 4 x (128x256x16) per k-block
//   warps 2..5  epilogue: TMEM -> registers -> global, double-buffered
//               accumulators so the epilogue of tile i overlaps the
//               mainloop of tile i+1 (2 x 256 TMEM columns = all 512).
// Every wait is bounded: on timeout the CTA records an error, drains what it
// issued, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "gemm.cuh"
#include "swiglu_math.cuh"
#include "tc_ptx.cuh"

namespace fcu {
namespace {

constexpr int BM = 128, BK = 64;
constexpr int UMMA_K = 16;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int NUM_THREADS = 192;
// Epilogue staging: per epilogue warp two 32-row x 128-byte boxes (32 fp32
// or 64 bf16 columns), 128B-swizzled, written out by TMA stores.
constexpr int EPI_BOX = 32 * 128;
constexpr int EPI_BYTES = 4 * 2 * EPI_BOX;
constexpr int GROUP_M = 16;                     // tile raster: GROUP_M m-blocks per n sweep

// Output tile width.  128 x 256 is the main tile; 128 x 128 doubles the tile
// count of narrow products that would otherwise leave SMs idle in the last
// wave (few tokens per GPU), at the same operand traffic per FLOP on A.
//
// PAIR: a cluster of two CTAs on two SMs computes one 256 x 256 tile with
// tcgen05 .cta_group::2 MMAs (M = 256).  Each CTA stages its own 128 rows of
// A and half (128 rows) of B, so a k-block costs an SM 32 KB of shared memory
// instead of 48 KB and the ring is 6 deep instead of 4: twice the B traffic
// per FLOP is saved and 50% more MMA time is covered by loads in flight.
// Each CTA's TMEM receives its own 128 rows x 256 columns, which its own
// epilogue warps write out.
template <int BN_, bool PAIR = false>
struct TileCfg {
  static constexpr int BN = BN_;                          // output columns per tile
  static constexpr int BNL = PAIR ? BN_ / 2 : BN_;        // B rows this CTA stages
  static constexpr int STAGES = (PAIR || BN_ != 256) ? 6 : 4;
  static constexpr int B_BYTES = BNL * BK * 2;            // 32 / 16 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // 48 / 32 KB
  static constexpr uint32_t TMEM_COLS = 2 * BN_;          // 512 / 256
  static constexpr size_t SMEM_BYTES =
      1024 /*align slack*/ + (size_t)STAGES * STAGE_BYTES + EPI_BYTES + 256;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// Epilogue modes (what the epilogue warps do with one fp32 accumulator row):
//   kOutF32      C[m,n] = acc            (beta = 1: C += acc)
//   kOutF32Res   C[m,n] = R[m,n] + acc   (residual add fused, R and C fp32)
//   kOutBF16     Cb[m,n] = bf16(acc)
//   kOutBF16Rope Cb[m,n] = bf16(rope(acc)) for n < rope_cols, bf16(acc) after:
//                interleaved pairs (2i, 2i+1) of each head_dim-wide head are
//                rotated by the (cos, sin) of position m % rope_T.
//   kOutSwiGLU   the gate|up projection: a 256-wide tile holds gate units
//                j0..j0+127 in accumulator columns [0,128) and the up units
//                of the same j in [128,256) (B is loaded as those two row
//                blocks); writes g and u to Cb [M, 2H] and silu(g) * u of the
//                bf16-rounded values to act [M, H] (through tmC2).
//   kOutSwiGLUBwd the down projection's input gradient d = bf16(acc) [M, H]
//                turned into dg | du [M, 2H] with the forward's g | u (aux).
enum : int { kOutF32 = 0, kOutF32Res = 1, kOutBF16 = 2, kOutBF16Rope = 3, kOutSwiGLU = 4, kOutSwiGLUBwd = 5 };

struct TcParams {
  int M, N, K;
  float *C;
  int64_t ldc;
  int beta;
  int a_mn, b_mn;
  int tiles_m, tiles_n;
  int row_major;           // tile raster (tile_coords)
  int *err;
  int mode;
  const float *R;          // kOutF32Res (row stride ldc)
  __nv_bfloat16 *Cb;       // kOutBF16* (row stride ldc)
  const float2 *rope;      // [rope_T][head_dim/2] (cos, sin)
  int rope_T, rope_cols, head_dim;
  int splits;              // K slices per output tile (1 = no split)
  float *ws;               // split-K partial tiles [splits][ws_rows][ldc]
  int ws_rows;             // M rounded up to the 128-row tile
  int tma_out;             // 1: epilogue stores through shared memory + TMA (tmC)
  int H;                   // kOutSwiGLU*: hidden units
  const __nv_bfloat16 *aux;  // kOutSwiGLUBwd: g | u [M, 2H]
};

using namespace tc;

// Tile t of the raster.  row_major: n fastest, so the few column tiles that
// share one row block of A run side by side in the same wave and A streams
// from DRAM once (products a few tiles wide: every wave then holds whole
// rows of tiles, and B, re-read by every row, stays in L2).  Otherwise
// groups of GROUP_M row blocks swept m fastest, column by column.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int row_major, int &tm, int &tn) {
  if (row_major) {
    tm = t / tiles_n;
    tn = t - tm * tiles_n;
    return;
  }
  const int per_group = GROUP_M * tiles_n;
  const int g = t / per_group;
  const int first = g * GROUP_M;
  const int gm = min(GROUP_M, tiles_m - first);
  const int r = t - g * per_group;
  tm = first + r % gm;
  tn = r / gm;
}

// Writes columns [nb, nb+32) of output row gm from one TMEM load.
__device__ __forceinline__ void store_chunk(const TcParams &p, int64_t gm, int nb,
                                            const uint32_t (&r)[32]) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
  const bool full = nb + 32 <= p.N;
  if (p.mode == kOutF32 || p.mode == kOutF32Res) {
    float *crow = p.C + gm * p.ldc;
    const float *rrow = p.mode == kOutF32Res ? p.R + gm * p.ldc : nullptr;
    const bool vec = full && ((p.ldc & 3) == 0) && (((uintptr_t)p.C & 15) == 0) &&
                     (rrow == nullptr || ((uintptr_t)p.R & 15) == 0);
    if (vec) {
      float4 *dst = reinterpret_cast<float4 *>(crow + nb);
      const float4 *src = rrow ? reinterpret_cast<const float4 *>(rrow + nb) : nullptr;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        if (src || p.beta) {
          const float4 a = src ? src[i] : dst[i];
          o.x += a.x;
          o.y += a.y;
          o.z += a.z;
          o.w += a.w;
        }
        dst[i] = o;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; i++) {
        if (nb + i < p.N) {
          float o = v[i];
          if (rrow) o += rrow[nb + i];
          else if (p.beta) o += crow[nb + i];
          crow[nb + i] = o;
        }
      }
    }
    return;
  }
  if (p.mode == kOutBF16Rope && nb < p.rope_cols) {
    const int64_t pos = gm % p.rope_T;
    const int half = p.head_dim >> 1;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const int pi = ((nb + 2 * i) % p.head_dim) >> 1;
      const float2 cs = p.rope[pos * half + pi];
      const float a = v[2 * i], b = v[2 * i + 1];
      v[2 * i] = a * cs.x - b * cs.y;
      v[2 * i + 1] = a * cs.y + b * cs.x;
    }
  }
  __nv_bfloat16 *brow = p.Cb + gm * p.ldc;
  if (full && ((p.ldc & 7) == 0) && (((uintptr_t)p.Cb & 15) == 0)) {
    uint4 *dst = reinterpret_cast<uint4 *>(brow + nb);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint4 o;
      o.x = pack2_bf16(v[8 * i], v[8 * i + 1]);
      o.y = pack2_bf16(v[8 * i + 2], v[8 * i + 3]);
      o.z = pack2_bf16(v[8 * i + 4], v[8 * i + 5]);
      o.w = pack2_bf16(v[8 * i + 6], v[8 * i + 7]);
      dst[i] = o;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; i++)
      if (nb + i < p.N) brow[nb + i] = __float2bfloat16_rn(v[i]);
  }
}

// SW selects the epilogue at compile time: 0 the generic modes, 1
// kOutSwiGLU, 2 kOutSwiGLUBwd (each instantiation holds one epilogue, so the
// register allocation of one does not constrain the others).  PAIR: launched
// in clusters of two, one 256-row tile per cluster (see TileCfg); p.tiles_m
// then counts 256-row tiles.
template <int BN_, int SW, bool PAIR = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC,
                        const __grid_constant__ CUtensorMap tmC2, TcParams p) {
  fcu::pdl_trigger();
  using Cfg = TileCfg<BN_, PAIR>;
  constexpr int BN = Cfg::BN;
  constexpr int BNL = Cfg::BNL;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int B_BYTES = Cfg::B_BYTES;
  constexpr int STAGE_BYTES = Cfg::STAGE_BYTES;
  constexpr uint32_t TMEM_COLS = Cfg::TMEM_COLS;
  constexpr int TILE_M = PAIR ? 2 * BM : BM;   // output rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_BYTES;
  uint8_t *sEpi = sB + STAGES * B_BYTES;
  uint64_t *full = (uint64_t *)(sEpi + EPI_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;   // [2]
  uint64_t *tempty = tfull + 2;       // [2]
  uint64_t *mma_done = tempty + 2;    // [1]
  uint32_t *tmem_slot = (uint32_t *)(mma_done + 1);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // PAIR: rank 0 of the cluster issues the MMAs; its full barriers count the
  // bytes both CTAs load and its tempty barriers the epilogue warps of both.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], PAIR ? 8 : 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (PAIR) cluster_sync();   // both CTAs' barriers exist before either signals the other's
  if (warp == 1) {
    if (PAIR) tmem_alloc2(tmem_slot, TMEM_COLS);
    else tmem_alloc(tmem_slot, TMEM_COLS);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();   // the previous kernel's outputs are complete from here on
  // The barriers of the MMA-issuing CTA, as shared::cluster addresses.
  const uint32_t full_cl = PAIR ? mapa_shared(smem_u32(full), 0) : smem_u32(full);
  const uint32_t tempty_cl = PAIR ? mapa_shared(smem_u32(tempty), 0) : smem_u32(tempty);

  // Work units: (output tile, K slice).  With split-K (p.splits > 1) unit u
  // covers k-blocks [kb0, kb1) of slice u / num_tiles of tile u % num_tiles;
  // its partial tile goes to the workspace and a reduction kernel adds the
  // slices in order.  Slice-major order keeps the units in flight on the
  // same K range, so each k-block of both operands is fetched from DRAM
  // about once and reused from L2 by every tile that needs it.
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int nk = (p.K + BK - 1) / BK;
  const int units = num_tiles * p.splits;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    int it = 0;
    bool ok = true;
    // One load into this CTA's stage; PAIR completes it on the MMA CTA's barrier.
    auto load = [&](void *dst, const CUtensorMap *map, int c0, int c1, int s) {
      if (PAIR) tma_load_2d_pair(dst, map, c0, c1, full_cl + 8u * (uint32_t)s);
      else tma_load_2d(dst, map, c0, c1, &full[s]);
    };
    for (int u = unit0; u < units && ok; u += ustep) {
      const int sp = u / num_tiles, t = u - sp * num_tiles;
      const int kb0 = (int)((int64_t)nk * sp / p.splits);
      const int kb1 = (int)((int64_t)nk * (sp + 1) / p.splits);
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, p.row_major, tm, tn);
      // this CTA's A rows and B rows (PAIR: rank 1 takes the second half of each)
      const int m0 = tm * TILE_M + (int)rank * BM, n0 = tn * BN + (int)rank * BNL;
      for (int kb = kb0; kb < kb1; kb++, it++) {
        const int s = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        if (rank == 0) mbar_expect_tx(&full[s], PAIR ? 2 * STAGE_BYTES : STAGE_BYTES);
        uint8_t *a = sA + s * A_BYTES;
        uint8_t *b = sB + s * B_BYTES;
        const int k0 = kb * BK;
        if (!p.a_mn) {
          load(a, &tmA, k0, m0, s);
        } else {
#pragma unroll
          for (int j = 0; j < BM / 64; j++) load(a + j * BK * 128, &tmA, m0 + 64 * j, k0, s);
        }
        if (SW == 1) {
          // gate rows j0.. then up rows H + j0.. of the same 128 hidden units
          // (PAIR: rank 0 stages the gate rows, rank 1 the up rows)
          if (!PAIR || rank == 0) load(b, &tmB, k0, tn * 128, s);
          if (!PAIR || rank == 1) load(PAIR ? b : b + 128 * 128, &tmB, k0, p.H + tn * 128, s);
        } else if (!p.b_mn) {
          load(b, &tmB, k0, n0, s);
        } else {
#pragma unroll
          for (int j = 0; j < BNL / 64; j++) load(b + j * BK * 128, &tmB, n0 + 64 * j, k0, s);
        }
      }
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 1);
    }
    // Drain: every copy this thread issued has landed before the CTA exits.
    // The wait ignores the abort flag (another role may have set it): the
    // copies always complete, and none may still write this CTA's shared
    // memory once it has exited.  PAIR: the full barriers live in rank 0 and
    // count both CTAs' copies, so rank 0 drains for both, and the cluster
    // barrier before exit holds rank 1 until then.
    if (rank == 0)
      for (int i = it - STAGES < 0 ? 0 : it - STAGES; i < it; i++)
        mbar_wait_drain(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u);
  } else if (warp == 1 && PAIR && rank == 1) {
    // The peer's MMAs write this CTA's TMEM: wait for their completion
    // (signalled by rank 0's final commit) before TMEM is freed.
    mbar_wait_drain(mma_done, 0);
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp; elect.sync picks the issuing lane)
    const uint32_t idesc = instr_desc_bf16(p.a_mn, p.b_mn, TILE_M, BN);
    const uint64_t dA0 = p.a_mn ? desc_mn(smem_u32(sA), BK) : desc_k(smem_u32(sA));
    const uint64_t dB0 = p.b_mn ? desc_mn(smem_u32(sB), BK) : desc_k(smem_u32(sB));
    const uint64_t kA = p.a_mn ? kDescMNStep : kDescKStep, kB = p.b_mn ? kDescMNStep : kDescKStep;
    // PAIR: each commit arrives on this CTA's barrier and on the peer's
    // barrier at the same offset (two separate commits, one per CTA).
    auto commit = [&](uint64_t *bar) {
      if (PAIR) {
        umma2_commit_w(smem_u32(bar));
        umma2_commit_w(mapa_shared(smem_u32(bar), 1));
      } else {
        umma_commit_w(bar);
      }
    };
    int it = 0, ti = 0;
    bool ok = true;
    for (int u = unit0; u < units && ok; u += ustep, ti++) {
      const int sp = u / num_tiles;
      const int kb0 = (int)((int64_t)nk * sp / p.splits);
      const int kb1 = (int)((int64_t)nk * (sp + 1) / p.splits);
      const int acc = ti & 1;
      const uint32_t aph = (uint32_t)(ti >> 1) & 1u;
      if (!(PAIR ? warp_wait_cl(&tempty[acc], aph ^ 1u, abort_flag) : warp_wait(&tempty[acc], aph ^ 1u, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
      for (int kb = kb0; kb < kb1; kb++, it++) {
        const int s = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!warp_wait(&full[s], ph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a = dA0 + (uint64_t)s * (A_BYTES >> 4);
        const uint64_t b = dB0 + (uint64_t)s * (B_BYTES >> 4);
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; k++) {
          if (PAIR) umma2_bf16_w(d_tmem, a + k * kA, b + k * kB, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          else umma_bf16_w(d_tmem, a + k * kA, b + k * kB, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
        }
        commit(&empty[s]);  // frees the stage once these MMAs have read it
      }
      if (!ok) break;
      commit(&tfull[acc]);  // accumulator complete
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 2);
    }
    commit(mma_done);
    mbar_wait_drain(mma_done, 0);   // every MMA issued has completed before TMEM is freed
  } else if (warp >= 2) {
    // ---------------- epilogue
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    int ti = 0;
    bool ok = true;
    TcParams part = p;   // split-K: plain fp32 stores of this slice's partial tile
    part.mode = kOutF32;
    part.beta = 0;
    // TMA epilogue: fp32 outputs in 32-column boxes, bf16 in 64-column boxes.
    const bool bf16_out = p.splits == 1 && p.mode >= kOutBF16;
    const int cw = bf16_out ? 64 : 32;
    uint8_t *stg = sEpi + q * 2 * EPI_BOX;
    int seq = 0;                        // boxes this warp has stored (staging buffer = seq & 1)
    // Frees accumulator `acc` for the MMA issuer (PAIR: on rank 0's barrier).
    auto release_acc = [&](int acc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && rank == 1) mbar_arrive_remote(tempty_cl + 8u * (uint32_t)acc);
        else mbar_arrive(&tempty[acc]);
      }
    };
    for (int u = unit0; u < units; u += ustep, ti++) {
      const int sp = u / num_tiles, t = u - sp * num_tiles;
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, p.row_major, tm, tn);
      const int acc = ti & 1;
      const uint32_t aph = (uint32_t)(ti >> 1) & 1u;
      if (!warp_wait(&tfull[acc], aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int mrow0 = tm * TILE_M + (int)rank * BM;   // first output row of this CTA's accumulator
      const int64_t gm = (int64_t)mrow0 + row;
      const int n0 = tn * BN;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      if (SW == 0 && !p.tma_out) {
        if (p.splits > 1) part.C = p.ws + (int64_t)sp * p.ws_rows * p.ldc;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          uint32_t r[32];
          tmem_ld32(tbase + (uint32_t)(c * 32), r);
          if (gm < p.M) store_chunk(p.splits > 1 ? part : p, gm, n0 + c * 32, r);
        }
        release_acc(acc);
        continue;
      }
      const int m_box = mrow0 + q * 32;            // first output row of this warp's boxes
      // One 32-row x 64-column bf16 box of packed words w through the
      // staging buffer to `map` at column x.
      auto emit_bf16 = [&](const uint32_t *w, const CUtensorMap *map, int x) {
        uint8_t *box = stg + (seq & 1) * EPI_BOX;
        if (lane == 0) bulk_wait_read<1>();        // the store that last used this buffer has read it
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; j++)
          *reinterpret_cast<uint4 *>(box + lane * 128 + ((j ^ (lane & 7)) << 4)) =
              make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && m_box < p.M) {
          tma_store_2d(map, box, x, m_box);
          bulk_commit();
        }
        seq++;
      };
      // 64 accumulator columns from col as 32 bf16 pairs.
      auto load_bf16x64 = [&](int col, uint32_t *w) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
          uint32_t r[32];
          tmem_ld32(tbase + (uint32_t)(col + 32 * h), r);
#pragma unroll
          for (int i = 0; i < 16; i++)
            w[16 * h + i] = pack2_bf16(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
        }
      };
      if (SW == 1) {
        const int j0 = tn * 128;
#pragma unroll 1
        for (int c = 0; c < 2; c++) {
          uint32_t gw[32], uw[32];
          load_bf16x64(c * 64, gw);
          load_bf16x64(128 + c * 64, uw);
          if (c == 1) release_acc(acc);            // accumulator no longer needed
          emit_bf16(gw, &tmC, j0 + c * 64);
          emit_bf16(uw, &tmC, p.H + j0 + c * 64);
#pragma unroll
          for (int i = 0; i < 32; i++) gw[i] = swiglu_fwd_pair(gw[i], uw[i]);
          emit_bf16(gw, &tmC2, j0 + c * 64);
        }
        continue;
      }
      if (SW == 2) {
        const int nb = (min(BN, p.N - n0) + 63) / 64;   // p.N = H, a multiple of 64
        // this row's forward g and u for box c (8 x 16 bytes of each), loaded
        // one box ahead so their latency overlaps the previous box's work
        auto load_gu = [&](int c, uint4 (&g4)[8], uint4 (&u4)[8]) {
          if (gm < p.M && c < nb) {
            const uint4 *gp = reinterpret_cast<const uint4 *>(p.aux + gm * 2 * p.H + n0 + c * 64);
            const uint4 *up = reinterpret_cast<const uint4 *>(p.aux + gm * 2 * p.H + p.H + n0 + c * 64);
#pragma unroll
            for (int i = 0; i < 8; i++) {
              g4[i] = __ldg(gp + i);
              u4[i] = __ldg(up + i);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 8; i++) g4[i] = u4[i] = make_uint4(0u, 0u, 0u, 0u);
          }
        };
        uint4 g4[8], u4[8];
        load_gu(0, g4, u4);
#pragma unroll 1
        for (int c = 0; c < nb; c++) {
          const int j = n0 + c * 64;
          uint32_t r0[32], r1[32];
          tmem_ld32_nw(tbase + (uint32_t)(c * 64), r0);
          tmem_ld32_nw(tbase + (uint32_t)(c * 64 + 32), r1);
          uint4 gn[8], un[8];
          load_gu(c + 1, gn, un);
          tmem_wait_ld_r(r0);
          tmem_wait_ld_r(r1);
          if (c == nb - 1) release_acc(acc);       // accumulator no longer needed
          // dg goes through staging buffer 0 and du through buffer 1, both
          // written 32 columns at a time
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
#pragma unroll
          for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const uint4 ga = g4[4 * h + i], ua = u4[4 * h + i];
              const uint32_t gw[4] = {ga.x, ga.y, ga.z, ga.w};
              const uint32_t uw[4] = {ua.x, ua.y, ua.z, ua.w};
              uint32_t og[4], ou[4];
#pragma unroll
              for (int k = 0; k < 4; k++) {
                const uint32_t *r = h ? r1 : r0;
                const uint32_t dw = pack2_bf16(__uint_as_float(r[8 * i + 2 * k]), __uint_as_float(r[8 * i + 2 * k + 1]));
                swiglu_bwd_pair(dw, gw[k], uw[k], og[k], ou[k]);
              }
              const int off = lane * 128 + (((4 * h + i) ^ (lane & 7)) << 4);
              *reinterpret_cast<uint4 *>(stg + off) = make_uint4(og[0], og[1], og[2], og[3]);
              *reinterpret_cast<uint4 *>(stg + EPI_BOX + off) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && m_box < p.M) {
            tma_store_2d(&tmC, stg, j, m_box);
            tma_store_2d(&tmC, stg + EPI_BOX, p.H + j, m_box);
            bulk_commit();
          }
#pragma unroll
          for (int i = 0; i < 8; i++) {
            g4[i] = gn[i];
            u4[i] = un[i];
          }
        }
        if (nb == 0) release_acc(acc);
        continue;
      }
      const int nbox = min(BN, p.N - n0) > 0 ? (min(BN, p.N - n0) + cw - 1) / cw : 0;
      // The accumulator columns of box c are loaded while box c - 1 is
      // converted and stored (r0 | r1: the box after the one in v).
      uint32_t r0[32], r1[32];
      if (nbox > 0) {
        tmem_ld32_nw(tbase, r0);
        if (bf16_out) tmem_ld32_nw(tbase + 32u, r1);
        tmem_wait_ld_r(r0);
        if (bf16_out) tmem_wait_ld_r(r1);
      }
      // RoPE (cos, sin) of this row's position for a box's 32 column pairs
      // (a box's 64 columns lie inside one head: head_dim % 64 == 0).  Every
      // box of the row uses the same 32 pairs when heads are 64 wide, so they
      // are loaded once per tile and again only when a box's pair offset in
      // its head differs from the one held.
      float2 cs[32];
      int cs_at = -1;
#pragma unroll 1
      for (int c = 0; c < nbox; c++) {
        const int n = n0 + c * cw;
        const bool rope_box = bf16_out && p.mode == kOutBF16Rope && n < p.rope_cols && gm < p.M;
        const int cs_off = rope_box ? (n % p.head_dim) / 2 : -1;
        if (rope_box && cs_off != cs_at) {
          const int half = p.head_dim >> 1;
          const float4 *cs4 = reinterpret_cast<const float4 *>(p.rope + (gm % p.rope_T) * half + cs_off);
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const float4 t = cs4[i];
            cs[2 * i] = make_float2(t.x, t.y);
            cs[2 * i + 1] = make_float2(t.z, t.w);
          }
          cs_at = cs_off;
        }
        float v[64];
#pragma unroll
        for (int i = 0; i < 32; i++) {
          v[i] = __uint_as_float(r0[i]);
          v[32 + i] = bf16_out ? __uint_as_float(r1[i]) : 0.f;
        }
        const bool more = c + 1 < nbox;
        if (more) {
          tmem_ld32_nw(tbase + (uint32_t)((c + 1) * cw), r0);
          if (bf16_out) tmem_ld32_nw(tbase + (uint32_t)((c + 1) * cw + 32), r1);
        } else {
          release_acc(acc);                        // every column of the accumulator is loaded
        }
        uint8_t *box = stg + (seq & 1) * EPI_BOX;
        if (lane == 0) bulk_wait_read<1>();        // the store that last used this buffer has read it
        __syncwarp();
        if (!bf16_out) {
#pragma unroll
          for (int j = 0; j < 8; j++)
            *reinterpret_cast<float4 *>(box + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
          if (rope_box) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
              const float a = v[2 * i], b = v[2 * i + 1];
              v[2 * i] = a * cs[i].x - b * cs[i].y;
              v[2 * i + 1] = a * cs[i].y + b * cs[i].x;
            }
          }
#pragma unroll
          for (int j = 0; j < 8; j++)
            *reinterpret_cast<uint4 *>(box + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_uint4(pack2_bf16(v[8 * j], v[8 * j + 1]), pack2_bf16(v[8 * j + 2], v[8 * j + 3]),
                           pack2_bf16(v[8 * j + 4], v[8 * j + 5]), pack2_bf16(v[8 * j + 6], v[8 * j + 7]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && m_box < p.M) {
          const int y = p.splits > 1 ? sp * p.ws_rows + m_box : m_box;
          if (p.splits == 1 && p.beta) tma_reduce_add_2d(&tmC, box, n, y);
          else tma_store_2d(&tmC, box, n, y);
          bulk_commit();
        }
        seq++;
        if (more) {
          tmem_wait_ld_r(r0);
          if (bf16_out) tmem_wait_ld_r(r1);
        }
      }
      if (nbox == 0) release_acc(acc);
    }
    if (lane == 0) bulk_wait_all();
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.err, 3);
    }
  }
  tc_fence_before();
  __syncwarp();
  // PAIR: neither CTA exits (or frees TMEM) while the other may still signal
  // its barriers, read its shared memory or write its TMEM.
  if (PAIR) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    if (PAIR) tmem_dealloc2(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ fp32 -> bf16
__global__ void to_bf16_kernel(const float *__restrict__ x, int64_t n, __nv_bfloat16 *__restrict__ y) {
  fcu::pdl_trigger();
  const int64_t n4 = n >> 2;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = x4[i];
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t *>(&a);
    o.y = *reinterpret_cast<uint32_t *>(&b);
    reinterpret_cast<uint2 *>(y)[i] = o;
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

int tc_get_encode() {
  if (g_encode) return FCU_OK;
  cudaDriverEntryPointQueryResult q;
  void *fn = nullptr;
  FCU_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess || !fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return FCU_ERR_UNSUPPORTED;
  }
  g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  return FCU_OK;
}

static int make_map_dt(CUtensorMap *map, CUtensorMapDataType dt, int esize, const void *base,
                       uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_cols,
                       uint32_t box_rows) {
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride * (uint64_t)esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu stride=%llu box=%ux%u", (int)r,
              (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)row_stride,
              box_cols, box_rows);
    return FCU_ERR_CUDA;
  }
  return FCU_OK;
}

int tc_make_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                uint64_t row_stride, uint32_t box_cols, uint32_t box_rows) {
  return make_map_dt(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, cols, row_stride, box_cols,
                     box_rows);
}

int tc_make_map_f32(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                    uint64_t row_stride, uint32_t box_cols, uint32_t box_rows) {
  return make_map_dt(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, rows, cols, row_stride, box_cols,
                     box_rows);
}

namespace {

struct Workspace {
  void *ptr = nullptr;
  size_t bytes = 0;
  int *err = nullptr;
};

// Per-context bf16 operand workspace (grown on demand, never shrunk).
int workspace(fcu_ctx *ctx, size_t bytes, void **out, int **err) {
  static thread_local Workspace *ws_by_dev[64] = {nullptr};
  Workspace *&ws = ws_by_dev[ctx->device & 63];
  if (!ws) ws = new Workspace();
  if (!ws->err) {
    FCU_CHECK_CUDA(cudaMalloc(&ws->err, sizeof(int)));
    FCU_CHECK_CUDA(cudaMemsetAsync(ws->err, 0, sizeof(int), ctx->stream));
  }
  if (bytes > ws->bytes) {
    if (ws->ptr) {
      FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
      FCU_CHECK_CUDA(cudaFree(ws->ptr));
      ws->ptr = nullptr;
      ws->bytes = 0;
    }
    FCU_CHECK_CUDA(cudaMalloc(&ws->ptr, bytes));
    ws->bytes = bytes;
  }
  *out = ws->ptr;
  *err = ws->err;
  return FCU_OK;
}

// Split-K partial tiles (grown on demand, never shrunk).
int partials(fcu_ctx *ctx, size_t bytes, void **out) {
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

// Split-K epilogue: out = mode(sum over slices s = 0..splits-1 of ws[s]),
// summed in slice order (deterministic), for every output mode of the GEMM
// epilogue.  One thread per pair of adjacent columns (RoPE rotates pairs).
__global__ void splitk_reduce_kernel(TcParams p) {
  fcu::pdl_trigger();
  const int64_t hp = (p.N + 1) / 2;  // column pairs per row
  const int64_t pairs = (int64_t)p.M * hp, mn = (int64_t)p.ws_rows * p.ldc;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < pairs; e += stride) {
    const int64_t row = e / hp;
    const int c = (int)(e - row * hp) * 2;
    const bool two = c + 1 < p.N;
    const int64_t o = row * p.ldc + c;
    float s0 = 0.f, s1 = 0.f;
    for (int k = 0; k < p.splits; k++) {
      s0 += p.ws[(int64_t)k * mn + o];
      if (two) s1 += p.ws[(int64_t)k * mn + o + 1];
    }
    if (p.mode == kOutF32 || p.mode == kOutF32Res) {
      const float *add = p.mode == kOutF32Res ? p.R : (p.beta ? p.C : nullptr);
      if (add) {
        s0 += add[o];
        if (two) s1 += add[o + 1];
      }
      p.C[o] = s0;
      if (two) p.C[o + 1] = s1;
    } else {
      if (p.mode == kOutBF16Rope && c < p.rope_cols && two) {
        const float2 cs = p.rope[(row % p.rope_T) * (p.head_dim >> 1) + ((c % p.head_dim) >> 1)];
        const float a = s0, b = s1;
        s0 = a * cs.x - b * cs.y;
        s1 = a * cs.y + b * cs.x;
      }
      p.Cb[o] = __float2bfloat16_rn(s0);
      if (two) p.Cb[o + 1] = __float2bfloat16_rn(s1);
    }
  }
}

// The same with four adjacent columns per thread (16-byte loads of every
// slice, one 16- or 8-byte store), for N % 4 == 0 and 16-byte aligned outputs.
__global__ void splitk_reduce4_kernel(TcParams p) {
  fcu::pdl_trigger();
  const int64_t q4 = p.N / 4;                   // column quads per row
  const int64_t quads = (int64_t)p.M * q4, mn = (int64_t)p.ws_rows * p.ldc;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < quads; e += stride) {
    const int64_t row = e / q4;
    const int c = (int)(e - row * q4) * 4;
    const int64_t o = row * p.ldc + c;
    float4 a = *reinterpret_cast<const float4 *>(p.ws + o);
    for (int k = 1; k < p.splits; k++) {
      const float4 b = *reinterpret_cast<const float4 *>(p.ws + (int64_t)k * mn + o);
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    if (p.mode == kOutF32 || p.mode == kOutF32Res) {
      const float *add = p.mode == kOutF32Res ? p.R : (p.beta ? p.C : nullptr);
      if (add) {
        const float4 b = *reinterpret_cast<const float4 *>(add + o);
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      *reinterpret_cast<float4 *>(p.C + o) = a;
    } else {
      if (p.mode == kOutBF16Rope && c < p.rope_cols) {
        const float2 *cs = p.rope + (row % p.rope_T) * (p.head_dim >> 1) + ((c % p.head_dim) >> 1);
        const float x0 = a.x, y0 = a.y, x1 = a.z, y1 = a.w;
        a.x = x0 * cs[0].x - y0 * cs[0].y;
        a.y = x0 * cs[0].y + y0 * cs[0].x;
        a.z = x1 * cs[1].x - y1 * cs[1].y;
        a.w = x1 * cs[1].y + y1 * cs[1].x;
      }
      *reinterpret_cast<uint2 *>(p.Cb + o) = make_uint2(pack2_bf16(a.x, a.y), pack2_bf16(a.z, a.w));
    }
  }
}

int convert(fcu_ctx *ctx, const float *x, int64_t n, __nv_bfloat16 *y) {
  FCU_REQUIRE(((uintptr_t)x & 15) == 0, "tensor-core path: fp32 operand must be 16-byte aligned");
  int64_t work = (n >> 2) > 0 ? (n >> 2) : 1;
  int blocks = (int)((work + 255) / 256);
  if (blocks > 16 * ctx->num_sms) blocks = 16 * ctx->num_sms;
  to_bf16_kernel<<<blocks, 256, 0, ctx->stream>>>(x, n, y);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

bool gemm_tc_supported(GemmOp op, int64_t M, int64_t N, int64_t K) {
  // TMA needs 16-byte row strides: every row length of a bf16 operand a
  // multiple of 8 elements.
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return false;
  switch (op) {
    case GemmOp::kFwd: return K % 8 == 0;                  // A[M,K], B[N,K]
    case GemmOp::kDx: return K % 8 == 0 && N % 8 == 0;     // A[M,K], B[K,N]
    case GemmOp::kDw: return M % 8 == 0 && N % 8 == 0;     // A[K,M], B[K,N]
  }
  return false;
}

struct TcOut {
  int mode = kOutF32;
  float *C = nullptr;
  int beta = 0;
  const float *R = nullptr;
  __nv_bfloat16 *Cb = nullptr;
  const float2 *rope = nullptr;
  int rope_T = 1, rope_cols = 0, head_dim = 2;
  __nv_bfloat16 *Cb2 = nullptr;       // kOutSwiGLU: act [M, H]
  const __nv_bfloat16 *aux = nullptr; // kOutSwiGLUBwd: g | u [M, 2H]
};

namespace {

// FORGECU_GEMM_PAIR=0 keeps every product on single-CTA tiles; =1 takes the
// CTA-pair tile wherever the shape allows it; unset, the pair tile runs the
// products with at least two waves of 256 x 256 tiles and no split-K.
int pair_setting() {
  const char *e = getenv("FORGECU_GEMM_PAIR");
  return (e && (e[0] == '0' || e[0] == '1')) ? e[0] - '0' : -1;
}

// Clusters of two GEMM CTAs that fit on the device at once (every pair
// instantiation has the same block and shared-memory size); 0 when none fits.
int pair_slots(fcu_ctx *ctx, int *out) {
  static int slots = -1;
  if (slots < 0) {
    auto kern = gemm_bf16_tc_kernel<256, 0, true>;
    FCU_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)TileCfg<256, true>::SMEM_BYTES));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (ctx->num_sms / 2));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = TileCfg<256, true>::SMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    FCU_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    slots = n > 0 ? n : 0;
  }
  *out = slots;
  return FCU_OK;
}

// K slices for a product of `tiles` output tiles (of M x N outputs in all)
// and nk k-blocks on `slots` concurrent units, from a cost model in units of
// one k-block on every slot: units are dealt round-robin to the persistent
// CTAs, so a split into sp slices costs ceil(tiles * sp / slots) waves of
// ceil(nk / sp) k-blocks plus a fixed per-unit overhead (pipeline fill and
// the partial tile's epilogue, about 4 k-blocks), and each slice adds its
// partial tile's write and read-back (8 bytes per output at the copy
// bandwidth; a k-block wave takes about 0.45 us, as measured on the batch-8
// weight gradients).  1 = no split; at most 16 slices of at least 16
// k-blocks each.
int choose_splits(int64_t tiles, int nk, int64_t slots, int64_t outputs) {
  constexpr double kUnitOverhead = 4.0;
  const double reduce_per_slice = (double)outputs * 8.0 / 6.0e12 / 0.45e-6;
  const int hi = nk / 16 < 16 ? nk / 16 : 16;
  int best = 1;
  double best_t = (double)((tiles + slots - 1) / slots) * (nk + kUnitOverhead);
  for (int sp = 2; sp <= hi; sp++) {
    const double t = (double)((tiles * sp + slots - 1) / slots) * ((nk + sp - 1) / sp + kUnitOverhead) +
                     sp * reduce_per_slice;
    if (t < best_t) {
      best = sp;
      best_t = t;
    }
  }
  return best;
}

}  // namespace

// How one product runs: the tile (CTA pair or single CTA, width bn), the K
// slices and the raster.  A pure function of the shape, the output mode and
// the device (num_sms SMs; slots_pair CTA pairs fit at once, 0: none), so
// the host can state the plan without a GPU (fcu_gemm_plan).  setting is
// FORGECU_GEMM_PAIR (-1 unset, 0 never, 1 wherever the shape allows).
//   Tile: the CTA pair (256 x 256 over two SMs) whenever the product has at
//   least two waves of pair tiles, or a contraction long enough to split;
//   otherwise single-CTA 128 x 256 tiles, or 128 x 128 where those would
//   leave SMs idle in the last wave.
//   Split-K when a product has too few output tiles to fill the GPU twice
//   over and a long contraction (the weight gradients, whose contraction
//   runs over every token; the LM-head input gradient): choose_splits.
//   Raster n-fastest when a wave holds at least two whole rows of tiles.
struct GemmPlan {
  bool pair;          // CTA-pair tile (256 x 256 over two SMs)
  int bn;             // output columns per tile
  int splits;         // K slices (1: none)
  bool row_major;     // n-fastest raster
  int tiles_m, tiles_n;
};

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int mode, int num_sms, int slots_pair, int setting) {
  GemmPlan g;
  const int nk = (int)((K + BK - 1) / BK);
  const bool swiglu = mode == kOutSwiGLU || mode == kOutSwiGLUBwd;
  const int64_t tiles256 = ((M + BM - 1) / BM) * ((N + 255) / 256);
  const int64_t tiles_pair = ((M + 255) / 256) * ((N + 255) / 256);
  g.pair = slots_pair > 0 && M > BM && setting != 0 &&
           (setting == 1 || tiles_pair >= num_sms || (!swiglu && nk >= 32));
  const int slots = g.pair ? slots_pair : num_sms;   // concurrent work units
  const int64_t tiles = g.pair ? tiles_pair : tiles256;
  g.splits = 1;
  if (!swiglu && tiles < 2 * slots && nk >= 32) g.splits = choose_splits(tiles, nk, slots, M * N);
  // (the SwiGLU forward pairs gate and up halves in one 256-wide tile)
  g.bn = (!g.pair && mode != kOutSwiGLU && g.splits == 1 && tiles256 < 2 * num_sms && N > 128) ? 128 : 256;
  const int tile_m = g.pair ? 2 * BM : BM;
  g.tiles_m = (int)((M + tile_m - 1) / tile_m);
  g.tiles_n = mode == kOutSwiGLU ? (int)(N / 256) : (int)((N + g.bn - 1) / g.bn);
  g.row_major = 2 * g.tiles_n <= slots;
  return g;
}

namespace {

// Launches one instantiation (its shared-memory opt-in set on first use).
// PAIR instantiations launch in clusters of two CTAs; `units` caps the grid
// at one cluster (PAIR) or CTA per work unit.
template <int BN_, int SW, bool PAIR>
int launch_tc(fcu_ctx *ctx, int units, const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tc,
              const CUtensorMap &tc2, const TcParams &p) {
  using Cfg = TileCfg<BN_, PAIR>;
  auto kern = gemm_bf16_tc_kernel<BN_, SW, PAIR>;
  static bool attr_set = false;
  int max_clusters = 0;
  if (PAIR) {
    const int rc = pair_slots(ctx, &max_clusters);
    if (rc) return rc;
    if (max_clusters < 1) {
      set_error("no CTA pair of the tensor-core GEMM fits on this device");
      return FCU_ERR_UNSUPPORTED;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = ctx->stream;
  cfg.attrs = attr;
  int na = 0;
  if (PAIR) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 2;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  if (!attr_set) {
    FCU_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM_BYTES));
    attr_set = true;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.numAttrs = na;
  const int cap = PAIR ? max_clusters : ctx->num_sms;
  const int n = units < cap ? units : cap;
  cfg.gridDim = dim3(PAIR ? 2 * n : n);
  FCU_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, tc2, p));
  return FCU_OK;
}

}  // namespace

// out[M,N] = A . B in the layouts of `op` (bf16 operands), written as `o` says.
int gemm_bf16_tc(fcu_ctx *ctx, GemmOp op, const __nv_bfloat16 *A, const __nv_bfloat16 *B,
                 int64_t M, int64_t N, int64_t K, const TcOut &o, int *err) {
  int rc = tc_get_encode();
  if (rc) return rc;
  int slots_pair = 0;
  if (pair_setting() != 0 && (rc = pair_slots(ctx, &slots_pair))) return rc;
  const GemmPlan plan = plan_gemm(M, N, K, o.mode, ctx->num_sms, slots_pair, pair_setting());
  const bool pair = plan.pair;
  const int splits = plan.splits, bn = plan.bn;
  const bool swiglu = o.mode == kOutSwiGLU || o.mode == kOutSwiGLUBwd;
  const uint32_t b_rows = pair ? 128u : (uint32_t)bn;   // B rows one CTA stages
  CUtensorMap ta, tb;
  int a_mn = 0, b_mn = 0;
  switch (op) {
    case GemmOp::kFwd:
      rc = tc_make_map(&ta, A, M, K, K, 64, BM);
      if (!rc) rc = tc_make_map(&tb, B, N, K, K, 64, o.mode == kOutSwiGLU ? 128u : b_rows);
      break;
    case GemmOp::kDx:
      b_mn = 1;
      rc = tc_make_map(&ta, A, M, K, K, 64, BM);
      if (!rc) rc = tc_make_map(&tb, B, K, N, N, 64, BK);
      break;
    case GemmOp::kDw:
      a_mn = b_mn = 1;
      rc = tc_make_map(&ta, A, K, M, M, 64, BK);
      if (!rc) rc = tc_make_map(&tb, B, K, N, N, 64, BK);
      break;
  }
  if (rc) return rc;
  TcParams p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.C = o.C;
  p.ldc = N;
  p.beta = o.beta;
  p.mode = o.mode;
  p.R = o.R;
  p.Cb = o.Cb;
  p.rope = o.rope;
  p.rope_T = o.rope_T;
  p.rope_cols = o.rope_cols;
  p.head_dim = o.head_dim;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  const int tile_m = pair ? 2 * BM : BM;
  p.tiles_m = plan.tiles_m;
  p.tiles_n = plan.tiles_n;
  p.H = o.mode == kOutSwiGLU ? (int)(N / 2) : (int)N;
  p.aux = o.aux;
  p.err = err;
  p.splits = splits;
  p.ws = nullptr;
  p.ws_rows = p.tiles_m * tile_m;
  if (splits > 1) {
    void *w = nullptr;
    rc = partials(ctx, sizeof(float) * (size_t)splits * (size_t)p.ws_rows * (size_t)N, &w);
    if (rc) return rc;
    p.ws = (float *)w;
  }
  // TMA epilogue: needs 16-byte aligned output rows; the fp32 + residual
  // epilogue keeps the direct stores.
  CUtensorMap tc, tc2;
  memset(&tc, 0, sizeof(tc));
  memset(&tc2, 0, sizeof(tc2));
  p.tma_out = 0;
  if (swiglu) {
    // g | u (or dg | du) [M, 2H] and, forward, act [M, H]: 64-column boxes
    const uint64_t H = (uint64_t)p.H;
    rc = tc_make_map(&tc, o.Cb, M, 2 * H, 2 * H, 64, 32);
    if (!rc && o.mode == kOutSwiGLU) rc = tc_make_map(&tc2, o.Cb2, M, H, H, 64, 32);
    if (rc) return rc;
    p.tma_out = 1;
  } else if (splits > 1) {
    if (N % 4 == 0) {
      rc = tc_make_map_f32(&tc, p.ws, (uint64_t)splits * p.ws_rows, N, N, 32, 32);
      if (rc) return rc;
      p.tma_out = 1;
    }
  } else if (o.mode == kOutF32) {
    if (N % 4 == 0 && ((uintptr_t)o.C & 15) == 0) {
      rc = tc_make_map_f32(&tc, o.C, M, N, N, 32, 32);
      if (rc) return rc;
      p.tma_out = 1;
    }
  } else if (o.mode == kOutBF16 || o.mode == kOutBF16Rope) {
    if (N % 8 == 0 && ((uintptr_t)o.Cb & 15) == 0 && (o.mode == kOutBF16 || o.head_dim % 64 == 0)) {
      rc = tc_make_map(&tc, o.Cb, M, N, N, 64, 32);
      if (rc) return rc;
      p.tma_out = 1;
    }
  }
  p.row_major = plan.row_major;
  const int units = p.tiles_m * p.tiles_n * p.splits;
  const int sw = o.mode == kOutSwiGLU ? 1 : o.mode == kOutSwiGLUBwd ? 2 : 0;
  if (pair) {
    rc = sw == 1 ? launch_tc<256, 1, true>(ctx, units, ta, tb, tc, tc2, p)
       : sw == 2 ? launch_tc<256, 2, true>(ctx, units, ta, tb, tc, tc2, p)
                 : launch_tc<256, 0, true>(ctx, units, ta, tb, tc, tc2, p);
  } else if (bn == 256) {
    rc = sw == 1 ? launch_tc<256, 1, false>(ctx, units, ta, tb, tc, tc2, p)
       : sw == 2 ? launch_tc<256, 2, false>(ctx, units, ta, tb, tc, tc2, p)
                 : launch_tc<256, 0, false>(ctx, units, ta, tb, tc, tc2, p);
  } else {
    rc = sw == 2 ? launch_tc<128, 2, false>(ctx, units, ta, tb, tc, tc2, p)
                 : launch_tc<128, 0, false>(ctx, units, ta, tb, tc, tc2, p);
  }
  if (rc) return rc;
  FCU_CHECK_LAUNCH();
  if (p.splits > 1) {
    const bool vec = N % 4 == 0 && (((uintptr_t)p.C | (uintptr_t)p.R | (uintptr_t)p.ws) & 15) == 0 &&
                     ((uintptr_t)p.Cb & 7) == 0 && (p.mode != kOutBF16Rope || p.head_dim % 4 == 0);
    const int64_t work = vec ? M * (N / 4) : M * ((N + 1) / 2);
    int blocks = (int)((work + 255) / 256);
    if (blocks > 16 * ctx->num_sms) blocks = 16 * ctx->num_sms;
    if (blocks < 1) blocks = 1;
    if (vec)
      splitk_reduce4_kernel<<<blocks, 256, 0, ctx->stream>>>(p);
    else
      splitk_reduce_kernel<<<blocks, 256, 0, ctx->stream>>>(p);
    FCU_CHECK_LAUNCH();
  }
  return FCU_OK;
}

int gemm_tc(fcu_ctx *ctx, GemmOp op, const float *A, const float *B, float *C, int64_t M, int64_t N,
            int64_t K, int beta) {
  if (ctx->precision != FCU_PREC_BF16) {
    set_error("precision mode %d has no tensor-core kernel in this build", ctx->precision);
    return FCU_ERR_UNSUPPORTED;
  }
  if (!gemm_tc_supported(op, M, N, K) || ((uintptr_t)A & 15) || ((uintptr_t)B & 15))
    return gemm_simt(ctx->stream, op, A, B, C, M, N, K, beta);
  // Element counts of the two operands in this op's layout.
  const int64_t na = (op == GemmOp::kDw) ? K * M : M * K;
  const int64_t nb = (op == GemmOp::kFwd) ? N * K : K * N;
  const size_t off_b = round_up((size_t)na * 2, 1024);
  void *ws = nullptr;
  int *err = nullptr;
  int rc = workspace(ctx, off_b + round_up((size_t)nb * 2, 1024), &ws, &err);
  if (rc) return rc;
  __nv_bfloat16 *Ab = (__nv_bfloat16 *)ws;
  __nv_bfloat16 *Bb = (__nv_bfloat16 *)((uint8_t *)ws + off_b);
  rc = convert(ctx, A, na, Ab);
  if (!rc) rc = convert(ctx, B, nb, Bb);
  TcOut o;
  o.C = C;
  o.beta = beta;
  if (!rc) rc = gemm_bf16_tc(ctx, op, Ab, Bb, M, N, K, o, err);
  return rc;
}

// ---------------------------------------------------------------- fp32 on the tensor cores
// FCU_PREC_FP32_TC: every fp32 operand x is split into three bf16 parts,
// x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1) (each difference is
// exact in fp32), and the product is the sum of the six part products
// a_i b_j with i + j <= 2, laid out as one bf16 contraction six times as
// long: A' = [a0 a0 a0 a1 a1 a2], B' = [b0 b1 b2 b0 b1 b0] along K.  The
// dropped terms are about 2^-24 of |a b|, so the result carries fp32-level
// error (the products are exact and accumulate in fp32, as the tcgen05 GEMM
// does for bf16).  Every matmulT contraction runs as the forward form
// C[M,N] = A'[M,6K'] . B'[N,6K']^T: the split kernel reads its operand
// transposed where the op needs it and pads K to a multiple of 8 with zeros,
// so any shape runs on the tensor cores.  The contraction runs in chunks of
// 128 (C accumulates in fp32 between them).
namespace {

constexpr int kSplitTile = 32;
constexpr uint32_t kPatA = 0u | 0u << 2 | 0u << 4 | 1u << 6 | 1u << 8 | 2u << 10;   // a0 a0 a0 a1 a1 a2
constexpr uint32_t kPatB = 0u | 1u << 2 | 2u << 4 | 0u << 6 | 1u << 8 | 0u << 10;   // b0 b1 b2 b0 b1 b0

// S[r, c] = src[r * rs + c * cs], r < R, c < L.  dst [R, 6 * Lp] bf16 with
// dst[r, j * Lp + c] = part pat_j of S[r, c] (zero for L <= c < Lp).
__global__ void __launch_bounds__(256) split6_kernel(const float *__restrict__ src, int64_t R, int64_t L,
                                                     int64_t rs, int64_t cs, int64_t Lp, uint32_t pat,
                                                     __nv_bfloat16 *__restrict__ dst) {
  fcu::pdl_trigger();
  __shared__ float tile[kSplitTile][kSplitTile + 1];
  const int tx = threadIdx.x, ty = threadIdx.y;   // 32 x 8
  const int64_t r0 = (int64_t)blockIdx.y * kSplitTile, c0 = (int64_t)blockIdx.x * kSplitTile;
  if (cs == 1) {   // rows contiguous: read along c
    for (int i = ty; i < kSplitTile; i += 8) {
      const int64_t r = r0 + i, c = c0 + tx;
      tile[i][tx] = (r < R && c < L) ? src[r * rs + c] : 0.f;
    }
  } else {         // transposed read: consecutive threads walk r
    for (int i = ty; i < kSplitTile; i += 8) {
      const int64_t r = r0 + tx, c = c0 + i;
      tile[tx][i] = (r < R && c < L) ? src[r * rs + c * cs] : 0.f;
    }
  }
  __syncthreads();
  for (int i = ty; i < kSplitTile; i += 8) {
    const int64_t r = r0 + i, c = c0 + tx;
    if (r >= R || c >= Lp) continue;
    const float x = tile[i][tx];
    const __nv_bfloat16 p0 = __float2bfloat16_rn(x);
    const float e1 = x - __bfloat162float(p0);
    const __nv_bfloat16 p1 = __float2bfloat16_rn(e1);
    const __nv_bfloat16 p2 = __float2bfloat16_rn(e1 - __bfloat162float(p1));
    const __nv_bfloat16 parts[3] = {p0, p1, p2};
    __nv_bfloat16 *row = dst + r * 6 * Lp + c;
#pragma unroll
    for (int j = 0; j < 6; j++) row[j * Lp] = parts[(pat >> (2 * j)) & 3];
  }
}

int split6(fcu_ctx *ctx, const float *src, int64_t R, int64_t L, int64_t rs, int64_t cs, int64_t Lp, uint32_t pat,
           __nv_bfloat16 *dst) {
  dim3 grid((unsigned)((Lp + kSplitTile - 1) / kSplitTile), (unsigned)((R + kSplitTile - 1) / kSplitTile));
  FCU_REQUIRE(grid.y <= 65535, "fp32 tensor-core split: %lld rows", (long long)R);
  split6_kernel<<<grid, dim3(32, 8), 0, ctx->stream>>>(src, R, L, rs, cs, Lp, pat, dst);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // namespace

int gemm_split6(fcu_ctx *ctx, GemmOp op, const float *A, const float *B, float *C, int64_t M, int64_t N,
                int64_t K, int beta) {
  // Strides of the two operands as S_a[m, k] and S_b[n, k] (contraction k).
  int64_t ars, acs, brs, bcs;
  switch (op) {
    case GemmOp::kFwd: ars = K, acs = 1, brs = K, bcs = 1; break;   // A[M,K], B[N,K]
    case GemmOp::kDx: ars = K, acs = 1, brs = 1, bcs = N; break;    // A[M,K], B[K,N]
    default: ars = 1, acs = M, brs = 1, bcs = N; break;             // A[K,M], B[K,N]
  }
  // Contraction chunks of kTcChunk: the tensor cores accumulate at most
  // 6 x kTcChunk products per output (their fp32 accumulation does not round
  // each addition to nearest, so its error grows with the number of terms:
  // relL2 2e-5 against double over a 12,288-term contraction), and the chunks
  // are added into C by the GEMM epilogue in IEEE fp32.
  constexpr int64_t kTcChunk = 128;
  const int64_t chunk = K < kTcChunk ? K : kTcChunk;
  const int64_t Lp_max = (chunk + 7) / 8 * 8;
  const size_t bytes_a = round_up((size_t)M * 6 * Lp_max * 2, 1024);
  void *ws = nullptr;
  int *err = nullptr;
  int rc = workspace(ctx, bytes_a + round_up((size_t)N * 6 * Lp_max * 2, 1024), &ws, &err);
  if (rc) return rc;
  __nv_bfloat16 *Ab = (__nv_bfloat16 *)ws, *Bb = (__nv_bfloat16 *)((uint8_t *)ws + bytes_a);
  for (int64_t k0 = 0; k0 < K; k0 += chunk) {
    const int64_t L = K - k0 < chunk ? K - k0 : chunk, Lp = (L + 7) / 8 * 8;
    rc = split6(ctx, A + k0 * acs, M, L, ars, acs, Lp, kPatA, Ab);
    if (!rc) rc = split6(ctx, B + k0 * bcs, N, L, brs, bcs, Lp, kPatB, Bb);
    if (rc) return rc;
    TcOut o;
    o.C = C;
    o.beta = (beta || k0 > 0) ? 1 : 0;
    rc = gemm_bf16_tc(ctx, GemmOp::kFwd, Ab, Bb, M, N, 6 * Lp, o, err);
    if (rc) return rc;
  }
  return FCU_OK;
}

// (cos, sin) table [T][width] in fp32 for the RoPE epilogues, rounded once
// from the double angles of ropeRows (src/L2/tensor.js:141-143); entries past
// head_dim/2 (a table for heads carried 64 columns wide) are the identity.
__global__ void rope_table_f32_kernel(float2 *tab, int T, int width, int head_dim, double theta) {
  fcu::pdl_trigger();
  const int half = head_dim / 2;
  const int64_t n = (int64_t)T * width;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = e / width, i = e % width;
    if (i >= half) {
      tab[e] = make_float2(1.f, 0.f);
      continue;
    }
    const double ang = (double)pos / pow(theta, (double)(2 * i) / (double)head_dim);
    double s, c;
    sincos(ang, &s, &c);
    tab[e] = make_float2((float)c, (float)s);
  }
}

int rope_table_f32(fcu_ctx *ctx, int T, int head_dim, double theta, const float2 **out, int width) {
  struct Tab {
    float2 *p = nullptr;
    int T = 0, head_dim = 0;
    double theta = 0;
  };
  // one cached table per device for each kind: [T][head_dim/2] and the
  // 64-column padded [T][32]
  static thread_local Tab tabs[2][64];
  if (width <= 0) width = head_dim / 2;
  Tab &t = tabs[width != head_dim / 2][ctx->device & 63];
  if (!t.p || t.T < T || t.head_dim != head_dim || t.theta != theta) {
    if (t.p) {
      FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
      FCU_CHECK_CUDA(cudaFree(t.p));
      t.p = nullptr;
    }
    FCU_CHECK_CUDA(cudaMalloc(&t.p, sizeof(float2) * (size_t)T * width));
    rope_table_f32_kernel<<<256, 256, 0, ctx->stream>>>(t.p, T, width, head_dim, theta);
    FCU_CHECK_LAUNCH();
    t.T = T;
    t.head_dim = head_dim;
    t.theta = theta;
  }
  *out = t.p;
  return FCU_OK;
}

}  // namespace fcu

extern "C" int fcu_gemm_bf16(fcu_ctx *ctx, int op, const void *A, const void *B, int64_t M,
                             int64_t N, int64_t K, const fcu_gemm_out *out) {
  using namespace fcu;
  FCU_CTX(ctx);
  FCU_REQUIRE(out != nullptr && A && B, "fcu_gemm_bf16: null argument");
  FCU_REQUIRE(op >= 0 && op <= 2, "fcu_gemm_bf16: unknown op %d", op);
  const GemmOp gop = (GemmOp)op;
  FCU_REQUIRE(gemm_tc_supported(gop, M, N, K),
              "fcu_gemm_bf16: shape M=%lld N=%lld K=%lld has a row length that is not a multiple "
              "of 8 elements (TMA needs 16-byte rows)",
              (long long)M, (long long)N, (long long)K);
  FCU_REQUIRE((((uintptr_t)A | (uintptr_t)B) & 15) == 0, "fcu_gemm_bf16: operands must be 16-byte aligned");
  FCU_REQUIRE(out->out != nullptr, "fcu_gemm_bf16: null output");
  TcOut o;
  switch (out->mode) {
    case FCU_OUT_F32:
      o.mode = kOutF32;
      o.C = (float *)out->out;
      o.beta = out->accumulate ? 1 : 0;
      break;
    case FCU_OUT_F32_RESIDUAL:
      FCU_REQUIRE(out->residual != nullptr, "fcu_gemm_bf16: FCU_OUT_F32_RESIDUAL needs a residual");
      o.mode = kOutF32Res;
      o.C = (float *)out->out;
      o.R = out->residual;
      break;
    case FCU_OUT_BF16:
      o.mode = kOutBF16;
      o.Cb = (__nv_bfloat16 *)out->out;
      break;
    case FCU_OUT_BF16_ROPE: {
      FCU_REQUIRE(out->rope_T > 0 && out->head_dim > 0 && out->head_dim % 2 == 0,
                  "fcu_gemm_bf16: RoPE needs rope_T > 0 and an even head_dim (got %d, %d)",
                  out->rope_T, out->head_dim);
      FCU_REQUIRE(out->rope_cols >= 0 && out->rope_cols % 32 == 0 && out->rope_cols % out->head_dim == 0 &&
                      out->rope_cols <= N,
                  "fcu_gemm_bf16: rope_cols %d must be a multiple of 32 and of head_dim", out->rope_cols);
      o.mode = kOutBF16Rope;
      o.Cb = (__nv_bfloat16 *)out->out;
      o.rope_T = out->rope_T;
      o.rope_cols = out->rope_cols;
      o.head_dim = out->head_dim;
      int rc = rope_table_f32(ctx, out->rope_T, out->head_dim, out->rope_theta, &o.rope);
      if (rc) return rc;
      break;
    }
    case FCU_OUT_BF16_SWIGLU:
      FCU_REQUIRE(gop == GemmOp::kFwd, "fcu_gemm_bf16: FCU_OUT_BF16_SWIGLU needs op FCU_GEMM_FWD");
      FCU_REQUIRE(N % 256 == 0, "fcu_gemm_bf16: FCU_OUT_BF16_SWIGLU needs N = 2H with H %% 128 == 0 (N=%lld)",
                  (long long)N);
      FCU_REQUIRE(out->out2 != nullptr && ((((uintptr_t)out->out) | (uintptr_t)out->out2) & 15) == 0,
                  "fcu_gemm_bf16: FCU_OUT_BF16_SWIGLU needs 16-byte aligned out and out2");
      o.mode = kOutSwiGLU;
      o.Cb = (__nv_bfloat16 *)out->out;
      o.Cb2 = (__nv_bfloat16 *)out->out2;
      break;
    case FCU_OUT_BF16_SWIGLU_BWD:
      FCU_REQUIRE(N % 64 == 0, "fcu_gemm_bf16: FCU_OUT_BF16_SWIGLU_BWD needs N = H with H %% 64 == 0 (N=%lld)",
                  (long long)N);
      FCU_REQUIRE(out->aux != nullptr && ((((uintptr_t)out->out) | (uintptr_t)out->aux) & 15) == 0,
                  "fcu_gemm_bf16: FCU_OUT_BF16_SWIGLU_BWD needs 16-byte aligned out and aux");
      o.mode = kOutSwiGLUBwd;
      o.Cb = (__nv_bfloat16 *)out->out;
      o.aux = (const __nv_bfloat16 *)out->aux;
      break;
    default:
      set_error("fcu_gemm_bf16: unknown output mode %d", out->mode);
      return FCU_ERR_ARG;
  }
  void *ws = nullptr;
  int *err = nullptr;
  int rc = workspace(ctx, 0, &ws, &err);
  if (rc) return rc;
  return gemm_bf16_tc(ctx, gop, (const __nv_bfloat16 *)A, (const __nv_bfloat16 *)B, M, N, K, o, err);
}

// The plan fcu_gemm_bf16 follows for a product, from the same function, on
// the host alone (plan_gemm).
extern "C" int fcu_gemm_plan(int64_t M, int64_t N, int64_t K, int mode, int num_sms, int pair_slots,
                             int pair_setting, int *plan) {
  FCU_REQUIRE(plan != nullptr, "fcu_gemm_plan: null plan");
  FCU_REQUIRE(M > 0 && N > 0 && K > 0 && M <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX,
              "fcu_gemm_plan: shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  FCU_REQUIRE(num_sms > 0 && pair_slots >= 0, "fcu_gemm_plan: num_sms %d, pair_slots %d", num_sms, pair_slots);
  FCU_REQUIRE(mode >= FCU_OUT_F32 && mode <= FCU_OUT_BF16_SWIGLU_BWD, "fcu_gemm_plan: unknown mode %d", mode);
  const fcu::GemmPlan g =
      fcu::plan_gemm(M, N, K, mode, num_sms, pair_slots, pair_setting < 0 ? -1 : (pair_setting ? 1 : 0));
  plan[0] = g.pair ? 1 : 0;
  plan[1] = g.bn;
  plan[2] = g.splits;
  plan[3] = g.row_major ? 1 : 0;
  plan[4] = g.tiles_m;
  plan[5] = g.tiles_n;
  return FCU_OK;
}

namespace fcu {

int tc_error_word(fcu_ctx *ctx, int **err) {
  void *ws = nullptr;
  return workspace(ctx, 0, &ws, err);
}

int gemm_tc_error(fcu_ctx *ctx) {
  void *ws = nullptr;
  int *err = nullptr;
  int rc = workspace(ctx, 0, &ws, &err);
  if (rc) return rc;
  int h = 0;
  FCU_CHECK_CUDA(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  FCU_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  if (h) {
    set_error("tensor-core kernel: a bounded wait ran out (code %d)", h);
    FCU_CHECK_CUDA(cudaMemsetAsync(err, 0, sizeof(int), ctx->stream));   // reported once
    return FCU_ERR_TIMEOUT;
  }
  return FCU_OK;
}

namespace {

// One mbarrier whose phase 0 nothing completes: the bounded wait of the
// tensor-core kernels runs out after `cycles` and the error word records
// code 99, exactly as a stalled pipeline would, without faulting the GPU.
__global__ void selftest_wait_kernel(int *err, long long cycles) {
  fcu::pdl_trigger();
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    bool done = false;
    while (!(done = mbar_try_wait(&bar, 0)))
      if (clock64() - t0 > cycles) break;
    if (!done) atomicExch(err, 99);
  }
}

}  // namespace

}  // namespace fcu

extern "C" int fcu_selftest_bounded_wait(fcu_ctx *ctx, int64_t cycles) {
  using namespace fcu;
  FCU_CTX(ctx);
  FCU_REQUIRE(cycles >= 1000 && cycles <= 4000000000ll, "fcu_selftest_bounded_wait: cycles %lld",
              (long long)cycles);
  void *ws = nullptr;
  int *err = nullptr;
  int rc = workspace(ctx, 0, &ws, &err);
  if (rc) return rc;
  selftest_wait_kernel<<<1, 32, 0, ctx->stream>>>(err, (long long)cycles);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}
