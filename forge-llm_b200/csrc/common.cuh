// Shared definitions for the libforgecu.so kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "../../include/forgecu.h"

struct fcu_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int precision = FCU_PREC_FP32;
  int num_sms = 148;
  // Scratch owned by the context (grown on demand, freed by fcu_ctx_destroy).
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  // RoPE cos/sin table cache: (cos, sin) doubles for [rope_pos][rope_half].
  double2 *rope_tab = nullptr;
  int rope_pos = 0, rope_half = 0;
  double rope_theta = 0;
};

namespace fcu {

void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what, const char *file, int line);
// Returns a device buffer of at least `bytes` owned by ctx (reused across
// calls; contents undefined).
int ctx_scratch(fcu_ctx *ctx, size_t bytes, void **out);

inline int div_up(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Number of kernels this library has launched (fcu_launch_count).
void note_launch();

// Tensor-core attention (attn_tc.cu): head dims 16/32/64/128, 16-byte
// aligned operands.
bool attn_tc_supported(int dH, const void *Q, const void *K, const void *V);
int attn_fwd_tc(cudaStream_t st, const float *Q, const float *K, const float *V, int B, int T,
                int nH, int nKV, int dH, float *O, float *lse);
int attn_bwd_tc(cudaStream_t st, const float *dO, const float *Q, const float *K, const float *V,
                const float *lse, const float *delta, int B, int T, int nH, int nKV, int dH,
                float *dQ, float *dK, float *dV, int acc);

// The operator entries (fcu_attn_fwd / _bwd, bf16 mode) on the tcgen05
// kernels: fp32 operands packed to bf16 (attn_tmem.cu), heads of dH <= 64
// columns (dH % 4 == 0) carried 64 wide with zero padding; 16-byte aligned
// operands.
bool attn_tmem_op_supported(int dH, const void *a, const void *b, const void *c, const void *d);
int attn_fwd_op_tmem(fcu_ctx *ctx, const float *Q, const float *K, const float *V, int B, int T, int nH,
                     int nKV, int dH, float *O, float *lse);
int attn_bwd_op_tmem(fcu_ctx *ctx, const float *dO, const float *Q, const float *K, const float *V,
                     const float *O, const float *lse, int B, int T, int nH, int nKV, int dH, float *dQ,
                     float *dK, float *dV, int accumulate);

// tcgen05 attention (attn_tmem.cu) on a bf16 qkv buffer of 64-column heads
// (128-column heads for the forward at dh = 128);
// dh is the heads' true width (the softmax scale is 1/sqrt(dh); columns past
// dh must be zero).
bool attn_tmem_supported(int dH);
// The forward kernel also takes heads of 128 columns (the backward kernels
// only 64: at 128 the mma.sync backward runs).
bool attn_tmem_fwd_supported(int dH);
int attn_fwd_tmem(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV,
                  void *O, float *lse, int dh);
int attn_bwd_tmem(fcu_ctx *ctx, const void *dO, const void *qkv, int64_t ld_qkv, const void *O,
                  const float *lse, float *delta, int B, int T, int nH, int nKV, const float2 *rope,
                  void *dqkv, int split, float *pk, float *pv, int dh);
// The same kernels for heads narrower than 64 (dH % 4 == 0): the bf16
// buffers are re-laid out with zero-padded 64-column heads around the call.
bool attn_tmem_padded(int dH);
int attn_fwd_tmem_padded(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV, int dH,
                         void *O, float *lse);
int attn_bwd_tmem_padded(fcu_ctx *ctx, const void *dO, const void *qkv, int64_t ld_qkv, const void *O,
                         const float *lse, int B, int T, int nH, int nKV, int dH, double rope_theta, void *dqkv);

// (cos, sin) RoPE table [T][width] (width 0: head_dim/2; entries past
// head_dim/2 are the identity), cached per device (gemm_tc.cu).
int rope_table_f32(fcu_ctx *ctx, int T, int head_dim, double theta, const float2 **out, int width = 0);

// Programmatic dependent launch.  A kernel launched with launch_pdl may
// start while the previous kernel in the stream is finishing: it runs its
// prologue (barrier init, TMEM allocation) and must call pdl_wait() before
// it reads or writes any global memory.  Every kernel on the training step
// calls pdl_trigger() at its start, which lets such a dependent launch once
// all of its own CTAs are resident.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// FORGECU_NO_PDL=1 in the environment launches these kernels plainly.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace fcu

#define FCU_CHECK_CUDA(expr)                                                  \
  do {                                                                        \
    cudaError_t _e = (expr);                                                  \
    if (_e != cudaSuccess) return fcu::cuda_fail(_e, #expr, __FILE__, __LINE__); \
  } while (0)

#define FCU_CHECK_LAUNCH()           \
  do {                               \
    fcu::note_launch();              \
    FCU_CHECK_CUDA(cudaGetLastError()); \
  } while (0)

#define FCU_REQUIRE(cond, ...)            \
  do {                                    \
    if (!(cond)) {                        \
      fcu::set_error(__VA_ARGS__);        \
      return FCU_ERR_ARG;                 \
    }                                     \
  } while (0)

#define FCU_CTX(ctx) FCU_REQUIRE((ctx) != nullptr, "null fcu_ctx")

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum over blockDim.x threads (multiple of 32, <= 1024).  `sh`
// holds >= 32 entries.  Result valid in every thread.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T *sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  T r = lane < nw ? sh[lane] : T(0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}
