// SwiGLU arithmetic of the bf16 path (swigluRows, src/L2/tensor.js:272-290),
// on pairs of adjacent hidden units packed as bf16x2 words.  The standalone
// kernels (fused.cu) and the GEMM epilogues (gemm_tc.cu) both call these, so
// the fused and unfused paths round identically: g and u are the
// bf16-rounded gate and up values the forward stores, the results are
// rounded to bf16 once.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace fcu {

__device__ __forceinline__ float2 swiglu_unpack(uint32_t w) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&w);
  return __bfloat1622float2(v);
}

__device__ __forceinline__ uint32_t swiglu_pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// act = silu(g) * u = g / (1 + e^-g) * u
__device__ __forceinline__ uint32_t swiglu_fwd_pair(uint32_t gw, uint32_t uw) {
  const float2 g = swiglu_unpack(gw), u = swiglu_unpack(uw);
  const float a = g.x / (1.f + __expf(-g.x)) * u.x;
  const float b = g.y / (1.f + __expf(-g.y)) * u.y;
  return swiglu_pack(a, b);
}

// dg = d * u * (s + g s (1 - s)),  du = d * g * s,  s = sigmoid(g)
__device__ __forceinline__ void swiglu_bwd_pair(uint32_t dw, uint32_t gw, uint32_t uw, uint32_t &og,
                                                uint32_t &ou) {
  const float2 d = swiglu_unpack(dw), g = swiglu_unpack(gw), u = swiglu_unpack(uw);
  const float sx = 1.f / (1.f + __expf(-g.x)), sy = 1.f / (1.f + __expf(-g.y));
  og = swiglu_pack(d.x * u.x * (sx + g.x * sx * (1.f - sx)), d.y * u.y * (sy + g.y * sy * (1.f - sy)));
  ou = swiglu_pack(d.x * g.x * sx, d.y * g.y * sy);
}

}  // namespace fcu
