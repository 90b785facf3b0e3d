// Adam with global-norm clipping (src/L2/autograd.js:214-244).
//
// Two passes over the flat parameter vector: a deterministic double-precision
// sum of squares of the gradients (fixed grid, fixed reduction order), then
// one fused update pass that reads p, g, m, v once and writes p, m, v once
// (28 bytes per parameter).  The per-element arithmetic is in double, like the
// JS, with fp32 stores.
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;

__global__ void sumsq_partial_kernel(const float *__restrict__ g, int64_t n,
                                     double *__restrict__ part, int vec) {
  fcu::pdl_trigger();
  __shared__ double sh[32];
  double s = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n4 = vec ? (n >> 2) : 0;
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  // four float4 loads in flight per thread, four independent fp64 sums
  // (combined in a fixed order, so the result is deterministic)
  double s1 = 0, s2 = 0, s3 = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += 4 * stride) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 a = g4[i];
    const float4 b = i + stride < n4 ? g4[i + stride] : z;
    const float4 c = i + 2 * stride < n4 ? g4[i + 2 * stride] : z;
    const float4 d = i + 3 * stride < n4 ? g4[i + 3 * stride] : z;
    s += (double)a.x * a.x + (double)a.y * a.y + (double)a.z * a.z + (double)a.w * a.w;
    s1 += (double)b.x * b.x + (double)b.y * b.y + (double)b.z * b.z + (double)b.w * b.w;
    s2 += (double)c.x * c.x + (double)c.y * c.y + (double)c.z * c.z + (double)c.w * c.w;
    s3 += (double)d.x * d.x + (double)d.y * d.y + (double)d.z * d.z + (double)d.w * d.w;
  }
  s = (s + s1) + (s2 + s3);
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    s += (double)g[i] * g[i];
  s = block_sum(s, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

__global__ void sumsq_final_kernel(const double *__restrict__ part, int nblk,
                                   double *__restrict__ out, int acc) {
  fcu::pdl_trigger();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0;
    for (int b = 0; b < nblk; b++) s += part[b];
    out[0] = acc ? out[0] + s : s;
  }
}

struct Hyper {
  double lr, b1, b2, eps, wd, clip, bc1, bc2;
};

__device__ __forceinline__ void adam_elem(float &p, float g, float &m, float &v, double scale,
                                          const Hyper &h) {
  double gg = (double)g * scale + h.wd * (double)p;
  m = (float)(h.b1 * (double)m + (1.0 - h.b1) * gg);
  v = (float)(h.b2 * (double)v + (1.0 - h.b2) * gg * gg);
  double mh = (double)m / h.bc1;
  double vh = (double)v / h.bc2;
  p = (float)((double)p - h.lr * mh / (sqrt(vh) + h.eps));
}

__global__ void __launch_bounds__(kThreads, 3) adam_update_kernel(float *__restrict__ p, const float *__restrict__ g,
                                   float *__restrict__ m, float *__restrict__ v, int64_t n, Hyper h,
                                   const double *__restrict__ sumsq, double *__restrict__ info,
                                   int vec, __nv_bfloat16 *__restrict__ shadow,
                                   const Hyper *__restrict__ hdev) {
  fcu::pdl_trigger();
  if (hdev) h = *hdev;  // the on-device schedule of fcu_adam_step_sched
  const double gnorm = sqrt(sumsq[0]);
  const double scale = gnorm > h.clip ? h.clip / gnorm : 1.0;
  if (info && blockIdx.x == 0 && threadIdx.x == 0) {
    info[0] = gnorm;
    info[1] = scale;
    if (hdev) info[2] = h.lr;
  }
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t start = 0;
  if (vec) {
    const int64_t n4 = n >> 2;
    float4 *p4 = reinterpret_cast<float4 *>(p);
    float4 *m4 = reinterpret_cast<float4 *>(m);
    float4 *v4 = reinterpret_cast<float4 *>(v);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    // Two float4 groups per thread and iteration, all eight loads issued
    // before the fp64 arithmetic, so twice the bytes are in flight (the
    // update is otherwise bound by memory-level parallelism).
    auto update4 = [&](int64_t i, float4 pp, float4 gg, float4 mm, float4 vv) {
      adam_elem(pp.x, gg.x, mm.x, vv.x, scale, h);
      adam_elem(pp.y, gg.y, mm.y, vv.y, scale, h);
      adam_elem(pp.z, gg.z, mm.z, vv.z, scale, h);
      adam_elem(pp.w, gg.w, mm.w, vv.w, scale, h);
      p4[i] = pp;
      m4[i] = mm;
      v4[i] = vv;
      if (shadow) {
        __nv_bfloat162 a = __floats2bfloat162_rn(pp.x, pp.y), b = __floats2bfloat162_rn(pp.z, pp.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t *>(&a);
        u.y = *reinterpret_cast<uint32_t *>(&b);
        reinterpret_cast<uint2 *>(shadow)[i] = u;
      }
    };
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += 2 * stride) {
      const int64_t j = i + stride;
      const float4 pa = p4[i], ga = g4[i], ma = m4[i], va = v4[i];
      float4 pb = pa, gb = ga, mb = ma, vb = va;
      if (j < n4) {
        pb = p4[j];
        gb = g4[j];
        mb = m4[j];
        vb = v4[j];
      }
      update4(i, pa, ga, ma, va);
      if (j < n4) update4(j, pb, gb, mb, vb);
    }
    start = n4 << 2;
  }
  for (int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float pp = p[i], mm = m[i], vv = v[i];
    adam_elem(pp, g[i], mm, vv, scale, h);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (shadow) shadow[i] = __float2bfloat16_rn(pp);
  }
}

inline bool aligned16(const void *a) { return ((uintptr_t)a & 15) == 0; }

// Blocks of the sum-of-squares pass; its per-block partials sit at the head
// of the context scratch (callers place their own values after them).
inline int sumsq_nblk(const fcu_ctx *ctx) { return 4 * ctx->num_sms; }

int sumsq_impl(fcu_ctx *ctx, const float *g, int64_t n, double *out, int acc) {
  const int nblk = sumsq_nblk(ctx);
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(double) * nblk, &scr);
  if (rc) return rc;
  sumsq_partial_kernel<<<nblk, kThreads, 0, ctx->stream>>>(g, n, (double *)scr, aligned16(g) ? 1 : 0);
  FCU_CHECK_LAUNCH();
  sumsq_final_kernel<<<1, 32, 0, ctx->stream>>>((const double *)scr, nblk, out, acc);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

// The cosine lr and bias corrections of step t = ++(*t_dev), computed on the
// device so a captured step replays with the right schedule
// (src/L2/autograd.js:222,229,237-238).
__global__ void adam_sched_kernel(double lr0, double b1, double b2, double eps, double wd,
                                  double clip, double total, int32_t *__restrict__ t_dev,
                                  Hyper *__restrict__ out) {
  fcu::pdl_trigger();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int t = ++t_dev[0];
    double tt = (double)t / total;
    if (tt > 1) tt = 1;
    Hyper h;
    h.lr = lr0 * 0.5 * (1.0 + cos(M_PI * tt));
    h.b1 = b1;
    h.b2 = b2;
    h.eps = eps;
    h.wd = wd;
    h.clip = clip;
    h.bc1 = 1.0 - pow(b1, (double)t);
    h.bc2 = 1.0 - pow(b2, (double)t);
    *out = h;
  }
}

int update_impl(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                const fcu_adam_hyper *hh, const double *sumsq, double *info,
                __nv_bfloat16 *shadow = nullptr, const Hyper *hdev = nullptr) {
  Hyper h{0, 0, 0, 0, 0, 0, 1, 1};
  if (hh) h = Hyper{hh->lr, hh->b1, hh->b2, hh->eps, hh->wd, hh->clip, hh->bc1, hh->bc2};
  int vec = aligned16(p) && aligned16(g) && aligned16(m) && aligned16(v) &&
            (shadow == nullptr || ((uintptr_t)shadow & 7) == 0);
  int64_t work = vec ? (n >> 2) : n;
  int64_t blocks = (work + kThreads - 1) / kThreads;
  int64_t cap = 16 * (int64_t)ctx->num_sms;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  adam_update_kernel<<<(int)blocks, kThreads, 0, ctx->stream>>>(p, g, m, v, n, h, sumsq, info, vec,
                                                                 shadow, hdev);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

}  // namespace

extern "C" {

int fcu_sumsq(fcu_ctx *ctx, const float *g, int64_t n, double *sumsq_dev, int accumulate) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && g && sumsq_dev, "fcu_sumsq: bad args");
  return sumsq_impl(ctx, g, n, sumsq_dev, accumulate);
}

int fcu_adam_step_sumsq(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                        const fcu_adam_hyper *h, const double *sumsq_dev, double *info_dev) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && p && g && m && v && h && sumsq_dev, "fcu_adam_step: bad args");
  FCU_REQUIRE(h->bc1 > 0 && h->bc2 > 0, "fcu_adam_step: bias corrections must be > 0 (t >= 1)");
  if (n == 0) return FCU_OK;
  return update_impl(ctx, p, g, m, v, n, h, sumsq_dev, info_dev);
}

int fcu_adam_step(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                  const fcu_adam_hyper *h, double *info_dev) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && p && g && m && v && h, "fcu_adam_step: bad args");
  FCU_REQUIRE(h->bc1 > 0 && h->bc2 > 0, "fcu_adam_step: bias corrections must be > 0 (t >= 1)");
  if (n == 0) return FCU_OK;
  // The sum of squares lands in the tail of the context scratch, after the
  // per-block partials that sumsq_impl keeps at its head.
  const int nblk = sumsq_nblk(ctx);
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(double) * (nblk + 1), &scr);
  if (rc) return rc;
  double *ss = (double *)scr + nblk;
  rc = sumsq_impl(ctx, g, n, ss, 0);
  if (rc) return rc;
  return update_impl(ctx, p, g, m, v, n, h, ss, info_dev);
}

int fcu_adam_step_shadow(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                         const fcu_adam_hyper *h, const double *sumsq_dev, double *info_dev,
                         void *p_bf16) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && p && g && m && v && h && p_bf16, "fcu_adam_step_shadow: bad args");
  FCU_REQUIRE(h->bc1 > 0 && h->bc2 > 0, "fcu_adam_step_shadow: bias corrections must be > 0 (t >= 1)");
  if (n == 0) return FCU_OK;
  const double *ss = sumsq_dev;
  if (!ss) {
    const int nblk = sumsq_nblk(ctx);
    void *scr = nullptr;
    int rc = fcu::ctx_scratch(ctx, sizeof(double) * (nblk + 1), &scr);
    if (rc) return rc;
    double *own = (double *)scr + nblk;
    rc = sumsq_impl(ctx, g, n, own, 0);
    if (rc) return rc;
    ss = own;
  }
  return update_impl(ctx, p, g, m, v, n, h, ss, info_dev, (__nv_bfloat16 *)p_bf16);
}

int fcu_adam_step_sched(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                        const fcu_adam_sched *s, int32_t *t_dev, double *info_dev, void *p_bf16) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && p && g && m && v && s && t_dev, "fcu_adam_step_sched: bad args");
  FCU_REQUIRE(s->total_steps > 0, "fcu_adam_step_sched: total_steps must be > 0");
  if (n == 0) return FCU_OK;
  // scratch: [nblk partial sums][sum of squares][Hyper]
  const int nblk = sumsq_nblk(ctx);
  void *scr = nullptr;
  int rc = fcu::ctx_scratch(ctx, sizeof(double) * (nblk + 1) + sizeof(Hyper) + 64, &scr);
  if (rc) return rc;
  double *ss = (double *)scr + nblk;
  Hyper *hdev = (Hyper *)(((uintptr_t)(ss + 1) + 63) & ~(uintptr_t)63);
  adam_sched_kernel<<<1, 32, 0, ctx->stream>>>(s->lr, s->b1, s->b2, s->eps, s->wd, s->clip,
                                               s->total_steps, t_dev, hdev);
  FCU_CHECK_LAUNCH();
  rc = sumsq_impl(ctx, g, n, ss, 0);
  if (rc) return rc;
  return update_impl(ctx, p, g, m, v, n, nullptr, ss, info_dev, (__nv_bfloat16 *)p_bf16, hdev);
}

// The two halves of fcu_adam_step_sched for an optimizer whose update is
// split into pieces (a rank's shard of every bucket): advance the schedule
// once, then update each piece with the step's device-resident constants and
// a caller-supplied (e.g. all-reduced) gradient sum of squares.
int fcu_adam_sched_advance(fcu_ctx *ctx, const fcu_adam_sched *s, int32_t *t_dev, fcu_adam_hyper *h_dev) {
  FCU_CTX(ctx);
  FCU_REQUIRE(s && t_dev && h_dev && (((uintptr_t)h_dev & 7) == 0), "fcu_adam_sched_advance: bad args");
  FCU_REQUIRE(s->total_steps > 0, "fcu_adam_sched_advance: total_steps must be > 0");
  static_assert(sizeof(Hyper) == sizeof(fcu_adam_hyper), "Hyper mirrors fcu_adam_hyper");
  adam_sched_kernel<<<1, 32, 0, ctx->stream>>>(s->lr, s->b1, s->b2, s->eps, s->wd, s->clip,
                                               s->total_steps, t_dev, (Hyper *)h_dev);
  FCU_CHECK_LAUNCH();
  return FCU_OK;
}

int fcu_adam_update_dev(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                        const fcu_adam_hyper *h_dev, const double *sumsq_dev, double *info_dev,
                        void *p_bf16) {
  FCU_CTX(ctx);
  FCU_REQUIRE(n >= 0 && p && g && m && v && h_dev && sumsq_dev, "fcu_adam_update_dev: bad args");
  if (n == 0) return FCU_OK;
  return update_impl(ctx, p, g, m, v, n, nullptr, sumsq_dev, info_dev, (__nv_bfloat16 *)p_bf16,
                     (const Hyper *)h_dev);
}

}  // extern "C"
