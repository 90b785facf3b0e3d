/*
 * forgecu.h -- the C-ABI of libforgecu.so, the B200 (sm_100a) implementation
 * of forge-llm's training hot path.
 *
 * This is the drop-in boundary.  forge-llm's operators (src/L2/tensor.js,
 * src/L2/autograd.js, src/L6/train.js) keep their JavaScript signatures; a
 * host binding (N-API addon, ctypes, ...) marshals their typed arrays to
 * device buffers and calls the entry points below.  Each entry point cites
 * the JS function it replaces.
 *
 * Conventions
 *   - Every tensor is a plain device pointer to row-major, token-major data
 *     (fp32 unless the name says otherwise), exactly the Float32Array layout
 *     the JS uses.  Sizes are int64_t element counts.
 *   - Gradient outputs follow the JS `grad += ...` contract: an `accumulate`
 *     flag of 1 adds into the buffer, 0 overwrites it (the JS `??=` of a fresh
 *     zero array followed by `+=`).
 *   - All work is enqueued on the context's stream (fcu_ctx_set_stream) and
 *     returns without waiting; fcu_sync waits.  A context is not re-entrant.
 *   - Every function returns an fcu_status; FCU_OK is 0.  On any other value
 *     fcu_last_error() (thread-local) describes the failure.  Shapes are
 *     validated before anything is launched.
 */
#ifndef FORGECU_H
#define FORGECU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum {
  FCU_OK = 0,
  FCU_ERR_ARG = -1,        /* bad shape, null pointer, unsupported size */
  FCU_ERR_CUDA = -2,       /* a CUDA runtime/driver call failed */
  FCU_ERR_NCCL = -3,       /* a collective failed */
  FCU_ERR_TIMEOUT = -4,    /* a bounded wait ran out */
  FCU_ERR_UNSUPPORTED = -5 /* not available on this device / build */
} fcu_status;

/* Arithmetic used by the contractions (matmulT, attention).
 *   FP32    : fp32 operands and accumulation on the CUDA cores.  Parity mode:
 *             relL2 <= 1e-5 against the JS operators.
 *   FP32_TC : the matmulT contractions (matmulT fwd / dX / dW, linear) on the
 *             tensor cores at fp32-level accuracy: each fp32 operand is split
 *             into three bf16 parts, x = x0 + x1 + x2, and the six part
 *             products a_i b_j with i + j <= 2 run as one tcgen05 contraction
 *             six times as long (the dropped terms are ~2^-24 of |a b|).  Any
 *             shape (K padded with zeros).  Same parity bound as FP32;
 *             attention and the other operators as in FP32.
 *   BF16    : tensor cores (tcgen05 kind::f16) on bf16-rounded operands, fp32
 *             accumulate.  Looser bound, relL2 <= 1e-2 (stated per test). */
typedef enum { FCU_PREC_FP32 = 0, FCU_PREC_FP32_TC = 1, FCU_PREC_BF16 = 2 } fcu_precision;

typedef struct fcu_ctx fcu_ctx;

/* ---------------------------------------------------------------- context */
const char *fcu_last_error(void);
const char *fcu_version(void);
int fcu_ctx_create(int device, fcu_ctx **out);
int fcu_ctx_destroy(fcu_ctx *ctx);
int fcu_ctx_set_stream(fcu_ctx *ctx, void *cuda_stream); /* NULL = legacy default stream */
int fcu_ctx_set_precision(fcu_ctx *ctx, int precision);   /* fcu_precision */
int fcu_ctx_get_precision(const fcu_ctx *ctx);
int fcu_sync(fcu_ctx *ctx);
/* FCU_ERR_TIMEOUT if a kernel on this context recorded a bounded wait that
 * ran out (the kernel then returned early; its outputs are invalid).
 * Synchronises the context's stream; a recorded timeout is reported once
 * (the device word is cleared after it is read). */
int fcu_check_device_error(fcu_ctx *ctx);
/* Failure-detection self-test (no counterpart in the reference): one kernel
 * whose bounded mbarrier wait can never complete runs out after `cycles`
 * SM clocks (1e3..4e9) and records the timeout as the tensor-core kernels
 * do, without faulting the GPU; fcu_check_device_error then reports it and
 * the context stays usable. */
int fcu_selftest_bounded_wait(fcu_ctx *ctx, int64_t cycles);
/* Kernels launched by this library since it was loaded (all contexts). */
unsigned long long fcu_launch_count(void);
/* Bytes of per-row scratch the context currently holds (0 until an entry
 * point that needs scratch first runs; it only grows).  No counterpart in
 * the reference: hosts with a fixed memory budget read it to plan for it. */
int fcu_ctx_scratch_bytes(const fcu_ctx *ctx, size_t *out);

/* Device memory for hosts without an allocator of their own (the N-API
 * addon).  The Python host allocates through PyTorch instead. */
int fcu_malloc(fcu_ctx *ctx, size_t bytes, void **out);
int fcu_free(fcu_ctx *ctx, void *ptr);
int fcu_memcpy_h2d(fcu_ctx *ctx, void *dst, const void *src, size_t bytes);
int fcu_memcpy_d2h(fcu_ctx *ctx, void *dst, const void *src, size_t bytes);
int fcu_memset_zero(fcu_ctx *ctx, void *dst, size_t bytes);

/* ---------------------------------------------------------------- matmulT */
/* Y[M,N] = X[M,K] . W[N,K]^T.
 * Replaces matmulT forward, src/L2/tensor.js:34-36 (-> gemm, src/L0/numeric.js:111-129). */
int fcu_matmulT_fwd(fcu_ctx *ctx, const float *X, const float *W, float *Y, int64_t M, int64_t K,
                    int64_t N);

/* dX[M,K] (+)= dY[M,N] . W[N,K];  dW[N,K] (+)= dY^T . X.  Either output may be
 * NULL to skip it.  Replaces the matmulT closure, src/L2/tensor.js:37-52. */
int fcu_matmulT_bwd(fcu_ctx *ctx, const float *dY, const float *X, const float *W, float *dX,
                    int accumulate_dx, float *dW, int accumulate_dw, int64_t M, int64_t K,
                    int64_t N);

/* ---------------------------------------------------------------- fused bf16 path */
/* The building blocks TrainableTransformer's step uses in FCU_PREC_BF16 mode.
 * They compute the same contractions as the matmulT / causalAttn /
 * rmsNorm / swigluRows / crossEntropyMean entries above, but take bf16
 * operands produced directly by the previous kernel and fuse the glue the JS
 * does as separate ops (residual add, RoPE, bf16 copies of gradients), so no
 * fp32 -> bf16 conversion pass or column slice is ever run. */
enum { FCU_GEMM_FWD = 0, FCU_GEMM_DX = 1, FCU_GEMM_DW = 2 };
enum {
  FCU_OUT_F32 = 0,
  FCU_OUT_F32_RESIDUAL = 1,
  FCU_OUT_BF16 = 2,
  FCU_OUT_BF16_ROPE = 3,
  /* gate|up projection with swigluRows (tensor.js:272-290) in the epilogue:
   * op FCU_GEMM_FWD, B = [Wgate; Wup] with N = 2H rows, H % 128 == 0;
   * out = g | u bf16 [M, 2H] as BF16 would write it, out2 = silu(g) * u bf16
   * [M, H] from the bf16-rounded g and u (bit-identical to
   * fcu_swiglu_fwd_bf16 applied to out) */
  FCU_OUT_BF16_SWIGLU = 4,
  /* down-projection input gradient with the swigluRows backward in the
   * epilogue: N = H (H % 64 == 0), aux = the forward's g | u bf16 [M, 2H];
   * out = dg | du bf16 [M, 2H], computed from bf16(A.B) (bit-identical to
   * BF16 output followed by fcu_swiglu_bwd_bf16) */
  FCU_OUT_BF16_SWIGLU_BWD = 5
};

typedef struct {
  int mode;               /* FCU_OUT_* */
  void *out;              /* [M, N] fp32 (F32*) or bf16 (BF16*) */
  int accumulate;         /* FCU_OUT_F32: out += A.B */
  const float *residual;  /* FCU_OUT_F32_RESIDUAL: out = residual + A.B (addTensors, train.js:230) */
  int rope_T;             /* FCU_OUT_BF16_ROPE: position = row % rope_T (ropeRows posStride) */
  int rope_cols;          /* columns [0, rope_cols) are rotated (q and k of a fused qkv) */
  int head_dim;
  double rope_theta;
  void *out2;             /* FCU_OUT_BF16_SWIGLU: the activation output */
  const void *aux;        /* FCU_OUT_BF16_SWIGLU_BWD: the forward's gate|up values */
  /* (out2 and aux are read only in those two modes, so a caller that fills
   * just the fields above them keeps working for the other modes) */
} fcu_gemm_out;

/* One tcgen05 contraction on bf16 operands (fp32 accumulate) in the layouts
 * of matmulT: FCU_GEMM_FWD C = A[M,K].B[N,K]^T; FCU_GEMM_DX C = A[M,K].B[K,N];
 * FCU_GEMM_DW C = A[K,M]^T.B[K,N].  Every operand row length must be a multiple
 * of 8 elements and both operands 16-byte aligned. */
int fcu_gemm_bf16(fcu_ctx *ctx, int op, const void *A, const void *B, int64_t M, int64_t N,
                  int64_t K, const fcu_gemm_out *out);

/* The launch plan fcu_gemm_bf16 picks for an M x N x K product in output mode
 * `mode` (FCU_OUT_*), computed on the host without a device: plan[0] = 1 for
 * the CTA-pair tile (256 x 256 over two SMs, tcgen05 cta_group::2), plan[1] =
 * the tile width in columns, plan[2] = the K slices (1: no split-K), plan[3] =
 * 1 for the n-fastest tile raster, plan[4] / plan[5] = row / column tiles.
 * num_sms and pair_slots describe the device (148 SMs and 74 concurrent CTA
 * pairs on a B200; pair_slots 0 rules the pair tile out); pair_setting is the
 * FORGECU_GEMM_PAIR switch (-1 unset, 0 never, 1 wherever the shape allows).
 * Not in the reference: an introspection aid for the kernel choices. */
int fcu_gemm_plan(int64_t M, int64_t N, int64_t K, int mode, int num_sms, int pair_slots, int pair_setting,
                  int *plan);

/* rmsNorm forward (src/L2/tensor.js:103-113) writing bf16 out[T,D] and fp32
 * inv[T].  D % 4 == 0. */
int fcu_rmsnorm_fwd_bf16(fcu_ctx *ctx, const float *X, const float *w, int64_t T, int64_t D,
                         double eps, void *out_bf16, float *inv);

// Residual add fused into the next normalisation: Xout = X + A (fp32; the
// residual stream plus the branch output a GEMM wrote), then out / inv as
// fcu_rmsnorm_fwd_bf16 computes them from Xout.  D a multiple of 4.  Replaces an `addTensors(x, branch)` + `rmsNorm(x)` pair of the
// block (src/L6/train.js:145-147, 153 with the next block's :130 or :156).
int fcu_rmsnorm_fwd_bf16_add(fcu_ctx *ctx, const float *X, const float *A, const float *w, int64_t T,
                             int64_t D, double eps, float *Xout, void *out, float *inv);
/* rmsNorm backward (src/L2/tensor.js:114-127) fused with the residual
 * gradient: dX (+)= the rmsNorm input gradient (fp32, in place); if dX_bf16
 * is not NULL it receives bf16 of the final dX (the next GEMM's operand);
 * dw (+)= sum_t g*x*inv (deterministic).  D % 4 == 0, D <= 2048. */
int fcu_rmsnorm_bwd_fused(fcu_ctx *ctx, const float *dY, const float *X, const float *w,
                          const float *inv, int64_t T, int64_t D, float *dX, int accumulate_dx,
                          void *dX_bf16, float *dw, int accumulate_dw);
/* swigluRows (src/L2/tensor.js:272-290) over one bf16 [N, 2H] buffer whose
 * columns [0,H) are the gate and [H,2H) the up projection (the layout of
 * ffn_gate followed by ffn_up in paramList order): act[N,H] = silu(g)*u, and
 * backward dgu[N,2H] = (dact*u*silu'(g), dact*silu(g)).  H % 8 == 0. */
int fcu_swiglu_fwd_bf16(fcu_ctx *ctx, const void *gu, int64_t N, int64_t H, void *act);
int fcu_swiglu_bwd_bf16(fcu_ctx *ctx, const void *dact, const void *gu, int64_t N, int64_t H,
                        void *dgu);
/* crossEntropyMean forward (src/L2/tensor.js:393-407) whose unit gradient
 * (P - onehot)/T is written in bf16 (the LM-head backward's operand). */
int fcu_ce_fwd_bf16grad(fcu_ctx *ctx, const float *logits, const int32_t *targets, int64_t T,
                        int64_t V, float *loss_out, void *dlogits_bf16);
/* Causal GQA attention on bf16 operands read from one qkv buffer [B*T, ld]
 * (q heads at columns [0, nH*dH), k at [nH*dH, ..+nKV*dH), v after), O bf16
 * [B*T, nH*dH], lse fp32 [B, nH, T] (causalAttnBatch, src/L2/tensor.js:299-337). */
int fcu_attn_fwd_bf16(fcu_ctx *ctx, const void *qkv, int64_t ld_qkv, int B, int T, int nH, int nKV,
                      int dH, void *O, float *lse);
/* Its backward (src/L2/tensor.js:339-375): dq, dk, dv written in bf16 into
 * dqkv (same layout as qkv); when rope_theta > 0 the RoPE backward R^T
 * (src/L2/tensor.js:150-165, position = row % T) is applied to dq and dk. */
int fcu_attn_bwd_bf16(fcu_ctx *ctx, const void *dO, const void *qkv, int64_t ld_qkv, const void *O,
                      const float *lse, int B, int T, int nH, int nKV, int dH, double rope_theta,
                      void *dqkv);
/* y[i] = bf16(x[i]). */
int fcu_to_bf16(fcu_ctx *ctx, const float *x, int64_t n, void *y);
/* y[i] = bf16(y[i] * alpha_dev[0]) (a loss gradient other than 1). */
int fcu_scale_bf16_dev(fcu_ctx *ctx, void *y, int64_t n, const float *alpha_dev);

/* ---------------------------------------------------------------- embedding */
/* out[T,D] = W[ids[t], :].  Replaces embedLookup, src/L2/tensor.js:85-91. */
int fcu_embed_fwd(fcu_ctx *ctx, const float *W, const int32_t *ids, int64_t T, int64_t V,
                  int64_t D, float *out);
/* dW[ids[t], :] += dX[t, :], deterministic: every row of dW receives its terms
 * in ascending t, as the JS loop adds them (src/L2/tensor.js:92-98). */
int fcu_embed_bwd(fcu_ctx *ctx, const float *dX, const int32_t *ids, int64_t T, int64_t V,
                  int64_t D, float *dW);

/* ---------------------------------------------------------------- rmsNorm */
/* out = X * inv[t] * w, inv[t] = 1/sqrt(mean(X[t]^2) + eps) (stored).
 * Replaces rmsNorm forward, src/L2/tensor.js:103-113. */
int fcu_rmsnorm_fwd(fcu_ctx *ctx, const float *X, const float *w, int64_t T, int64_t D, double eps,
                    float *out, float *inv);
/* Replaces the rmsNorm closure, src/L2/tensor.js:114-127. */
int fcu_rmsnorm_bwd(fcu_ctx *ctx, const float *dY, const float *X, const float *w,
                    const float *inv, int64_t T, int64_t D, float *dX, int accumulate_dx,
                    float *dw, int accumulate_dw);

/* ---------------------------------------------------------------- ropeRows */
/* Interleaved-pair rotation, position pos0 + (posStride > 0 ? t % posStride : t).
 * Replaces ropeRows, src/L2/tensor.js:133-149; backward (R^T) :150-165. */
int fcu_rope_fwd(fcu_ctx *ctx, const float *X, int64_t T, int nHead, int dHead, int pos0,
                 double theta, int posStride, float *out);
int fcu_rope_bwd(fcu_ctx *ctx, const float *dY, int64_t T, int nHead, int dHead, int pos0,
                 double theta, int posStride, float *dX, int accumulate);

/* ---------------------------------------------------------------- sliceCols */
/* out[M,len] = X[:, off:off+len].  Replaces sliceCols, src/L2/tensor.js:170-183. */
int fcu_slicecols_fwd(fcu_ctx *ctx, const float *X, int64_t M, int64_t K, int64_t off,
                      int64_t len, float *out);
int fcu_slicecols_bwd(fcu_ctx *ctx, const float *dY, int64_t M, int64_t K, int64_t off,
                      int64_t len, float *dX, int accumulate);

/* ---------------------------------------------------------------- attention */
/* Causal attention with GQA (kv head = h / (nH/nKV)) over B sequences of T
 * tokens under the block-diagonal causal mask; B == 1 is causalAttn.
 * Q [B*T, nH*dH], K/V [B*T, nKV*dH], O like Q, lse [B, nH, T] = log-sum-exp
 * of each score row (kept for the backward instead of the JS's T x T P).
 * Replaces causalAttn (src/L2/tensor.js:191-229) and causalAttnBatch
 * (src/L2/tensor.js:299-337).  Requires nH % nKV == 0 and 1 <= dH <= 128. */
int fcu_attn_fwd(fcu_ctx *ctx, const float *Q, const float *K, const float *V, int B, int T,
                 int nH, int nKV, int dH, float *O, float *lse);
/* Replaces the attention closures, src/L2/tensor.js:231-267 / :339-375. */
int fcu_attn_bwd(fcu_ctx *ctx, const float *dO, const float *Q, const float *K, const float *V,
                 const float *O, const float *lse, int B, int T, int nH, int nKV, int dH,
                 float *dQ, float *dK, float *dV, int accumulate);

/* ---------------------------------------------------------------- swiglu */
/* out = G * sigmoid(G) * U.  Replaces swigluRows, src/L2/tensor.js:272-280. */
int fcu_swiglu_fwd(fcu_ctx *ctx, const float *G, const float *U, int64_t n, float *out);
/* Replaces the swigluRows closure, src/L2/tensor.js:281-289. */
int fcu_swiglu_bwd(fcu_ctx *ctx, const float *dO, const float *G, const float *U, int64_t n,
                   float *dG, float *dU, int accumulate);

/* ---------------------------------------------------------------- residual add */
/* out = a + b; backward passes g to both (src/L6/train.js:230-238). */
int fcu_add_fwd(fcu_ctx *ctx, const float *a, const float *b, int64_t n, float *out);
int fcu_add_bwd(fcu_ctx *ctx, const float *g, int64_t n, float *da, int accumulate_a, float *db,
                int accumulate_b);

/* ---------------------------------------------------------------- cross entropy */
/* Fused crossEntropyMean forward and unit-gradient pass (src/L2/tensor.js:393-417):
 * loss_out[0] = -(1/T) sum_t log softmax(logits_t)[targets_t]  (device scalar)
 * dunit[T,V]  = (softmax(logits_t) - onehot(targets_t)) / T
 * One read of logits; dunit may alias logits (in-place).  The backward of the
 * JS closure is then dLogits += g * dunit (fcu_axpy). */
int fcu_ce_fwd(fcu_ctx *ctx, const float *logits, const int32_t *targets, int64_t T, int64_t V,
               float *loss_out, float *dunit);

/* fcu_ce_fwd for callers that must not allocate device memory.  No
 * counterpart in the reference: it exists for hosts that plan every device
 * byte up front (an embedding runtime with a fixed memory pool, or an
 * N-API host whose buffers belong to another allocator), and for which a
 * cudaMalloc inside a training step is not allowed (it can fail under memory
 * pressure and it synchronises the whole device).  fcu_ce_fwd may allocate
 * its per-row scratch through the context on first use or growth; this entry
 * point never calls cudaMalloc, cudaFree or any allocating routine.
 * Its scratch is a fixed array compiled into the library: T <= 65536 rows
 * (256 KiB, held by every GPU that loads the library until the process
 * exits).  Larger T is rejected with FCU_ERR_ARG.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress, with that device
 * current) and caches it; make that first call before any stream capture.
 * The cached address belongs to the device's current primary context: after
 * cudaDeviceReset (or anything else that destroys that context) it is stale,
 * so a process that resets a device must not call this entry point on it
 * again.  All calls share the one array, so calls whose kernels overlap on
 * the GPU (other streams, other threads) race; calls on one stream are
 * ordered and safe.  Results equal fcu_ce_fwd's. */
int fcu_ce_fwd_static(fcu_ctx *ctx, const float *logits, const int32_t *targets, int64_t T,
                      int64_t V, float *loss_out, float *dunit);

/* y (+)= alpha_dev[0] * x, alpha read from device memory (a loss gradient). */
int fcu_axpy_dev(fcu_ctx *ctx, const float *alpha_dev, const float *x, int64_t n, float *y,
                 int accumulate);

/* ---------------------------------------------------------------- weightedSum */
/* out[0] = sum_i Y[i] t[i] (src/L2/tensor.js:380-389), device scalar. */
int fcu_wsum_fwd(fcu_ctx *ctx, const float *Y, const float *t, int64_t n, float *out);

/* ---------------------------------------------------------------- training windows */
/* The batch of train() (src/L6/train.js:256-262) gathered on the device from
 * a device-resident token stream: out[b*T1 + i] = data[starts[b] + i], or
 * data[n-1] past the end of the stream.  starts (device, B values) are drawn
 * on the host from the forge-llm RNG exactly as the JS draws them. */
int fcu_gather_windows(fcu_ctx *ctx, const int32_t *data, int64_t n, const int32_t *starts, int B,
                       int T1, int32_t *out);

/* ---------------------------------------------------------------- Adam */
typedef struct {
  double lr;    /* the cosine-scheduled lr of this step (autograd.js:229) */
  double b1, b2, eps, wd, clip;
  double bc1;   /* 1 - b1^t */
  double bc2;   /* 1 - b2^t */
} fcu_adam_hyper;

/* One Adam step over flat p/g/m/v of n elements (all params concatenated in
 * paramList order), with global-norm clipping: gnorm = ||g||_2 over all n,
 * scale = gnorm > clip ? clip/gnorm : 1, then per element
 * g' = g*scale + wd*p; m = b1 m + (1-b1) g'; v = b2 v + (1-b2) g'^2;
 * p -= lr * (m/bc1) / (sqrt(v/bc2) + eps).
 * info_dev (device, 2 doubles) receives {gnorm, scale}.
 * Replaces Adam.step, src/L2/autograd.js:221-243. */
int fcu_adam_step(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                  const fcu_adam_hyper *h, double *info_dev);

/* Same update with the gradient sum of squares supplied by the caller
 * (device double, e.g. after an all-reduce); info_dev as above. */
int fcu_adam_step_sumsq(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                        const fcu_adam_hyper *h, const double *sumsq_dev, double *info_dev);

/* sumsq_dev[0] (+)= sum g[i]^2 in double, deterministic. */
int fcu_sumsq(fcu_ctx *ctx, const float *g, int64_t n, double *sumsq_dev, int accumulate);

/* The constants of one Adam optimizer (the constructor options of
 * src/L2/autograd.js:215). */
typedef struct {
  double lr, b1, b2, eps, wd, clip, total_steps;
} fcu_adam_sched;

/* One Adam.step whose step counter lives on the device: t = ++t_dev[0], then
 * the cosine lr and bias corrections of step t are computed on the device
 * (src/L2/autograd.js:222,229,237-238), so a captured CUDA graph of a whole
 * training step replays with the right schedule.  Global-norm clipping as
 * fcu_adam_step.  info_dev (3 doubles) receives {gnorm, scale, lr}; p_bf16
 * may be NULL or the bf16 weight copy to refresh. */
int fcu_adam_step_sched(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                        const fcu_adam_sched *s, int32_t *t_dev, double *info_dev, void *p_bf16);

/* The halves of fcu_adam_step_sched, for an update split into pieces (a
 * data-parallel rank's shard of every gradient bucket; no counterpart in the
 * reference, whose Adam is one loop): fcu_adam_sched_advance increments
 * t_dev once and writes that step's constants to h_dev (device memory);
 * fcu_adam_update_dev then updates one piece with them and the caller's
 * gradient sum of squares (the global one, all-reduced over the ranks).
 * info_dev (3 doubles, may be NULL) receives {gnorm, scale, lr}. */
int fcu_adam_sched_advance(fcu_ctx *ctx, const fcu_adam_sched *s, int32_t *t_dev, fcu_adam_hyper *h_dev);
int fcu_adam_update_dev(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                        const fcu_adam_hyper *h_dev, const double *sumsq_dev, double *info_dev,
                        void *p_bf16);

/* Adam (fcu_adam_step semantics) that also writes bf16(p) into p_bf16, the
 * weight copy the bf16 GEMMs read.  sumsq_dev may be NULL (computed here). */
int fcu_adam_step_shadow(fcu_ctx *ctx, float *p, const float *g, float *m, float *v, int64_t n,
                         const fcu_adam_hyper *h, const double *sumsq_dev, double *info_dev,
                         void *p_bf16);

/* ---------------------------------------------------------------- RNG / init (host) */
/* xorshift128+ with splitmix32 seeding, Box-Muller normals: the seeded
 * generator every forge-llm config draws from (RNG, src/L0/numeric.js:27-49).
 * Host functions; they touch no device. */
typedef struct { uint32_t s0, s1; } fcu_rng;
void fcu_rng_init(fcu_rng *r, uint32_t seed);
double fcu_rng_next(fcu_rng *r);
double fcu_rng_normal(fcu_rng *r);
int fcu_rng_int(fcu_rng *r, int n);
/* out[i] = (float)(normal() * scale), i in [0, n): the `Float32Array` fill of
 * initWeights / randArr. */
void fcu_rng_fill_normal(fcu_rng *r, float *host_out, int64_t n, double scale);
void fcu_rng_fill_int(fcu_rng *r, int32_t *host_out, int64_t n, int range);

/* Model shape (Config, src/L6/transformer.js:29-53). */
typedef struct {
  int vocab, dim, n_layers, n_heads, n_kv_heads, hidden;
  double norm_eps, rope_theta;
} fcu_model_cfg;

/* Number of parameters in the flat layout below. */
int64_t fcu_model_num_params(const fcu_model_cfg *cfg);
/* initWeights (src/L6/train.js:33-57) into one flat host array in paramList
 * order (toParams, src/L6/train.js:60-78): tok_emb[V*D], ln_f[D], then per
 * layer ln1[D], ln2[D], wqkv[qkvOut*D], wo[D*qD], ffn_gate[H*D], ffn_up[H*D],
 * ffn_down[D*H]. */
int fcu_init_weights(const fcu_model_cfg *cfg, uint32_t seed, float *host_out);

/* ---------------------------------------------------------------- inference side (decode) */
/* GGML tensor types these kernels read (GGMLType, src/L3/quant.js:34-38).
 * FCU_GGML_Q4_0 / FCU_GGML_Q5_0 are decoded as the reference decodes them
 * (src/L3/quant.js:191-205: f16 d, then nibble j&1 of byte 2 + j/2, Q5_0
 * without its high bits), which is not ggml's own Q4_0 / Q5_0 layout. */
enum {
  FCU_GGML_F32 = 0,
  FCU_GGML_F16 = 1,
  FCU_GGML_Q4_0 = 2,
  FCU_GGML_Q5_0 = 6,
  FCU_GGML_Q8_0 = 8,
  FCU_GGML_Q4_K = 12,
  FCU_GGML_Q5_K = 13,
  FCU_GGML_Q6_K = 14
};
/* Bytes of one row of n elements (rowBytes, src/L3/quant.js:62); -1 for an
 * unsupported type.  Host function. */
int64_t fcu_ggml_row_bytes(int type, int64_t n);
/* Y[m, n] = sum_k W[n, k] X[m, k] for m < M: QuantLinear.forward
 * (src/L4/nn.js:27-32; dotQ src/L3/quant.js:215-310, matvec
 * src/L0/numeric.js:85-100 for F32) applied to M vectors in one pass over W.
 * W: N rows of K elements in GGML blocks (row n at n * fcu_ggml_row_bytes),
 * 16-byte aligned; X [M, K] fp32 16-byte aligned; Y [M, N] fp32.  K a
 * multiple of the type's block (32 or 256; any K for F32 / F16), one row at
 * most 24 KiB, K <= 24576.  fp32 accumulation (the JS accumulates in double). */
int fcu_quant_matvec(fcu_ctx *ctx, int type, const void *W, int64_t N, int64_t K, const float *X, int64_t M,
                     float *Y);
/* out[r, :] = dequantize(row rows[r] of W) (src/L3/quant.js:109-209),
 * bit-identical to the JS; rows NULL: rows 0..nrows-1.  An id outside [0, N)
 * gives a NaN row.  The quantized embedding lookup of
 * src/L6/transformer.js:122-132 is rows = the token ids. */
int fcu_dequantize_rows(fcu_ctx *ctx, int type, const void *W, int64_t N, int64_t K, const int32_t *rows,
                        int64_t nrows, float *out);
/* For each of B sequences, qkv row b ([q heads | k heads | v heads], dH each,
 * row stride ld_qkv floats): RoPE at position positions[b] (device) on the
 * q and k heads in place (applyRopeHead, src/L6/transformer.js:56-64, with
 * the fp32 table of ropeTable, src/L1/special.js:116-127), then k and v
 * written to that position's cache row (KVCache.put / PagedKVCache.put,
 * src/L5/attention.js:135-139, 166-171).  Cache row of position p of
 * sequence b: block_table[b * max_blocks + p / block_size] * block_size +
 * p % block_size (block_table NULL: block b * max_blocks + p / block_size);
 * rows are row_stride floats apart, kv head h at column h * dH.  A position
 * outside [0, max_blocks * block_size) leaves that sequence untouched. */
int fcu_decode_rope_kv(fcu_ctx *ctx, float *qkv, int64_t ld_qkv, int B, int nH, int nKV, int dH, double theta,
                       const int32_t *positions, float *k_cache, float *v_cache, int64_t row_stride,
                       const int32_t *block_table, int max_blocks, int block_size);
/* out[b, h*dH:(h+1)*dH] = attention of q head h of sequence b (q rows ld_q
 * floats apart) over cache positions [0, seq_lens[b]) (device; clamped to
 * max_blocks * block_size) with kv head h / (nH / nKV) and the given scale:
 * the decode loop of src/L6/transformer.js:157-172 with attentionDecode
 * (src/L5/attention.js:31-57).  A length of 0 gives zeros.  dH <= 256,
 * nH / nKV <= 16.  Sequences longer than 256 positions are split across CTAs
 * and merged; the partials use the context's scratch. */
int fcu_attn_decode(fcu_ctx *ctx, const float *q, int64_t ld_q, const float *k_cache, const float *v_cache,
                    int64_t row_stride, const int32_t *block_table, int max_blocks, int block_size,
                    const int32_t *seq_lens, int B, int nH, int nKV, int dH, double scale, float *out);

/* ---------------------------------------------------------------- data-parallel exchange */
/* NCCL over NVLink / NVSwitch, one communicator per GPU.  The reference has no
 * counterpart (it trains on one CPU thread); this is the exchange a
 * data-parallel host wraps around Adam.step (src/L2/autograd.js:214-244) when
 * TrainableTransformer's batch (src/L6/train.js:175-185) is split by sequence
 * over the GPUs: every rank averages the flat gradient buffer, bucket by
 * bucket while its backward continues, then takes the identical Adam step.
 *
 * NCCL is loaded at run time (libnccl.so.2, or the path in FORGECU_NCCL_LIB);
 * FCU_ERR_UNSUPPORTED if it cannot be.  Communicators are non-blocking
 * (ncclConfig_t.blocking = 0): every wait for NCCL is bounded, and a
 * communicator that misses a deadline or reports an asynchronous error is
 * aborted (ncclCommAbort, which also ends its kernels in flight) and the call
 * returns FCU_ERR_TIMEOUT / FCU_ERR_NCCL.  An aborted communicator only
 * accepts fcu_comm_destroy.
 *
 * Collectives are stream-ordered: each one starts on the communicator's own
 * stream once the work already queued on ctx's stream is done (an event), so
 * it overlaps what ctx launches next; fcu_comm_join makes ctx's stream wait
 * for all of them.  The fork and join are legal inside CUDA stream capture. */
typedef struct fcu_comm fcu_comm;
#define FCU_COMM_ID_BYTES 128
/* A fresh NCCL unique id: rank 0 makes it and the host hands the bytes to
 * every rank (a store, MPI, a file ...). */
int fcu_comm_unique_id(void *id_out);
/* Joins the nranks-rank communicator named by id as `rank`, on CUDA device
 * `device` (-1: the calling thread's current device, which must then be the
 * device of the contexts later passed with it).  Waits at most timeout_s for
 * every rank to join. */
int fcu_comm_init(int device, const void *id, int nranks, int rank, double timeout_s, fcu_comm **out);
/* Finalizes (bounded) and frees the communicator; after an abort it only frees. */
int fcu_comm_destroy(fcu_comm *comm);
int fcu_comm_abort(fcu_comm *comm);
/* nranks / rank / device (any output may be NULL); FCU_ERR_NCCL once aborted. */
int fcu_comm_info(const fcu_comm *comm, int *nranks, int *rank, int *device);
/* buf[0..n) = average over the ranks of buf (in place): one gradient bucket,
 * e.g. one layer's contiguous block of the flat gradient buffer. */
int fcu_allreduce_grads(fcu_ctx *ctx, fcu_comm *comm, float *buf, int64_t n);
/* ZeRO-1: rank r's slice buf[r*n/R, (r+1)*n/R) = average over the ranks of
 * that slice of buf (in place; n % nranks == 0). */
int fcu_reduce_scatter_grads(fcu_ctx *ctx, fcu_comm *comm, float *buf, int64_t n);
/* ZeRO-1: every rank's slice buf[r*n/R, (r+1)*n/R) gathered into all of buf
 * (in place); elem_bytes 4 (fp32 parameters) or 2 (their bf16 copy). */
int fcu_allgather_params(fcu_ctx *ctx, fcu_comm *comm, void *buf, int64_t n, int elem_bytes);
/* buf[0..n) = sum over the ranks (fp64, in place): the global gradient sum
 * of squares for Adam's norm clipping. */
int fcu_allreduce_sum_f64(fcu_ctx *ctx, fcu_comm *comm, double *buf, int64_t n);
/* ctx's stream waits for every collective launched on comm so far. */
int fcu_comm_join(fcu_ctx *ctx, fcu_comm *comm);
/* Host check between steps (not during stream capture): FCU_OK once every
 * collective launched since the last poll has finished; FCU_ERR_TIMEOUT if
 * they have not within timeout_s, FCU_ERR_NCCL on an asynchronous error (both
 * abort the communicator). */
int fcu_comm_poll(fcu_comm *comm, double timeout_s);
/* Measurement (no counterpart in the reference): time the next max_records
 * collectives and joins issued outside stream capture with CUDA events (0
 * stops; restarting discards earlier records). */
int fcu_comm_profile(fcu_comm *comm, int max_records);
/* Waits for the recorded events and writes 5 doubles per record: kind (0
 * all-reduce of fp32 gradients, 1 reduce-scatter, 2 all-gather, 3 fp64 sum,
 * 4 join), bytes, then in ms from the first record's ready time: ready (the
 * context's stream reached the call), start and end on the communicator's
 * stream (for a join: when ctx's stream could continue). */
int fcu_comm_profile_read(fcu_comm *comm, double *out, int max_records, int *n_out);

/* ---------------------------------------------------------------- misc */
/* y[i] *= alpha (data-parallel gradient averaging). */
int fcu_scale(fcu_ctx *ctx, float *y, int64_t n, float alpha);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* FORGECU_H */
