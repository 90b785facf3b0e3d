/*
 * forge_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of forge-llm's training hot path, used as the parity
 * checker for the CUDA kernels in forge-llm_b200/csrc.  Nothing in the
 * product links, loads or calls this file: only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline / reference legs of bench.py do.
 *
 * The reference is JavaScript.  Its numeric model is reproduced exactly:
 *   - scalar locals are IEEE double (JS `number`);
 *   - every store into a Float32Array rounds to fp32 (here: a (float) cast);
 *   - products of two fp32 values are exact in double, so loop order alone
 *     fixes every result; the file is built with -ffp-contract=off so no FMA
 *     changes a rounding the JS engine would not make.
 * Loop orders follow the cited JS line for line; where a loop is split for
 * threading, every output element still accumulates its terms in the same
 * order as the JS loop does.
 *
 * Citations are path:line inside the forge-llm project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define OR_API __attribute__((visibility("default")))

static int g_threads = 1;

OR_API void or_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }
OR_API int or_get_threads(void) { return g_threads; }

/* parallel_for(n, body, ctx): body(ctx, i) for i in [0, n), split into
 * g_threads contiguous chunks.  Each index runs exactly once, so results do
 * not depend on the thread count. */
typedef void (*pf_body)(void *ctx, int64_t i);
typedef struct { pf_body body; void *ctx; int64_t lo, hi; } pf_chunk;

static void *pf_run(void *arg) {
  pf_chunk *c = (pf_chunk *)arg;
  for (int64_t i = c->lo; i < c->hi; i++) c->body(c->ctx, i);
  return NULL;
}

static void parallel_for(int64_t n, pf_body body, void *ctx) {
  int nt = g_threads;
  if (nt > n) nt = (int)n;
  if (nt <= 1) {
    for (int64_t i = 0; i < n; i++) body(ctx, i);
    return;
  }
  pthread_t th[256];
  pf_chunk ch[256];
  for (int t = 0; t < nt; t++) {
    ch[t].body = body;
    ch[t].ctx = ctx;
    ch[t].lo = n * t / nt;
    ch[t].hi = n * (t + 1) / nt;
  }
  for (int t = 1; t < nt; t++) pthread_create(&th[t], NULL, pf_run, &ch[t]);
  pf_run(&ch[0]);
  for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------
 * RNG: xorshift128+ (32-bit lanes) seeded by splitmix32.
 * src/L0/numeric.js:27-49
 * ---------------------------------------------------------------------- */
typedef struct { uint32_t s0, s1; } or_rng;

static uint32_t splitmix32_next(uint32_t *s) {
  *s += 0x9e3779b9u;
  uint32_t z = *s;
  z = (z ^ (z >> 16)) * 0x21f0aaadu;
  z = (z ^ (z >> 15)) * 0x735a2d97u;
  return z ^ (z >> 15);
}

OR_API void or_rng_init(or_rng *r, uint32_t seed) {
  uint32_t s = seed ? seed : 1u; /* numeric.js:28  `seed >>> 0 || 1` */
  r->s0 = splitmix32_next(&s);
  r->s1 = splitmix32_next(&s);
}

OR_API double or_rng_next(or_rng *r) { /* numeric.js:34-41 */
  uint32_t x = r->s0, y = r->s1;
  r->s0 = y;
  x ^= x << 23;
  x ^= x >> 17;
  x ^= y;
  x ^= y >> 26;
  r->s1 = x;
  return (double)(uint32_t)(r->s1 + y) / 4294967296.0;
}

OR_API double or_rng_normal(or_rng *r) { /* numeric.js:43-46, Box-Muller */
  double u = or_rng_next(r);
  if (u < 1e-12) u = 1e-12;
  double v = or_rng_next(r);
  return sqrt(-2.0 * log(u)) * cos(2.0 * M_PI * v);
}

OR_API int or_rng_int(or_rng *r, int n) { /* numeric.js:48 */
  return (int)floor(or_rng_next(r) * n);
}

/* out[i] = f32(normal() * scale): verify.js:491-495 randArr, and the
 * `new Float32Array(n).map(() => rng.normal())` pattern of the tests
 * (scale 1). */
OR_API void or_rng_fill_normal(or_rng *r, float *out, int64_t n, double scale) {
  for (int64_t i = 0; i < n; i++) out[i] = (float)(or_rng_normal(r) * scale);
}

OR_API void or_rng_fill_int(or_rng *r, int32_t *out, int64_t n, int range) {
  for (int64_t i = 0; i < n; i++) out[i] = or_rng_int(r, range);
}

/* relL2(a, b) = sqrt(sum (a-b)^2 / sum a^2): numeric.js:152-156 */
OR_API double or_rel_l2(const float *a, const float *b, int64_t n) {
  double ns = 0, ds = 0;
  for (int64_t i = 0; i < n; i++) {
    double d = (double)a[i] - (double)b[i];
    ns += d * d;
    ds += (double)a[i] * (double)a[i];
  }
  return sqrt(ns / (ds != 0 ? ds : 1));
}

/* ------------------------------------------------------------------------
 * gemm: C[M,N] = A[M,K] . B[N,K]^T with four double partial sums.
 * src/L0/numeric.js:111-129.  matmulT's forward is exactly this call
 * (src/L2/tensor.js:34-36).
 * ---------------------------------------------------------------------- */
static inline float gemm_dot(const float *a, const float *b, int64_t K) {
  double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  int64_t k = 0;
  for (; k + 4 <= K; k += 4) {
    s0 += (double)a[k] * (double)b[k];
    s1 += (double)a[k + 1] * (double)b[k + 1];
    s2 += (double)a[k + 2] * (double)b[k + 2];
    s3 += (double)a[k + 3] * (double)b[k + 3];
  }
  double s = s0 + s1 + s2 + s3;
  for (; k < K; k++) s += (double)a[k] * (double)b[k];
  return (float)s;
}

typedef struct { float *C; const float *A, *B; int64_t N, K; } gemm_ctx;

static void gemm_row(void *p, int64_t m) {
  gemm_ctx *c = (gemm_ctx *)p;
  for (int64_t n = 0; n < c->N; n++) c->C[m * c->N + n] = gemm_dot(c->A + m * c->K, c->B + n * c->K, c->K);
}

OR_API void or_gemm(float *C, const float *A, const float *B, int64_t M, int64_t N, int64_t K) {
  gemm_ctx c = {C, A, B, N, K};
  parallel_for(M, gemm_row, &c);
}

/* matmulT backward, src/L2/tensor.js:37-52:
 *   for m, for n (skip g==0), for k: gX[m,k] += g*W[n,k]; gW[n,k] += g*X[m,k]
 * Every gX element accumulates in ascending n and every gW element in
 * ascending m, so the two halves can run as separate loops. */
typedef struct { const float *g, *W, *X; float *out; int64_t M, K, N, n0; } mmb_ctx;

static void mmb_dx_row(void *p, int64_t m) {
  mmb_ctx *c = (mmb_ctx *)p;
  float *gx = c->out + m * c->K;
  const float *gr = c->g + m * c->N;
  for (int64_t n = 0; n < c->N; n++) {
    float gn = gr[n];
    if (gn == 0.0f) continue;
    const float *w = c->W + n * c->K;
    for (int64_t k = 0; k < c->K; k++) gx[k] = (float)((double)gx[k] + (double)gn * (double)w[k]);
  }
}

static void mmb_dw_row(void *p, int64_t i) {
  mmb_ctx *c = (mmb_ctx *)p;
  int64_t n = c->n0 + i;
  float *gw = c->out + n * c->K;
  for (int64_t m = 0; m < c->M; m++) {
    float gn = c->g[m * c->N + n];
    if (gn == 0.0f) continue;
    const float *x = c->X + m * c->K;
    for (int64_t k = 0; k < c->K; k++) gw[k] = (float)((double)gw[k] + (double)gn * (double)x[k]);
  }
}

OR_API void or_matmulT_bwd_dx(const float *g, const float *W, float *gX, int64_t M, int64_t K,
                              int64_t N) {
  mmb_ctx c = {g, W, NULL, gX, M, K, N, 0};
  parallel_for(M, mmb_dx_row, &c);
}

/* Rows [n0, n1) of gW only (the full range is n0=0, n1=N). */
OR_API void or_matmulT_bwd_dw(const float *g, const float *X, float *gW, int64_t M, int64_t K,
                              int64_t N, int64_t n0, int64_t n1) {
  mmb_ctx c = {g, NULL, X, gW, M, K, N, n0};
  parallel_for(n1 - n0, mmb_dw_row, &c);
}

OR_API void or_matmulT_bwd(const float *g, const float *X, const float *W, float *gX, float *gW,
                           int64_t M, int64_t K, int64_t N) {
  or_matmulT_bwd_dx(g, W, gX, M, K, N);
  or_matmulT_bwd_dw(g, X, gW, M, K, N, 0, N);
}

/* ------------------------------------------------------------------------
 * embedLookup, src/L2/tensor.js:85-99
 * ---------------------------------------------------------------------- */
OR_API void or_embed_fwd(const float *W, const int32_t *ids, int64_t T, int64_t D, float *out) {
  for (int64_t t = 0; t < T; t++) memcpy(out + t * D, W + (int64_t)ids[t] * D, D * sizeof(float));
}

OR_API void or_embed_bwd(const float *g, const int32_t *ids, int64_t T, int64_t V, int64_t D,
                         float *gW) {
  for (int64_t t = 0; t < T; t++) {
    /* tensor.js:94-96: an out-of-range id indexes outside the Float32Array,
     * whose store is a no-op. */
    if (ids[t] < 0 || (int64_t)ids[t] >= V) continue;
    float *o = gW + (int64_t)ids[t] * D;
    const float *gr = g + t * D;
    for (int64_t d = 0; d < D; d++) o[d] = (float)((double)o[d] + (double)gr[d]);
  }
}

/* ------------------------------------------------------------------------
 * rmsNorm, src/L2/tensor.js:103-128.  inv[t] is a Float32Array in the JS.
 * ---------------------------------------------------------------------- */
OR_API void or_rmsnorm_fwd(const float *X, const float *w, int64_t T, int64_t D, double eps,
                           float *out, float *inv) {
  for (int64_t t = 0; t < T; t++) {
    const float *x = X + t * D;
    double ss = 0;
    for (int64_t i = 0; i < D; i++) ss += (double)x[i] * (double)x[i];
    double r = sqrt(ss / (double)D + eps);
    inv[t] = (float)(1.0 / r);
    double iv = (double)inv[t];
    for (int64_t i = 0; i < D; i++) out[t * D + i] = (float)((double)x[i] * iv * (double)w[i]);
  }
}

OR_API void or_rmsnorm_bwd(const float *g, const float *X, const float *w, const float *inv,
                           int64_t T, int64_t D, float *gX, float *gw) {
  for (int64_t t = 0; t < T; t++) {
    const float *x = X + t * D, *gr = g + t * D;
    double iv = (double)inv[t];
    double r = 1.0 / iv;
    double dot = 0;
    for (int64_t i = 0; i < D; i++) dot += (double)gr[i] * (double)w[i] * (double)x[i];
    double c = dot / ((double)D * r * r * r);
    for (int64_t i = 0; i < D; i++) {
      gX[t * D + i] = (float)((double)gX[t * D + i] +
                              ((double)gr[i] * (double)w[i] * iv - c * (double)x[i]));
      gw[i] = (float)((double)gw[i] + (double)gr[i] * (double)x[i] * iv);
    }
  }
}

/* ------------------------------------------------------------------------
 * ropeRows, src/L2/tensor.js:133-166: interleaved pairs, pos = pos0 +
 * (posStride > 0 ? t % posStride : t), freq = 1 / theta^(i/dHead).
 * ---------------------------------------------------------------------- */
OR_API void or_rope_fwd(const float *X, int64_t T, int nHead, int dHead, int pos0, double theta,
                        int posStride, float *out) {
  int64_t D = (int64_t)nHead * dHead;
  memcpy(out, X, T * D * sizeof(float));
  for (int64_t t = 0; t < T; t++) {
    double pos = (double)pos0 + (double)(posStride > 0 ? (t % posStride) : t);
    for (int h = 0; h < nHead; h++) {
      float *o = out + t * D + (int64_t)h * dHead;
      for (int i = 0; i < dHead; i += 2) {
        double freq = 1.0 / pow(theta, (double)i / (double)dHead);
        double ang = pos * freq, c = cos(ang), s = sin(ang);
        double a = o[i], b = o[i + 1];
        o[i] = (float)(a * c - b * s);
        o[i + 1] = (float)(a * s + b * c);
      }
    }
  }
}

OR_API void or_rope_bwd(const float *g, int64_t T, int nHead, int dHead, int pos0, double theta,
                        int posStride, float *gX) {
  int64_t D = (int64_t)nHead * dHead;
  for (int64_t t = 0; t < T; t++) {
    double pos = (double)pos0 + (double)(posStride > 0 ? (t % posStride) : t);
    for (int h = 0; h < nHead; h++) {
      int64_t hb = t * D + (int64_t)h * dHead;
      for (int i = 0; i < dHead; i += 2) {
        double freq = 1.0 / pow(theta, (double)i / (double)dHead);
        double ang = pos * freq, c = cos(ang), s = sin(ang);
        double ga = g[hb + i], gb = g[hb + i + 1];
        gX[hb + i] = (float)((double)gX[hb + i] + (ga * c + gb * s));
        gX[hb + i + 1] = (float)((double)gX[hb + i + 1] + (-ga * s + gb * c));
      }
    }
  }
}

/* ------------------------------------------------------------------------
 * sliceCols, src/L2/tensor.js:170-183
 * ---------------------------------------------------------------------- */
OR_API void or_slicecols_fwd(const float *X, int64_t M, int64_t K, int64_t off, int64_t len,
                             float *out) {
  for (int64_t m = 0; m < M; m++) memcpy(out + m * len, X + m * K + off, len * sizeof(float));
}

OR_API void or_slicecols_bwd(const float *g, int64_t M, int64_t K, int64_t off, int64_t len,
                             float *gX) {
  for (int64_t m = 0; m < M; m++)
    for (int64_t i = 0; i < len; i++) {
      float *p = gX + m * K + off + i;
      *p = (float)((double)*p + (double)g[m * len + i]);
    }
}

/* ------------------------------------------------------------------------
 * Causal attention with GQA, one sequence (B = 1: causalAttn,
 * src/L2/tensor.js:191-268) or B sequences under the block-diagonal causal
 * mask (causalAttnBatch, src/L2/tensor.js:299-376).  The two JS functions do
 * the same arithmetic per element; B = 1 reproduces causalAttn.
 * P is [B, nH, T, T] fp32 (the JS stores it, :197 / :305).
 * ---------------------------------------------------------------------- */
typedef struct {
  const float *Q, *K, *V, *g, *Pc;
  float *out, *P, *gQ, *gK, *gV;
  int B, T, nH, nKV, dH, group;
  double scale;
} attn_ctx;

static void attn_fwd_head(void *p, int64_t bh) {
  attn_ctx *c = (attn_ctx *)p;
  const int T = c->T, nH = c->nH, dH = c->dH;
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)c->nKV * dH;
  int b = (int)(bh / nH), h = (int)(bh % nH);
  int64_t base = (int64_t)b * T;
  int kvh = h / c->group;
  float *Pb = c->P + bh * (int64_t)T * T;
  float *s = (float *)malloc(sizeof(float) * (size_t)T);
  for (int t = 0; t < T; t++) {
    const float *q = c->Q + (base + t) * qD + (int64_t)h * dH;
    double mx = -INFINITY;
    for (int j = 0; j <= t; j++) {
      const float *k = c->K + (base + j) * kvD + (int64_t)kvh * dH;
      double acc = 0;
      for (int d = 0; d < dH; d++) acc += (double)q[d] * (double)k[d];
      acc *= c->scale;
      s[j] = (float)acc;
      if (acc > mx) mx = acc;
    }
    double sum = 0;
    for (int j = 0; j <= t; j++) {
      s[j] = (float)exp((double)s[j] - mx);
      sum += (double)s[j];
    }
    double inv = 1.0 / sum;
    for (int j = 0; j <= t; j++) {
      s[j] = (float)((double)s[j] * inv);
      Pb[(int64_t)t * T + j] = s[j];
    }
    float *o = c->out + (base + t) * qD + (int64_t)h * dH;
    for (int j = 0; j <= t; j++) {
      double pj = s[j];
      if (pj == 0) continue;
      const float *v = c->V + (base + j) * kvD + (int64_t)kvh * dH;
      for (int d = 0; d < dH; d++) o[d] = (float)((double)o[d] + pj * (double)v[d]);
    }
  }
  free(s);
}

OR_API void or_attn_fwd(const float *Q, const float *K, const float *V, int B, int T, int nH,
                        int nKV, int dH, float *out, float *P) {
  attn_ctx c;
  memset(&c, 0, sizeof c);
  c.Q = Q; c.K = K; c.V = V; c.out = out; c.P = P;
  c.B = B; c.T = T; c.nH = nH; c.nKV = nKV; c.dH = dH;
  c.group = nH / nKV < 1 ? 1 : nH / nKV;
  c.scale = 1.0 / sqrt((double)dH);
  memset(out, 0, sizeof(float) * (int64_t)B * T * nH * dH);
  parallel_for((int64_t)B * nH, attn_fwd_head, &c);
}

/* Backward.  Threads split over (sequence, kv head); inside a kv head the
 * group's q heads run in ascending h, so each gK / gV element receives its
 * terms in the same (h, t) order as the JS loop. */
static void attn_bwd_kvhead(void *p, int64_t bk) {
  attn_ctx *c = (attn_ctx *)p;
  const int T = c->T, nH = c->nH, nKV = c->nKV, dH = c->dH, group = c->group;
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)nKV * dH;
  const double scale = c->scale;
  int b = (int)(bk / nKV), kvh = (int)(bk % nKV);
  int64_t base = (int64_t)b * T;
  float *dP = (float *)malloc(sizeof(float) * (size_t)T);
  for (int h = kvh * group; h < (kvh + 1) * group && h < nH; h++) {
    const float *Pb = c->Pc + ((int64_t)b * nH + h) * (int64_t)T * T;
    for (int t = 0; t < T; t++) {
      const float *go = c->g + (base + t) * qD + (int64_t)h * dH;
      double dotP = 0;
      for (int j = 0; j <= t; j++) {
        const float *v = c->V + (base + j) * kvD + (int64_t)kvh * dH;
        double acc = 0;
        for (int d = 0; d < dH; d++) acc += (double)go[d] * (double)v[d];
        dP[j] = (float)acc;
        dotP += acc * (double)Pb[(int64_t)t * T + j];
      }
      const float *q = c->Q + (base + t) * qD + (int64_t)h * dH;
      float *gq = c->gQ + (base + t) * qD + (int64_t)h * dH;
      for (int j = 0; j <= t; j++) {
        double pj = Pb[(int64_t)t * T + j];
        if (pj == 0) continue;
        double dS = pj * ((double)dP[j] - dotP);
        float *gv = c->gV + (base + j) * kvD + (int64_t)kvh * dH;
        const float *k = c->K + (base + j) * kvD + (int64_t)kvh * dH;
        float *gk = c->gK + (base + j) * kvD + (int64_t)kvh * dH;
        for (int d = 0; d < dH; d++) gv[d] = (float)((double)gv[d] + pj * (double)go[d]);
        for (int d = 0; d < dH; d++) {
          gq[d] = (float)((double)gq[d] + dS * (double)k[d] * scale);
          gk[d] = (float)((double)gk[d] + dS * (double)q[d] * scale);
        }
      }
    }
  }
  free(dP);
}

OR_API void or_attn_bwd(const float *g, const float *Q, const float *K, const float *V,
                        const float *P, int B, int T, int nH, int nKV, int dH, float *gQ,
                        float *gK, float *gV) {
  attn_ctx c;
  memset(&c, 0, sizeof c);
  c.g = g; c.Q = Q; c.K = K; c.V = V; c.Pc = P; c.gQ = gQ; c.gK = gK; c.gV = gV;
  c.B = B; c.T = T; c.nH = nH; c.nKV = nKV; c.dH = dH;
  c.group = nH / nKV < 1 ? 1 : nH / nKV;
  c.scale = 1.0 / sqrt((double)dH);
  parallel_for((int64_t)B * nKV, attn_bwd_kvhead, &c);
}

/* ------------------------------------------------------------------------
 * swigluRows, src/L2/tensor.js:272-290.  The forward multiplies with the
 * double sigmoid; the backward reads the fp32-stored one.
 * ---------------------------------------------------------------------- */
OR_API void or_swiglu_fwd(const float *G, const float *U, int64_t n, float *out, float *sig) {
  for (int64_t i = 0; i < n; i++) {
    double g = G[i];
    double s = 1.0 / (1.0 + exp(-g));
    sig[i] = (float)s;
    out[i] = (float)(g * s * (double)U[i]);
  }
}

OR_API void or_swiglu_bwd(const float *g, const float *G, const float *U, const float *sig,
                          int64_t n, float *gG, float *gU) {
  for (int64_t i = 0; i < n; i++) {
    double s = sig[i], gv = G[i], gi = g[i];
    gG[i] = (float)((double)gG[i] + gi * (double)U[i] * (s + gv * s * (1.0 - s)));
    gU[i] = (float)((double)gU[i] + gi * (gv * s));
  }
}

/* ------------------------------------------------------------------------
 * crossEntropyMean, src/L2/tensor.js:393-417.  Returns the fp32 loss;
 * probs [T,V] is the normalised softmax the backward reads.
 * ---------------------------------------------------------------------- */
OR_API float or_ce_fwd(const float *logits, const int32_t *targets, int64_t T, int64_t V,
                       float *probs) {
  double loss = 0;
  for (int64_t t = 0; t < T; t++) {
    const float *l = logits + t * V;
    float *p = probs + t * V;
    double mx = -INFINITY;
    for (int64_t i = 0; i < V; i++)
      if ((double)l[i] > mx) mx = l[i];
    double s = 0;
    for (int64_t i = 0; i < V; i++) {
      double e = exp((double)l[i] - mx);
      p[i] = (float)e;
      s += e;
    }
    double lse = mx + log(s);
    loss += -((double)l[targets[t]] - lse);
    for (int64_t i = 0; i < V; i++) p[i] = (float)((double)p[i] / s);
  }
  return (float)(loss / (double)T);
}

OR_API void or_ce_bwd(float gout, const float *probs, const int32_t *targets, int64_t T,
                      int64_t V, float *gL) {
  double k = (double)gout / (double)T;
  for (int64_t t = 0; t < T; t++) {
    float *gl = gL + t * V;
    const float *p = probs + t * V;
    for (int64_t i = 0; i < V; i++) gl[i] = (float)((double)gl[i] + k * (double)p[i]);
    gl[targets[t]] = (float)((double)gl[targets[t]] - k);
  }
}

/* ------------------------------------------------------------------------
 * weightedSum, src/L2/tensor.js:380-389: out is a Float32Array(1), so the
 * running sum is rounded to fp32 after every term.
 * ---------------------------------------------------------------------- */
OR_API float or_wsum_fwd(const float *Y, const float *t, int64_t n) {
  float out = 0;
  for (int64_t i = 0; i < n; i++) out = (float)((double)out + (double)Y[i] * (double)t[i]);
  return out;
}

OR_API void or_wsum_bwd(float gout, const float *t, int64_t n, float *gY) {
  double k = gout;
  for (int64_t i = 0; i < n; i++) gY[i] = (float)((double)gY[i] + k * (double)t[i]);
}

/* ------------------------------------------------------------------------
 * linear (out[N] = W[N,K] . x) and softmaxCE, used by invariant I-30.
 * src/L2/autograd.js:47-58 (matvec src/L0/numeric.js:85-100) and :110-124.
 * ---------------------------------------------------------------------- */
OR_API void or_linear_fwd(const float *W, const float *x, int64_t N, int64_t K, float *out) {
  for (int64_t n = 0; n < N; n++) out[n] = gemm_dot(W + n * K, x, K);
}

OR_API void or_linear_bwd(const float *g, const float *W, const float *x, int64_t N, int64_t K,
                          float *gW, float *gx) {
  for (int64_t n = 0; n < N; n++) {
    double gn = g[n];
    for (int64_t k = 0; k < K; k++) {
      gW[n * K + k] = (float)((double)gW[n * K + k] + gn * (double)x[k]);
      gx[k] = (float)((double)gx[k] + gn * (double)W[n * K + k]);
    }
  }
}

OR_API float or_softmaxce_fwd(const float *logits, int64_t n, int target, float *p) {
  double m = -INFINITY;
  for (int64_t i = 0; i < n; i++)
    if ((double)logits[i] > m) m = logits[i];
  double s = 0;
  for (int64_t i = 0; i < n; i++) {
    p[i] = (float)exp((double)logits[i] - m);
    s += (double)p[i];
  }
  for (int64_t i = 0; i < n; i++) p[i] = (float)((double)p[i] / s);
  double pt = p[target];
  if (pt < 1e-40) pt = 1e-40;
  return (float)(-log(pt));
}

OR_API void or_softmaxce_bwd(float gout, const float *p, int64_t n, int target, float *gl) {
  double k = gout;
  for (int64_t i = 0; i < n; i++)
    gl[i] = (float)((double)gl[i] + k * ((double)p[i] - (i == target ? 1.0 : 0.0)));
}

/* ------------------------------------------------------------------------
 * Adam with global-norm clipping and cosine lr, src/L2/autograd.js:214-244,
 * over one flat vector that concatenates the params in paramList order (the
 * JS sums squares and updates params in that same order).  `t` is the step
 * counter AFTER the increment (autograd.js:222).  info = {lr, gnorm, scale}.
 * ---------------------------------------------------------------------- */
OR_API void or_adam_step(float *p, const float *grad, float *m, float *v, int64_t n, int t,
                         double lr0, double b1, double b2, double eps, double wd, double clip,
                         double total, double *info) {
  double tot = 0;
  for (int64_t i = 0; i < n; i++) tot += (double)grad[i] * (double)grad[i];
  double gnorm = sqrt(tot);
  double scale = gnorm > clip ? clip / gnorm : 1.0;
  double tt = (double)t / total;
  if (tt > 1) tt = 1;
  double lr = lr0 * 0.5 * (1.0 + cos(M_PI * tt));
  double bc1 = 1.0 - pow(b1, (double)t), bc2 = 1.0 - pow(b2, (double)t);
  for (int64_t i = 0; i < n; i++) {
    double g = (double)grad[i] * scale + wd * (double)p[i];
    m[i] = (float)(b1 * (double)m[i] + (1.0 - b1) * g);
    v[i] = (float)(b2 * (double)v[i] + (1.0 - b2) * g * g);
    double mh = (double)m[i] / bc1;
    double vh = (double)v[i] / bc2;
    p[i] = (float)((double)p[i] - lr * mh / (sqrt(vh) + eps));
  }
  info[0] = lr;
  info[1] = gnorm;
  info[2] = scale;
}

/* ------------------------------------------------------------------------
 * TrainableTransformer (src/L6/train.js:33-185) over a flat parameter
 * vector in toParams order (train.js:60-78):
 *   tok_emb[V*D], ln_f[D], then per layer ln1[D], ln2[D], wqkv[qkvOut*D],
 *   wo[D*qD], ffn_gate[H*D], ffn_up[H*D], ffn_down[D*H].
 * The LM head is tied to tok_emb (train.js:97).
 * ---------------------------------------------------------------------- */
typedef struct {
  int vocab, dim, n_layers, n_heads, n_kv_heads, hidden;
  double norm_eps, rope_theta;
} or_cfg;

typedef struct {
  int64_t tok_emb, ln_f;
  int64_t ln1, ln2, wqkv, wo, gate, up, down; /* offsets of layer 0 */
  int64_t layer_stride, total;
} or_layout;

static void or_make_layout(const or_cfg *c, or_layout *L) {
  int64_t D = c->dim, V = c->vocab, H = c->hidden;
  int64_t dH = c->dim / c->n_heads;
  int64_t qD = (int64_t)c->n_heads * dH;
  int64_t qkvOut = (int64_t)(c->n_heads + 2 * c->n_kv_heads) * dH;
  L->tok_emb = 0;
  L->ln_f = V * D;
  int64_t o = V * D + D;
  L->ln1 = o;
  L->ln2 = o + D;
  L->wqkv = o + 2 * D;
  L->wo = L->wqkv + qkvOut * D;
  L->gate = L->wo + D * qD;
  L->up = L->gate + H * D;
  L->down = L->up + H * D;
  L->layer_stride = (L->down + D * H) - o;
  L->total = o + L->layer_stride * c->n_layers;
}

OR_API int64_t or_model_num_params(const or_cfg *c) {
  or_layout L;
  or_make_layout(c, &L);
  return L.total;
}

/* initWeights, src/L6/train.js:33-57: one RNG, draws in the order
 * tok_emb, then per layer wqkv, wo (scaled by 1/sqrt(2L)), gate, up,
 * down (scaled); norm weights are ones. */
OR_API void or_init_weights(const or_cfg *c, uint32_t seed, float *P) {
  or_layout L;
  or_make_layout(c, &L);
  or_rng r;
  or_rng_init(&r, seed);
  const double std = 0.02;
  const double res = 1.0 / sqrt(2.0 * c->n_layers);
  int64_t D = c->dim, H = c->hidden;
  int64_t dH = c->dim / c->n_heads, qD = (int64_t)c->n_heads * dH;
  int64_t qkvOut = (int64_t)(c->n_heads + 2 * c->n_kv_heads) * dH;
  for (int64_t i = 0; i < (int64_t)c->vocab * D; i++) P[L.tok_emb + i] = (float)(or_rng_normal(&r) * std);
  for (int64_t i = 0; i < D; i++) P[L.ln_f + i] = 1.0f;
  for (int l = 0; l < c->n_layers; l++) {
    int64_t off = (int64_t)l * L.layer_stride;
    for (int64_t i = 0; i < D; i++) P[off + L.ln1 + i] = 1.0f;
    for (int64_t i = 0; i < D; i++) P[off + L.ln2 + i] = 1.0f;
    for (int64_t i = 0; i < qkvOut * D; i++) P[off + L.wqkv + i] = (float)(or_rng_normal(&r) * std);
    /* wo: dim*dim draws (train.js:50), the layout size D*qD equals it */
    for (int64_t i = 0; i < D * qD; i++) P[off + L.wo + i] = (float)(or_rng_normal(&r) * std);
    for (int64_t i = 0; i < D * qD; i++) P[off + L.wo + i] = (float)((double)P[off + L.wo + i] * res);
    for (int64_t i = 0; i < H * D; i++) P[off + L.gate + i] = (float)(or_rng_normal(&r) * std);
    for (int64_t i = 0; i < H * D; i++) P[off + L.up + i] = (float)(or_rng_normal(&r) * std);
    for (int64_t i = 0; i < D * H; i++) P[off + L.down + i] = (float)(or_rng_normal(&r) * std);
    for (int64_t i = 0; i < D * H; i++) P[off + L.down + i] = (float)((double)P[off + L.down + i] * res);
  }
}

static float *zalloc(int64_t n) { return (float *)calloc((size_t)(n > 0 ? n : 1), sizeof(float)); }

static void add_into(float *dst, const float *src, int64_t n) {
  for (int64_t i = 0; i < n; i++) dst[i] = (float)((double)dst[i] + (double)src[i]);
}

/* One forward (+ loss) and, when G != NULL, one backward of
 * TrainableTransformer.lossBatch (train.js:177-185; B == 1 is loss(),
 * train.js:166-171).  ids/targets are [B*T].  Gradients ACCUMULATE into G
 * (the JS `+=`, zeroGrad is the caller's job).  The backward replays the
 * tape in reverse creation order (autograd.js:126-133); where two ops feed
 * one tensor, its grad receives their terms in that reverse order.
 * If logits_out != NULL the [B*T, V] logits are copied there.
 * Returns the fp32 loss. */
OR_API float or_model_step(const or_cfg *c, const float *P, float *G, const int32_t *ids,
                           const int32_t *targets, int B, int T, float *logits_out) {
  or_layout Lo;
  or_make_layout(c, &Lo);
  const int64_t D = c->dim, V = c->vocab, H = c->hidden, N = (int64_t)B * T;
  const int nH = c->n_heads, nKV = c->n_kv_heads, dH = c->dim / c->n_heads;
  const int64_t qD = (int64_t)nH * dH, kvD = (int64_t)nKV * dH;
  const int64_t qkvOut = qD + 2 * kvD;
  const int nL = c->n_layers;
  const double eps = c->norm_eps, theta = c->rope_theta;

  typedef struct {
    float *x_in, *xn, *inv1, *qkv, *q, *k, *v, *qr, *kr, *att, *Pm, *ao, *x1, *xn2, *inv2, *g, *u,
        *sig, *act, *ff;
  } layer_act;
  layer_act *A = (layer_act *)calloc((size_t)nL, sizeof(layer_act));

  /* ---- forward, train.js:120-159 ---- */
  float *x = zalloc(N * D);
  or_embed_fwd(P + Lo.tok_emb, ids, N, D, x);
  for (int l = 0; l < nL; l++) {
    const int64_t off = (int64_t)l * Lo.layer_stride;
    layer_act *a = &A[l];
    a->x_in = x;
    a->xn = zalloc(N * D);
    a->inv1 = zalloc(N);
    or_rmsnorm_fwd(x, P + off + Lo.ln1, N, D, eps, a->xn, a->inv1);
    a->qkv = zalloc(N * qkvOut);
    or_gemm(a->qkv, a->xn, P + off + Lo.wqkv, N, qkvOut, D);
    a->q = zalloc(N * qD);
    a->k = zalloc(N * kvD);
    a->v = zalloc(N * kvD);
    or_slicecols_fwd(a->qkv, N, qkvOut, 0, qD, a->q);
    or_slicecols_fwd(a->qkv, N, qkvOut, qD, kvD, a->k);
    or_slicecols_fwd(a->qkv, N, qkvOut, qD + kvD, kvD, a->v);
    a->qr = zalloc(N * qD);
    a->kr = zalloc(N * kvD);
    or_rope_fwd(a->q, N, nH, dH, 0, theta, T, a->qr);
    or_rope_fwd(a->k, N, nKV, dH, 0, theta, T, a->kr);
    a->att = zalloc(N * qD);
    a->Pm = zalloc((int64_t)B * nH * T * T);
    or_attn_fwd(a->qr, a->kr, a->v, B, T, nH, nKV, dH, a->att, a->Pm);
    a->ao = zalloc(N * D);
    or_gemm(a->ao, a->att, P + off + Lo.wo, N, D, qD);
    a->x1 = zalloc(N * D);
    for (int64_t i = 0; i < N * D; i++) a->x1[i] = (float)((double)x[i] + (double)a->ao[i]);
    a->xn2 = zalloc(N * D);
    a->inv2 = zalloc(N);
    or_rmsnorm_fwd(a->x1, P + off + Lo.ln2, N, D, eps, a->xn2, a->inv2);
    a->g = zalloc(N * H);
    a->u = zalloc(N * H);
    or_gemm(a->g, a->xn2, P + off + Lo.gate, N, H, D);
    or_gemm(a->u, a->xn2, P + off + Lo.up, N, H, D);
    a->act = zalloc(N * H);
    a->sig = zalloc(N * H);
    or_swiglu_fwd(a->g, a->u, N * H, a->act, a->sig);
    a->ff = zalloc(N * D);
    or_gemm(a->ff, a->act, P + off + Lo.down, N, D, H);
    float *x2 = zalloc(N * D);
    for (int64_t i = 0; i < N * D; i++) x2[i] = (float)((double)a->x1[i] + (double)a->ff[i]);
    x = x2;
  }
  float *xf = zalloc(N * D), *invf = zalloc(N);
  or_rmsnorm_fwd(x, P + Lo.ln_f, N, D, eps, xf, invf);
  float *logits = zalloc(N * V);
  or_gemm(logits, xf, P + Lo.tok_emb, N, V, D);
  float *probs = zalloc(N * V);
  float loss = or_ce_fwd(logits, targets, N, V, probs);
  if (logits_out) memcpy(logits_out, logits, sizeof(float) * N * V);

  /* ---- backward (reverse tape) ---- */
  if (G) {
    float *gLogits = zalloc(N * V);
    or_ce_bwd(1.0f, probs, targets, N, V, gLogits);
    float *gxf = zalloc(N * D);
    or_matmulT_bwd(gLogits, xf, P + Lo.tok_emb, gxf, G + Lo.tok_emb, N, D, V);
    free(gLogits);
    float *gx = zalloc(N * D); /* grad of the last residual output */
    or_rmsnorm_bwd(gxf, x, P + Lo.ln_f, invf, N, D, gx, G + Lo.ln_f);
    free(gxf);
    for (int l = nL - 1; l >= 0; l--) {
      const int64_t off = (int64_t)l * Lo.layer_stride;
      layer_act *a = &A[l];
      /* x2 = add(x1, ff) */
      float *gx1 = zalloc(N * D), *gff = zalloc(N * D);
      add_into(gx1, gx, N * D);
      add_into(gff, gx, N * D);
      free(gx);
      /* ff = matmulT(act, down) */
      float *gact = zalloc(N * H);
      or_matmulT_bwd(gff, a->act, P + off + Lo.down, gact, G + off + Lo.down, N, H, D);
      free(gff);
      /* act = swiglu(g, u) */
      float *gg = zalloc(N * H), *gu = zalloc(N * H);
      or_swiglu_bwd(gact, a->g, a->u, a->sig, N * H, gg, gu);
      free(gact);
      /* u = matmulT(xn2, up) was created after g = matmulT(xn2, gate) */
      float *gxn2 = zalloc(N * D);
      or_matmulT_bwd(gu, a->xn2, P + off + Lo.up, gxn2, G + off + Lo.up, N, D, H);
      or_matmulT_bwd(gg, a->xn2, P + off + Lo.gate, gxn2, G + off + Lo.gate, N, D, H);
      free(gg);
      free(gu);
      /* xn2 = rmsNorm(x1, ln2) */
      or_rmsnorm_bwd(gxn2, a->x1, P + off + Lo.ln2, a->inv2, N, D, gx1, G + off + Lo.ln2);
      free(gxn2);
      /* x1 = add(x_in, ao) */
      float *gxin = zalloc(N * D), *gao = zalloc(N * D);
      add_into(gxin, gx1, N * D);
      add_into(gao, gx1, N * D);
      free(gx1);
      /* ao = matmulT(att, wo) */
      float *gatt = zalloc(N * qD);
      or_matmulT_bwd(gao, a->att, P + off + Lo.wo, gatt, G + off + Lo.wo, N, qD, D);
      free(gao);
      /* att = attn(qr, kr, v) */
      float *gqr = zalloc(N * qD), *gkr = zalloc(N * kvD), *gv = zalloc(N * kvD);
      or_attn_bwd(gatt, a->qr, a->kr, a->v, a->Pm, B, T, nH, nKV, dH, gqr, gkr, gv);
      free(gatt);
      /* kr = rope(k), then qr = rope(q) */
      float *gk = zalloc(N * kvD), *gq = zalloc(N * qD);
      or_rope_bwd(gkr, N, nKV, dH, 0, theta, T, gk);
      or_rope_bwd(gqr, N, nH, dH, 0, theta, T, gq);
      free(gkr);
      free(gqr);
      /* v, k, q = sliceCols(qkv) (reverse creation order) */
      float *gqkv = zalloc(N * qkvOut);
      or_slicecols_bwd(gv, N, qkvOut, qD + kvD, kvD, gqkv);
      or_slicecols_bwd(gk, N, qkvOut, qD, kvD, gqkv);
      or_slicecols_bwd(gq, N, qkvOut, 0, qD, gqkv);
      free(gv);
      free(gk);
      free(gq);
      /* qkv = matmulT(xn, wqkv) */
      float *gxn = zalloc(N * D);
      or_matmulT_bwd(gqkv, a->xn, P + off + Lo.wqkv, gxn, G + off + Lo.wqkv, N, D, qkvOut);
      free(gqkv);
      /* xn = rmsNorm(x_in, ln1) */
      or_rmsnorm_bwd(gxn, a->x_in, P + off + Lo.ln1, a->inv1, N, D, gxin, G + off + Lo.ln1);
      free(gxn);
      gx = gxin;
    }
    /* x = embedLookup(tok_emb, ids) */
    or_embed_bwd(gx, ids, N, c->vocab, D, G + Lo.tok_emb);
    free(gx);
  }

  /* ---- free ---- */
  for (int l = 0; l < nL; l++) {
    layer_act *a = &A[l];
    free(a->x_in);
    free(a->xn); free(a->inv1); free(a->qkv); free(a->q); free(a->k); free(a->v);
    free(a->qr); free(a->kr); free(a->att); free(a->Pm); free(a->ao); free(a->x1);
    free(a->xn2); free(a->inv2); free(a->g); free(a->u); free(a->sig); free(a->act); free(a->ff);
  }
  free(x);
  free(A);
  free(xf); free(invf); free(logits); free(probs);
  return loss;
}
