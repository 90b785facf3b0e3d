/*
 * forge_oracle_infer.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of forge-llm's inference-side kernels: the GGUF block
 * formats of src/L3/quant.js (quantizers, dequantize, dotQ), matvec and dot
 * (src/L0/numeric.js), QuantLinear.forward (src/L4/nn.js:27-32), the three
 * single-query attentions of src/L5/attention.js, the vector rmsnorm /
 * softmax / ropeTable of src/L1/special.js and the inference forward of
 * src/L6/transformer.js.  It is the parity checker for the decode kernels in
 * forge-llm_b200/csrc/{quant,decode}.cu; the product never links it.
 *
 * Numeric model as in forge_oracle.c: scalar locals are double, every store
 * into a Float32Array is a (float) cast, Uint8Array / Int8Array stores wrap
 * modulo 256, -ffp-contract=off.  Math.round is restated exactly (ties toward
 * +infinity), and quant.js's `rnd` (ties away from zero) on top of it.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))
#define QK_K 256

/* ---------------------------------------------------------------- helpers */
static double js_round(double v) { /* Math.round: nearest integer, ties toward +inf */
  double r = floor(v);
  if (v - r >= 0.5) r += 1.0;
  return r;
}
static double rnd(double v) { return v < 0 ? -js_round(-v) : js_round(v); } /* quant.js:318 */
static double clampd(double v, double a, double b) { return v < a ? a : v > b ? b : v; } /* quant.js:319 */

static float g_fp16[65536];
/* fp16Table, quant.js:67-80 */
__attribute__((constructor)) static void fp16_table_build(void) {
  for (uint32_t h = 0; h < 65536; h++) {
    uint32_t s = (h & 0x8000) >> 15, e = (h & 0x7c00) >> 10, f = h & 0x03ff;
    float v;
    if (e == 0) {
      v = (float)((s ? -1.0 : 1.0) * 5.9604644775390625e-8 * (double)f);
    } else {
      uint32_t bits = e == 31 ? ((s << 31) | (f ? 0x7fc00000u : 0x7f800000u))
                              : ((s << 31) | ((e + 112) << 23) | (f << 13));
      memcpy(&v, &bits, 4);
    }
    g_fp16[h] = v;
  }
}
static double h2f(const uint8_t *u8, int64_t i) { return g_fp16[u8[i] | (u8[i + 1] << 8)]; }

OR_API float or_fp16_to_fp32(int h) { return g_fp16[h & 0xffff]; }

/* fp32ToFp16, special.js:151-168 (note: Math.round, not round-to-even) */
OR_API int or_fp32_to_fp16(double x) {
  if (!isfinite(x)) return x > 0 ? 0x7c00 : x < 0 ? 0xfc00 : 0x7e00;
  int s = x < 0 ? 0x8000 : 0;
  x = fabs(x);
  if (x < 6.103515625e-5) {
    int q = (int)js_round(x * 16777216.0);
    return s | (q & 0x3ff);
  }
  int e = 0;
  while (x >= 2) { x /= 2; e++; }
  while (x < 1) { x *= 2; e--; }
  int m = (int)js_round((x - 1) * 1024);
  if (m == 1024) { e++; m = 0; }
  int ex = e + 15;
  if (ex >= 31) return s | 0x7c00;
  return s | (ex << 10) | m;
}

/* getScaleMinK4Into, quant.js:98-106 */
static void scale_min_k4(int j, const uint8_t *q, int64_t base, int *sc, int *mn) {
  if (j < 4) {
    *sc = q[base + j] & 63;
    *mn = q[base + j + 4] & 63;
  } else {
    *sc = (q[base + j + 4] & 0xF) | ((q[base + j - 4] >> 6) << 4);
    *mn = (q[base + j + 4] >> 4) | ((q[base + j] >> 6) << 4);
  }
}

/* TYPE_INFO, quant.js:42-55: elements and bytes per block */
OR_API int or_block_size(int type) {
  switch (type) {
    case 0: case 1: return 1;
    case 2: case 3: case 6: case 7: case 8: case 9: return 32;
    case 12: case 13: case 14: case 15: return 256;
    default: return 0;
  }
}
OR_API int or_block_bytes(int type) {
  switch (type) {
    case 0: return 4;   case 1: return 2;   case 2: return 18;  case 3: return 20;
    case 6: return 22;  case 7: return 24;  case 8: return 34;  case 9: return 36;
    case 12: return 144; case 13: return 176; case 14: return 210; case 15: return 292;
    default: return 0;
  }
}
/* rowBytes, quant.js:62 */
OR_API int64_t or_row_bytes(int type, int64_t n) {
  int bs = or_block_size(type);
  return bs ? (n + bs - 1) / bs * or_block_bytes(type) : -1;
}

/* ---------------------------------------------------------------- numeric.js */
/* dot, numeric.js:52-61 */
static double dot_f(const float *a, const float *b, int64_t n) {
  double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  int64_t i = 0;
  for (; i + 4 <= n; i += 4) {
    s0 += (double)a[i] * b[i];
    s1 += (double)a[i + 1] * b[i + 1];
    s2 += (double)a[i + 2] * b[i + 2];
    s3 += (double)a[i + 3] * b[i + 3];
  }
  double s = s0 + s1 + s2 + s3;
  for (; i < n; i++) s += (double)a[i] * b[i];
  return s;
}
OR_API double or_dot(const float *a, const float *b, int64_t n) { return dot_f(a, b, n); }

/* matvec, numeric.js:85-100 */
OR_API void or_matvec(float *out, const float *W, const float *x, int64_t N, int64_t K) {
  for (int64_t n = 0; n < N; n++) {
    const int64_t base = n * K;
    double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int64_t k = 0;
    for (; k + 4 <= K; k += 4) {
      s0 += (double)W[base + k] * x[k];
      s1 += (double)W[base + k + 1] * x[k + 1];
      s2 += (double)W[base + k + 2] * x[k + 2];
      s3 += (double)W[base + k + 3] * x[k + 3];
    }
    double s = s0 + s1 + s2 + s3;
    for (; k < K; k++) s += (double)W[base + k] * x[k];
    out[n] = (float)s;
  }
}

/* ---------------------------------------------------------------- dequantize, quant.js:109-209 */
OR_API int or_dequantize(int type, const uint8_t *u8, int64_t n, float *out, int64_t byteOff) {
  switch (type) {
    case 0:
      memcpy(out, u8 + byteOff, (size_t)n * 4);
      return 0;
    case 1:
      for (int64_t i = 0; i < n; i++) out[i] = g_fp16[u8[byteOff + 2 * i] | (u8[byteOff + 2 * i + 1] << 8)];
      return 0;
    case 8: {
      const int64_t nb = n >> 5;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 34;
        const double d = h2f(u8, base);
        for (int j = 0; j < 32; j++) out[b * 32 + j] = (float)((double)(int8_t)u8[base + 2 + j] * d);
      }
      return 0;
    }
    case 12: {
      const int64_t nb = n >> 8;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 144;
        const double d = h2f(u8, base), dmin = h2f(u8, base + 2);
        const int64_t scB = base + 4, qsB = base + 16;
        int is = 0;
        for (int j = 0; j < QK_K; j += 64) {
          int sc, mn;
          scale_min_k4(is, u8, scB, &sc, &mn);
          const double d1 = d * sc, n1 = dmin * mn;
          scale_min_k4(is + 1, u8, scB, &sc, &mn);
          const double d2 = d * sc, n2 = dmin * mn;
          for (int l = 0; l < 32; l++) out[b * 256 + j + l] = (float)(d1 * (u8[qsB + (j >> 1) + l] & 0xF) - n1);
          for (int l = 0; l < 32; l++) out[b * 256 + j + 32 + l] = (float)(d2 * (u8[qsB + (j >> 1) + l] >> 4) - n2);
          is += 2;
        }
      }
      return 0;
    }
    case 13: {
      const int64_t nb = n >> 8;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 176;
        const double d = h2f(u8, base), dmin = h2f(u8, base + 2);
        const int64_t scB = base + 4, qhB = base + 16, qsB = base + 48;
        int is = 0, u1 = 1, u2 = 2;
        for (int j = 0; j < QK_K; j += 64) {
          int sc, mn;
          scale_min_k4(is, u8, scB, &sc, &mn);
          const double d1 = d * sc, n1 = dmin * mn;
          scale_min_k4(is + 1, u8, scB, &sc, &mn);
          const double d2 = d * sc, n2 = dmin * mn;
          for (int l = 0; l < 32; l++)
            out[b * 256 + j + l] = (float)(d1 * ((u8[qsB + (j >> 1) + l] & 0xF) + ((u8[qhB + l] & u1) ? 16 : 0)) - n1);
          for (int l = 0; l < 32; l++)
            out[b * 256 + j + 32 + l] = (float)(d2 * ((u8[qsB + (j >> 1) + l] >> 4) + ((u8[qhB + l] & u2) ? 16 : 0)) - n2);
          is += 2;
          u1 <<= 2;
          u2 <<= 2;
        }
      }
      return 0;
    }
    case 14: {
      const int64_t nb = n >> 8;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 210;
        const double d = h2f(u8, base + 208);
        const int64_t qlB = base, qhB = base + 128, scB = base + 192;
        for (int n2 = 0; n2 < QK_K; n2 += 128) {
          const int hB = n2 >> 2, sB = n2 >> 4;
          for (int l = 0; l < 32; l++) {
            const int is = l >> 4;
            const int q1 = ((u8[qlB + (n2 >> 1) + l] & 0xF) | ((u8[qhB + hB + l] & 3) << 4)) - 32;
            const int q2 = ((u8[qlB + (n2 >> 1) + l + 32] & 0xF) | (((u8[qhB + hB + l] >> 2) & 3) << 4)) - 32;
            const int q3 = ((u8[qlB + (n2 >> 1) + l] >> 4) | (((u8[qhB + hB + l] >> 4) & 3) << 4)) - 32;
            const int q4 = ((u8[qlB + (n2 >> 1) + l + 32] >> 4) | (((u8[qhB + hB + l] >> 6) & 3) << 4)) - 32;
            out[b * 256 + n2 + l] = (float)(d * (int8_t)u8[scB + sB + is] * q1);
            out[b * 256 + n2 + 32 + l] = (float)(d * (int8_t)u8[scB + sB + is + 2] * q2);
            out[b * 256 + n2 + 64 + l] = (float)(d * (int8_t)u8[scB + sB + is + 4] * q3);
            out[b * 256 + n2 + 96 + l] = (float)(d * (int8_t)u8[scB + sB + is + 6] * q4);
          }
        }
      }
      return 0;
    }
    case 2:
    case 6: {
      /* quant.js:191-205: f16 d, then nibble j&1 of byte 2 + j/2 (q - 8 for
       * type 2; type 6 reads the same nibbles unshifted) */
      const int64_t nb = n >> 5, bb = or_block_bytes(type);
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * bb;
        const double d = h2f(u8, base);
        for (int j = 0; j < 32; j++) {
          const int u = u8[base + 2 + (j >> 1)];
          const int q = (j & 1) ? (u >> 4) : (u & 0xF);
          out[b * 32 + j] = (float)((type == 2 ? q - 8 : q) * d);
        }
      }
      return 0;
    }
    default:
      return -1;
  }
}

/* ---------------------------------------------------------------- dotQ, quant.js:215-310 */
OR_API double or_dotq(int type, const uint8_t *u8, const float *x, int64_t n, int64_t xOff, int64_t byteOff) {
  switch (type) {
    case 0: {
      float *f = (float *)malloc((size_t)n * 4);
      memcpy(f, u8 + byteOff, (size_t)n * 4);
      double s = dot_f(f, x + xOff, n);
      free(f);
      return s;
    }
    case 1: {
      double s = 0;
      for (int64_t i = 0; i < n; i++)
        s += (double)g_fp16[u8[byteOff + 2 * i] | (u8[byteOff + 2 * i + 1] << 8)] * x[xOff + i];
      return s;
    }
    case 8: {
      const int64_t nb = n >> 5;
      double s = 0;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 34;
        const double d = h2f(u8, base);
        double t0 = 0, t1 = 0, t2 = 0, t3 = 0;
        for (int j = 0; j < 32; j += 4) {
          t0 += (double)(int8_t)u8[base + 2 + j] * x[xOff + b * 32 + j];
          t1 += (double)(int8_t)u8[base + 3 + j] * x[xOff + b * 32 + j + 1];
          t2 += (double)(int8_t)u8[base + 4 + j] * x[xOff + b * 32 + j + 2];
          t3 += (double)(int8_t)u8[base + 5 + j] * x[xOff + b * 32 + j + 3];
        }
        s += (t0 + t1 + t2 + t3) * d;
      }
      return s;
    }
    case 12: {
      const int64_t nb = n >> 8;
      double s = 0;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 144;
        const double d = h2f(u8, base), dmin = h2f(u8, base + 2);
        const int64_t scB = base + 4, qsB = base + 16, xb = xOff + b * 256;
        int is = 0;
        for (int j = 0; j < QK_K; j += 64) {
          int sc, mn;
          scale_min_k4(is, u8, scB, &sc, &mn);
          const double d1 = d * sc, m1 = dmin * mn;
          scale_min_k4(is + 1, u8, scB, &sc, &mn);
          const double d2 = d * sc, m2 = dmin * mn;
          for (int l = 0; l < 32; l++) s += (d1 * (u8[qsB + (j >> 1) + l] & 0xF) - m1) * x[xb + j + l];
          for (int l = 0; l < 32; l++) s += (d2 * (u8[qsB + (j >> 1) + l] >> 4) - m2) * x[xb + j + 32 + l];
          is += 2;
        }
      }
      return s;
    }
    case 13: {
      const int64_t nb = n >> 8;
      double s = 0;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 176;
        const double d = h2f(u8, base), dmin = h2f(u8, base + 2);
        const int64_t scB = base + 4, qhB = base + 16, qsB = base + 48, xb = xOff + b * 256;
        int is = 0, u1 = 1, u2 = 2;
        for (int j = 0; j < QK_K; j += 64) {
          int sc, mn;
          scale_min_k4(is, u8, scB, &sc, &mn);
          const double d1 = d * sc, m1 = dmin * mn;
          scale_min_k4(is + 1, u8, scB, &sc, &mn);
          const double d2 = d * sc, m2 = dmin * mn;
          for (int l = 0; l < 32; l++)
            s += (d1 * ((u8[qsB + (j >> 1) + l] & 0xF) + ((u8[qhB + l] & u1) ? 16 : 0)) - m1) * x[xb + j + l];
          for (int l = 0; l < 32; l++)
            s += (d2 * ((u8[qsB + (j >> 1) + l] >> 4) + ((u8[qhB + l] & u2) ? 16 : 0)) - m2) * x[xb + j + 32 + l];
          is += 2;
          u1 <<= 2;
          u2 <<= 2;
        }
      }
      return s;
    }
    case 14: {
      const int64_t nb = n >> 8;
      double s = 0;
      for (int64_t b = 0; b < nb; b++) {
        const int64_t base = byteOff + b * 210;
        const double d = h2f(u8, base + 208);
        const int64_t qlB = base, qhB = base + 128, scB = base + 192, xb = xOff + b * 256;
        for (int nn = 0; nn < QK_K; nn += 128) {
          const int hB = nn >> 2, sB = nn >> 4, lb = nn >> 1;
          for (int l = 0; l < 32; l++) {
            const int is = l >> 4;
            const int qh = u8[qhB + hB + l];
            const int q1 = ((u8[qlB + lb + l] & 0xF) | ((qh & 3) << 4)) - 32;
            const int q2 = ((u8[qlB + lb + l + 32] & 0xF) | (((qh >> 2) & 3) << 4)) - 32;
            const int q3 = ((u8[qlB + lb + l] >> 4) | (((qh >> 4) & 3) << 4)) - 32;
            const int q4 = ((u8[qlB + lb + l + 32] >> 4) | (((qh >> 6) & 3) << 4)) - 32;
            const int s1 = (int8_t)u8[scB + sB + is], s2 = (int8_t)u8[scB + sB + is + 2],
                      s3 = (int8_t)u8[scB + sB + is + 4], s4 = (int8_t)u8[scB + sB + is + 6];
            s += d * ((double)s1 * q1 * x[xb + nn + l] + (double)s2 * q2 * x[xb + nn + 32 + l] +
                      (double)s3 * q3 * x[xb + nn + 64 + l] + (double)s4 * q4 * x[xb + nn + 96 + l]);
          }
        }
      }
      return s;
    }
    default: { /* quant.js:308: dot of the dequantized row */
      float *f = (float *)malloc((size_t)n * 4);
      if (or_dequantize(type, u8, n, f, byteOff)) {
        free(f);
        return NAN;
      }
      double s = dot_f(f, x + xOff, n);
      free(f);
      return s;
    }
  }
}

/* QuantLinear.forward, nn.js:27-32: out[N] = W . x */
OR_API void or_quantlinear_fwd(int type, const uint8_t *bytes, const float *x, int64_t N, int64_t K,
                               float *out, int64_t xOff) {
  if (type == 0) {
    or_matvec(out, (const float *)bytes, x + xOff, N, K);
    return;
  }
  const int64_t rb = or_row_bytes(type, K);
  for (int64_t n = 0; n < N; n++) out[n] = (float)or_dotq(type, bytes, x, K, xOff, n * rb);
}

/* ---------------------------------------------------------------- quantizers */
/* quantizeRowF16, quant.js:321-325 */
OR_API void or_quantize_f16(const float *x, int64_t n, uint8_t *out) {
  for (int64_t i = 0; i < n; i++) {
    const int h = or_fp32_to_fp16(x[i]);
    out[2 * i] = (uint8_t)(h & 0xff);
    out[2 * i + 1] = (uint8_t)(h >> 8);
  }
}

/* quantizeRowQ8_0, quant.js:328-339 */
OR_API void or_quantize_q8_0(const float *x, int64_t n, uint8_t *out) {
  const int64_t nb = n >> 5;
  for (int64_t b = 0; b < nb; b++) {
    double amax = 0;
    for (int j = 0; j < 32; j++) {
      const double v = fabs((double)x[b * 32 + j]);
      if (v > amax) amax = v;
    }
    const double d = amax / 127, id = d ? 1 / d : 0;
    const int h = or_fp32_to_fp16(d);
    out[b * 34] = (uint8_t)(h & 0xff);
    out[b * 34 + 1] = (uint8_t)(h >> 8);
    for (int j = 0; j < 32; j++)
      out[b * 34 + 2 + j] = (uint8_t)((int)clampd(rnd((double)x[b * 32 + j] * id), -128, 127) & 0xff);
  }
}

/* makeQxQuants, quant.js:382-412 (rmse_type 1, no importance matrix) */
static double make_qx_quants(int n, int nmax, const float *x, int8_t *L) {
  double max = 0, amax = 0;
  for (int i = 0; i < n; i++) {
    const double ax = fabs((double)x[i]);
    if (ax > amax) {
      amax = ax;
      max = x[i];
    }
  }
  if (amax < 1e-30) {
    for (int i = 0; i < n; i++) L[i] = 0;
    return 0;
  }
  double iscale = -nmax / max;
  double sumlx = 0, suml2 = 0;
  for (int i = 0; i < n; i++) {
    const double l = clampd(rnd(iscale * x[i]), -nmax, nmax - 1);
    L[i] = (int8_t)(int)l;
    const double w = (double)x[i] * x[i];
    sumlx += w * x[i] * l;
    suml2 += w * l * l;
  }
  double scale = suml2 ? sumlx / suml2 : 0;
  double best = scale * sumlx;
  for (int is = -9; is <= 9; is++) {
    if (is == 0) continue;
    iscale = -(nmax + 0.1 * is) / max;
    sumlx = 0;
    suml2 = 0;
    for (int i = 0; i < n; i++) {
      const double l = clampd(rnd(iscale * x[i]), -nmax, nmax - 1);
      const double w = (double)x[i] * x[i];
      sumlx += w * x[i] * l;
      suml2 += w * l * l;
    }
    if (suml2 > 0 && sumlx * sumlx > best * suml2) {
      for (int i = 0; i < n; i++) L[i] = (int8_t)(int)clampd(rnd(iscale * x[i]), -nmax, nmax - 1);
      scale = sumlx / suml2;
      best = scale * sumlx;
    }
  }
  return scale;
}

/* quantizeRowQ6K, quant.js:345-379 */
OR_API void or_quantize_q6_k(const float *x, int64_t n, uint8_t *out) {
  const int64_t nb = n >> 8;
  int8_t L[QK_K];
  float scales[QK_K / 16];
  memset(out, 0, (size_t)nb * 210);
  memset(L, 0, sizeof L);
  for (int64_t b = 0; b < nb; b++) {
    double maxScale = 0, maxAbs = 0;
    for (int ib = 0; ib < 16; ib++) {
      const double s = make_qx_quants(16, 32, x + b * 256 + ib * 16, L + ib * 16);
      scales[ib] = (float)s;
      const double a = fabs(s);
      if (a > maxAbs) {
        maxAbs = a;
        maxScale = s;
      }
    }
    if (maxAbs < 1e-30) continue;
    const double iscale = -128 / maxScale;
    const int dh = or_fp32_to_fp16(1 / iscale);
    const int64_t base = b * 210;
    out[base + 208] = (uint8_t)(dh & 0xff);
    out[base + 209] = (uint8_t)(dh >> 8);
    for (int ib = 0; ib < 16; ib++) {
      double v = rnd(iscale * scales[ib]);
      if (v > 127) v = 127;
      out[base + 192 + ib] = (uint8_t)((int)v & 0xff);
    }
    const double d = g_fp16[dh & 0xffff];
    for (int j = 0; j < 16; j++) {
      const double dd = d * (int8_t)out[base + 192 + j];
      if (!dd) {
        for (int ii = 0; ii < 16; ii++) L[j * 16 + ii] = 32;
        continue;
      }
      for (int ii = 0; ii < 16; ii++)
        L[j * 16 + ii] = (int8_t)((int)clampd(rnd(x[b * 256 + j * 16 + ii] / dd), -32, 31) + 32);
    }
    for (int j = 0; j < QK_K; j += 128) {
      const int64_t p = base + (j >> 1);
      for (int l = 0; l < 32; l++) {
        const int q1 = L[j + l] & 0xF, q2 = L[j + l + 32] & 0xF, q3 = L[j + l + 64] & 0xF, q4 = L[j + l + 96] & 0xF;
        out[p + l] = (uint8_t)(q1 | (q3 << 4));
        out[p + l + 32] = (uint8_t)(q2 | (q4 << 4));
        out[base + 128 + (j >> 2) + l] = (uint8_t)((L[j + l] >> 4) | ((L[j + l + 32] >> 4) << 2) |
                                                   ((L[j + l + 64] >> 4) << 4) | ((L[j + l + 96] >> 4) << 6));
      }
    }
  }
}

/* makeQkx2Quants, quant.js:421-472 */
static double make_qkx2_quants(int n, int nmax, const float *x, const float *weights, uint8_t *L,
                               float *theMinOut, uint8_t *Laux, double rmin, double rdelta, int nstep,
                               int useMad) {
  double min = x[0], max = x[0];
  double sumW = weights[0], sumX = (double)weights[0] * x[0];
  for (int i = 1; i < n; i++) {
    const double v = x[i];
    if (v < min) min = v;
    if (v > max) max = v;
    const double w = weights[i];
    sumW += w;
    sumX += w * v;
  }
  if (min > 0) min = 0;
  if (max == min) {
    for (int i = 0; i < n; i++) L[i] = 0;
    theMinOut[0] = (float)-min;
    return 0;
  }
  double iscale = nmax / (max - min);
  double scale = 1 / iscale;
  double best = 0;
  for (int i = 0; i < n; i++) {
    const double l = clampd(rnd(iscale * (x[i] - min)), 0, nmax);
    L[i] = (uint8_t)(int)l;
    double diff = scale * l + min - x[i];
    diff = useMad ? fabs(diff) : diff * diff;
    best += weights[i] * diff;
  }
  if (nstep < 1) {
    theMinOut[0] = (float)-min;
    return scale;
  }
  for (int is = 0; is <= nstep; is++) {
    iscale = (rmin + rdelta * is + nmax) / (max - min);
    double sumL = 0, sumL2 = 0, sumXL = 0;
    for (int i = 0; i < n; i++) {
      const double l = clampd(rnd(iscale * (x[i] - min)), 0, nmax);
      Laux[i] = (uint8_t)(int)l;
      const double w = weights[i];
      sumL += w * l;
      sumL2 += w * l * l;
      sumXL += w * l * x[i];
    }
    const double D = sumW * sumL2 - sumL * sumL;
    if (D > 0) {
      double thisScale = (sumW * sumXL - sumX * sumL) / D;
      double thisMin = (sumL2 * sumX - sumL * sumXL) / D;
      if (thisMin > 0) {
        thisMin = 0;
        thisScale = sumXL / sumL2;
      }
      double cur = 0;
      for (int i = 0; i < n; i++) {
        double diff = thisScale * Laux[i] + thisMin - x[i];
        diff = useMad ? fabs(diff) : diff * diff;
        cur += weights[i] * diff;
      }
      if (cur < best) {
        for (int i = 0; i < n; i++) L[i] = Laux[i];
        best = cur;
        scale = thisScale;
        min = thisMin;
      }
    }
  }
  theMinOut[0] = (float)-min;
  return scale;
}

/* the 6-bit scale / min packing shared by quantizeRowQ5K and quantizeRowQ4K
 * (quant.js:505-512, 572-579) */
static void pack_scales_k4(uint8_t *out, int64_t base, const uint8_t *ls, const uint8_t *lm) {
  for (int j = 0; j < 8; j++) {
    if (j < 4) {
      out[base + 4 + j] = ls[j];
      out[base + 4 + j + 4] = lm[j];
    } else {
      out[base + 4 + j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
      out[base + 4 + j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
      out[base + 4 + j] |= (uint8_t)((lm[j] >> 4) << 6);
    }
  }
}

/* quantizeRowQ5K, quant.js:480-539 */
OR_API void or_quantize_q5_k(const float *x, int64_t n, uint8_t *out) {
  const int64_t nb = n >> 8;
  uint8_t L[QK_K], Laux[32], ls[8], lm[8];
  float weights[32], mins[8], scales[8], tm[1];
  memset(out, 0, (size_t)nb * 176);
  memset(L, 0, sizeof L);
  for (int64_t b = 0; b < nb; b++) {
    const float *xb = x + b * 256;
    double maxScale = 0, maxMin = 0;
    for (int j = 0; j < 8; j++) {
      double sumX2 = 0;
      for (int l = 0; l < 32; l++) {
        const double v = xb[j * 32 + l];
        sumX2 += v * v;
      }
      const double avX = sqrt(sumX2 / 32);
      for (int l = 0; l < 32; l++) weights[l] = (float)(avX + fabs((double)xb[j * 32 + l]));
      scales[j] = (float)make_qkx2_quants(32, 31, xb + j * 32, weights, L + j * 32, tm, Laux, -0.5, 0.1, 15, 0);
      mins[j] = tm[0];
      if (scales[j] > maxScale) maxScale = scales[j];
      if (mins[j] > maxMin) maxMin = mins[j];
    }
    const double invScale = maxScale > 0 ? 63 / maxScale : 0;
    const double invMin = maxMin > 0 ? 63 / maxMin : 0;
    const int64_t base = b * 176;
    for (int j = 0; j < 8; j++) {
      double a = rnd(invScale * scales[j]), c = rnd(invMin * mins[j]);
      ls[j] = (uint8_t)(int)(a < 63 ? a : 63);
      lm[j] = (uint8_t)(int)(c < 63 ? c : 63);
    }
    pack_scales_k4(out, base, ls, lm);
    const int dh = or_fp32_to_fp16(maxScale / 63), dhm = or_fp32_to_fp16(maxMin / 63);
    out[base] = (uint8_t)(dh & 0xff);
    out[base + 1] = (uint8_t)(dh >> 8);
    out[base + 2] = (uint8_t)(dhm & 0xff);
    out[base + 3] = (uint8_t)(dhm >> 8);
    const double d = g_fp16[dh & 0xffff], dmin = g_fp16[dhm & 0xffff];
    for (int j = 0; j < 8; j++) {
      int sc, mn;
      scale_min_k4(j, out, base + 4, &sc, &mn);
      const double dd = d * sc, dm = dmin * mn;
      if (!dd) continue;
      for (int l = 0; l < 32; l++) {
        const double v = xb[j * 32 + l];
        L[j * 32 + l] = (uint8_t)(int)clampd(rnd((v + dm) / dd), 0, 31);
      }
    }
    int m1 = 1, m2 = 2;
    for (int jj = 0; jj < QK_K; jj += 64) {
      for (int l = 0; l < 32; l++) {
        int l1 = L[jj + l];
        if (l1 > 15) {
          l1 -= 16;
          out[base + 16 + l] |= (uint8_t)m1;
        }
        int l2 = L[jj + l + 32];
        if (l2 > 15) {
          l2 -= 16;
          out[base + 16 + l] |= (uint8_t)m2;
        }
        out[base + 48 + (jj >> 1) + l] = (uint8_t)(l1 | (l2 << 4));
      }
      m1 <<= 2;
      m2 <<= 2;
    }
  }
}

/* quantizeRowQ4K, quant.js:547-592 (the closed-form writer) */
OR_API void or_quantize_q4_k(const float *x, int64_t n, uint8_t *out) {
  const int64_t nb = n >> 8;
  float mins[8], scales[8];
  uint8_t L[QK_K], lsArr[8], lmArr[8];
  memset(out, 0, (size_t)nb * 144);
  for (int64_t b = 0; b < nb; b++) {
    double maxScale = 0, maxMin = 0;
    for (int j = 0; j < 8; j++) {
      double mn = INFINITY, mx = -INFINITY;
      for (int l = 0; l < 32; l++) {
        const double v = x[b * 256 + j * 32 + l];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
      }
      if (mn > 0) mn = 0;
      scales[j] = (float)((mx - mn) / 15);
      mins[j] = (float)-mn;
      if (scales[j] > maxScale) maxScale = scales[j];
      if (mins[j] > maxMin) maxMin = mins[j];
    }
    const double d = maxScale / 63, dm = maxMin / 63;
    const int64_t base = b * 144;
    const int dh = or_fp32_to_fp16(d), dh2 = or_fp32_to_fp16(dm);
    out[base] = (uint8_t)(dh & 0xff);
    out[base + 1] = (uint8_t)(dh >> 8);
    out[base + 2] = (uint8_t)(dh2 & 0xff);
    out[base + 3] = (uint8_t)(dh2 >> 8);
    for (int j = 0; j < 8; j++) {
      lsArr[j] = (uint8_t)(int)clampd(rnd(scales[j] / (d ? d : 1)), 0, 63);
      lmArr[j] = (uint8_t)(int)clampd(rnd(fabs((double)mins[j]) / (dm ? dm : 1)), 0, 63);
    }
    pack_scales_k4(out, base, lsArr, lmArr);
    for (int j = 0; j < 8; j++) {
      int sc, mnq;
      scale_min_k4(j, out, base + 4, &sc, &mnq);
      const double dd = d * sc, mm = dm * mnq;
      for (int l = 0; l < 32; l++) {
        const double v = x[b * 256 + j * 32 + l];
        L[j * 32 + l] = (uint8_t)(int)clampd(rnd(dd ? (v + mm) / dd : 0), 0, 15);
      }
    }
    for (int j = 0; j < QK_K; j += 64)
      for (int l = 0; l < 32; l++) out[base + 16 + (j >> 1) + l] = (uint8_t)(L[j + l] | (L[j + l + 32] << 4));
  }
}

/* quantizeRow, quant.js:594-604; returns the byte count or -1 */
OR_API int64_t or_quantize_row(int type, const float *x, int64_t n, uint8_t *out) {
  switch (type) {
    case 0: memcpy(out, x, (size_t)n * 4); return n * 4;
    case 1: or_quantize_f16(x, n, out); return n * 2;
    case 8: or_quantize_q8_0(x, n, out); return (n >> 5) * 34;
    case 12: or_quantize_q4_k(x, n, out); return (n >> 8) * 144;
    case 13: or_quantize_q5_k(x, n, out); return (n >> 8) * 176;
    case 14: or_quantize_q6_k(x, n, out); return (n >> 8) * 210;
    default: return -1;
  }
}

/* ---------------------------------------------------------------- attention.js */
/* softmax, special.js:66-74 */
static void softmax_f(float *out, const float *x, int64_t n) {
  double m = -INFINITY;
  for (int64_t i = 0; i < n; i++) if (x[i] > m) m = x[i];
  double s = 0;
  for (int64_t i = 0; i < n; i++) {
    const double e = exp((double)x[i] - m);
    out[i] = (float)e;
    s += e;
  }
  const double inv = 1 / s;
  for (int64_t i = 0; i < n; i++) out[i] = (float)(out[i] * inv);
}

/* attentionDecode, attention.js:31-57 */
OR_API void or_attention_decode(float *out, const float *q, const float *K, const float *V, int64_t n,
                                int64_t d, double scale, int causal, int64_t qOff, int64_t kOff) {
  float *sc = (float *)malloc((size_t)(n > 0 ? n : 1) * 4);
  double mx = -INFINITY;
  for (int64_t j = 0; j < n; j++) {
    if (causal && j > qOff) {
      sc[j] = -INFINITY;
      continue;
    }
    const int64_t kb = kOff + j * d;
    double acc = 0;
    for (int64_t i = 0; i < d; i++) acc += (double)q[i] * K[kb + i];
    const double v = acc * scale;
    sc[j] = (float)v;
    if (v > mx) mx = v;
  }
  for (int64_t i = 0; i < d; i++) out[i] = 0;
  double l = 0;
  for (int64_t j = 0; j < n; j++) {
    const double p = sc[j] == -INFINITY ? 0 : exp((double)sc[j] - mx);
    if (p == 0) continue;
    l += p;
    const int64_t vb = kOff + j * d;
    for (int64_t i = 0; i < d; i++) out[i] = (float)(out[i] + p * V[vb + i]);
  }
  const double inv = 1 / (l ? l : 1);
  for (int64_t i = 0; i < d; i++) out[i] = (float)(out[i] * inv);
  free(sc);
}

/* attentionNaive, attention.js:63-79 */
OR_API void or_attention_naive(float *out, const float *q, const float *K, const float *V, int64_t n,
                               int64_t d, double scale, int causal, int64_t qOff, int64_t kOff) {
  float *s = (float *)malloc((size_t)(n > 0 ? n : 1) * 4);
  for (int64_t j = 0; j < n; j++) {
    if (causal && j > qOff) {
      s[j] = -INFINITY;
      continue;
    }
    double acc = 0;
    for (int64_t i = 0; i < d; i++) acc += (double)q[i] * K[kOff + j * d + i];
    s[j] = (float)(acc * scale);
  }
  softmax_f(s, s, n);
  for (int64_t i = 0; i < d; i++) out[i] = 0;
  for (int64_t j = 0; j < n; j++) {
    const double p = s[j];
    if (p == 0) continue;
    for (int64_t i = 0; i < d; i++) out[i] = (float)(out[i] + p * V[kOff + j * d + i]);
  }
  free(s);
}

/* flashAttention, attention.js:89-125 */
OR_API void or_flash_attention(float *out, const float *q, const float *K, const float *V, int64_t n,
                               int64_t d, double scale, int causal, int64_t qOff, int64_t kOff, int block) {
  const int64_t end = causal ? (n < qOff + 1 ? n : qOff + 1) : n;
  for (int64_t i = 0; i < d; i++) out[i] = 0;
  if (end <= 0) return;
  float *s = (float *)malloc((size_t)block * 4);
  double m = -INFINITY, l = 0;
  for (int64_t b = 0; b < end; b += block) {
    const int64_t e = b + block < end ? b + block : end;
    double mb = -INFINITY;
    for (int64_t j = b; j < e; j++) {
      const int64_t kb = kOff + j * d;
      double acc = 0;
      for (int64_t i = 0; i < d; i++) acc += (double)q[i] * K[kb + i];
      const double v = acc * scale;
      s[j - b] = (float)v;
      if (v > mb) mb = v;
    }
    const double mNew = m > mb ? m : mb;
    const double alpha = m == -INFINITY ? 0 : exp(m - mNew);
    double lNew = l * alpha;
    if (alpha != 1)
      for (int64_t i = 0; i < d; i++) out[i] = (float)(out[i] * alpha);
    for (int64_t j = b; j < e; j++) {
      const double p = exp((double)s[j - b] - mNew);
      lNew += p;
      const int64_t vb = kOff + j * d;
      for (int64_t i = 0; i < d; i++) out[i] = (float)(out[i] + p * V[vb + i]);
    }
    m = mNew;
    l = lNew;
  }
  const double inv = 1 / (l ? l : 1);
  for (int64_t i = 0; i < d; i++) out[i] = (float)(out[i] * inv);
  free(s);
}

/* ---------------------------------------------------------------- special.js vector ops */
/* rmsnorm, special.js:46-50 (rms, numeric.js:74-78) */
OR_API void or_rmsnorm_vec(float *out, const float *x, const float *w, int64_t n, double eps) {
  double s = 0;
  for (int64_t i = 0; i < n; i++) {
    const double v = x[i];
    s += v * v;
  }
  const double r = sqrt(s / n);
  const double ss = 1 / sqrt(r * r + eps);
  for (int64_t i = 0; i < n; i++) out[i] = (float)((double)x[i] * ss * w[i]);
}

/* ropeTable, special.js:116-127: cos / sin [maxPos][dim/2] as Float32Array */
OR_API void or_rope_table(int64_t maxPos, int dim, double theta, float *cosT, float *sinT) {
  for (int64_t p = 0; p < maxPos; p++)
    for (int i = 0; i < dim; i += 2) {
      const double freq = 1 / pow(theta, (double)i / dim);
      const double ang = (double)p * freq;
      cosT[p * (dim / 2) + i / 2] = (float)cos(ang);
      sinT[p * (dim / 2) + i / 2] = (float)sin(ang);
    }
}

/* applyRopeHead, transformer.js:56-64 */
static void apply_rope_head(float *x, int64_t base, int dHead, int64_t pos, const float *cosT, const float *sinT) {
  const int half = dHead >> 1;
  const int64_t cp = pos * half;
  for (int i = 0; i < dHead; i += 2) {
    const double c = cosT[cp + (i >> 1)], s = sinT[cp + (i >> 1)];
    const double a = x[base + i], b = x[base + i + 1];
    x[base + i] = (float)(a * c - b * s);
    x[base + i + 1] = (float)(a * s + b * c);
  }
}

/* ---------------------------------------------------------------- Transformer.forward */
/* The inference forward of transformer.js:134-185 for one token, with the
 * weights as QuantLinear byte streams.  Weights (all in one struct):
 *   tok_emb: type tok_type, [V, D] (also the LM head: wcls = tok_emb);
 *   per layer l: ln1[D], ln2[D] fp32 and wqkv [qkvOut, D], wo [D, D],
 *   gate [H, D], up [H, D], down [D, H] of type w_type;
 *   ln_f[D].
 * cacheK / cacheV: KVCache [nLayers, maxSeq, kvDim] (attention.js:128-154). */
typedef struct {
  int vocab, dim, n_layers, n_heads, n_kv_heads, hidden, max_seq;
  double norm_eps, rope_theta;
  int tok_type, w_type;
  const uint8_t *tok_emb;
  const float *ln_f;
  const float *const *ln1, *const *ln2;
  const uint8_t *const *wqkv, *const *wo, *const *gate, *const *up, *const *down;
} or_infer_model;

OR_API void or_transformer_forward(const or_infer_model *m, int token, int64_t pos, float *cacheK,
                                   float *cacheV, float *logits) {
  const int D = m->dim, H = m->hidden, nH = m->n_heads, nKV = m->n_kv_heads;
  const int dH = D / nH, kvDim = nKV * dH, qkvOut = (nH + 2 * nKV) * dH, g = nH / nKV;
  float *x = (float *)calloc(D, 4), *xb = (float *)calloc(D, 4), *xb2 = (float *)calloc(D, 4);
  float *q = (float *)calloc(qkvOut, 4), *att = (float *)calloc(D, 4);
  float *hg = (float *)calloc(H, 4), *hu = (float *)calloc(H, 4);
  float *tmpK = (float *)calloc((size_t)(pos + 1) * dH, 4), *tmpV = (float *)calloc((size_t)(pos + 1) * dH, 4);
  float *cosT = (float *)malloc((size_t)m->max_seq * (dH / 2) * 4), *sinT = (float *)malloc((size_t)m->max_seq * (dH / 2) * 4);
  or_rope_table(m->max_seq, dH, m->rope_theta, cosT, sinT);
  /* _embed, transformer.js:122-132 */
  if (m->tok_type == 0)
    memcpy(x, m->tok_emb + (int64_t)token * D * 4, (size_t)D * 4);
  else
    or_dequantize(m->tok_type, m->tok_emb, D, x, token * or_row_bytes(m->tok_type, D));
  for (int l = 0; l < m->n_layers; l++) {
    or_rmsnorm_vec(xb, x, m->ln1[l], D, m->norm_eps);
    or_quantlinear_fwd(m->w_type, m->wqkv[l], xb, qkvOut, D, q, 0);
    int off = 0;
    for (int h = 0; h < nH; h++, off += dH) apply_rope_head(q, off, dH, pos, cosT, sinT);
    for (int h = 0; h < nKV; h++, off += dH) apply_rope_head(q, off, dH, pos, cosT, sinT);
    /* cache.put(l, pos, K, V) */
    const int64_t co = ((int64_t)l * m->max_seq + pos) * kvDim;
    memcpy(cacheK + co, q + nH * dH, (size_t)kvDim * 4);
    memcpy(cacheV + co, q + nH * dH + kvDim, (size_t)kvDim * 4);
    for (int i = 0; i < D; i++) att[i] = 0;
    const int64_t n = pos + 1;
    for (int kvh = 0; kvh < nKV; kvh++) {
      /* gatherKV: the kv head's rows [0, n) of layer l */
      for (int64_t p = 0; p < n; p++) {
        const int64_t src = ((int64_t)l * m->max_seq + p) * kvDim + kvh * dH;
        memcpy(tmpK + p * dH, cacheK + src, (size_t)dH * 4);
        memcpy(tmpV + p * dH, cacheV + src, (size_t)dH * 4);
      }
      for (int gi = 0; gi < g; gi++) {
        const int h = kvh * g + gi;
        if (h >= nH) break;
        or_attention_decode(att + h * dH, q + h * dH, tmpK, tmpV, n, dH, 1 / sqrt((double)dH), 1, pos, 0);
      }
    }
    or_quantlinear_fwd(m->w_type, m->wo[l], att, D, D, xb2, 0);
    for (int i = 0; i < D; i++) x[i] = (float)((double)x[i] + xb2[i]);
    or_rmsnorm_vec(xb, x, m->ln2[l], D, m->norm_eps);
    /* SwiGLU.forward, nn.js:56-66 */
    or_quantlinear_fwd(m->w_type, m->gate[l], xb, H, D, hg, 0);
    or_quantlinear_fwd(m->w_type, m->up[l], xb, H, D, hu, 0);
    for (int i = 0; i < H; i++) {
      const double gv = hg[i];
      hg[i] = (float)((gv / (1 + exp(-gv))) * hu[i]);
    }
    or_quantlinear_fwd(m->w_type, m->down[l], hg, D, H, xb2, 0);
    for (int i = 0; i < D; i++) x[i] = (float)((double)x[i] + xb2[i]);
  }
  or_rmsnorm_vec(xb, x, m->ln_f, D, m->norm_eps);
  or_quantlinear_fwd(m->tok_type, m->tok_emb, xb, m->vocab, D, logits, 0);
  free(x); free(xb); free(xb2); free(q); free(att); free(hg); free(hu); free(tmpK); free(tmpV);
  free(cosT); free(sinT);
}
