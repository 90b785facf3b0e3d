// Host-side seeded generator and weight initialisation (no device code).
// The generator is forge-llm's RNG (src/L0/numeric.js:27-49): xorshift128+ on
// two 32-bit lanes, seeded through splitmix32, Box-Muller normals.  Weight
// init follows initWeights (src/L6/train.js:33-57).
#include <math.h>

#include "common.cuh"

namespace {

uint32_t splitmix32(uint32_t *s) {
  *s += 0x9e3779b9u;
  uint32_t z = *s;
  z = (z ^ (z >> 16)) * 0x21f0aaadu;
  z = (z ^ (z >> 15)) * 0x735a2d97u;
  return z ^ (z >> 15);
}

struct Layout {
  int64_t ln1, ln2, wqkv, wo, gate, up, down, stride, total, head;
};

Layout layout_of(const fcu_model_cfg *c) {
  const int64_t D = c->dim, V = c->vocab, H = c->hidden;
  const int64_t dH = c->dim / c->n_heads, qD = (int64_t)c->n_heads * dH;
  const int64_t qkvOut = (int64_t)(c->n_heads + 2 * c->n_kv_heads) * dH;
  Layout L;
  L.head = V * D + D;
  L.ln1 = 0;
  L.ln2 = D;
  L.wqkv = 2 * D;
  L.wo = L.wqkv + qkvOut * D;
  L.gate = L.wo + D * qD;
  L.up = L.gate + H * D;
  L.down = L.up + H * D;
  L.stride = L.down + D * H;
  L.total = L.head + L.stride * c->n_layers;
  return L;
}

}  // namespace

extern "C" {

void fcu_rng_init(fcu_rng *r, uint32_t seed) {
  uint32_t s = seed ? seed : 1u;
  r->s0 = splitmix32(&s);
  r->s1 = splitmix32(&s);
}

double fcu_rng_next(fcu_rng *r) {
  uint32_t x = r->s0, y = r->s1;
  r->s0 = y;
  x ^= x << 23;
  x ^= x >> 17;
  x ^= y;
  x ^= y >> 26;
  r->s1 = x;
  return (double)(uint32_t)(r->s1 + y) / 4294967296.0;
}

double fcu_rng_normal(fcu_rng *r) {
  double u = fcu_rng_next(r);
  if (u < 1e-12) u = 1e-12;
  double v = fcu_rng_next(r);
  return sqrt(-2.0 * log(u)) * cos(2.0 * M_PI * v);
}

int fcu_rng_int(fcu_rng *r, int n) { return (int)floor(fcu_rng_next(r) * n); }

void fcu_rng_fill_normal(fcu_rng *r, float *out, int64_t n, double scale) {
  for (int64_t i = 0; i < n; i++) out[i] = (float)(fcu_rng_normal(r) * scale);
}

void fcu_rng_fill_int(fcu_rng *r, int32_t *out, int64_t n, int range) {
  for (int64_t i = 0; i < n; i++) out[i] = fcu_rng_int(r, range);
}

int64_t fcu_model_num_params(const fcu_model_cfg *c) {
  if (!c || c->n_heads <= 0 || c->n_kv_heads <= 0) return -1;
  return layout_of(c).total;
}

int fcu_init_weights(const fcu_model_cfg *c, uint32_t seed, float *P) {
  FCU_REQUIRE(c && P, "fcu_init_weights: null argument");
  FCU_REQUIRE(c->n_heads > 0 && c->n_kv_heads > 0 && c->n_heads % c->n_kv_heads == 0,
              "GQA requires nHeads (%d) divisible by nKvHeads (%d)", c->n_heads, c->n_kv_heads);
  const Layout L = layout_of(c);
  const int64_t D = c->dim, V = c->vocab, H = c->hidden;
  const int64_t dH = c->dim / c->n_heads, qD = (int64_t)c->n_heads * dH;
  const int64_t qkvOut = (int64_t)(c->n_heads + 2 * c->n_kv_heads) * dH;
  fcu_rng r;
  fcu_rng_init(&r, seed);
  const double std = 0.02, res = 1.0 / sqrt(2.0 * c->n_layers);
  fcu_rng_fill_normal(&r, P, V * D, std);
  for (int64_t i = 0; i < D; i++) P[V * D + i] = 1.0f;
  for (int l = 0; l < c->n_layers; l++) {
    float *b = P + L.head + (int64_t)l * L.stride;
    for (int64_t i = 0; i < D; i++) b[L.ln1 + i] = 1.0f;
    for (int64_t i = 0; i < D; i++) b[L.ln2 + i] = 1.0f;
    fcu_rng_fill_normal(&r, b + L.wqkv, qkvOut * D, std);
    fcu_rng_fill_normal(&r, b + L.wo, D * qD, std);
    for (int64_t i = 0; i < D * qD; i++) b[L.wo + i] = (float)((double)b[L.wo + i] * res);
    fcu_rng_fill_normal(&r, b + L.gate, H * D, std);
    fcu_rng_fill_normal(&r, b + L.up, H * D, std);
    fcu_rng_fill_normal(&r, b + L.down, D * H, std);
    for (int64_t i = 0; i < D * H; i++) b[L.down + i] = (float)((double)b[L.down + i] * res);
  }
  return FCU_OK;
}

}  // extern "C"
