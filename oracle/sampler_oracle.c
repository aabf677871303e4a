/*
 * sampler_oracle.c — TEST INFRASTRUCTURE ONLY (CPU oracle; never linked into the product).
 *
 * CPU restatement of the reference's Gumbel-max sampler (fused_sampler_ops.py:54-93):
 *   u = tl.rand(seed + row, col)          Philox4x32-10, key (seed+row as Triton does), counter
 *                                          (col, 0, 0, 0), first output word, Triton's
 *                                          uint_to_uniform_float (triton/language/random.py)
 *   u = min(max(u, 1e-10), 1 - 1e-7)      fused_sampler_ops.py:67
 *   g = -log(-log(u))                     fused_sampler_ops.py:68
 *   sample = first argmax(x + g), amax = first argmax(x)     fused_sampler_ops.py:69-81
 * with the temperature division of the logits processor (x / T, IEEE) applied first.
 *
 * Philox4x32-10 is restated from Salmon et al., "Parallel random numbers: as easy as 1, 2, 3"
 * (SC'11).  The logarithm is the same published atanh-series construction as the product's
 * (written independently here): x = 2^e m, s = (m-1)/(m+1), log m = 2 atanh(s), with IEEE
 * single-precision operations in a fixed order so CPU and GPU agree bit for bit.
 * Build: see oracle/build_oracle.py (gcc -O2 -ffp-contract=off, no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

void oracle_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    c1 = (uint32_t)p1;
    c3 = (uint32_t)p0;
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* key words of tl.rand(seed + row, .): a seed that fits int32 is an i32 kernel argument, so
 * seed + row wraps in 32 bits and is then sign-extended to 64 bits before the split. */
void oracle_row_key(int64_t seed, int64_t row, uint32_t key[2]) {
  if (seed >= -2147483648LL && seed <= 2147483647LL) {
    const int32_t s = (int32_t)((uint32_t)seed + (uint32_t)row);
    key[0] = (uint32_t)s;
    key[1] = s < 0 ? 0xffffffffu : 0u;
  } else {
    const uint64_t s = (uint64_t)(seed + row);
    key[0] = (uint32_t)s;
    key[1] = (uint32_t)(s >> 32);
  }
}

float oracle_uniform(uint32_t w) {
  int32_t x = (int32_t)w;
  if (x < 0) x = -x - 1;
  return (float)x * u2f(0x2fffffffu); /* largest float below 2^-31 */
}

float oracle_log(float x) {
  const uint32_t b = f2u(x);
  int e = (int)(b >> 23) - 127;
  float m = u2f((b & 0x007fffffu) | 0x3f800000u);
  if (m > u2f(0x3fb504f3u)) { m = m * 0.5f; e += 1; }
  const float f = m - 1.0f;
  const float s = f / (2.0f + f);
  const float z = s * s;
  float p = fmaf(z, 0x1.745d18p-3f, 0x1.c71c72p-3f);
  p = fmaf(z, p, 0x1.24924ap-2f);
  p = fmaf(z, p, 0x1.99999ap-2f);
  p = fmaf(z, p, 0x1.555556p-1f);
  p = fmaf(z, p, 2.0f);
  const float lm = s * p;
  const float ef = (float)e;
  return fmaf(ef, 0x1.62e400p-1f, fmaf(ef, 0x1.7f7d1cp-20f, lm));
}

float oracle_gumbel(uint32_t w) {
  float u = oracle_uniform(w);
  u = fminf(fmaxf(u, 0x1.b7cdfep-34f), 0x1.fffffcp-1f);
  return -oracle_log(-oracle_log(u));
}

uint32_t oracle_philox_w0(uint32_t col, const uint32_t key[2]) {
  const uint32_t ctr[4] = {col, 0u, 0u, 0u};
  uint32_t out[4];
  oracle_philox4x32_10(ctr, key, out);
  return out[0];
}

/* Per row: q = x / T (skipped when T == 1), samp = first argmax(q + g), amax = first argmax(q). */
void oracle_gumbel_argmax(const float* x, int64_t rows, int64_t V, float temperature, int64_t seed,
                          int64_t* samp, int64_t* amax, int nthreads) {
  const int do_div = temperature != 1.0f;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t r = 0; r < rows; ++r) {
    uint32_t key[2];
    oracle_row_key(seed, r, key);
    const float* xr = x + r * V;
    float bg = -INFINITY, bq = -INFINITY;
    int64_t bgi = 0, bqi = 0;
    int have_g = 0, have_q = 0;
    for (int64_t c = 0; c < V; ++c) {
      const float q = do_div ? xr[c] / temperature : xr[c];
      if (!have_q || q > bq) { bq = q; bqi = c; have_q = 1; }
      const float v = q + oracle_gumbel(oracle_philox_w0((uint32_t)c, key));
      if (!have_g || v > bg) { bg = v; bgi = c; have_g = 1; }
    }
    if (samp) samp[r] = bgi;
    if (amax) amax[r] = bqi;
  }
}

/* Noise table for tests: g[r, c] for c < V. */
void oracle_gumbel_noise(int64_t rows, int64_t V, int64_t seed, float* g) {
  for (int64_t r = 0; r < rows; ++r) {
    uint32_t key[2];
    oracle_row_key(seed, r, key);
    for (int64_t c = 0; c < V; ++c) g[r * V + c] = oracle_gumbel(oracle_philox_w0((uint32_t)c, key));
  }
}

/* Check (test helper): the product's reciprocal-plus-correction quotient equals IEEE x / t for n
 * pseudo-random normal x.  Returns the number of mismatches. */
int64_t oracle_markstein_mismatches(float t, int64_t n, uint32_t seed) {
  const float r = 1.0f / t;
  int64_t bad = 0;
  uint32_t st = seed ? seed : 1u;
  for (int64_t i = 0; i < n; ++i) {
    st ^= st << 13; st ^= st >> 17; st ^= st << 5;
    uint32_t bits = st;
    /* exponents in [2^-40, 2^40]: the range logits live in, far from overflow/underflow */
    uint32_t ex = 87u + (bits >> 24) % 80u;
    float x = u2f(((bits & 1u) << 31) | (ex << 23) | (bits & 0x7fffffu));
    const float q = x * r;
    const float rem = fmaf(-q, t, x);
    const float qm = fmaf(rem, r, q);
    const float qi = x / t;
    if (f2u(qm) != f2u(qi)) ++bad;
  }
  return bad;
}
