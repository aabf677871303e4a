// knx_math.cuh — bit-reproducible random and logarithm routines for the sampler.
//
// Philox4x32-10 is the counter-based generator of Salmon, Moraes, Dror and Shaw, "Parallel
// random numbers: as easy as 1, 2, 3" (SC'11).  The round structure, multipliers and Weyl key
// increments below are the published ones; the key/counter assignment and the uint->uniform map
// follow Triton's tl.rand (triton/language/random.py: philox_impl, randint, uint_to_uniform_float),
// which the reference calls at fused_sampler_ops.py:66.
//
// knx_log is this library's own natural logarithm, built only from IEEE-rounded +, *, fma and
// division so that a CPU restatement with the same operation sequence reproduces it bit for bit:
//   x = 2^e * m, m in [sqrt(1/2), sqrt(2));  f = m - 1;  s = f / (2 + f);
//   log(m) = 2*atanh(s) = s * (2 + z*(2/3 + z*(2/5 + z*(2/7 + z*(2/9 + z*2/11))))),  z = s*s
// (the Taylor series of atanh; |s| <= 0.1716 so the first omitted term is below 2^-28 relative),
//   log(x) = e*ln2_hi + (e*ln2_lo + log(m))   with ln2 split so e*ln2_hi is exact.
// Valid for positive normal x, which is all the Gumbel transform feeds it.
#pragma once
#include <stdint.h>

namespace knx {

constexpr uint32_t PHILOX_M0 = 0xD2511F53u;  // multiplier applied to counter word 0
constexpr uint32_t PHILOX_M1 = 0xCD9E8D57u;  // multiplier applied to counter word 2
constexpr uint32_t PHILOX_W0 = 0x9E3779B9u;  // Weyl increment, key word 0
constexpr uint32_t PHILOX_W1 = 0xBB67AE85u;  // Weyl increment, key word 1

// First output word of Philox4x32-10 for counter (c0, 0, 0, 0) and key (k0, k1).
__device__ __forceinline__ uint32_t philox_w0(uint32_t c0, uint32_t k0, uint32_t k1) {
  uint32_t c1 = 0u, c2 = 0u, c3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(PHILOX_M0, c0), lo0 = PHILOX_M0 * c0;
    const uint32_t hi2 = __umulhi(PHILOX_M1, c2), lo2 = PHILOX_M1 * c2;
    const uint32_t n0 = hi2 ^ c1 ^ k0;
    const uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo2;
    c2 = n2;
    c3 = lo0;
    k0 += PHILOX_W0;
    k1 += PHILOX_W1;
  }
  return c0;
}

// philox_w0 for two counters under one key: the same rounds, with the key schedule shared.
__device__ __forceinline__ void philox_w0_x2(uint32_t a0, uint32_t b0, uint32_t k0, uint32_t k1,
                                             uint32_t& wa, uint32_t& wb) {
  uint32_t a1 = 0u, a2 = 0u, a3 = 0u, b1 = 0u, b2 = 0u, b3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t ha0 = __umulhi(PHILOX_M0, a0), la0 = PHILOX_M0 * a0;
    const uint32_t ha2 = __umulhi(PHILOX_M1, a2), la2 = PHILOX_M1 * a2;
    const uint32_t hb0 = __umulhi(PHILOX_M0, b0), lb0 = PHILOX_M0 * b0;
    const uint32_t hb2 = __umulhi(PHILOX_M1, b2), lb2 = PHILOX_M1 * b2;
    const uint32_t na0 = ha2 ^ a1 ^ k0, na2 = ha0 ^ a3 ^ k1;
    const uint32_t nb0 = hb2 ^ b1 ^ k0, nb2 = hb0 ^ b3 ^ k1;
    a0 = na0; a1 = la2; a2 = na2; a3 = la0;
    b0 = nb0; b1 = lb2; b2 = nb2; b3 = lb0;
    k0 += PHILOX_W0;
    k1 += PHILOX_W1;
  }
  wa = a0;
  wb = b0;
}

// Triton's uint_to_uniform_float for 32-bit words: reinterpret as int32, fold negatives with
// -x-1, convert to fp32 (round to nearest) and scale by the largest float below 2^-31.
__device__ __forceinline__ float uint_to_uniform(uint32_t w) {
  int32_t x = static_cast<int32_t>(w);
  x = x < 0 ? -x - 1 : x;
  return __fmul_rn(__int2float_rn(x), __uint_as_float(0x2fffffffu));
}

__device__ __forceinline__ float knx_log(float x) {
  const uint32_t bits = __float_as_uint(x);
  int e = static_cast<int>(bits >> 23) - 127;
  float m = __uint_as_float((bits & 0x007fffffu) | 0x3f800000u);  // [1, 2)
  if (m > __uint_as_float(0x3fb504f3u)) {                          // > sqrt(2)
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  const float f = __fsub_rn(m, 1.0f);
  const float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
  const float z = __fmul_rn(s, s);
  float p = __fmaf_rn(z, 0x1.745d18p-3f, 0x1.c71c72p-3f);  // 2/11, 2/9
  p = __fmaf_rn(z, p, 0x1.24924ap-2f);                      // 2/7
  p = __fmaf_rn(z, p, 0x1.99999ap-2f);                      // 2/5
  p = __fmaf_rn(z, p, 0x1.555556p-1f);                      // 2/3
  p = __fmaf_rn(z, p, 2.0f);
  const float lm = __fmul_rn(s, p);
  const float ef = static_cast<float>(e);
  return __fmaf_rn(ef, 0x1.62e400p-1f, __fmaf_rn(ef, 0x1.7f7d1cp-20f, lm));
}

// Gumbel noise exactly as fused_sampler_ops.py:66-69: clamp u to [1e-10, 1-1e-7], -log(-log u).
__device__ __forceinline__ float gumbel_from_word(uint32_t w) {
  float u = uint_to_uniform(w);
  u = fminf(fmaxf(u, 0x1.b7cdfep-34f), 0x1.fffffcp-1f);
  return -knx_log(-knx_log(u));
}

// Upper bound of gumbel_from_word over all inputs: u <= 1-1e-7 gives -log(u) >= 1.19e-7,
// so g <= -log(1.19e-7) = 15.94.  Used to skip elements that cannot win the Gumbel argmax.
constexpr float GUMBEL_MAX = 15.95f;

// IEEE x / t for normal x and t via the reciprocal plus one Markstein correction:
//   r = RN(1/t), q = RN(x*r), rem = x - q*t (exact by fma), RN(q + rem*r) == RN(x/t).
__device__ __forceinline__ float div_rn_by(float x, float t, float r) {
  const float q = __fmul_rn(x, r);
  const float rem = __fmaf_rn(-q, t, x);
  return __fmaf_rn(rem, r, q);
}

// The |x| range in which div_rn_by is the IEEE quotient for t > 0: x * r and x / t stay below
// 3e38 (no overflow), and |x| >= 2^-100 * max(t, 1) keeps the quotient normal and the remainder
// x - q*t (a multiple of 2^(e_x - 46)) representable.  Zeros, infinities, NaN and values outside
// the range take the IEEE division itself (div_exact).
__device__ __forceinline__ float div_fast_lo(float t) { return 0x1p-100f * fmaxf(t, 1.0f); }
__device__ __forceinline__ float div_fast_hi(float t) { return 3.0e38f * fminf(t, 1.0f); }
__device__ __forceinline__ float div_exact(float x, float t, float r, float lo, float hi) {
  const float a = fabsf(x);
  return (a >= lo && a <= hi) ? div_rn_by(x, t, r) : __fdiv_rn(x, t);
}

}  // namespace knx
