// knx_rms_row.cuh — one RMSNorm row by one warp (the body of rmsnorm_kernel, shared with the
// fused RMSNorm + router kernel so that both produce the same bits).
#pragma once
#include <type_traits>

#include "knx_common.cuh"

namespace knx {
namespace rms {

constexpr int RMS_MAX_VEC = 16;  // 16 lanes-vectors * 8 elements * 32 lanes = 4096 elements

template <typename T>
KNX_DEVINL void unpack8(const uint4& v, float (&f)[8]);
template <>
KNX_DEVINL void unpack8<__half>(const uint4& v, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <>
KNX_DEVINL void unpack8<__nv_bfloat16>(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Eight weights starting at element 8v, as fp32 (WT = void: no weight, all ones).  WS: w points
// to shared memory (a plain load instead of the read-only global path).
template <typename WT, bool WS = false>
KNX_DEVINL void load_w8(const void* w, int v, float (&f)[8]) {
  if constexpr (std::is_same<WT, void>::value) {
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = 1.0f;
  } else if constexpr (std::is_same<WT, float>::value) {
    const float4* p = reinterpret_cast<const float4*>(w) + 2 * v;
    const float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else if constexpr (WS) {
    unpack8<WT>(reinterpret_cast<const uint4*>(w)[v], f);
  } else {
    unpack8<WT>(__ldg(reinterpret_cast<const uint4*>(w) + v), f);
  }
}

template <typename T>
KNX_DEVINL T from_f32(float v, bool round_bf16) {
  if (round_bf16) v = __bfloat162float(__float2bfloat16_rn(v));
  if constexpr (std::is_same<T, __half>::value) {
    return __float2half_rn(v);
  } else {
    return __float2bfloat16_rn(v);
  }
}

// One row: y = x * (1 / sqrt(sum(x^2) / cols + eps)) * w, optionally also the MoE K-interleaved
// f16 copy p (xperm).  The row is read once with 16-byte loads and kept in registers (up to
// RMS_MAX_VEC vectors per lane); wider rows are re-read for the second pass.  Returns 1/rms.
// WS: the weights are in shared memory (same arithmetic).
template <typename T, typename WT, bool WS = false>
KNX_DEVINL float rms_row(const T* __restrict__ xrow, const void* __restrict__ w,
                         T* __restrict__ yrow, __half* __restrict__ prow, int cols, float eps,
                         bool round_bf16, int lane) {
  const int nvec = cols >> 3;  // 8 elements per 16-byte vector
  const uint4* xr = reinterpret_cast<const uint4*>(xrow);
  uint4 cache[RMS_MAX_VEC];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < RMS_MAX_VEC; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      cache[i] = ldg_nc_v4(xr + v);
      float f[8];
      unpack8<T>(cache[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
  }
  for (int v = lane + 32 * RMS_MAX_VEC; v < nvec; v += 32) {
    float f[8];
    unpack8<T>(xr[v], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
  }
  ss = warp_sum(ss);
  const float ms = __fadd_rn(__fdiv_rn(ss, static_cast<float>(cols)), eps);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ms));

  uint4* yr = reinterpret_cast<uint4*>(yrow);
  uint4* pr = prow ? reinterpret_cast<uint4*>(prow) : nullptr;
  auto emit = [&](int v, const uint4& c) {
    float f[8], wf[8];
    unpack8<T>(c, f);
    load_w8<WT, WS>(w, v, wf);
    T out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t = __fmul_rn(f[j], inv);
      if constexpr (!std::is_same<WT, void>::value) t = __fmul_rn(t, wf[j]);
      out[j] = from_f32<T>(t, round_bf16);
    }
    yr[v] = *reinterpret_cast<uint4*>(out);
    if (pr) {
      // MoE K-interleave inside each 8-group: position p(i) = 2*(i%4) + i/4 holds element i.
      __half hp[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float t;
        if constexpr (std::is_same<T, __half>::value) {
          t = __half2float(out[j]);
        } else {
          t = __bfloat162float(out[j]);
        }
        hp[2 * (j & 3) + (j >> 2)] = __float2half_rn(t);
      }
      pr[v] = *reinterpret_cast<uint4*>(hp);
    }
  };
#pragma unroll
  for (int i = 0; i < RMS_MAX_VEC; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) emit(v, cache[i]);
  }
  for (int v = lane + 32 * RMS_MAX_VEC; v < nvec; v += 32) emit(v, xr[v]);
  return inv;
}

}  // namespace rms
}  // namespace knx
