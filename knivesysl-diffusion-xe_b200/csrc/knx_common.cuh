// knx_common.cuh — shared device helpers for the sm_100a kernels (PTX wrappers, f16 packing,
// launch checks).  Everything here is header-only and internal to libknx.so.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "knx.h"

#define KNX_DEVINL __device__ __forceinline__
#define KNX_HOST_DEVINL __host__ __device__ __forceinline__

namespace knx {

// Number of SMs on the current device (cached per device id; B200 = 148).
int num_sms();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device); thread-safe.
int set_max_dyn_smem(const void* func, int bytes);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KNX_OK : KNX_E_LAUNCH;
}

// Programmatic dependent launch.  Every kernel of libknx.so is launched with launch_pdl, which
// lets it start (CTA launch, prologue) while the previous kernel on the stream finishes, and calls
// pdl_wait_trigger() before it touches global memory: that waits until the previous kernel has
// completed and its writes are visible (at once when the previous launch was an ordinary one),
// then allows the next kernel to start launching in turn.  The next kernel is only scheduled once
// every CTA of this one has started, so an early start never takes an SM this kernel still needs.
// (The ws down GEMM with per-task readiness skips the wait: it synchronises with gate_up through
// per-task counters instead; knx_moe_hw.cu.)
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? KNX_OK
                                                                                      : KNX_E_LAUNCH;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- small PTX wrappers -------------------------------------------------------------------

KNX_DEVINL void pdl_wait_trigger() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

KNX_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async copy global -> shared (L2 only, bypass L1).  src_bytes < 16 zero-fills the rest.
KNX_DEVINL void cp_async16(void* smem, const void* gmem, int src_bytes = 16) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(src_bytes));
}
KNX_DEVINL void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
KNX_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
KNX_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Streaming 16-byte global load that does not allocate in L1 (read-once data).
KNX_DEVINL uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

KNX_DEVINL uint32_t lds32(uint32_t addr) {
  uint32_t r;
  asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(r) : "r"(addr));
  return r;
}
KNX_DEVINL void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}
// 32-bit shared load at addr + OFF (the offset folded into the instruction's immediate)
template <int OFF>
KNX_DEVINL uint32_t lds32_at(uint32_t addr) {
  uint32_t r;
  asm volatile("ld.shared.u32 %0, [%1+%2];\n" : "=r"(r) : "r"(addr), "n"(OFF));
  return r;
}
KNX_DEVINL __half lds16h(uint32_t addr) {
  unsigned short r;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(r) : "r"(addr));
  return __ushort_as_half(r);
}
KNX_DEVINL void sts16h(uint32_t addr, __half v) {
  asm volatile("st.shared.u16 [%0], %1;\n" ::"r"(addr), "h"(__half_as_ushort(v)) : "memory");
}
KNX_DEVINL uint4 lds128(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(addr));
  return r;
}
KNX_DEVINL void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// lop3 with immediate truth table: (a & b) | c  -> 0xEA
KNX_DEVINL uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

KNX_DEVINL uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

KNX_DEVINL uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
KNX_DEVINL __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// D = A(16x16, row) * B(16x8, col) + C, f16 inputs, f32 accumulate (legacy warp MMA).
KNX_DEVINL void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- the MoE K-interleave -------------------------------------------------------------------
// Within every group of 8 consecutive k, activations are stored in the order
//   [k0, k4, k1, k5, k2, k6, k3, k7]
// so that one 16-byte shared load yields the two m16n8k16 B-fragments that match the nibble
// pairs (k, k+4) produced by the magic-number dequant below.  Actual k = i (0..7) lives at
// position p(i) = 2*(i%4) + i/4.  The permutation is a bijection inside each 8-group, so the
// GEMM result is the same sum over k, only the summation order inside the tensor core changes.
KNX_DEVINL int kperm_pos(int i) { return 2 * (i & 3) + (i >> 2); }

// Dequantise the 8 nibbles of one u32 (row bytes 4q..4q+3, nibble i = k 8q+i, low nibble = even
// k) into four f16x2 A-fragment registers:  w0 = (k0,k4)  w1 = (k1,k5)  w2 = (k2,k6)  w3 = (k3,k7).
// 0x6400 is f16 1024: OR-ing a low nibble into the mantissa gives h = 1024 + n exactly; a high
// nibble lands at h = 1024 + 16n.  Per (row, group) the caller supplies
//   s  = (s, s),   s16 = (s/16, s/16)
// and, for ZINT (integer zero-points 0..15, what quantize_w4 produces):
//   c  = 1024 + z,  c16 = 1024 + 16z      w = (h - c) * s    = RN16((n - z) * s)     exact
//                                          w = (h - c16) * s16 = RN16((n - z) * s)   exact
// i.e. bit-identical to the fp32 dequant rounded once (dequant_w4);  otherwise (any fp16 z):
//   c  = z,  c16 = 16z                     w = RN16(RN16(n - z) * s)
// which is the fp16 arithmetic of the reference kernel, (w - z) * s (fused_moe_w4_v2.py:126-128).
// (s/16 is exact for s >= 2^-10; smaller scales round their last bits.)
template <bool ZINT>
KNX_DEVINL void dequant8(uint32_t u, __half2 s, __half2 s16, __half2 c, __half2 c16,
                         uint32_t (&w)[4]) {
  const uint32_t MAG = 0x64006400u;
  const uint32_t p0 = lop3_and_or(u, 0x000F000Fu, MAG);
  const uint32_t p1 = lop3_and_or(u, 0x00F000F0u, MAG);
  const uint32_t u8 = u >> 8;
  const uint32_t p2 = lop3_and_or(u8, 0x000F000Fu, MAG);
  const uint32_t p3 = lop3_and_or(u8, 0x00F000F0u, MAG);
  if constexpr (ZINT) {
    w[0] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(p0), c), s));
    w[1] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(p1), c16), s16));
    w[2] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(p2), c), s));
    w[3] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(p3), c16), s16));
  } else {
    const __half2 k1024 = u32_as_h2(MAG);
    w[0] = h2_as_u32(__hmul2(__hsub2(__hsub2(u32_as_h2(p0), k1024), c), s));
    w[1] = h2_as_u32(__hmul2(__hsub2(__hsub2(u32_as_h2(p1), k1024), c16), s16));
    w[2] = h2_as_u32(__hmul2(__hsub2(__hsub2(u32_as_h2(p2), k1024), c), s));
    w[3] = h2_as_u32(__hmul2(__hsub2(__hsub2(u32_as_h2(p3), k1024), c16), s16));
  }
}

// Per (row, group) dequant constants, packed as two f16x2: {s, c} and {s/16, c16} (see dequant8).
template <bool ZINT>
KNX_DEVINL uint2 make_sz(__half s, __half z) {
  const float sf = __half2float(s), zf = __half2float(z);
  const __half s16 = __float2half_rn(sf * 0.0625f);
  const __half c = ZINT ? __float2half_rn(1024.0f + zf) : z;
  const __half c16 = __float2half_rn(ZINT ? 1024.0f + 16.0f * zf : 16.0f * zf);
  uint2 r;
  r.x = (static_cast<uint32_t>(__half_as_ushort(c)) << 16) | __half_as_ushort(s);
  r.y = (static_cast<uint32_t>(__half_as_ushort(c16)) << 16) | __half_as_ushort(s16);
  return r;
}

KNX_DEVINL float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

KNX_DEVINL float load_as_float(const void* p, int dtype, int64_t i) {
  if (dtype == KNX_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == KNX_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

KNX_DEVINL int64_t load_as_i64(const void* p, int dtype, int64_t i) {
  if (dtype == KNX_I64) return reinterpret_cast<const int64_t*>(p)[i];
  return reinterpret_cast<const int32_t*>(p)[i];
}

}  // namespace knx
