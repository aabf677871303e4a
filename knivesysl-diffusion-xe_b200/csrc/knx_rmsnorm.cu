// knx_rmsnorm.cu — single-launch RMSNorm (replaces fused_rmsnorm.py:10-32).
//
// One warp per row, two rows per CTA (a 256-row canvas spreads over 128 SMs).  A row is read
// once with 16-byte loads and kept in registers (up to RMS_MAX_VEC vectors per lane, 4096 16-bit
// elements per row); wider rows are re-read from L2 for the second pass.  The weight is read with
// 16-byte loads in its own dtype.  Math is fp32: ms = sum(x^2)/cols + eps,
// y = x * (1/sqrt(ms)) * w.  HBM-bound: 2 * rows * cols * 2 bytes + cols * 2 bytes of weight.
#include <type_traits>

#include "knx_common.cuh"
#include "knx_rms_row.cuh"

namespace knx {
namespace {

constexpr int RMS_WARPS = 2;
using namespace rms;

template <typename T, typename WT>
__global__ void __launch_bounds__(RMS_WARPS * 32)
    rmsnorm_kernel(const T* __restrict__ x, const void* __restrict__ w,
                   T* __restrict__ y, __half* __restrict__ xperm, int64_t rows, int cols,
                   float eps, bool round_bf16) {
  pdl_wait_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RMS_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  rms_row<T, WT>(x + row * cols, w, y + row * cols, xperm ? xperm + row * cols : nullptr, cols, eps,
                 round_bf16, lane);
}

}  // namespace
}  // namespace knx

extern "C" int knx_rmsnorm(const void* x, const void* w, int w_dtype, void* y, void* xperm,
                           int64_t rows, int64_t cols, float eps, int dtype, int flags,
                           void* stream) {
  using namespace knx;
  if (rows < 0 || cols <= 0 || (cols % 8) != 0 || cols > (1 << 24)) return KNX_E_INVALID;
  if (dtype != KNX_F16 && dtype != KNX_BF16) return KNX_E_INVALID;
  if (w != nullptr && w_dtype != KNX_F16 && w_dtype != KNX_BF16 && w_dtype != KNX_F32)
    return KNX_E_INVALID;
  if (!aligned(x, 16) || !aligned(y, 16) || (xperm && !aligned(xperm, 16))) return KNX_E_ALIGN;
  if (rows == 0) return KNX_OK;
  const bool rb = (flags & KNX_RMS_ROUND_BF16) != 0;
  if (w != nullptr && !aligned(w, 16)) return KNX_E_ALIGN;
  const dim3 grid(static_cast<unsigned>((rows + RMS_WARPS - 1) / RMS_WARPS));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto xt, auto wt) {
    using T = decltype(xt);
    using WT = std::remove_pointer_t<decltype(wt)>;
    (void)launch_pdl(rmsnorm_kernel<T, WT>, grid, RMS_WARPS * 32, 0, s, static_cast<const T*>(x), w,
                     static_cast<T*>(y), static_cast<__half*>(xperm), rows, static_cast<int>(cols),
                     eps, rb);
  };
  auto with_w = [&](auto xt) {
    if (w == nullptr) launch(xt, static_cast<void*>(nullptr));
    else if (w_dtype == KNX_F16) launch(xt, static_cast<__half*>(nullptr));
    else if (w_dtype == KNX_BF16) launch(xt, static_cast<__nv_bfloat16*>(nullptr));
    else launch(xt, static_cast<float*>(nullptr));
  };
  if (dtype == KNX_F16) with_w(__half{});
  else with_w(__nv_bfloat16{});
  return launch_status();
}
