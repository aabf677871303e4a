// knx_topk.cuh — the router's per-token softmax / top-k / renormalise by one warp (shared by
// router_topk_kernel and the fused RMSNorm + router kernel, so both give the same bits).
#pragma once
#include "knx_common.cuh"

namespace knx {

constexpr int TK_MAXE = 256;  // experts at most
constexpr int TK_PER = TK_MAXE / 32;

// l[i]: the logit of expert lane + 32 i (-inf for e >= E).  Top-k by logit, ties to the lower
// expert id; weights are the selected softmax probabilities renormalised to sum 1.  Lane k < topk
// writes selection k.
KNX_DEVINL void topk_select(const float (&l_in)[TK_PER], int E, int topk, int lane,
                            int32_t* __restrict__ ids_row, float* __restrict__ w_row) {
  constexpr int PER = TK_PER;
  float l[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    l[i] = l_in[i];
    mx = fmaxf(mx, l[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) den += (lane + 32 * i < E) ? expf(l[i] - mx) : 0.f;
  den = warp_sum(den);
  // top-k selection: k rounds of a warp-wide (max value, min index) reduction; lane k keeps
  // selection k (topk <= 16), so nothing goes through local memory
  float my_p = 0.f;
  int my_i = 0;
  float psum = 0.f;
  for (int k = 0; k < topk; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (l[i] > bv || (l[i] == bv && e < bi))) {
        bv = l[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == bi) l[i] = -INFINITY;  // remove the winner
    const float p = expf(bv - mx) / den;
    if (lane == k) {
      my_p = p;
      my_i = bi;
    }
    psum += p;
  }
  if (lane < topk) {
    ids_row[lane] = my_i;
    w_row[lane] = my_p / psum;
  }
}

}  // namespace knx
