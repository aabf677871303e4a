// knx_topk.cuh — the router's per-token softmax / top-k / renormalise by one warp (shared by
// router_topk_kernel and the fused RMSNorm + router kernel, so both give the same bits).
#pragma once
#include "knx_common.cuh"

namespace knx {

constexpr int TK_MAXE = 256;  // experts at most
constexpr int TK_PER = TK_MAXE / 32;

// Order-preserving map of a non-NaN float to uint32 (larger float -> larger key), and back.
KNX_DEVINL uint32_t tk_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
KNX_DEVINL float tk_unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// l[i]: the logit of expert lane + 32 i (-inf for e >= E).  Top-k by logit, ties to the lower
// expert id; weights are the selected softmax probabilities renormalised to sum 1.  Lane k < topk
// writes selection k.  Each selection round is two warp reductions (the largest key, then the
// lowest expert id holding it); the probabilities of the k winners are then formed in parallel,
// each as expf(l - max) / den, and summed in selection order (the arithmetic of a sequential
// round-by-round evaluation, bit for bit).
// PER: logits per lane that can be valid (32 * PER >= E; the entries past it are -inf and add
// exact zeros), TOPK: topk at compile time (0: the runtime value).  Every instantiation gives the
// same bits for the same inputs.
template <int PER, int TOPK>
KNX_DEVINL void topk_select_t(const float (&l_in)[TK_PER], int E, int topk_rt, int lane,
                              int32_t* __restrict__ ids_row, float* __restrict__ w_row) {
  static_assert(PER <= TK_PER, "logits per lane");
  const int topk = TOPK > 0 ? TOPK : topk_rt;
  float l[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    l[i] = l_in[i];
    mx = fmaxf(mx, l[i]);
  }
  mx = tk_unkey(__reduce_max_sync(0xffffffffu, tk_key(fmaxf(mx, -INFINITY))));
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) den += (lane + 32 * i < E) ? expf(l[i] - mx) : 0.f;
  den = warp_sum(den);
  float my_v = -INFINITY;
  int my_i = 0;
#pragma unroll
  for (int k = 0; k < (TOPK > 0 ? TOPK : topk); ++k) {
    // this lane's best: the lowest expert id among its largest values (never NaN)
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
    const uint32_t key = tk_key(bv);
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
    const int win = static_cast<int>(
        __reduce_min_sync(0xffffffffu, key == kmax ? static_cast<uint32_t>(bi) : 0xffffffffu));
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == win) l[i] = -INFINITY;  // remove the winner
    if (lane == k) {
      my_v = tk_unkey(kmax);
      my_i = win;
    }
  }
  const float p = lane < topk ? expf(my_v - mx) / den : 0.f;
  float psum = 0.f;
#pragma unroll
  for (int k = 0; k < (TOPK > 0 ? TOPK : topk); ++k) psum += __shfl_sync(0xffffffffu, p, k);
  if (lane < topk) {
    ids_row[lane] = my_i;
    w_row[lane] = p / psum;
  }
}


// The routine for E experts (<= 256) and topk (<= 16): specialised for 8 selections and for the
// logits per lane that E needs.
KNX_DEVINL void topk_select(const float (&l)[TK_PER], int E, int topk, int lane,
                            int32_t* __restrict__ ids_row, float* __restrict__ w_row) {
  const int per = (E + 31) / 32;
  if (topk == 8) {
    if (per <= 2) topk_select_t<2, 8>(l, E, topk, lane, ids_row, w_row);
    else if (per <= 4) topk_select_t<4, 8>(l, E, topk, lane, ids_row, w_row);
    else topk_select_t<8, 8>(l, E, topk, lane, ids_row, w_row);
  } else {
    if (per <= 2) topk_select_t<2, 0>(l, E, topk, lane, ids_row, w_row);
    else if (per <= 4) topk_select_t<4, 0>(l, E, topk, lane, ids_row, w_row);
    else topk_select_t<8, 0>(l, E, topk, lane, ids_row, w_row);
  }
}

}  // namespace knx
