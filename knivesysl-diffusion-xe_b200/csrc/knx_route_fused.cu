// knx_route_fused.cu — RMSNorm + router logits + top-k in one launch, for canvases whose router
// fits one thread-block cluster per 32 tokens (E = 64 or 128).
//
// A cluster of E/64 x 4 CTAs owns 32 tokens: CTA (eb, split) computes the partial logits of
// experts [64 eb, 64 eb + 64) over the K-split `split` (H/4 columns), exactly as
// router_logits_kernel does (same 64-column chunks, same m16n8k16 sequence per output), so the
// partials are the same numbers.  The steps:
//   1. one 1-D bulk copy per row brings the split's K-slice of the 32 token rows and of the 64
//      expert rows (96 copies in flight at once), and one more the norm weights;
//   2. meanwhile each warp normalises whole rows with the RMSNorm row routine of
//      rmsnorm_kernel (rms::rms_row: same loads, same summation order; the weights from shared
//      memory), writing y and the MoE K-interleaved copy, and publishes 1/rms in shared memory —
//      the cluster's CTAs share the 32 rows, 4 or 8 each;
//   3. after a cluster barrier every CTA reads the 32 values of 1/rms over distributed shared
//      memory and normalises its K-slice in place with the same formula as the row routine;
//   4. the MMAs produce the [32 x 64] partial tile (16 tokens x 16 experts per warp), kept in
//      shared memory;
//   5. after a second cluster barrier each warp takes one token, sums the four K-split partials
//      of every expert in split order over distributed shared memory (router_topk_kernel's
//      order), adds the bias and runs the shared softmax / top-k routine (topk_select).
// So y, the interleaved copy, the logits, ids and weights are bit-identical to knx_rmsnorm +
// knx_router_topk.  A third cluster barrier keeps every CTA's tile alive until all reads are done.
#include <cooperative_groups.h>

#include <type_traits>

#include "knx_common.cuh"
#include "knx_rms_row.cuh"
#include "knx_sm100.cuh"
#include "knx_topk.cuh"

namespace cg = cooperative_groups;

namespace knx {
namespace {

constexpr int RF_TOK = 32;                        // tokens per cluster (8 clusters: one wave)
constexpr int RF_EXP = 64;                        // experts per CTA
constexpr int RF_KSPLIT = 4;                      // K-splits (= router_logits_kernel's)
constexpr int RF_BK = 64;                         // k per MMA chunk
constexpr int RF_THREADS = 256;                   // 8 warps
constexpr int RF_MAX_CHUNKS = 15;                 // H <= 3840
constexpr int RF_ROWS = RF_TOK + RF_EXP;          // token rows, then expert rows, per CTA
// A row's K-slice (H/4 f16) padded by 16 bytes: rows 4 banks apart, so the fragment loads of the
// 8 row groups x 4 lanes hit 32 different banks.
constexpr int rf_row_stride(int H) { return (H / RF_KSPLIT) * 2 + 16; }
constexpr size_t rf_part_off(int H) { return static_cast<size_t>(RF_ROWS) * rf_row_stride(H); }
constexpr size_t rf_nw_off(int H) { return rf_part_off(H) + (RF_TOK * RF_EXP + 8 + RF_TOK + 8) * 4; }
constexpr size_t rf_bar_off(int H) { return rf_nw_off(H) + static_cast<size_t>(H) * 2; }
constexpr size_t rf_smem_bytes(int H) { return rf_bar_off(H) + 16; }  // + two mbarriers

// NEB: expert blocks of 64 (E = 64 NEB).
template <int NEB>
__global__ void __launch_bounds__(RF_THREADS)
    route_fused_kernel(const __half* __restrict__ x, const __half* __restrict__ nw, float eps,
                       bool round_bf16, const __half* __restrict__ wr, const float* __restrict__ bias, int T, int H,
                       int E, int topk, __half* __restrict__ y, __half* __restrict__ xperm,
                       float* __restrict__ logits_out, int32_t* __restrict__ ids,
                       float* __restrict__ weights) {
  pdl_wait_trigger();
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t rf_smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  constexpr int neb = NEB;             // expert blocks (the cluster's y extent)
  constexpr int PER = 2 * NEB;         // logits per lane in the top-k
  const int csize = neb * RF_KSPLIT;   // CTAs per cluster
  const int rank = static_cast<int>(cluster.block_rank());  // = eb + neb * split
  const int eb = blockIdx.y, split = blockIdx.z;
  const int t0 = blockIdx.x * RF_TOK;
  const int kper = H / RF_KSPLIT, nchunk = kper / RF_BK, kbeg = split * kper;
  const int e0 = eb * RF_EXP;
  const int RS = rf_row_stride(H);
  uint8_t* slices = rf_smem;                                   // [96 rows][RS]: K-slice per row
  float* part = reinterpret_cast<float*>(rf_smem + rf_part_off(H));  // [32][64]
  float* inv_pub = part + RF_TOK * RF_EXP;                     // [8] 1/rms of own rows
  float* inv_all = inv_pub + 8;                                // [32] the cluster's rows
  __half* nwf = reinterpret_cast<__half*>(rf_smem + rf_nw_off(H));  // [H] norm weights
  uint64_t* bar = reinterpret_cast<uint64_t*>(rf_smem + rf_bar_off(H));  // slices, norm weights

  // 1. one bulk copy per row K-slice (token rows first, then expert rows) and one of the norm
  //    weights, each group on its own mbarrier
  if (tid == 0) {
    sm100::mbar_init(&bar[0], 1);
    sm100::mbar_init(&bar[1], 1);
    sm100::fence_mbar_init();
    sm100::mbar_arrive_expect_tx(&bar[0], static_cast<uint32_t>(RF_ROWS * kper * 2));
    sm100::mbar_arrive_expect_tx(&bar[1], static_cast<uint32_t>(H * 2));
    sm100::bulk_load(nwf, nw, static_cast<uint32_t>(H * 2), &bar[1]);
  }
  __syncthreads();
  // issued by warps 4-7, which have no RMSNorm row: warps 0-3 start their rows at once
  if (tid >= RF_THREADS / 2 && tid < RF_THREADS / 2 + RF_ROWS) {
    const int r = tid - RF_THREADS / 2;
    const __half* src;
    if (r < RF_TOK) {
      const int t = t0 + r;
      src = x + static_cast<int64_t>(t < T ? t : T - 1) * H + kbeg;
    } else {
      src = wr + static_cast<int64_t>(e0 + r - RF_TOK) * H + kbeg;
    }
    sm100::bulk_load(slices + r * RS, src, static_cast<uint32_t>(kper * 2), &bar[0]);
  }

  // 2. RMSNorm of this CTA's rows of the cluster's 32 (whole rows, one warp per row)
  const int rpc = RF_TOK / csize;  // 4 or 8
  if (warp < rpc) (void)sm100::mbar_wait(&bar[1], 0);  // norm weights in shared memory
  for (int r = warp; r < rpc; r += RF_THREADS / 32) {
    const int t = t0 + rank * rpc + r;
    float inv = 0.f;
    if (t < T)
      inv = rms::rms_row<__half, __half, true>(x + static_cast<int64_t>(t) * H, nwf,
                                               y + static_cast<int64_t>(t) * H,
                                               xperm ? xperm + static_cast<int64_t>(t) * H : nullptr,
                                               H, eps, round_bf16, lane);
    if (lane == 0) inv_pub[r] = inv;
  }
  cluster.sync();  // 1/rms of every row of the cluster published

  // 3. the 32 values of 1/rms, then the K-slice normalised in place (the row routine's formula)
  if (tid < RF_TOK) {
    const float* src = cluster.map_shared_rank(inv_pub, tid / rpc);
    inv_all[tid] = src[tid % rpc];
  }
  // a wait that ran out leaves the slices undefined but keeps every CTA on the cluster barriers
  (void)sm100::mbar_wait(&bar[0], 0);
  (void)sm100::mbar_wait(&bar[1], 0);
  __syncthreads();
  const int vpr = kper / 8;  // 16-byte vectors per row slice
  // thread i of the CTA takes vectors i, i + 256, ... of the 32 x vpr: (row, vector) advanced
  // incrementally; the bf16 rounding flag is folded at compile time
  auto normalise = [&](auto rb) {
    constexpr bool RB = decltype(rb)::value;
    const int dr = RF_THREADS / vpr, dv = RF_THREADS - dr * vpr;
    const uint32_t wbase = smem_u32(nwf + kbeg);
    auto advance = [&](int& r, int& v) {
      v += dv;
      r += dr;
      if (v >= vpr) {
        v -= vpr;
        ++r;
      }
    };
    auto emit = [&](uint32_t a, const uint4& xv, const uint4& wv, float inv) {
      float f[8], wf[8];
      rms::unpack8<__half>(xv, f);
      rms::unpack8<__half>(wv, wf);
      __half out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        out[j] = rms::from_f32<__half>(__fmul_rn(__fmul_rn(f[j], inv), wf[j]), RB);
      const uint4 o = *reinterpret_cast<const uint4*>(out);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(o.x), "r"(o.y), "r"(o.z),
                   "r"(o.w)
                   : "memory");
    };
    int r = tid / vpr, v = tid - r * vpr;
    // two vectors per pass: both loads are issued before either store
    while (r < RF_TOK) {
      int r2 = r, v2 = v;
      advance(r2, v2);
      const uint32_t a1 = smem_u32(slices + r * RS + v * 16);
      const uint4 x1 = lds128(a1), w1 = lds128(wbase + 16u * v);
      const float i1 = inv_all[r];
      if (r2 < RF_TOK) {
        const uint32_t a2 = smem_u32(slices + r2 * RS + v2 * 16);
        const uint4 x2 = lds128(a2), w2 = lds128(wbase + 16u * v2);
        const float i2 = inv_all[r2];
        emit(a1, x1, w1, i1);
        emit(a2, x2, w2, i2);
      } else {
        emit(a1, x1, w1, i1);
      }
      r = r2;
      v = v2;
      advance(r, v);
    }
  };
  if (round_bf16) normalise(std::true_type{});
  else normalise(std::false_type{});
  __syncthreads();

  // 4. partial logits of this K-split: warp w takes tokens [16 (w & 1), +16) (one m16 tile) and
  //    experts [16 (w >> 1), +16) (two n8 tiles)
  const int tm = 16 * (warp & 1), en = 16 * (warp >> 1);
  // two accumulator sets (even / odd k16 steps), added once at the end: half the dependent
  // MMA chain; the fused and the standalone router use the same order
  float acc[2][2][4] = {};
  for (int c = 0; c < nchunk; ++c) {
    const uint32_t bx = smem_u32(slices) + c * (RF_BK * 2);
    const uint32_t bw = bx + RF_TOK * RS;
#pragma unroll
    for (int ks = 0; ks < RF_BK / 16; ++ks) {
      const int kb = ks * 32 + q * 4;  // byte offset of k = 16*ks + 2q
      const uint32_t a0 = lds32(bx + (tm + g) * RS + kb);
      const uint32_t a1 = lds32(bx + (tm + g + 8) * RS + kb);
      const uint32_t a2 = lds32(bx + (tm + g) * RS + kb + 16);
      const uint32_t a3 = lds32(bx + (tm + g + 8) * RS + kb + 16);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t b0 = lds32(bw + (en + 8 * nt + g) * RS + kb);
        const uint32_t b1 = lds32(bw + (en + 8 * nt + g) * RS + kb + 16);
        mma_16816(acc[nt][ks & 1], a0, a1, a2, a3, b0, b1);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int e = en + 8 * nt + 2 * q;
    part[(tm + g) * RF_EXP + e] = acc[nt][0][0] + acc[nt][1][0];
    part[(tm + g) * RF_EXP + e + 1] = acc[nt][0][1] + acc[nt][1][1];
    part[(tm + g + 8) * RF_EXP + e] = acc[nt][0][2] + acc[nt][1][2];
    part[(tm + g + 8) * RF_EXP + e + 1] = acc[nt][0][3] + acc[nt][1][3];
  }
  cluster.sync();  // every partial tile of the cluster complete

  // 5. one warp per token: split partials in split order, bias, softmax / top-k
  for (int j = rank * rpc + warp; j < (rank + 1) * rpc; j += RF_THREADS / 32) {
    const int t = t0 + j;
    if (t >= T) continue;  // warp-uniform
    // every partial (and bias) load first, all in flight together; then the sums in split order
    float pv[PER][RF_KSPLIT], bv[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        const int ebk = e / RF_EXP, el = e - ebk * RF_EXP;
#pragma unroll
        for (int s = 0; s < RF_KSPLIT; ++s)
          pv[i][s] = cluster.map_shared_rank(part, ebk + neb * s)[j * RF_EXP + el];
        bv[i] = bias ? bias[e] : 0.f;
      }
    }
    float l[TK_PER];
#pragma unroll
    for (int i = 0; i < TK_PER; ++i) {
      const int e = lane + 32 * i;
      float v = -INFINITY;
      if (i >= PER) {  // experts past E
        l[i] = v;
        continue;
      }
      if (e < E) {
        v = 0.f;
#pragma unroll
        for (int s = 0; s < RF_KSPLIT; ++s) v += pv[i][s];
        if (bias) v += bv[i];
        if (logits_out) logits_out[static_cast<int64_t>(t) * E + e] = v;
      }
      l[i] = v;
    }
    if (topk == 8)
      topk_select_t<PER, 8>(l, E, topk, lane, ids + static_cast<int64_t>(t) * topk,
                            weights + static_cast<int64_t>(t) * topk);
    else
      topk_select_t<PER, 0>(l, E, topk, lane, ids + static_cast<int64_t>(t) * topk,
                            weights + static_cast<int64_t>(t) * topk);
  }
  cluster.sync();  // no CTA leaves while another still reads its tile
}

}  // namespace
}  // namespace knx

extern "C" int knx_rmsnorm_router_topk(const void* x, const void* norm_w, float eps, int flags,
                                       const void* wr, const float* bias, int64_t T, int64_t H, int E, int topk,
                                       void* y, void* xperm, float* logits_out, int32_t* ids,
                                       float* weights, void* stream) {
  using namespace knx;
  if (T < 0 || H <= 0 || T > (1 << 24) || topk < 1 || topk > 16 || topk > E) return KNX_E_INVALID;
  if ((H % 256) != 0 || H / 256 > RF_MAX_CHUNKS || (E != 64 && E != 128)) return KNX_E_UNSUPPORTED;
  if (!aligned(x, 16) || !aligned(norm_w, 16) || !aligned(wr, 16) || !aligned(y, 16) ||
      (xperm && !aligned(xperm, 16)))
    return KNX_E_ALIGN;
  if (T == 0) return KNX_OK;
  const int neb = E / RF_EXP;
  auto kern = neb == 1 ? route_fused_kernel<1> : route_fused_kernel<2>;
  if (set_max_dyn_smem(reinterpret_cast<const void*>(kern),
                       static_cast<int>(rf_smem_bytes(RF_MAX_CHUNKS * 256))) != KNX_OK)
    return KNX_E_DEVICE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((T + RF_TOK - 1) / RF_TOK), neb, RF_KSPLIT);
  cfg.blockDim = dim3(RF_THREADS);
  cfg.dynamicSmemBytes = rf_smem_bytes(static_cast<int>(H));
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(neb);
  attr[0].val.clusterDim.z = RF_KSPLIT;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, static_cast<const __half*>(x),
                         static_cast<const __half*>(norm_w), eps,
                         (flags & KNX_RMS_ROUND_BF16) != 0, static_cast<const __half*>(wr),
                         bias, static_cast<int>(T), static_cast<int>(H), E, topk,
                         static_cast<__half*>(y), static_cast<__half*>(xperm), logits_out, ids,
                         weights) != cudaSuccess)
    return KNX_E_LAUNCH;
  return launch_status();
}
