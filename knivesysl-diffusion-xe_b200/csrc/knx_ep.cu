// knx_ep.cu — the device pieces of the expert-parallel MoE layer (experts sharded over ranks,
// tokens data-parallel), which the host drives between two NCCL all-to-all exchanges:
//
//   source rank: align (global expert ids) -> knx_gather_rows (pairs in sorted order: expert, then
//                pair index t*topk+k) -> all-to-all (dispatch)
//   expert rank: knx_ep_layout (received rows, source-major, re-slotted expert-major) ->
//                knx_moe_w4_grouped (gate_up + GELU, down) -> knx_gather_rows (back to receive
//                order) -> all-to-all (return)
//   source rank: knx_moe_combine (fixed k order, the single-GPU combine)
//
// Every pair's down output is computed by the same engine from the same activation row and
// weights as on one GPU, and the returned rows reach the combine in the single-GPU slot order, so
// the layer output is bit-identical to the single-GPU layer at any rank count (the engine is
// chosen from the job-wide tokens per expert, identically on every rank).
#include "knx_common.cuh"
#include "knx_internal.cuh"

namespace knx {
namespace {

// dst[i, :] = src[idx[i] / div, :] (16-byte vectors; idx < 0: a zero row)
__global__ void gather_rows_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ idx,
                                   int div, int64_t n, int vec_per_row, uint4* __restrict__ dst) {
  pdl_wait_trigger();
  const int64_t i = blockIdx.y * static_cast<int64_t>(gridDim.x) + blockIdx.x;
  if (i >= n) return;
  const int r = idx[i];
  uint4* d = dst + i * vec_per_row;
  if (r < 0) {
    for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) d[v] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* sp = src + static_cast<int64_t>(r / div) * vec_per_row;
  for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) d[v] = ldg_nc_v4(sp + v);
}

constexpr int EPL_MAX = 4096;  // sources x local experts handled by the layout kernel

// Received rows arrive grouped by source, then by local expert, then in the source's pair order.
// The local GEMMs want them grouped by expert: slot order (expert e, source s, j).  Every block
// rebuilds the small prefix tables, then maps slots grid-stride.
__global__ void ep_layout_kernel(const int32_t* __restrict__ cnt, int S, int El, int64_t R,
                                 int32_t* __restrict__ offsets, int32_t* __restrict__ rows,
                                 int32_t* __restrict__ inv) {
  pdl_wait_trigger();
  __shared__ int slot_base[EPL_MAX];  // [e][s]: first slot of (e, s)
  __shared__ int recv_base[EPL_MAX];  // [e][s]: first received row of (s, e)
  __shared__ int off[257];
  __shared__ int src_start[65];
  const int tid = threadIdx.x;
  if (tid == 0) {
    int acc = 0;
    for (int s = 0; s < S; ++s) {
      src_start[s] = acc;
      for (int e = 0; e < El; ++e) acc += cnt[s * El + e];
    }
    acc = 0;
    for (int e = 0; e < El; ++e) {
      off[e] = acc;
      for (int s = 0; s < S; ++s) acc += cnt[s * El + e];
    }
    off[El] = acc;
  }
  __syncthreads();
  for (int e = tid; e < El; e += blockDim.x) {
    int a = off[e];
    for (int s = 0; s < S; ++s) {
      slot_base[e * S + s] = a;
      a += cnt[s * El + e];
    }
  }
  for (int s = tid; s < S; s += blockDim.x) {
    int a = src_start[s];
    for (int e = 0; e < El; ++e) {
      recv_base[e * S + s] = a;
      a += cnt[s * El + e];
    }
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int e = tid; e <= El; e += blockDim.x) offsets[e] = off[e];
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + tid; i < R;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int lo = 0, hi = El - 1;  // last expert with off[e] <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (off[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int e = lo;
    int s = S - 1;
    while (s > 0 && slot_base[e * S + s] > i) --s;
    const int r = recv_base[e * S + s] + static_cast<int>(i - slot_base[e * S + s]);
    rows[i] = r;
    inv[r] = static_cast<int32_t>(i);
  }
}

struct GroupedWs {
  int4* tasks;
  int32_t* ntasks;
  int32_t* counters;
  int n_counters;
  __half* out2;
  size_t bytes;
};

GroupedWs carve_grouped(uint8_t* base, int64_t R, int64_t I, int E) {
  GroupedWs w{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + o : nullptr;
    o += (bytes + 255) & ~size_t(255);
    return p;
  };
  const int64_t max_tasks = (R + MIN_TASK_TOKENS - 1) / MIN_TASK_TOKENS + E;
  w.tasks = reinterpret_cast<int4*>(take(size_t(max_tasks) * 16));
  w.ntasks = reinterpret_cast<int32_t*>(take(16));
  w.counters = reinterpret_cast<int32_t*>(take(size_t(gemm_counter_ints(max_tasks)) * 4));
  w.n_counters = static_cast<int>(gemm_counter_ints(max_tasks));
  w.out2 = reinterpret_cast<__half*>(take(size_t(R) * I * 2));
  w.bytes = o;
  return w;
}

}  // namespace
}  // namespace knx

extern "C" int knx_gather_rows(const void* src, int64_t src_rows, int64_t row_bytes,
                               const int32_t* idx, int div, int64_t n, void* dst, void* stream) {
  using namespace knx;
  if (src_rows < 0 || n < 0 || row_bytes <= 0 || div <= 0 || (row_bytes % 16) != 0)
    return KNX_E_INVALID;
  if (!aligned(src, 16) || !aligned(dst, 16)) return KNX_E_ALIGN;
  if (n == 0) return KNX_OK;
  const int vpr = static_cast<int>(row_bytes / 16);
  const unsigned gx = static_cast<unsigned>(n < 65535 ? n : 65535);
  const unsigned gy = static_cast<unsigned>((n + gx - 1) / gx);
  const int threads = vpr < 256 ? ((vpr + 31) / 32) * 32 : 256;
  (void)launch_pdl(gather_rows_kernel, dim3(gx, gy), threads, 0, static_cast<cudaStream_t>(stream),
                   static_cast<const uint4*>(src), idx, div, n, vpr, static_cast<uint4*>(dst));
  return launch_status();
}

extern "C" int knx_ep_layout(const int32_t* recv_counts, int S, int El, int64_t R,
                             int32_t* offsets, int32_t* rows, int32_t* inv, void* stream) {
  using namespace knx;
  if (S <= 0 || S > 64 || El <= 0 || El > 256 || S * El > EPL_MAX || R < 0 || R > (1LL << 30))
    return KNX_E_INVALID;
  const int64_t blocks = R > 0 ? (R + 255) / 256 : 1;
  (void)launch_pdl(ep_layout_kernel, static_cast<unsigned>(blocks < 1184 ? blocks : 1184), 256, 0,
                   static_cast<cudaStream_t>(stream), recv_counts, S, El, R, offsets, rows, inv);
  return launch_status();
}

extern "C" size_t knx_moe_w4_grouped_workspace_size(int64_t R, int64_t H, int64_t I, int E) {
  if (R < 0 || H <= 0 || I <= 0 || E <= 0) return 0;
  (void)H;
  return knx::carve_grouped(nullptr, R, I, E).bytes;
}

extern "C" int knx_moe_w4_grouped(const void* xrows, const int32_t* rows, int64_t R,
                                  const int32_t* offsets, const uint8_t* gu_q, const void* gu_s,
                                  const void* gu_z, const uint8_t* dn_q, const void* dn_s,
                                  const void* dn_z, int64_t H, int64_t I, int E, int gs_gu,
                                  int gs_dn, int flags, int64_t tokens_per_expert,
                                  void* workspace, size_t workspace_bytes, void* out3,
                                  int32_t* err, void* stream) {
  using namespace knx;
  const bool zint = (flags & KNX_W4_INT_ZEROS) != 0;
  if (R < 0 || H <= 0 || I <= 0 || E <= 0 || E > 256) return KNX_E_INVALID;
  if ((H % 256) != 0 || (I % 64) != 0 || H > (1 << 20) || I > (1 << 20)) return KNX_E_UNSUPPORTED;
  if (gs_gu <= 0 || gs_dn <= 0 || (gs_gu % 32) != 0 || (gs_dn % 32) != 0 || (H % gs_gu) != 0 ||
      (I % gs_dn) != 0)
    return KNX_E_INVALID;
  if (H / gs_gu > 56 || I / gs_dn > 56) return KNX_E_UNSUPPORTED;
  if (!aligned(xrows, 16) || !aligned(out3, 16) || !aligned(gu_q, 16) || !aligned(dn_q, 16) ||
      !aligned(gu_s, 16) || !aligned(gu_z, 16) || !aligned(dn_s, 16) || !aligned(dn_z, 16) ||
      !aligned(workspace, 256))
    return KNX_E_ALIGN;
  if (R == 0) return KNX_OK;
  if (workspace == nullptr || workspace_bytes < knx_moe_w4_grouped_workspace_size(R, H, I, E))
    return KNX_E_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GroupedWs w = carve_grouped(static_cast<uint8_t*>(workspace), R, I, E);
  const int eng = moe_engine(flags, tokens_per_expert, H, I, gs_gu, gs_dn);
  int st = launch_tasks_from_offsets(offsets, E, engine_task_tokens(eng), w.tasks, w.ntasks,
                                     w.counters,
                                     eng == KNX_W4_WARP_WS ? w.n_counters : GEMM_COUNTERS, s);
  if (st != KNX_OK) return st;
  GemmArgs ga{};
  ga.xp = static_cast<const __half*>(xrows);
  ga.sorted_pair = rows;  // slot -> row of xrows (topk 1); NULL: row = slot
  ga.topk = 1;
  ga.offsets = offsets; ga.tasks = w.tasks; ga.ntasks = w.ntasks; ga.counters = w.counters;
  ga.gu_q = gu_q; ga.gu_s = static_cast<const __half*>(gu_s); ga.gu_z = static_cast<const __half*>(gu_z);
  ga.dn_q = dn_q; ga.dn_s = static_cast<const __half*>(dn_s); ga.dn_z = static_cast<const __half*>(dn_z);
  ga.E = E; ga.H = H; ga.I = I; ga.gs_gu = gs_gu; ga.gs_dn = gs_dn; ga.zint = zint;
  ga.out2 = w.out2; ga.out3 = static_cast<__half*>(out3); ga.pairs = R; ga.err = err;
  return run_moe_gemms(ga, eng, -1, s);
}

extern "C" int knx_moe_combine(const void* out3, const int32_t* inv, const void* topk_w,
                               int w_dtype, int64_t T, int topk, int64_t H, int out_dtype,
                               void* out, void* stream) {
  using namespace knx;
  if (T < 0 || topk <= 0 || topk > 16 || H <= 0 || (H % 8) != 0) return KNX_E_INVALID;
  if (out_dtype != KNX_F16 && out_dtype != KNX_BF16) return KNX_E_INVALID;
  if (w_dtype != KNX_F16 && w_dtype != KNX_BF16 && w_dtype != KNX_F32) return KNX_E_INVALID;
  if (!aligned(out3, 16) || !aligned(out, 16)) return KNX_E_ALIGN;
  if (T == 0) return KNX_OK;
  return launch_combine(static_cast<const __half*>(out3), inv, topk_w, w_dtype, T, topk, H,
                        out_dtype, out, static_cast<cudaStream_t>(stream));
}
