// knx_ep_p2p.cu — expert-parallel dispatch and return by direct stores into the peers' memory
// over NVLink, with no host synchronisation and no collective library in the data path.
//
// Experts are sharded round-robin: rank r owns the global experts e = el * world + r, local
// index el (a skewed router, e.g. one biased towards low expert ids, then loads every rank
// alike).  Each rank owns one symmetric region (the same layout on every rank, mapped into every
// peer's address space): barrier flags, the [world][E] matrix of per-expert pair counts, the
// receive rows and the return rows.  One layer:
//   knx_ep_p2p_counts    this rank's counts into every peer's matrix row `rank`; barrier; then
//                        (one CTA) every offset of the exchange from the full matrix — the plan;
//   knx_ep_p2p_dispatch  each of this rank's pairs (its align order: expert, then pair index)
//                        is copied into the owning rank's receive rows at its final slot, so the
//                        receiver's rows are already in the grouped GEMMs' order (local expert,
//                        then source rank, then the source's order);
//   knx_ep_p2p_barrier   every rank's stores have landed;
//   (knx_moe_w4_grouped on the receive rows, offsets from the plan)
//   knx_ep_p2p_return    each result row goes back into its source rank's return rows at the
//                        source's align slot; barrier; knx_moe_combine there.
// The rows every GEMM sees and the order the combine reads them in are those of the single-GPU
// layer, so the output is bit-identical to it (as with the NCCL exchange).
//
// Barriers are epoch counters: a rank stores `epoch` into flag `rank` of every peer (release,
// system scope) and waits until all its own flags have reached it (acquire).  Epochs only grow,
// so no flag is ever reset.  Every wait gives up after 2 s and sets KNX_DEV_TIMEOUT.  When the
// counts barrier gives up, the count matrix may be partial, so the plan is written empty: no
// expert slot (dest_base < 0: the dispatch stores nothing), no receive rows (the grouped GEMMs and
// the return do nothing).  The layer's output is then invalid and the error word says so.
#include "knx_common.cuh"
#include "knx_internal.cuh"
#include "knx_sm100.cuh"

namespace knx {
namespace {

constexpr int P2P_MAX_WORLD = 8;
constexpr int P2P_MAX_E = 256;

KNX_DEVINL void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
KNX_DEVINL uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread: publish `epoch` to every rank, wait (bounded) until every rank published it here.
KNX_DEVINL bool p2p_barrier(uint32_t* const* peer_flags, int rank, int world, uint32_t epoch,
                            int32_t* err) {
  __threadfence_system();
  for (int r = 0; r < world; ++r) st_release_sys(peer_flags[r] + rank, epoch);
  const uint32_t* mine = peer_flags[rank];
  const uint64_t t0 = sm100::globaltimer();
  for (int s = 0; s < world; ++s) {
    while (static_cast<int32_t>(ld_acquire_sys(mine + s) - epoch) < 0) {
      if (sm100::globaltimer() - t0 > 2000000000ull) {
        if (err) atomicOr(err, KNX_DEV_TIMEOUT);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// Every thread's peer stores of this CTA are ordered before one system-scope fence (the CTA
// barrier makes them visible to thread 0, whose fence is cumulative); the next barrier kernel's
// release stores then publish them.  One fence per CTA instead of one per warp.
KNX_DEVINL void cta_fence_system() {
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
}

KNX_DEVINL int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Exclusive scan of a[0..n) by one warp into out[0..n], out[n] = total.
KNX_DEVINL void warp_excl_scan(const int* a, int n, int* out, int lane) {
  int run = 0;
  for (int c = 0; c < n; c += 32) {
    const int v = c + lane < n ? a[c + lane] : 0;
    const int incl = warp_incl_scan(v, lane);
    if (c + lane < n) out[c + lane] = run + incl - v;
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) out[n] = run;
}

// plan layout (int32): dest_base[E] | recv_off[El + 1] | seg_start[El*world + 1] | src_base[El*world]
__global__ void __launch_bounds__(256)
    p2p_counts_kernel(const int32_t* __restrict__ counts, int E, int El, int rank, int world,
                      int32_t* const* __restrict__ peer_cnt, uint32_t* const* __restrict__ peer_flags,
                      uint32_t epoch, int32_t* __restrict__ plan, int32_t* __restrict__ err) {
  pdl_wait_trigger();
  __shared__ int tot_own[P2P_MAX_E];  // pairs per expert from all ranks, owner-major [r][el]
  __shared__ int own_off[P2P_MAX_E + P2P_MAX_WORLD];   // per owner: scan of tot over its experts
  __shared__ int srcpre[P2P_MAX_WORLD][P2P_MAX_E + 1];  // per source: scan of its counts
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int r = 0; r < world; ++r)
    for (int e = tid; e < E; e += blockDim.x) peer_cnt[r][rank * E + e] = counts[e];
  __shared__ int met;
  __syncthreads();
  if (tid == 0) met = p2p_barrier(peer_flags, rank, world, epoch, err) ? 1 : 0;
  __syncthreads();
  int32_t* dest_base = plan;
  int32_t* recv_off = dest_base + E;
  int32_t* seg_start = recv_off + El + 1;
  int32_t* src_base = seg_start + El * world + 1;
  if (!met) {  // the empty plan (see the file comment)
    for (int e = tid; e < E; e += blockDim.x) dest_base[e] = -1;
    for (int i = tid; i <= El; i += blockDim.x) recv_off[i] = 0;
    for (int i = tid; i <= El * world; i += blockDim.x) seg_start[i] = 0;
    return;
  }
  const int32_t* cnt = peer_cnt[rank];  // [world][E], complete after the barrier
  for (int e = tid; e < E; e += blockDim.x) {
    int a = 0;
    for (int s = 0; s < world; ++s) a += cnt[s * E + e];
    tot_own[(e % world) * El + e / world] = a;
  }
  __syncthreads();
  if (warp < world) {
    warp_excl_scan(cnt + warp * E, E, srcpre[warp], lane);
    // owner `warp`: offsets of its local experts in its receive rows
    warp_excl_scan(tot_own + warp * El, El, own_off + warp * (El + 1), lane);
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    const int r = e % world, el = e / world;
    int a = own_off[r * (El + 1) + el];
    for (int s = 0; s < rank; ++s) a += cnt[s * E + e];
    dest_base[e] = a;  // first slot of this rank's pairs of expert e in owner r's rows
  }
  for (int el = tid; el <= El; el += blockDim.x) recv_off[el] = own_off[rank * (El + 1) + el];
  for (int i = tid; i < El * world; i += blockDim.x) {
    const int el = i / world, s = i - el * world, e = el * world + rank;
    int a = own_off[rank * (El + 1) + el];
    for (int s2 = 0; s2 < s; ++s2) a += cnt[s2 * E + e];
    seg_start[i] = a;            // first local row from source s for local expert el
    src_base[i] = srcpre[s][e];  // that source's align slot of its first pair of expert e
  }
  if (tid == 0) seg_start[El * world] = own_off[rank * (El + 1) + El];
}

// One warp per source slot j (this rank's align order): the pair's activation row into the
// owning rank's receive rows.
__global__ void __launch_bounds__(256)
    p2p_dispatch_kernel(const uint4* __restrict__ xp, int vpr, int topk,
                        const int32_t* __restrict__ sorted_pair,
                        const int32_t* __restrict__ offsets, int E, int El,
                        const int32_t* __restrict__ plan, uint4* const* __restrict__ peer_rows,
                        int64_t n_cap) {
  pdl_wait_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (j < n_cap && j < offsets[E]) {
    int lo = 0, hi = E - 1;  // the expert of slot j: last e with offsets[e] <= j
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (offsets[mid] <= j) lo = mid; else hi = mid - 1;
    }
    const int e = lo, r = e % (E / El);  // owner: round-robin sharding
    if (plan[e] >= 0) {                  // plan[e] < 0: the counts barrier gave up (empty plan)
      const int64_t dst = plan[e] + (j - offsets[e]);
      const uint4* s = xp + static_cast<int64_t>(sorted_pair[j] / topk) * vpr;
      uint4* d = peer_rows[r] + dst * vpr;
      for (int v = lane; v < vpr; v += 32) d[v] = ldg_nc_v4(s + v);
    }
  }
  cta_fence_system();
}

// One warp per local row j (expert-major): the result row back into its source rank's return
// rows at the source's align slot.
__global__ void __launch_bounds__(256)
    p2p_return_kernel(const uint4* __restrict__ out3, int vpr, int El, int world,
                      const int32_t* __restrict__ plan, int E, uint4* const* __restrict__ peer_ret,
                      int64_t r_cap) {
  pdl_wait_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int32_t* seg_start = plan + E + El + 1;
  const int32_t* src_base = seg_start + El * world + 1;
  const int nseg = El * world;
  if (j < r_cap && j < seg_start[nseg]) {
    int lo = 0, hi = nseg - 1;  // last segment (el, s) starting at or before j
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seg_start[mid] <= j) lo = mid; else hi = mid - 1;
    }
    const int s = lo % world;
    const int64_t dst = src_base[lo] + (j - seg_start[lo]);
    const uint4* src = out3 + j * vpr;
    uint4* d = peer_ret[s] + dst * vpr;
    for (int v = lane; v < vpr; v += 32) d[v] = ldg_nc_v4(src + v);
  }
  cta_fence_system();
}

// Dispatch, then the barrier, in one launch.  Warps take the slots in a grid-stride loop (the
// expert of a slot by binary search over the offsets staged in shared memory); every CTA orders
// its peer stores before one system-scope fence and then counts itself in `arrive`; the CTA that
// arrives last resets the counter and runs the epoch barrier.  A CTA's fence precedes its
// increment, and the last CTA fences again after reading the full count, so every CTA's stores
// are ordered before the release stores of the epoch (fence-to-fence synchronisation through the
// counter).
__global__ void __launch_bounds__(256)
    p2p_dispatch_bar_kernel(const uint4* __restrict__ xp, int vpr, int topk,
                            const int32_t* __restrict__ sorted_pair,
                            const int32_t* __restrict__ offsets, int E, int El,
                            const int32_t* __restrict__ plan, uint4* const* __restrict__ peer_rows,
                            int64_t n_cap, uint32_t* const* __restrict__ peer_flags, int rank,
                            int world, uint32_t epoch, uint32_t* __restrict__ arrive,
                            int32_t* __restrict__ err) {
  pdl_wait_trigger();
  __shared__ int s_off[P2P_MAX_E + 1];
  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_off[i] = offsets[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const int64_t nslots = min(n_cap, static_cast<int64_t>(s_off[E]));
  const int64_t step = static_cast<int64_t>(gridDim.x) * wpb;
  for (int64_t j = blockIdx.x * static_cast<int64_t>(wpb) + (threadIdx.x >> 5); j < nslots;
       j += step) {
    int lo = 0, hi = E - 1;  // the expert of slot j: last e with offsets[e] <= j
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_off[mid] <= j) lo = mid; else hi = mid - 1;
    }
    const int e = lo, r = e % (E / El);  // owner: round-robin sharding
    if (plan[e] >= 0) {                  // plan[e] < 0: the counts barrier gave up (empty plan)
      const int64_t dst = plan[e] + (j - s_off[e]);
      const uint4* src = xp + static_cast<int64_t>(sorted_pair[j] / topk) * vpr;
      uint4* d = peer_rows[r] + dst * vpr;
      for (int v = lane; v < vpr; v += 32) d[v] = ldg_nc_v4(src + v);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(arrive, 1u) == gridDim.x - 1) {
      *arrive = 0u;  // the next launch starts after this kernel has completed
      p2p_barrier(peer_flags, rank, world, epoch, err);
    }
  }
}

// Return, then the barrier, in one launch (the same pattern as p2p_dispatch_bar_kernel; the
// segment of a local row by binary search over the segment starts staged in shared memory).
__global__ void __launch_bounds__(256)
    p2p_return_bar_kernel(const uint4* __restrict__ out3, int vpr, int El, int world,
                          const int32_t* __restrict__ plan, int E,
                          uint4* const* __restrict__ peer_ret, int64_t r_cap,
                          uint32_t* const* __restrict__ peer_flags, int rank, uint32_t epoch,
                          uint32_t* __restrict__ arrive, int32_t* __restrict__ err) {
  pdl_wait_trigger();
  __shared__ int s_seg[P2P_MAX_E + 1];
  const int32_t* seg_start = plan + E + El + 1;
  const int32_t* src_base = seg_start + El * world + 1;
  const int nseg = El * world;
  for (int i = threadIdx.x; i <= nseg; i += blockDim.x) s_seg[i] = seg_start[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const int64_t nrows = min(r_cap, static_cast<int64_t>(s_seg[nseg]));
  const int64_t step = static_cast<int64_t>(gridDim.x) * wpb;
  for (int64_t j = blockIdx.x * static_cast<int64_t>(wpb) + (threadIdx.x >> 5); j < nrows;
       j += step) {
    int lo = 0, hi = nseg - 1;  // last segment (el, s) starting at or before j
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_seg[mid] <= j) lo = mid; else hi = mid - 1;
    }
    const int s = lo % world;
    const int64_t dst = src_base[lo] + (j - s_seg[lo]);
    const uint4* src = out3 + j * vpr;
    uint4* d = peer_ret[s] + dst * vpr;
    for (int v = lane; v < vpr; v += 32) d[v] = ldg_nc_v4(src + v);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(arrive, 1u) == gridDim.x - 1) {
      *arrive = 0u;
      p2p_barrier(peer_flags, rank, world, epoch, err);
    }
  }
}

__global__ void p2p_barrier_kernel(uint32_t* const* __restrict__ peer_flags, int rank, int world,
                                   uint32_t epoch, int32_t* __restrict__ err) {
  pdl_wait_trigger();
  if (threadIdx.x == 0) p2p_barrier(peer_flags, rank, world, epoch, err);
}

}  // namespace
}  // namespace knx

extern "C" size_t knx_ep_p2p_plan_ints(int E, int El, int world) {
  if (E <= 0 || El <= 0 || world <= 0) return 0;
  return static_cast<size_t>(E) + El + 1 + static_cast<size_t>(El) * world + 1 +
         static_cast<size_t>(El) * world;
}

extern "C" int knx_ep_p2p_counts(const int32_t* counts, int E, int El, int rank, int world,
                                 int32_t* const* peer_cnt, uint32_t* const* peer_flags,
                                 uint32_t epoch, int32_t* plan, int32_t* err, void* stream) {
  using namespace knx;
  if (world < 1 || world > P2P_MAX_WORLD || rank < 0 || rank >= world || E < 1 || E > P2P_MAX_E ||
      El < 1 || El * world != E)
    return KNX_E_INVALID;
  (void)launch_pdl(p2p_counts_kernel, 1, 256, 0, static_cast<cudaStream_t>(stream), counts, E, El,
                   rank, world, peer_cnt, peer_flags, epoch, plan, err);
  return launch_status();
}

extern "C" int knx_ep_p2p_dispatch(const void* xp, int64_t H, int topk, const int32_t* sorted_pair,
                                   const int32_t* offsets, int E, int El, const int32_t* plan,
                                   void* const* peer_rows, int64_t n_cap, void* stream) {
  using namespace knx;
  if (H <= 0 || (H % 8) != 0 || topk < 1 || E < 1 || El < 1 || n_cap < 0) return KNX_E_INVALID;
  if (!aligned(xp, 16)) return KNX_E_ALIGN;
  if (n_cap == 0) return KNX_OK;
  const int64_t blocks = (n_cap + 7) / 8;
  (void)launch_pdl(p2p_dispatch_kernel, static_cast<unsigned>(blocks), 256, 0,
                   static_cast<cudaStream_t>(stream), static_cast<const uint4*>(xp),
                   static_cast<int>(H / 8), topk, sorted_pair, offsets, E, El, plan,
                   reinterpret_cast<uint4* const*>(peer_rows), n_cap);
  return launch_status();
}

extern "C" int knx_ep_p2p_return(const void* out3, int64_t H, int El, int world, int E,
                                 const int32_t* plan, void* const* peer_ret, int64_t r_cap,
                                 void* stream) {
  using namespace knx;
  if (H <= 0 || (H % 8) != 0 || El < 1 || world < 1 || E < 1 || r_cap < 0) return KNX_E_INVALID;
  if (!aligned(out3, 16)) return KNX_E_ALIGN;
  if (r_cap == 0) return KNX_OK;
  const int64_t blocks = (r_cap + 7) / 8;
  (void)launch_pdl(p2p_return_kernel, static_cast<unsigned>(blocks), 256, 0,
                   static_cast<cudaStream_t>(stream), static_cast<const uint4*>(out3),
                   static_cast<int>(H / 8), El, world, plan, E,
                   reinterpret_cast<uint4* const*>(peer_ret), r_cap);
  return launch_status();
}

// Copy grid of the fused exchange kernels: enough warps for the rows, at most two CTAs per SM.
static unsigned p2p_grid(int64_t rows) {
  const int64_t need = (rows + 7) / 8;
  const int64_t cap = 2 * static_cast<int64_t>(knx::num_sms());
  return static_cast<unsigned>(need < cap ? (need > 0 ? need : 1) : cap);
}

extern "C" int knx_ep_p2p_dispatch_barrier(const void* xp, int64_t H, int topk,
                                           const int32_t* sorted_pair, const int32_t* offsets,
                                           int E, int El, const int32_t* plan,
                                           void* const* peer_rows, int64_t n_cap,
                                           uint32_t* const* peer_flags, int rank, int world,
                                           uint32_t epoch, uint32_t* arrive, int32_t* err,
                                           void* stream) {
  using namespace knx;
  if (H <= 0 || (H % 8) != 0 || topk < 1 || E < 1 || E > P2P_MAX_E || El < 1 || n_cap < 0 ||
      world < 1 || world > P2P_MAX_WORLD || rank < 0 || rank >= world || arrive == nullptr)
    return KNX_E_INVALID;
  if (!aligned(xp, 16)) return KNX_E_ALIGN;
  (void)launch_pdl(p2p_dispatch_bar_kernel, p2p_grid(n_cap), 256, 0,
                   static_cast<cudaStream_t>(stream), static_cast<const uint4*>(xp),
                   static_cast<int>(H / 8), topk, sorted_pair, offsets, E, El, plan,
                   reinterpret_cast<uint4* const*>(peer_rows), n_cap, peer_flags, rank, world,
                   epoch, arrive, err);
  return launch_status();
}

extern "C" int knx_ep_p2p_return_barrier(const void* out3, int64_t H, int El, int world, int E,
                                         const int32_t* plan, void* const* peer_ret,
                                         int64_t r_cap, uint32_t* const* peer_flags, int rank,
                                         uint32_t epoch, uint32_t* arrive, int32_t* err,
                                         void* stream) {
  using namespace knx;
  if (H <= 0 || (H % 8) != 0 || El < 1 || world < 1 || world > P2P_MAX_WORLD || E < 1 ||
      E > P2P_MAX_E || El * world > P2P_MAX_E || r_cap < 0 || rank < 0 || rank >= world ||
      arrive == nullptr)
    return KNX_E_INVALID;
  if (!aligned(out3, 16)) return KNX_E_ALIGN;
  (void)launch_pdl(p2p_return_bar_kernel, p2p_grid(r_cap), 256, 0,
                   static_cast<cudaStream_t>(stream), static_cast<const uint4*>(out3),
                   static_cast<int>(H / 8), El, world, plan, E,
                   reinterpret_cast<uint4* const*>(peer_ret), r_cap, peer_flags, rank, epoch,
                   arrive, err);
  return launch_status();
}

extern "C" int knx_ep_p2p_barrier(uint32_t* const* peer_flags, int rank, int world,
                                  uint32_t epoch, int32_t* err, void* stream) {
  using namespace knx;
  if (world < 1 || world > P2P_MAX_WORLD || rank < 0 || rank >= world) return KNX_E_INVALID;
  (void)launch_pdl(p2p_barrier_kernel, 1, 32, 0, static_cast<cudaStream_t>(stream), peer_flags,
                   rank, world, epoch, err);
  return launch_status();
}
