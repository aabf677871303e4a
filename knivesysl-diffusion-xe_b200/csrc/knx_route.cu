// knx_route.cu — router (logits, softmax, top-k, renormalise) and the token->expert
// permutation (deterministic counting sort), plus the activation K-interleave copy.
//
// Reference behaviour followed:
//   * moe_align (fused_moe_w4.py:15-51): stable sort of flat pairs p = t*topk + k by expert,
//     ids == E are "dropped" and sort to the end; BM-padded block layout with pad sentinels
//     Nexp (rows) and E (blocks); inv[p] = padded slot (0 for dropped pairs).
//   * router (DiffusionGemma, not vendored; specified as softmax -> top-k -> renormalise).
#include "knx_common.cuh"
#include "knx_internal.cuh"
#include "knx_topk.cuh"

namespace knx {
namespace {

// ------------------------------------------------------------------------------------------
// Router logits: grid (ceil(T/32), E/32, RT_KSPLIT); each CTA computes a [32 token x 32 expert]
// partial over one K split with m16n8k16 MMAs.  The split's 64-k chunks stream through a
// cp.async ring of up to RT_RING chunks, all issued up front (at H = 2816 the whole split is in
// flight at once: one memory round trip instead of one per chunk); chunks are consumed in order.
// Partials go to part[split][T][E]; the top-k kernel sums the splits in fixed order
// (deterministic).
constexpr int RT_TOK = 32, RT_EXP = 32, RT_BK = 64, RT_KSPLIT = 4;
constexpr int RT_ROWB = RT_BK * 2 + 16;  // 144-byte padded smem rows: conflict-free u32 loads
constexpr int RT_RING = 16;              // chunks in flight at most
constexpr int RT_CHUNK_BYTES = (RT_TOK + RT_EXP) * RT_ROWB;

// cp.async.wait_group with a run-time count (0..15): the instruction takes an immediate.
KNX_DEVINL void cp_async_wait_upto(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    case 7: cp_async_wait<7>(); break;
    case 8: cp_async_wait<8>(); break;
    case 9: cp_async_wait<9>(); break;
    case 10: cp_async_wait<10>(); break;
    case 11: cp_async_wait<11>(); break;
    case 12: cp_async_wait<12>(); break;
    case 13: cp_async_wait<13>(); break;
    case 14: cp_async_wait<14>(); break;
    default: cp_async_wait<15>(); break;
  }
}

__global__ void __launch_bounds__(128)
    router_logits_kernel(const __half* __restrict__ x, const __half* __restrict__ wr, int T,
                         int H, int E, float* __restrict__ part) {
  pdl_wait_trigger();
  extern __shared__ __align__(16) uint8_t rt_ring[];  // [ring][x rows | w rows]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int t0 = blockIdx.x * RT_TOK, e0 = blockIdx.y * RT_EXP;
  const int kper = H / RT_KSPLIT;  // multiple of RT_BK (host checks H % 256 == 0)
  const int kbeg = blockIdx.z * kper;
  const int nchunk = kper / RT_BK;
  const int ring = nchunk < RT_RING ? nchunk : RT_RING;

  // chunk c -> ring slot c % ring: token rows then expert rows, RT_ROWB bytes each
  auto load = [&](int c) {
    uint8_t* slot = rt_ring + (c % ring) * RT_CHUNK_BYTES;
    const int k0 = kbeg + c * RT_BK;
    for (int i = tid; i < (RT_TOK + RT_EXP) * 8; i += 128) {
      const int r = i >> 3, ch = i & 7;
      const __half* src;
      if (r < RT_TOK) {
        const int t = t0 + r;
        src = x + static_cast<int64_t>(t < T ? t : T - 1) * H + k0 + ch * 8;
      } else {
        src = wr + static_cast<int64_t>(e0 + r - RT_TOK) * H + k0 + ch * 8;
      }
      cp_async16(slot + r * RT_ROWB + ch * 16, src);
    }
    cp_async_commit();
  };

  // warp tile: tokens [16*(warp&1), +16) as MMA rows, experts [16*(warp>>1), +16) as 2 n8 tiles
  const int tm = 16 * (warp & 1), en = 16 * (warp >> 1);
  // two accumulator sets (even / odd k16 steps), added once at the end: half the dependent
  // MMA chain; the fused and the standalone router use the same order
  float acc[2][2][4] = {};
  int issued = 0;
  for (; issued < ring; ++issued) load(issued);
  for (int c = 0; c < nchunk; ++c) {
    cp_async_wait_upto(issued - 1 - c);  // chunk c has landed (newer chunks may be in flight)
    __syncthreads();
    const uint32_t bx = smem_u32(rt_ring + (c % ring) * RT_CHUNK_BYTES);
    const uint32_t bw = bx + RT_TOK * RT_ROWB;
#pragma unroll
    for (int ks = 0; ks < RT_BK / 16; ++ks) {
      const int kb = ks * 32 + q * 4;  // byte offset of k = 16*ks + 2q
      const uint32_t a0 = lds32(bx + (tm + g) * RT_ROWB + kb);
      const uint32_t a1 = lds32(bx + (tm + g + 8) * RT_ROWB + kb);
      const uint32_t a2 = lds32(bx + (tm + g) * RT_ROWB + kb + 16);
      const uint32_t a3 = lds32(bx + (tm + g + 8) * RT_ROWB + kb + 16);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t b0 = lds32(bw + (en + 8 * nt + g) * RT_ROWB + kb);
        const uint32_t b1 = lds32(bw + (en + 8 * nt + g) * RT_ROWB + kb + 16);
        mma_16816(acc[nt][ks & 1], a0, a1, a2, a3, b0, b1);
      }
    }
    __syncthreads();  // every warp is done with the slot before it is refilled
    if (issued < nchunk) load(issued++);
  }
  float* out = part + static_cast<int64_t>(blockIdx.z) * T * E;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int e = e0 + en + 8 * nt + 2 * q;
    const int ta = t0 + tm + g, tb = ta + 8;
    if (ta < T) {
      out[static_cast<int64_t>(ta) * E + e] = acc[nt][0][0] + acc[nt][1][0];
      out[static_cast<int64_t>(ta) * E + e + 1] = acc[nt][0][1] + acc[nt][1][1];
    }
    if (tb < T) {
      out[static_cast<int64_t>(tb) * E + e] = acc[nt][0][2] + acc[nt][1][2];
      out[static_cast<int64_t>(tb) * E + e + 1] = acc[nt][0][3] + acc[nt][1][3];
    }
  }
}

// One warp per token: sum the K-split partials in order, add bias, softmax, top-k by logit
// (ties -> lower expert id), renormalise the selected probabilities.
__global__ void __launch_bounds__(256)
    router_topk_kernel(const float* __restrict__ part, const float* __restrict__ bias, int T,
                       int E, int topk, float* __restrict__ logits_out, int32_t* __restrict__ ids,
                       float* __restrict__ weights) {
  pdl_wait_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  constexpr int PER = TK_PER;
  float l[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    float v = -INFINITY;
    if (e < E) {
      v = 0.f;
      for (int s = 0; s < RT_KSPLIT; ++s) v += part[(static_cast<int64_t>(s) * T + t) * E + e];
      if (bias) v += bias[e];
      if (logits_out) logits_out[static_cast<int64_t>(t) * E + e] = v;
    }
    l[i] = v;
  }
  topk_select(l, E, topk, lane, ids + static_cast<int64_t>(t) * topk,
              weights + static_cast<int64_t>(t) * topk);
}

// ------------------------------------------------------------------------------------------
// Counting sort (one CTA, 1024 threads).  Each warp ranks a contiguous run of pairs by the lanes
// holding the same expert id (match_by_bits), so the rank of pair p inside its expert is
//   (pairs of that expert in earlier warps) + (earlier pairs in the same warp),
// which is exactly the stable order.  Also builds the GEMM task list (expert token chunks of at
// most m_max, ordered by chunk size descending, then expert, then chunk; each task is
// (expert, first token in the expert, tokens, first slot)) and zeroes the GEMMs' counters.
constexpr int AL_THREADS = 1024;
constexpr int AL_WH = 33;  // per-expert row of the 32 warps' counts, padded: [E][AL_WH]

// Mask of the lanes whose v equals this lane's (0 <= v < 2^nbits, nbits warp-uniform): one ballot
// per bit, the same mask as __match_any_sync and measured cheaper on B200.
KNX_DEVINL unsigned match_by_bits(int v, int nbits) {
  unsigned peers = 0xffffffffu;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (v >> b) & 1;
    const unsigned bb = __ballot_sync(0xffffffffu, bit);
    peers &= bit ? bb : ~bb;
  }
  return peers;
}
KNX_DEVINL int bits_for(int maxv) {  // bits to hold 0..maxv
  int n = 1;
  while ((1 << n) <= maxv) ++n;
  return n;
}

// Exclusive scans of three values at once over blockDim.x threads in thread order (one pass, two
// barriers).  sbuf: >= 99 ints.
__device__ void block_excl_scan3(const int (&v)[3], int* sbuf, int (&ex)[3], int (&tot)[3]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl[3] = {v[0], v[1], v[2]};
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int n = __shfl_up_sync(0xffffffffu, incl[k], o);
      if (lane >= o) incl[k] += n;
    }
  }
  if (lane == 31)
    for (int k = 0; k < 3; ++k) sbuf[33 * k + warp] = incl[k];
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int wv = lane < nw ? sbuf[33 * k + lane] : 0;
      int wi = wv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += n;
      }
      if (lane < nw) sbuf[33 * k + lane] = wi - wv;
      if (lane == 31) sbuf[33 * k + 32] = wi;
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    ex[k] = sbuf[33 * k + warp] + incl[k] - v[k];
    tot[k] = sbuf[33 * k + 32];
  }
  __syncthreads();
}

// The label of pair p: ids[p] (0..E-1; E or anything outside means dropped), through the
// optional relabelling table (a permutation of 0..E-1; a label outside it is an invalid id).
// Returns E for a dropped or invalid pair and sets `bad` for an invalid one.
KNX_DEVINL int pair_label(const void* ids, int ids_dtype, int64_t p, int E,
                          const int32_t* __restrict__ relabel, int& bad) {
  int64_t v = load_as_i64(ids, ids_dtype, p);
  if (v < 0 || v > E) {
    bad = 1;
    return E;
  }
  if (relabel && v < E) {
    v = relabel[v];
    if (v < 0 || v >= E) {
      bad = 1;
      return E;
    }
  }
  return static_cast<int>(v);
}

__global__ void __launch_bounds__(AL_THREADS)
    align_kernel(const void* __restrict__ ids, int ids_dtype, int T, int topk, int E, int block_m,
                 int m_max, int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                 int32_t* __restrict__ sorted_pair, int32_t* __restrict__ inv,
                 int32_t* __restrict__ sorted_rows, int32_t* __restrict__ expert_ids,
                 int32_t* __restrict__ padded_inv, int4* __restrict__ tasks,
                 int32_t* __restrict__ ntasks, int32_t* __restrict__ work_counters,
                 int n_work_counters, int32_t* __restrict__ err,
                 const int32_t* __restrict__ relabel) {
  pdl_wait_trigger();
  extern __shared__ __align__(16) uint8_t sm_raw[];
  const int N = T * topk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per_warp = ((N + AL_THREADS - 1) / AL_THREADS) * 32;
  const int npad = (N + 7) & ~7;
  int16_t* sid = reinterpret_cast<int16_t*>(sm_raw);
  int16_t* srank = sid + npad;
  int* whist = reinterpret_cast<int*>(srank + npad);  // [E][AL_WH]: counts of the 32 warps
  int* soff = whist + AL_WH * E;                       // [E+1]
  int* spblk = soff + E + 1;                           // [E+1]
  int* scan_buf = spblk + E + 1;                       // [100]
  int* size_hist = scan_buf + 100;                     // [m_max+1]
  int* scnt = size_hist + m_max + 1;                   // [E] pairs per expert
  int* rhist = scnt + E;                               // [8][m_max+1] remainder counts per warp
  const int RH = m_max + 1;

  for (int i = tid; i < AL_WH * E; i += AL_THREADS) whist[i] = 0;
  for (int i = tid; i <= m_max; i += AL_THREADS) size_hist[i] = 0;
  for (int i = tid; i < n_work_counters; i += AL_THREADS) work_counters[i] = 0;
  int bad = 0;
  for (int p = tid; p < N; p += AL_THREADS)
    sid[p] = static_cast<int16_t>(pair_label(ids, ids_dtype, p, E, relabel, bad));
  if (bad && err) atomicOr(err, KNX_DEV_BAD_EXPERT_ID);
  __syncthreads();

  const unsigned lt_mask = (1u << lane) - 1u;
  const int p0 = warp * per_warp;
  const int ebits = bits_for(E);
  for (int r = 0; r < per_warp; r += 32) {
    const int p = p0 + r + lane;
    const bool valid = p < N;
    const int e = valid ? sid[p] : E;
    const unsigned peers = match_by_bits(e, ebits);
    const int before = __popc(peers & lt_mask);
    const int leader = __ffs(peers) - 1;
    const int prev = (e < E) ? whist[e * AL_WH + warp] : 0;
    __syncwarp();
    if (e < E && lane == leader) whist[e * AL_WH + warp] = prev + __popc(peers);
    __syncwarp();
    if (valid) srank[p] = static_cast<int16_t>(e < E ? prev + before : -1);
  }
  __syncthreads();

  // per expert: exclusive prefix of the 32 warps' counts (in place) and the expert's total.  C
  // consecutive lanes share an expert (C = 8 for E <= 128, else 4), each summing 32 / C warps in
  // order, then a segmented shuffle scan across the C lanes.
  {
    const int lc = E <= 128 ? 3 : 2;
    const int C = 1 << lc, wpc = 32 >> lc;
    const int e = tid >> lc, c = tid & (C - 1);
    int part[8];
    int run = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      part[w] = run;
      if (w < wpc && e < E) run += whist[e * AL_WH + c * wpc + w];
    }
    int incl = run;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o, C);
      if (o < C && c >= o) incl += n;
    }
    const int excl = incl - run;
#pragma unroll
    for (int w = 0; w < 8; ++w)
      if (w < wpc && e < E) whist[e * AL_WH + c * wpc + w] = excl + part[w];
    const int tot = __shfl_sync(0xffffffffu, incl, C - 1, C);
    if (c == 0 && e < E) scnt[e] = tot;
  }
  __syncthreads();

  int cnt = 0, nblk = 0, nfull = 0, rem = 0;
  const int e_me = tid;  // E <= AL_THREADS
  if (e_me < E) {
    cnt = scnt[e_me];
    nblk = block_m > 0 ? (cnt + block_m - 1) / block_m : 0;
    nfull = cnt / m_max;
    rem = cnt % m_max;
  }
  int ex[3], tot3[3];
  block_excl_scan3({cnt, nblk, nfull}, scan_buf, ex, tot3);
  const int off = ex[0], pblk = ex[1], fpre = ex[2];
  const int total_valid = tot3[0], total_blk = tot3[1], total_full = tot3[2];
  if (e_me < E) {
    soff[e_me] = off;
    spblk[e_me] = pblk;
    if (counts) counts[e_me] = cnt;
    if (offsets) offsets[e_me] = off;
    if (rem > 0) atomicAdd(&size_hist[rem], 1);
  }
  if (tid == 0) {
    soff[E] = total_valid;
    spblk[E] = total_blk;
    if (offsets) offsets[E] = total_valid;
    size_hist[m_max] = total_full;
  }
  const int max_blocks = block_m > 0 ? (N + block_m - 1) / block_m + E : 0;
  const int cap = max_blocks * block_m;
  if (block_m > 0 && sorted_rows) {
    for (int i = tid; i < cap; i += AL_THREADS) sorted_rows[i] = N;
  }
  __syncthreads();

  for (int p = tid; p < N; p += AL_THREADS) {
    const int e = sid[p];
    if (e < E) {
      const int w = p / per_warp;
      const int rank = whist[e * AL_WH + w] + srank[p];
      const int slot = soff[e] + rank;
      if (sorted_pair) sorted_pair[slot] = p;
      if (inv) inv[p] = slot;
      if (block_m > 0) {
        const int ps = spblk[e] * block_m + rank;
        if (sorted_rows) sorted_rows[ps] = p;
        if (padded_inv) padded_inv[p] = ps;
      }
    } else {
      if (inv) inv[p] = -1;
      if (block_m > 0 && padded_inv) padded_inv[p] = 0;
    }
  }
  if (sorted_pair)
    for (int s = total_valid + tid; s < N; s += AL_THREADS) sorted_pair[s] = N;
  if (block_m > 0 && expert_ids) {
    for (int b = tid; b < max_blocks; b += AL_THREADS) {
      // expert e with spblk[e] <= b < spblk[e+1]; b >= total -> E (upper_bound search)
      int lo = 0, hi = E;  // find first e in [0,E] with spblk[e] > b, answer = that - 1
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (spblk[mid + 1] > b) hi = mid; else lo = mid + 1;
      }
      expert_ids[b] = (b < total_blk) ? lo : E;
    }
  }

  // task list: sizes descending; size_hist[s] becomes the number of tasks with size > s
  if (tasks) {
    for (int i = tid; i < 8 * RH; i += AL_THREADS) rhist[i] = 0;
    __syncthreads();  // placement above still reads whist; rhist zeroed
    // rank of this expert's remainder task among the experts with the same remainder, in expert
    // order: lanes of one warp by match_by_bits, earlier warps through rhist
    const int r = (e_me < E && rem > 0) ? rem : -1;
    const unsigned peers = match_by_bits(r + 1, bits_for(m_max + 1));
    const int rank_w = __popc(peers & lt_mask);
    if (r > 0 && lane == __ffs(peers) - 1) rhist[warp * RH + r] = __popc(peers);
    __syncthreads();
    if (warp == 0) {
      // reverse exclusive scan over sizes s = m_max .. 1 (position i = m_max - s), four per lane
      int v[4], a = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = 4 * lane + j;
        v[j] = i < m_max ? size_hist[m_max - i] : 0;
        a += v[j];
      }
      int incl = a;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      int base = incl - a;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = 4 * lane + j;
        if (i < m_max) size_hist[m_max - i] = base;
        base += v[j];
      }
      if (lane == 31) *ntasks = incl;
    }
    __syncthreads();
    if (e_me < E && cnt > 0) {
      for (int j = 0; j < nfull; ++j)
        tasks[size_hist[m_max] + fpre + j] = make_int4(e_me, j * m_max, m_max, off + j * m_max);
      if (rem > 0) {
        int before_same = rank_w;
        for (int w2 = 0; w2 < warp; ++w2) before_same += rhist[w2 * RH + rem];
        tasks[size_hist[rem] + before_same] =
            make_int4(e_me, nfull * m_max, rem, off + nfull * m_max);
      }
    }
  }
}

// Task list (expert token chunks of at most m) from per-expert slot offsets, largest chunks first
// (full chunks in expert order, then remainders by size, in expert order within a size), plus the
// task count and n_counters zeroed counters: the same list the align kernel builds.  One CTA.
__global__ void tasks_from_offsets_kernel(const int32_t* __restrict__ offsets, int E, int m,
                                          int4* __restrict__ tasks, int32_t* __restrict__ ntasks,
                                          int32_t* __restrict__ counters, int n_counters) {
  pdl_wait_trigger();
  __shared__ int full_pre[257];
  __shared__ int rem_of[256];
  __shared__ int rem_cnt[MAX_TASK_TOKENS + 1];
  __shared__ int rem_start[MAX_TASK_TOKENS + 1];
  const int tid = threadIdx.x;
  for (int r = tid; r <= m; r += blockDim.x) rem_cnt[r] = 0;
  for (int i = tid; i < n_counters; i += blockDim.x) counters[i] = 0;
  __syncthreads();
  if (tid < E) {
    const int rem = (offsets[tid + 1] - offsets[tid]) % m;
    rem_of[tid] = rem;
    if (rem > 0) atomicAdd(&rem_cnt[rem], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      full_pre[e] = acc;
      acc += (offsets[e + 1] - offsets[e]) / m;
    }
    full_pre[E] = acc;
    for (int r = m - 1; r >= 1; --r) {
      rem_start[r] = acc;
      acc += rem_cnt[r];
    }
    *ntasks = acc;
  }
  __syncthreads();
  if (tid < E) {
    const int cnt = offsets[tid + 1] - offsets[tid];
    const int nfull = cnt / m, rem = cnt % m;
    const int first = offsets[tid];
    for (int j = 0; j < nfull; ++j)
      tasks[full_pre[tid] + j] = make_int4(tid, j * m, m, first + j * m);
    if (rem > 0) {
      int before = 0;
      for (int e = 0; e < tid; ++e) before += rem_of[e] == rem;
      tasks[rem_start[rem] + before] = make_int4(tid, nfull * m, rem, first + nfull * m);
    }
  }
}

// ---- counting sort for more pairs than one CTA holds (N > ALIGN_MAX_PAIRS), unpadded form ----
// LA1: each CTA of AL_THREADS takes LB consecutive pairs and writes its per-expert counts and
//      every pair's stable rank inside the block (warp ranks by __match_any_sync, warp prefixes);
// LA2: one CTA turns the block counts into expert offsets and per-(block, expert) slot bases;
// LA3: pair p of block b with expert e goes to slot base[b][e] + rank.  Stable in p overall.
constexpr int LB = 4096;  // pairs per block

__global__ void __launch_bounds__(AL_THREADS)
    align_large_count_kernel(const void* __restrict__ ids, int ids_dtype, int64_t N, int E,
                             int32_t* __restrict__ blkcnt, int32_t* __restrict__ lrank,
                             int32_t* __restrict__ err, const int32_t* __restrict__ relabel) {
  pdl_wait_trigger();
  __shared__ int whist[32 * 256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b0 = static_cast<int64_t>(blockIdx.x) * LB;
  for (int i = tid; i < 32 * E; i += AL_THREADS) whist[i] = 0;
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  constexpr int PER_WARP = LB / 32;
  int my_e[PER_WARP / 32], my_r[PER_WARP / 32];
  int bad = 0;
#pragma unroll
  for (int r = 0; r < PER_WARP / 32; ++r) {
    const int64_t p = b0 + warp * PER_WARP + r * 32 + lane;
    int e = E;
    if (p < N) e = pair_label(ids, ids_dtype, p, E, relabel, bad);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int before = __popc(peers & lt_mask);
    const int leader = __ffs(peers) - 1;
    const int prev = e < E ? whist[warp * E + e] : 0;
    __syncwarp();
    if (e < E && lane == leader) whist[warp * E + e] = prev + __popc(peers);
    __syncwarp();
    my_e[r] = e;
    my_r[r] = prev + before;
  }
  if (bad && err) atomicOr(err, KNX_DEV_BAD_EXPERT_ID);
  __syncthreads();
  if (tid < E) {  // exclusive prefix over warps, block total
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = whist[w * E + tid];
      whist[w * E + tid] = run;
      run += c;
    }
    blkcnt[static_cast<int64_t>(blockIdx.x) * E + tid] = run;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < PER_WARP / 32; ++r) {
    const int64_t p = b0 + warp * PER_WARP + r * 32 + lane;
    if (p < N) lrank[p] = my_e[r] < E ? whist[warp * E + my_e[r]] + my_r[r] : -1;
  }
}

__global__ void __launch_bounds__(256)
    align_large_scan_kernel(const int32_t* __restrict__ blkcnt, int nblk, int E,
                            int32_t* __restrict__ blkbase, int32_t* __restrict__ counts,
                            int32_t* __restrict__ offsets) {
  pdl_wait_trigger();
  __shared__ int tot[257];
  const int e = threadIdx.x;
  int c = 0;
  if (e < E)
    for (int b = 0; b < nblk; ++b) c += blkcnt[static_cast<int64_t>(b) * E + e];
  if (e < E) tot[e] = c;
  __syncthreads();
  if (e == 0) {
    int acc = 0;
    for (int i = 0; i < E; ++i) {
      const int t = tot[i];
      tot[i] = acc;
      acc += t;
    }
    tot[E] = acc;
    if (offsets) offsets[E] = acc;
  }
  __syncthreads();
  if (e < E) {
    if (counts) counts[e] = c;
    if (offsets) offsets[e] = tot[e];
    int a = tot[e];
    for (int b = 0; b < nblk; ++b) {
      blkbase[static_cast<int64_t>(b) * E + e] = a;
      a += blkcnt[static_cast<int64_t>(b) * E + e];
    }
  }
}

__global__ void align_large_scatter_kernel(const void* __restrict__ ids, int ids_dtype, int64_t N,
                                           int E, const int32_t* __restrict__ blkbase,
                                           const int32_t* __restrict__ lrank,
                                           const int32_t* __restrict__ offsets,
                                           int32_t* __restrict__ sorted_pair,
                                           int32_t* __restrict__ inv,
                                           const int32_t* __restrict__ relabel) {
  pdl_wait_trigger();
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= N) return;
  const int r = lrank[p];
  if (r < 0) {
    if (inv) inv[p] = -1;
  } else {
    int bad = 0;  // a valid pair here (lrank >= 0): its label is in range
    const int e = pair_label(ids, ids_dtype, p, E, relabel, bad);
    const int slot = blkbase[(p / LB) * E + e] + r;
    if (sorted_pair) sorted_pair[slot] = static_cast<int32_t>(p);
    if (inv) inv[p] = slot;
  }
  if (sorted_pair && p >= offsets[E]) sorted_pair[p] = static_cast<int32_t>(N);  // tail
}

// Activation copy into the MoE K-interleave (f16 out; f16 or bf16 in).  One thread per 16 bytes.
template <typename T>
__global__ void permute_act_kernel(const T* __restrict__ x, __half* __restrict__ xp, int64_t nvec) {
  pdl_wait_trigger();
  const int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (v >= nvec) return;
  const uint4 raw = ldg_nc_v4(reinterpret_cast<const uint4*>(x) + v);
  const T* e = reinterpret_cast<const T*>(&raw);
  __half hp[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float f;
    if constexpr (std::is_same<T, __half>::value) {
      f = __half2float(e[j]);
    } else {
      f = __bfloat162float(e[j]);
    }
    hp[2 * (j & 3) + (j >> 2)] = __float2half_rn(f);
  }
  reinterpret_cast<uint4*>(xp)[v] = *reinterpret_cast<uint4*>(hp);
}

}  // namespace

constexpr int RT_KSPLIT_PUBLIC = RT_KSPLIT;

size_t align_smem_bytes(int N, int E, int m_max) {
  const int npad = (N + 7) & ~7;
  return static_cast<size_t>(npad) * 4 +
         static_cast<size_t>(AL_WH * E + 2 * (E + 1) + 100 + m_max + 1 + E + 8 * (m_max + 1)) * 4;
}

bool align_supported(int64_t N, int E) {
  return N <= ALIGN_MAX_PAIRS && E >= 1 && E <= ALIGN_MAX_EXPERTS;
}

int launch_align(const void* ids, int ids_dtype, int T, int topk, int E, int block_m, int m_max,
                 int32_t* counts, int32_t* offsets, int32_t* sorted_pair, int32_t* inv,
                 int32_t* sorted_rows, int32_t* expert_ids, int32_t* padded_inv, int4* tasks,
                 int32_t* ntasks, int32_t* work_counters, int n_work_counters, int32_t* err,
                 cudaStream_t stream, const int32_t* relabel) {
  const int N = T * topk;
  if (tasks && (m_max < 1 || m_max > MAX_TASK_TOKENS)) return KNX_E_UNSUPPORTED;  // one warp scan
  const size_t smem = align_smem_bytes(N, E, m_max);
  if (set_max_dyn_smem(reinterpret_cast<const void*>(align_kernel), 200 * 1024) != KNX_OK)
    return KNX_E_DEVICE;
  (void)launch_pdl(align_kernel, 1, AL_THREADS, smem, stream, ids, ids_dtype, T, topk, E, block_m,
                   m_max, counts, offsets, sorted_pair, inv, sorted_rows, expert_ids, padded_inv,
                   tasks, ntasks, work_counters, n_work_counters, err, relabel);
  return launch_status();
}

int launch_permute(const void* x, int dtype, __half* xp, int64_t elems, cudaStream_t stream) {
  const int64_t nvec = elems / 8;
  if (nvec == 0) return KNX_OK;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((nvec + threads - 1) / threads);
  if (dtype == KNX_F16) {
    (void)launch_pdl(permute_act_kernel<__half>, blocks, threads, 0, stream,
                     static_cast<const __half*>(x), xp, nvec);
  } else {
    (void)launch_pdl(permute_act_kernel<__nv_bfloat16>, blocks, threads, 0, stream,
                     static_cast<const __nv_bfloat16*>(x), xp, nvec);
  }
  return launch_status();
}

size_t align_large_scratch_bytes(int64_t N, int E) {
  const int64_t nblk = (N + LB - 1) / LB;
  return static_cast<size_t>(N) * 4 + 2 * static_cast<size_t>(nblk) * E * 4 + 256;
}

int launch_align_large(const void* ids, int ids_dtype, int64_t N, int E, int32_t* counts,
                       int32_t* offsets, int32_t* sorted_pair, int32_t* inv, void* scratch,
                       int32_t* err, cudaStream_t s, const int32_t* relabel) {
  if (E > 256 || N > (1LL << 30)) return KNX_E_UNSUPPORTED;
  if (N == 0) return KNX_OK;
  const int nblk = static_cast<int>((N + LB - 1) / LB);
  int32_t* lrank = static_cast<int32_t*>(scratch);
  int32_t* blkcnt = lrank + ((N + 63) & ~int64_t(63));
  int32_t* blkbase = blkcnt + static_cast<int64_t>(nblk) * E;
  (void)launch_pdl(align_large_count_kernel, nblk, AL_THREADS, 0, s, ids, ids_dtype, N, E, blkcnt,
                   lrank, err, relabel);
  (void)launch_pdl(align_large_scan_kernel, 1, 256, 0, s, blkcnt, nblk, E, blkbase, counts,
                   offsets);
  (void)launch_pdl(align_large_scatter_kernel, static_cast<unsigned>((N + 255) / 256), 256, 0, s,
                   ids, ids_dtype, N, E, blkbase, lrank, offsets, sorted_pair, inv, relabel);
  return launch_status();
}

int launch_tasks_from_offsets(const int32_t* offsets, int E, int m, int4* tasks, int32_t* ntasks,
                              int32_t* counters, int n_counters, cudaStream_t s) {
  if (E > 256 || m < 1 || m > MAX_TASK_TOKENS || n_counters < 0) return KNX_E_UNSUPPORTED;
  (void)launch_pdl(tasks_from_offsets_kernel, 1, 256, 0, s, offsets, E, m, tasks, ntasks, counters,
                   n_counters);
  return launch_status();
}

}  // namespace knx

// ------------------------------------------------------------------------------------------
extern "C" size_t knx_router_workspace_size(int64_t T, int E) {
  return static_cast<size_t>(knx::RT_KSPLIT_PUBLIC) * static_cast<size_t>(T > 0 ? T : 0) *
             static_cast<size_t>(E > 0 ? E : 0) * sizeof(float) + 256;
}

extern "C" int knx_router_topk(const void* x, const void* wr, const float* bias, int64_t T,
                               int64_t H, int E, int topk, float* logits_out, int32_t* ids,
                               float* weights, void* workspace, size_t workspace_bytes,
                               void* stream) {
  using namespace knx;
  if (T < 0 || H <= 0 || (H % 256) != 0 || E < 32 || (E % 32) != 0 || E > 256 || topk < 1 ||
      topk > 16 || topk > E || H > (1 << 24) || T > (1 << 24))
    return KNX_E_INVALID;
  if (!aligned(x, 16) || !aligned(wr, 16)) return KNX_E_ALIGN;
  if (T == 0) return KNX_OK;
  if (workspace == nullptr || workspace_bytes < knx_router_workspace_size(T, E))
    return KNX_E_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  const dim3 g1(static_cast<unsigned>((T + RT_TOK - 1) / RT_TOK), E / RT_EXP, RT_KSPLIT);
  const int nchunk = static_cast<int>(H / RT_KSPLIT / RT_BK);
  const size_t smem = static_cast<size_t>(nchunk < RT_RING ? nchunk : RT_RING) * RT_CHUNK_BYTES;
  if (set_max_dyn_smem(reinterpret_cast<const void*>(router_logits_kernel),
                       RT_RING * RT_CHUNK_BYTES) != KNX_OK)
    return KNX_E_DEVICE;
  (void)launch_pdl(router_logits_kernel, g1, 128, smem, s, static_cast<const __half*>(x),
                   static_cast<const __half*>(wr), static_cast<int>(T), static_cast<int>(H), E,
                   part);
  int st = launch_status();
  if (st != KNX_OK) return st;
  (void)launch_pdl(router_topk_kernel, static_cast<unsigned>((T + 7) / 8), 256, 0, s, part, bias,
                   static_cast<int>(T), E, topk, logits_out, ids, weights);
  return launch_status();
}

extern "C" size_t knx_moe_align_large_scratch_size(int64_t N, int E) {
  if (N < 0 || E <= 0) return 0;
  return knx::align_large_scratch_bytes(N, E);
}

extern "C" int knx_moe_align_large(const void* topk_ids, int ids_dtype, int64_t T, int topk, int E,
                                   int32_t* counts, int32_t* offsets, int32_t* sorted_pair,
                                   int32_t* inv, void* scratch, size_t scratch_bytes, int32_t* err,
                                   void* stream) {
  using namespace knx;
  if (T < 0 || topk < 1 || topk > 64 || E < 1 || E > ALIGN_MAX_EXPERTS) return KNX_E_INVALID;
  if (ids_dtype != KNX_I32 && ids_dtype != KNX_I64) return KNX_E_INVALID;
  const int64_t N = T * topk;
  if (N > (1LL << 30)) return KNX_E_UNSUPPORTED;
  if (N == 0) return KNX_OK;
  if (scratch == nullptr || scratch_bytes < align_large_scratch_bytes(N, E)) return KNX_E_WORKSPACE;
  if (!aligned(scratch, 16)) return KNX_E_ALIGN;
  return launch_align_large(topk_ids, ids_dtype, N, E, counts, offsets, sorted_pair, inv, scratch,
                            err, static_cast<cudaStream_t>(stream));
}

extern "C" int knx_moe_align_relabeled(const void* topk_ids, int ids_dtype, int64_t T, int topk,
                                       int E, const int32_t* relabel, int32_t* counts,
                                       int32_t* offsets, int32_t* sorted_pair, int32_t* inv,
                                       void* scratch, size_t scratch_bytes, int32_t* err,
                                       void* stream) {
  using namespace knx;
  if (T < 0 || topk < 1 || topk > 64 || E < 1 || E > ALIGN_MAX_EXPERTS || relabel == nullptr)
    return KNX_E_INVALID;
  if (ids_dtype != KNX_I32 && ids_dtype != KNX_I64) return KNX_E_INVALID;
  const int64_t N = T * topk;
  if (N == 0) return KNX_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (align_supported(N, E))
    return launch_align(topk_ids, ids_dtype, static_cast<int>(T), topk, E, 0, 1, counts, offsets,
                        sorted_pair, inv, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0,
                        err, s, relabel);
  if (scratch == nullptr || scratch_bytes < align_large_scratch_bytes(N, E)) return KNX_E_WORKSPACE;
  if (!aligned(scratch, 16)) return KNX_E_ALIGN;
  return launch_align_large(topk_ids, ids_dtype, N, E, counts, offsets, sorted_pair, inv, scratch,
                            err, s, relabel);
}

extern "C" int knx_moe_align(const void* topk_ids, int ids_dtype, int64_t T, int topk, int E,
                             int block_m, int32_t* counts, int32_t* offsets, int32_t* sorted_pair,
                             int32_t* inv, int32_t* sorted_rows, int32_t* expert_ids,
                             int32_t* padded_inv, int32_t* err, void* stream) {
  using namespace knx;
  if (T < 0 || topk < 1 || topk > 64 || E < 1 || block_m < 0) return KNX_E_INVALID;
  if (ids_dtype != KNX_I32 && ids_dtype != KNX_I64) return KNX_E_INVALID;
  const int64_t N = T * topk;
  if (!align_supported(N, E)) return KNX_E_UNSUPPORTED;
  if (N == 0) return KNX_OK;
  return launch_align(topk_ids, ids_dtype, static_cast<int>(T), topk, E, block_m, 1, counts,
                      offsets, sorted_pair, inv, sorted_rows, expert_ids, padded_inv, nullptr,
                      nullptr, nullptr, 0, err, static_cast<cudaStream_t>(stream));
}
