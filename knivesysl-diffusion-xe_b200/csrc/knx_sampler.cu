// knx_sampler.cu — one streaming pass over fp32 logits that yields, per row, the entropy of
// softmax(x/T), the Gumbel-max sample and the plain argmax; plus the entropy-bound acceptance
// mask and the stable-and-confident stop test.
//
// Reference semantics: fused_sampler_ops.py:22-93 (entropy, Gumbel argmax), fast_sampler.py:32-65
// (acceptance, stop), fast_sampler.py:92 (seed mixing, done by the caller).
//
// Layout / work split: a row of V logits is cut into a power-of-two number of chunks; a work item
// is (row, chunk) and persistent CTAs pull items from a counter.  Each warp streams 512 columns
// per step (4 float4 per lane) and keeps
//   * an online softmax state (m, sp, t): sp = sum e^(q-m) minus the max element's 1, t =
//     sum (q-m) e^(q-m), so H = log1p(sp) - t/(1+sp) is a sum of two non-negative terms and keeps
//     its relative precision for peaked (near-zero entropy) rows;
//   * the running argmax of q;
//   * the running Gumbel winner.  Gumbel noise is bounded above by GUMBEL_MAX, so an element with
//     q + GUMBEL_MAX < W (W = best q+g seen anywhere in the row so far, shared through a per-row
//     atomic) cannot win and its Philox draw is skipped.  Candidates are compacted per warp so
//     the 35-instruction Philox runs on full warps.  Skipping never changes the result, only
//     the work, so the output is bit-identical whatever the schedule.
// Chunk partials are merged by the last CTA of each row in chunk order (deterministic).
#include "knx_common.cuh"
#include "knx_math.cuh"
#include "knx_sm100.cuh"

namespace knx {
namespace {

constexpr int SP_THREADS = 256;
constexpr int SP_WARPS = SP_THREADS / 32;
constexpr int SP_TILE = 512;                 // columns per warp step
constexpr int SP_TARGET_CHUNK = 32768;       // columns per work item (before power-of-2 rounding)

struct __align__(16) Part {
  float m, s, t, bq;
  int bqi, bgi;
  float bg, pad;
};

// order-preserving map float -> uint32 (for atomicMax on the per-row Gumbel bound)
KNX_DEVINL uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
KNX_DEVINL float fdecode(uint32_t k) {
  if (k < 0x00800000u) return -INFINITY;  // zero-initialised bound = no bound yet
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}

KNX_DEVINL float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
constexpr float LOG2E = 1.4426950408889634f;

// Online-softmax state (m, sp, t) of a set of logits q:  m = max q,  S = sum e^(q-m) = 1 + sp
// (sp excludes one element equal to the max, so tiny entropies keep their relative precision),
// t = sum (q-m) e^(q-m) <= 0.  Entropy = log S - t/S = log1p(sp) - t/(1+sp).  m = -inf: empty.
KNX_DEVINL void sm_merge(float& m, float& sp, float& t, float m2, float sp2, float t2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2; sp = sp2; t = t2;
    return;
  }
  if (m >= m2) {
    const float a = ex2((m2 - m) * LOG2E), S2 = 1.0f + sp2;
    t = t + a * (t2 + (m2 - m) * S2);
    sp = sp + a * S2;
  } else {
    const float a = ex2((m - m2) * LOG2E), S1 = 1.0f + sp;
    t = t2 + a * (t + (m - m2) * S1);
    sp = sp2 + a * S1;
    m = m2;
  }
}
KNX_DEVINL void arg_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

// Final index of a row.  A row with no element that could win (every q is -inf or NaN) keeps
// index 0, as the reference's scan does: its running index starts at 0 and moves only on a
// strict improvement of the running best (fused_sampler_ops.py:55-81).
KNX_DEVINL int64_t row_index(int i) { return i == 0x7fffffff ? 0 : i; }

KNX_DEVINL void row_key(int64_t seed, int seed_is32, int64_t row, uint32_t& k0, uint32_t& k1) {
  if (seed_is32) {
    // Triton passes a 32-bit seed as i32: seed + row wraps in i32, then sign-extends to u64.
    const int32_t s = static_cast<int32_t>(static_cast<uint32_t>(seed) + static_cast<uint32_t>(row));
    k0 = static_cast<uint32_t>(s);
    k1 = s < 0 ? 0xffffffffu : 0u;
  } else {
    const uint64_t s = static_cast<uint64_t>(seed + row);
    k0 = static_cast<uint32_t>(s);
    k1 = static_cast<uint32_t>(s >> 32);
  }
}

template <bool VEC>
__global__ void __launch_bounds__(SP_THREADS, 3)
    sampler_kernel(const float* __restrict__ logits, int64_t rows, int V, float temp, float rtemp,
                   int do_div, int64_t seed, int seed_is32, int want_gumbel, int nchunks,
                   int chunk_cols, Part* __restrict__ parts, uint32_t* __restrict__ row_ticket,
                   uint32_t* __restrict__ row_bound, int* __restrict__ work_counter,
                   float* __restrict__ entropy, int64_t* __restrict__ samp,
                   int64_t* __restrict__ amax) {
  pdl_wait_trigger();
  const float dlo = div_fast_lo(temp), dhi = div_fast_hi(temp);  // fast-division range
  __shared__ int s_item;
  __shared__ int s_last;
  __shared__ Part s_wpart[SP_WARPS];
  __shared__ int cq_col[SP_WARPS][SP_TILE];
  __shared__ float cq_q[SP_WARPS][SP_TILE];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nitems = rows * nchunks;

  for (;;) {
    if (tid == 0) s_item = atomicAdd(work_counter, 1);
    __syncthreads();
    const int64_t item = s_item;
    if (item >= nitems) break;
    const int64_t row = item / nchunks;
    const int chunk = static_cast<int>(item - row * nchunks);
    const int c_beg = min(V, chunk * chunk_cols);
    const int c_end = min(V, c_beg + chunk_cols);
    // warp sub-range, multiple of 4 columns
    const int per_warp = (((c_end - c_beg) + SP_WARPS * 4 - 1) / (SP_WARPS * 4)) * 4;
    const int w_beg = min(c_end, c_beg + warp * per_warp);
    const int w_end = min(c_end, w_beg + per_warp);
    const float* xr = logits + row * static_cast<int64_t>(V);
    uint32_t k0 = 0, k1 = 0;
    row_key(seed, seed_is32, row, k0, k1);

    float m = -INFINITY, s = 0.f, t = 0.f;
    float bq = -INFINITY, bg = -INFINITY;
    int bqi = 0x7fffffff, bgi = 0x7fffffff;
    float W = -INFINITY;
    bool first = true;
    for (int base = w_beg; base < w_end; base += SP_TILE) {
      float qv[16];
      unsigned valid = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c0 = base + 128 * j + 4 * lane;
        if (VEC) {
          if (c0 < w_end) {  // w_end - c0 is a multiple of 4 when VEC
            const float4 v = __ldcs(reinterpret_cast<const float4*>(xr + c0));
            qv[4 * j] = v.x; qv[4 * j + 1] = v.y; qv[4 * j + 2] = v.z; qv[4 * j + 3] = v.w;
            valid |= 0xfu << (4 * j);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c0 + c < w_end) {
              qv[4 * j + c] = __ldcs(xr + c0 + c);
              valid |= 1u << (4 * j + c);
            }
          }
        }
      }
      float tm = -INFINITY;
      int ti = 0x7fffffff, imax = -1;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (valid & (1u << i)) {
          if (do_div) qv[i] = div_exact(qv[i], temp, rtemp, dlo, dhi);
          if (qv[i] > tm) {
            tm = qv[i];
            ti = base + 128 * (i >> 2) + 4 * lane + (i & 3);
            imax = i;
          }
        } else {
          qv[i] = -INFINITY;
        }
      }
      if (valid) {
        int skip = -1;  // the element that becomes the running max contributes the implicit 1
        if (tm > m) {
          if (m != -INFINITY) {
            const float a = ex2((m - tm) * LOG2E), S = 1.0f + s;
            t = a * (t + (m - tm) * S);
            s = a * S;
          } else {
            s = 0.f;
            t = 0.f;
          }
          m = tm;
          skip = imax;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if ((valid & (1u << i)) && qv[i] != -INFINITY && i != skip) {
            const float d = qv[i] - m;
            const float e = ex2(d * LOG2E);
            s += e;
            t = fmaf(d, e, t);
          }
        }
        if (tm > bq) {
          bq = tm;
          bqi = ti;
        }
      }
      if (want_gumbel) {
        if (first) {  // bootstrap the bound with each lane's tile maximum
          first = false;
          if (valid) {
            const float v = tm + gumbel_from_word(philox_w0(static_cast<uint32_t>(ti), k0, k1));
            arg_merge(bg, bgi, v, ti);
          }
          float wm = bg;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
          W = fmaxf(W, wm);
        }
        unsigned cm = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if ((valid & (1u << i)) && !(qv[i] + GUMBEL_MAX < W)) cm |= 1u << i;
        const int n = __popc(cm);
        int incl = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        if (total > 0) {
          int pos = incl - n;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (cm & (1u << i)) {
              cq_col[warp][pos] = base + 128 * (i >> 2) + 4 * lane + (i & 3);
              cq_q[warp][pos] = qv[i];
              ++pos;
            }
          }
          __syncwarp();
          for (int i = lane; i < total; i += 32) {
            const int col = cq_col[warp][i];
            const float v = cq_q[warp][i] + gumbel_from_word(philox_w0(static_cast<uint32_t>(col), k0, k1));
            arg_merge(bg, bgi, v, col);
          }
          __syncwarp();
        }
        float wm = bg;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
        uint32_t old = 0;
        if (lane == 0) old = atomicMax(row_bound + row, fkey(wm));
        old = __shfl_sync(0xffffffffu, old, 0);
        W = fmaxf(fmaxf(W, wm), fdecode(old));
      }
    }
    // warp reductions (fixed butterfly order)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float t2 = __shfl_xor_sync(0xffffffffu, t, o);
      const float bq2 = __shfl_xor_sync(0xffffffffu, bq, o);
      const int bqi2 = __shfl_xor_sync(0xffffffffu, bqi, o);
      const float bg2 = __shfl_xor_sync(0xffffffffu, bg, o);
      const int bgi2 = __shfl_xor_sync(0xffffffffu, bgi, o);
      // merge in a symmetric way so both partners hold the same result
      float ma = m, sa = s, ta = t, mb = m2, sb = s2, tb = t2;
      if ((lane & o) != 0) {  // canonical order: lower lane first
        ma = m2; sa = s2; ta = t2; mb = m; sb = s; tb = t;
      }
      sm_merge(ma, sa, ta, mb, sb, tb);
      m = ma; s = sa; t = ta;
      arg_merge(bq, bqi, bq2, bqi2);
      arg_merge(bg, bgi, bg2, bgi2);
    }
    if (lane == 0) {
      Part p;
      p.m = m; p.s = s; p.t = t; p.bq = bq; p.bqi = bqi; p.bg = bg; p.bgi = bgi; p.pad = 0.f;
      s_wpart[warp] = p;
    }
    __syncthreads();
    if (tid == 0) {
      Part acc = s_wpart[0];
      for (int w = 1; w < SP_WARPS; ++w) {
        const Part p = s_wpart[w];
        sm_merge(acc.m, acc.s, acc.t, p.m, p.s, p.t);
        arg_merge(acc.bq, acc.bqi, p.bq, p.bqi);
        arg_merge(acc.bg, acc.bgi, p.bg, p.bgi);
      }
      parts[item] = acc;
      __threadfence();
      const uint32_t tk = atomicAdd(row_ticket + row, 1u);
      s_last = (tk + 1u) == static_cast<uint32_t>(nchunks);
    }
    __syncthreads();
    if (s_last && tid == 0) {
      __threadfence();
      const float4* pr = reinterpret_cast<const float4*>(parts + row * nchunks);
      float4 a = __ldcg(pr), b = __ldcg(pr + 1);
      Part acc;
      acc.m = a.x; acc.s = a.y; acc.t = a.z; acc.bq = a.w;
      acc.bqi = __float_as_int(b.x); acc.bgi = __float_as_int(b.y); acc.bg = b.z; acc.pad = 0.f;
      for (int c = 1; c < nchunks; ++c) {
        a = __ldcg(pr + 2 * c);
        b = __ldcg(pr + 2 * c + 1);
        sm_merge(acc.m, acc.s, acc.t, a.x, a.y, a.z);
        arg_merge(acc.bq, acc.bqi, a.w, __float_as_int(b.x));
        arg_merge(acc.bg, acc.bgi, b.z, __float_as_int(b.y));
      }
      if (entropy) entropy[row] = log1pf(acc.s) - acc.t / (1.0f + acc.s);
      if (amax) amax[row] = row_index(acc.bqi);
      if (samp) samp[row] = row_index(acc.bgi);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------
// Streaming variant for V % 4 == 0 (the configs' 262144-wide rows): one persistent CTA per SM.
//   * work items are quarter rows (SX_CHUNK = 65536 columns, 8 stages), assigned statically in
//     contiguous blocks (CTA c takes items c*n .. c*n + n - 1), so all roles walk the same
//     sequence without a work queue, and a CTA mostly takes a row's quarters one after another:
//     its Gumbel bound carries over from quarter to quarter (measured 4-7 us per step faster at
//     T = 0.4-0.7 than CTA c taking items c, c + grid, ...);
//   * warp 16 streams each item through a ring of 4 x 32 KB shared-memory stages with 1-D bulk
//     copies (128 KB in flight per SM, what HBM needs at full rate);
//   * warps 0-15 each take 512 columns of every 8192-column stage.  The running maximum and the
//     argmax are kept per warp, so their updates are rare, uniform branches; the common path per
//     element is the IEEE division by the temperature, a max and five operations of the entropy
//     update (log2 units).  Gumbel candidates are pruned against the best q + g seen so far in
//     the row — this CTA's warps share it through shared memory at once, the other CTAs of the
//     row through a fire-and-forget atomic max on the per-row bound, which warp 18 keeps copying
//     into shared memory; a stale bound only prunes less, never wrongly;
//   * warp 17 merges the 16 warp partials of each item (in warp order) into parts[item], double
//     buffered so the math warps never wait for it; rows are finished by row_merge_kernel.
// Every decision (argmax ties, Gumbel winner, merge order) is the same as sampler_kernel's, so the
// sampled and argmax indices are identical; the entropy agrees to fp32 rounding.
constexpr int SX_COLS = 8192;               // columns per stage
constexpr int SX_BYTES = SX_COLS * 4;
constexpr int SX_CHUNK = 8 * SX_COLS;       // columns per work item
constexpr int SX_RING = 4;
constexpr int SX_WARPS = 16;                // math warps
constexpr int SX_THREADS = (SX_WARPS + 3) * 32;
// Philox chains per lane in one pass over the deferred candidates (32 candidates each).  Two
// beat four on B200 (8-10 us per step at T 0.4-0.6).
constexpr int SX_CHAINS = 2;
// Deferred Gumbel candidates per warp.  Once SX_FLUSH (one full pass) are pending, the whole
// multiples of SX_FLUSH are evaluated and the rest stays for the next tile, so a tile (at most
// SP_TILE candidates) always fits on top of the at most SX_FLUSH - 1 left over; the last flush
// of an item takes everything.
constexpr int SX_FLUSH = 32 * SX_CHAINS;
constexpr int SX_CQ = SP_TILE + SX_FLUSH;
constexpr size_t SX_SMEM = 128 + static_cast<size_t>(SX_RING) * SX_BYTES +
                           static_cast<size_t>(SX_WARPS) * SX_CQ * 8;

struct SxCtrl {
  uint64_t full[SX_RING], empty[SX_RING];
  uint64_t pfull[2], pempty[2];
  unsigned long long wbound;  // (row << 32) | fkey(best q + g): rows only grow along a CTA's items
  long long cur_row;          // row of the item math warp 0 is on (for the bound relay)
  int done;                   // math warps finished
  int abort;
};

KNX_DEVINL uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
KNX_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
KNX_DEVINL int warp_min_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// bf16 bits of v rounded to nearest even; NaN -> 0x7FC0 (torch's float -> bfloat16 conversion)
KNX_DEVINL uint32_t bf16_bits(float v) {
  return v != v ? 0x7FC0u : static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
}
KNX_DEVINL uint32_t bf16x2_bits(float lo, float hi) { return bf16_bits(lo) | (bf16_bits(hi) << 16); }

// Self-conditioning copy (SC): besides the sampling results the pass writes
//   sc_out[r, :] = finished[r / canvas_len] ? sc_prev[r, :] : bf16(x[r, :] / T)
// (x / T the same IEEE quotient the sampler uses), i.e. the reference step's
// where(finished, previous self-conditioning logits, processed logits).to(bfloat16).
template <bool SC>
__global__ void __launch_bounds__(SX_THREADS, 1)
    sampler_stream_kernel(const float* __restrict__ logits, int64_t rows, int V, float temp,
                          float rtemp, int do_div, int64_t seed, int seed_is32, int want_gumbel,
                          int nchunks, Part* __restrict__ parts, uint32_t* __restrict__ row_bound,
                          int* __restrict__ err, __nv_bfloat16* __restrict__ sc_out,
                          const __nv_bfloat16* __restrict__ sc_prev,
                          const uint8_t* __restrict__ finished, int canvas_len) {
  pdl_wait_trigger();
  const float dlo = div_fast_lo(temp), dhi = div_fast_hi(temp);  // fast-division range
  using namespace sm100;
  extern __shared__ uint8_t sx_raw[];
  __shared__ SxCtrl c;
  __shared__ Part s_wpart[2][SX_WARPS];
  // 128-byte aligned ring, by an offset from sx_raw; the math warps read it and their candidate
  // buffers through explicit shared-memory loads and stores (shared addresses)
  uint8_t* ring = sx_raw + ((128u - (smem_u32(sx_raw) & 127u)) & 127u);
  const uint32_t ring_s = smem_u32(ring);
  const uint32_t cq_col = ring_s + SX_RING * SX_BYTES;      // int [SX_WARPS][SX_CQ]
  const uint32_t cq_q = cq_col + SX_WARPS * SX_CQ * 4;      // float [SX_WARPS][SX_CQ]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nitems = rows * nchunks;
  const int64_t per_cta = (nitems + gridDim.x - 1) / gridDim.x;
  const int64_t it_beg = blockIdx.x * per_cta, it_end = min(nitems, it_beg + per_cta);
  if (tid == 0) {
    for (int i = 0; i < SX_RING; ++i) { mbar_init(&c.full[i], 1); mbar_init(&c.empty[i], SX_WARPS); }
    for (int i = 0; i < 2; ++i) { mbar_init(&c.pfull[i], SX_WARPS); mbar_init(&c.pempty[i], 1); }
    c.wbound = 0ull;
    c.cur_row = -1;
    c.done = 0;
    c.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort_flag = &c.abort;
  auto fail = [&]() {
    *abort_flag = 1;
    atomicOr(err, KNX_DEV_TIMEOUT);
  };

  if (warp == SX_WARPS) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t u = 0;
      for (int64_t item = it_beg; item < it_end && !*abort_flag; ++item) {
        const int64_t row = item / nchunks;
        const int chunk = static_cast<int>(item - row * nchunks);
        const int c_beg = min(V, chunk * SX_CHUNK), c_end = min(V, c_beg + SX_CHUNK);
        const float* xr = logits + row * static_cast<int64_t>(V);
        for (int c0 = c_beg; c0 < c_end; c0 += SX_COLS, ++u) {
          const int slot = u % SX_RING;
          if (!mbar_wait(&c.empty[slot], ((u / SX_RING) & 1) ^ 1, 2000000000ull, 128)) {
            fail();
            break;
          }
          const uint32_t bytes = static_cast<uint32_t>(min(SX_COLS, c_end - c0)) * 4u;
          mbar_arrive_expect_tx(&c.full[slot], bytes);
          bulk_load(ring + slot * SX_BYTES, xr + c0, bytes, &c.full[slot]);
        }
      }
      // copies already issued land before the CTA exits (bounded)
      for (uint32_t x = u > SX_RING ? u - SX_RING : 0; x < u; ++x)
        mbar_wait(&c.full[x % SX_RING], (x / SX_RING) & 1);
    }
    __syncwarp();
  } else if (warp == SX_WARPS + 1) {
    // ------------------------------------------------------------ item merger
    if (lane == 0) {
      int k = 0;
      for (int64_t item = it_beg; item < it_end; ++item, ++k) {
        const int b = k & 1;
        if (*abort_flag || !mbar_wait(&c.pfull[b], (k >> 1) & 1, 2000000000ull, 64)) {
          if (!*abort_flag) fail();
          break;
        }
        Part acc = s_wpart[b][0];
        for (int w = 1; w < SX_WARPS; ++w) {
          const Part pw = s_wpart[b][w];
          sm_merge(acc.m, acc.s, acc.t, pw.m, pw.s, pw.t);
          arg_merge(acc.bq, acc.bqi, pw.bq, pw.bqi);
          arg_merge(acc.bg, acc.bgi, pw.bg, pw.bgi);
        }
        parts[item] = acc;
        mbar_arrive(&c.pempty[b]);
      }
    }
    __syncwarp();
  } else if (warp == SX_WARPS + 2) {
    // ------------------------------------------------------------ bound relay
    // Copies the global per-row Gumbel bound (other CTAs' best q + g for the row) into this CTA's
    // shared bound, so no math warp waits on a global round trip.  Bounded by a time limit.
    if (lane == 0 && want_gumbel) {
      const uint64_t t0 = globaltimer();
      volatile long long* vrow = &c.cur_row;
      volatile int* vdone = &c.done;
      while (*vdone < SX_WARPS && !*abort_flag && globaltimer() - t0 < 4000000000ull) {
        const long long r = *vrow;
        if (r >= 0) {
          const uint32_t v = ld_relaxed_u32(row_bound + r);
          if (v) atomicMax(&c.wbound, (static_cast<unsigned long long>(r) << 32) | v);
        }
        __nanosleep(256);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ math warps
    uint32_t u = 0;
    const float L = LOG2E;
    int k = 0;
    const uint32_t wcol = cq_col + warp * SX_CQ * 4;  // this warp's deferred Gumbel candidates
    const uint32_t wq = cq_q + warp * SX_CQ * 4;
    for (int64_t item = it_beg; item < it_end; ++item, ++k) {
      const int64_t row = item / nchunks;
      const int chunk = static_cast<int>(item - row * nchunks);
      const int c_beg = min(V, chunk * SX_CHUNK), c_end = min(V, c_beg + SX_CHUNK);
      uint32_t k0 = 0, k1 = 0;
      row_key(seed, seed_is32, row, k0, k1);
      if (warp == 0 && lane == 0) *reinterpret_cast<volatile long long*>(&c.cur_row) = row;
      bool sc_keep = false;  // SC: the row's canvas has finished, copy its previous logits
      if constexpr (SC) sc_keep = finished != nullptr && finished[row / canvas_len] != 0;
      // entropy state: m (warp-uniform running max), per lane sp = sum of 2^d2 over the lane's
      // elements except the one element that carries the implicit 1, t2 = sum d2 * 2^d2
      float m = -INFINITY, m2 = -INFINITY, sp = 0.f, t2 = 0.f;
      float bq = -INFINITY;  // warp-uniform argmax
      int bqi = 0x7fffffff;
      float bg = -INFINITY;  // per-lane Gumbel winner
      int bgi = 0x7fffffff;
      float W = -INFINITY;  // best exact q + g known for the row (warp view)
      bool first = true;
      int nbuf = 0;         // deferred candidates in wcol/wq
      // Evaluates deferred candidates, 64 at a time (two Philox chains per lane): all of them on
      // the item's last flush, else the whole multiples of 64, the rest moving to the front of
      // the buffer.  Each is re-tested against the newest bound; its Philox word is then screened
      // with the exact-safe test u >= e^(-e^(-y)) - 2e-6 (y = best - q, u the clamped uniform;
      // q + g(u) >= best needs u >= e^(-e^(-y)), and the approximate exponentials err by far less
      // than the margin), and only survivors get the exact Gumbel value and enter the argmax.  The
      // test is written !(u < ...) so that y = inf - inf (a q = +inf candidate once the bound is
      // +inf) keeps the candidate: of several +inf elements the first must still win.
      auto flush = [&](bool last) {
        __syncwarp();
        const float thr_now = W - GUMBEL_MAX;
        const int nproc = last ? nbuf : nbuf - nbuf % SX_FLUSH;
        for (int i0 = 0; i0 < nproc; i0 += 32 * SX_CHAINS) {
          // SX_CHAINS independent Philox chains per lane (latency hiding), in column order
          uint32_t wv[SX_CHAINS];
          float qv[SX_CHAINS];
          int colv[SX_CHAINS];
#pragma unroll
          for (int r = 0; r < SX_CHAINS; ++r) {
            const int i = i0 + 32 * r + lane;
            qv[r] = i < nproc ? __uint_as_float(lds32(wq + 4 * i)) : -INFINITY;
            colv[r] = i < nproc ? static_cast<int>(lds32(wcol + 4 * i)) : 0;
          }
          if constexpr (SX_CHAINS == 2) {
            if (nproc - i0 > 32) {  // both chains hold candidates: one pass, key schedule once
              philox_w0_x2(static_cast<uint32_t>(colv[0]), static_cast<uint32_t>(colv[1]), k0,
                           k1, wv[0], wv[1]);
            } else {
              wv[0] = qv[0] < thr_now ? 0u : philox_w0(static_cast<uint32_t>(colv[0]), k0, k1);
              wv[1] = 0u;
            }
          } else {
#pragma unroll
            for (int r = 0; r < SX_CHAINS; ++r)
              wv[r] = qv[r] < thr_now ? 0u : philox_w0(static_cast<uint32_t>(colv[r]), k0, k1);
          }
#pragma unroll
          for (int r = 0; r < SX_CHAINS; ++r) {
            if (!(qv[r] < thr_now)) {
              const float u = fminf(fmaxf(uint_to_uniform(wv[r]), 0x1.b7cdfep-34f), 0x1.fffffcp-1f);
              const float y = fmaxf(W, bg) - qv[r];
              const float umin = ex2(-ex2(-y * L) * L);
              if (!(u < umin - 2e-6f)) arg_merge(bg, bgi, qv[r] + gumbel_from_word(wv[r]), colv[r]);
            }
          }
        }
        // the left-over (< SX_FLUSH) moves to the front: read both halves, then write
        const int rem = nbuf - nproc;
        if (rem > 0) {
          uint32_t cc[2] = {0u, 0u}, qq[2] = {0u, 0u};
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            if (32 * r + lane < rem) {
              cc[r] = lds32(wcol + 4 * (nproc + 32 * r + lane));
              qq[r] = lds32(wq + 4 * (nproc + 32 * r + lane));
            }
          }
          __syncwarp();
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            if (32 * r + lane < rem) {
              sts32(wcol + 4 * (32 * r + lane), cc[r]);
              sts32(wq + 4 * (32 * r + lane), qq[r]);
            }
          }
        }
        __syncwarp();
        nbuf = rem;
        const float wm = warp_max(bg);
        if (wm > W) {
          W = wm;
          if (lane == 0) {
            atomicMax(&c.wbound, (static_cast<unsigned long long>(row) << 32) | fkey(wm));
            atomicMax(row_bound + row, fkey(wm));  // result unused: a reduction
          }
        }
      };
      for (int c0 = c_beg; c0 < c_end; c0 += SX_COLS, ++u) {
        const int slot = u % SX_RING;
        bool ok = !*abort_flag;
        if (ok && !mbar_wait(&c.full[slot], (u / SX_RING) & 1)) {
          fail();
          ok = false;
        }
        const int scols = min(SX_COLS, c_end - c0);
        const int base = warp * SP_TILE;  // this warp's columns inside the stage
        if (ok && base < scols) {
          const uint32_t sx = ring_s + slot * SX_BYTES;
          float q[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int cl = base + 128 * j + 4 * lane;
            if (cl < scols) {  // scols - cl is a multiple of 4
              const uint4 v = lds128(sx + 4 * cl);
              q[4 * j] = __uint_as_float(v.x); q[4 * j + 1] = __uint_as_float(v.y);
              q[4 * j + 2] = __uint_as_float(v.z); q[4 * j + 3] = __uint_as_float(v.w);
            } else {
              q[4 * j] = q[4 * j + 1] = q[4 * j + 2] = q[4 * j + 3] = -INFINITY;
            }
          }
          if (do_div) {
            float xhi = 0.f, xlo = INFINITY;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              xhi = fmaxf(xhi, fabsf(q[i]));
              xlo = fminf(xlo, fabsf(q[i]));
            }
            if (__all_sync(0xffffffffu, xhi <= dhi && xlo >= dlo)) {  // Markstein = IEEE quotient
#pragma unroll
              for (int i = 0; i < 16; ++i) q[i] = div_rn_by(q[i], temp, rtemp);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) q[i] = div_exact(q[i], temp, rtemp, dlo, dhi);
            }
          }
          if constexpr (SC) {
            const int64_t rb = row * static_cast<int64_t>(V) + c0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int cl = base + 128 * j + 4 * lane;
              if (cl < scols) {
                uint2 o;
                if (sc_keep) {
                  o = *reinterpret_cast<const uint2*>(sc_prev + rb + cl);
                } else {
                  o.x = bf16x2_bits(q[4 * j], q[4 * j + 1]);
                  o.y = bf16x2_bits(q[4 * j + 2], q[4 * j + 3]);
                }
                __stcs(reinterpret_cast<uint2*>(sc_out + rb + cl), o);
              }
            }
          }
          float tm = q[0];
#pragma unroll
          for (int i = 1; i < 16; ++i) tm = fmaxf(tm, q[i]);
          const float wmx = warp_max(tm);
          const int col0 = c0 + base + 4 * lane;  // column of q[0]; q[i] at col0 + 128*(i>>2) + (i&3)
          if (wmx > bq || wmx > m) {  // rare: a new maximum of the item in this tile
            int fc = 0x7fffffff, fi = -1;  // this lane's first element equal to wmx
#pragma unroll
            for (int i = 15; i >= 0; --i) {
              if (q[i] == wmx) {
                fi = i;
                fc = col0 + 128 * (i >> 2) + (i & 3);
              }
            }
            const int wfc = warp_min_i(fc);
            if (wmx > bq) {
              bq = wmx;
              bqi = wfc;
            }
            if (wmx > m) {
              if (m != -INFINITY) {  // move the implicit 1 to the new maximum: lane 0 takes the old one
                const float a = ex2((m - wmx) * L);
                t2 = a * (t2 + (m - wmx) * L * sp);
                sp = a * sp;
                if (lane == 0) {
                  t2 += a * (m - wmx) * L;
                  sp += a;
                }
              }
              m = wmx;
              m2 = wmx * L;
              const int skip = (fc == wfc) ? fi : -1;  // the element carrying the new implicit 1
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (i != skip) {
                  const float d2 = fmaxf(fmaf(q[i], L, -m2), -1000.0f);
                  const float e = ex2(d2);
                  sp += e;
                  t2 = fmaf(d2, e, t2);
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float d2 = fmaxf(fmaf(q[i], L, -m2), -1000.0f);
                const float e = ex2(d2);
                sp += e;
                t2 = fmaf(d2, e, t2);
              }
            }
          } else if (m != -INFINITY) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float d2 = fmaxf(fmaf(q[i], L, -m2), -1000.0f);
              const float e = ex2(d2);
              sp += e;
              t2 = fmaf(d2, e, t2);
            }
          }
          if (want_gumbel) {
            if (first) {  // bootstrap the bound with each lane's tile maximum
              first = false;
              if (tm != -INFINITY) {
                int im = 0;
#pragma unroll
                for (int i = 15; i >= 0; --i)
                  if (q[i] == tm) im = i;
                const int ci = col0 + 128 * (im >> 2) + (im & 3);
                arg_merge(bg, bgi, tm + gumbel_from_word(philox_w0(static_cast<uint32_t>(ci), k0, k1)), ci);
              }
              W = fmaxf(W, warp_max(bg));
            }
            {
              const unsigned long long sb = *reinterpret_cast<volatile unsigned long long*>(&c.wbound);
              if (static_cast<int64_t>(sb >> 32) == row) W = fmaxf(W, fdecode(static_cast<uint32_t>(sb)));
            }
            const float thr = W - GUMBEL_MAX;
            unsigned cm = 0;
            if (!(tm < thr)) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (!(q[i] < thr) && q[i] != -INFINITY) cm |= 1u << i;
            }
            if (__any_sync(0xffffffffu, cm != 0)) {
              const int n = __popc(cm);
              int incl = n;
#pragma unroll
              for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
              }
              const int total = __shfl_sync(0xffffffffu, incl, 31);
              int pos = nbuf + incl - n;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (cm & (1u << i)) {
                  sts32(wcol + 4 * pos, static_cast<uint32_t>(col0 + 128 * (i >> 2) + (i & 3)));
                  sts32(wq + 4 * pos, __float_as_uint(q[i]));
                  ++pos;
                }
              }
              nbuf += total;
              if (nbuf >= SX_FLUSH) flush(false);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.empty[slot]);
      }
      if (want_gumbel && nbuf > 0) flush(true);
      // ---- item result: m and the argmax are warp-uniform; sp, t2 add up in a fixed tree
      float spw = sp, t2w = t2;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        spw += __shfl_xor_sync(0xffffffffu, spw, o);
        t2w += __shfl_xor_sync(0xffffffffu, t2w, o);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float bgo = __shfl_xor_sync(0xffffffffu, bg, o);
        const int bgio = __shfl_xor_sync(0xffffffffu, bgi, o);
        arg_merge(bg, bgi, bgo, bgio);
      }
      if (lane == 0) {
        const int b = k & 1;
        if (!*abort_flag && !mbar_wait(&c.pempty[b], ((k >> 1) & 1) ^ 1, 2000000000ull, 32)) fail();
        Part pt;
        pt.m = m; pt.s = spw; pt.t = t2w * 0.6931471805599453f; pt.bq = bq; pt.bqi = bqi;
        pt.bg = bg; pt.bgi = bgi; pt.pad = 0.f;
        if (m == -INFINITY) { pt.s = 0.f; pt.t = 0.f; }
        s_wpart[b][warp] = pt;
        mbar_arrive(&c.pfull[b]);
      }
      __syncwarp();
    }
    if (lane == 0) atomicAdd(&c.done, 1);
  }
  __syncthreads();
}

// Finishes each row from its chunk partials, merged in chunk order (one thread per row).
__global__ void row_merge_kernel(const Part* __restrict__ parts, int64_t rows, int nchunks,
                                 float* __restrict__ entropy, int64_t* __restrict__ samp,
                                 int64_t* __restrict__ amax) {
  pdl_wait_trigger();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const Part* pr = parts + row * nchunks;
  Part acc = pr[0];
  for (int ch = 1; ch < nchunks; ++ch) {
    const Part p = pr[ch];
    sm_merge(acc.m, acc.s, acc.t, p.m, p.s, p.t);
    arg_merge(acc.bq, acc.bqi, p.bq, p.bqi);
    arg_merge(acc.bg, acc.bgi, p.bg, p.bgi);
  }
  if (entropy) entropy[row] = log1pf(acc.s) - acc.t / (1.0f + acc.s);
  if (amax) amax[row] = row_index(acc.bqi);
  if (samp) samp[row] = row_index(acc.bgi);
}

// ------------------------------------------------------------------------------------------
// Acceptance mask + stop test, one CTA per batch row, one thread per canvas position.
__global__ void __launch_bounds__(1024)
    accept_stop_kernel(const float* __restrict__ ent, const int64_t* __restrict__ cur,
                       const int64_t* __restrict__ prop, int B, int L, float bound,
                       uint8_t* __restrict__ mask, int64_t* __restrict__ out,
                       const int64_t* __restrict__ argmax, int64_t* __restrict__ history, int S,
                       float conf, uint8_t* __restrict__ finished) {
  pdl_wait_trigger();
  __shared__ float sh[1024];
  __shared__ float sorted[1024];
  __shared__ uint8_t msorted[1024];
  const int b = blockIdx.x, i = threadIdx.x;
  const bool act = i < L;
  const int64_t gi = static_cast<int64_t>(b) * L + i;
  const float h = act ? ent[gi] : 0.f;
  if (act) sh[i] = h;
  __syncthreads();
  int rank = 0;
  if (act) {
    for (int j = 0; j < L; ++j) {
      const float hj = sh[j];
      rank += (hj < h) || (hj == h && j < i);
    }
    sorted[rank] = h;
  }
  __syncthreads();
  if (i == 0) {
    double acc = 0.0;
    for (int k = 0; k < L; ++k) {
      acc += static_cast<double>(sorted[k]);
      const float c = static_cast<float>(acc);
      msorted[k] = __fsub_rn(c, sorted[k]) <= bound;
    }
  }
  __syncthreads();
  if (act) {
    const uint8_t mk = msorted[rank];
    if (mask) mask[gi] = mk;
    if (out) out[gi] = mk ? prop[gi] : cur[gi];
  }
  if (finished) {
    int eq = 1;
    if (S > 0 && act) {
      const int64_t a = argmax[gi];
      for (int sidx = 0; sidx < S; ++sidx)
        eq &= history[(static_cast<int64_t>(sidx) * B + b) * L + i] == a;
      for (int sidx = 0; sidx + 1 < S; ++sidx)
        history[(static_cast<int64_t>(sidx) * B + b) * L + i] =
            history[(static_cast<int64_t>(sidx + 1) * B + b) * L + i];
      history[(static_cast<int64_t>(S - 1) * B + b) * L + i] = a;
    }
    const int stable = __syncthreads_and(eq);
    if (i == 0) {
      double acc = 0.0;
      for (int k = 0; k < L; ++k) acc += static_cast<double>(sh[k]);
      const float mean = static_cast<float>(acc / static_cast<double>(L));
      finished[b] = (stable && mean < conf) ? 1 : 0;
    }
  }
}

}  // namespace

size_t sampler_ws_layout(int64_t rows, int64_t V, int* nchunks_out, int* chunk_cols_out,
                         size_t* off_ticket, size_t* off_bound, size_t* off_counter) {
  int nch = 1;
  while (static_cast<int64_t>(nch) * SP_TARGET_CHUNK < V && nch < (1 << 20)) nch <<= 1;
  int64_t cols = (V + nch - 1) / nch;
  cols = ((cols + SP_TILE - 1) / SP_TILE) * SP_TILE;
  if (nchunks_out) *nchunks_out = nch;
  if (chunk_cols_out) *chunk_cols_out = static_cast<int>(cols);
  size_t o = static_cast<size_t>(rows) * nch * sizeof(Part);
  o = (o + 255) & ~size_t(255);
  if (off_ticket) *off_ticket = o;
  o += static_cast<size_t>(rows) * 4;
  o = (o + 255) & ~size_t(255);
  if (off_bound) *off_bound = o;
  o += static_cast<size_t>(rows) * 4;
  o = (o + 255) & ~size_t(255);
  if (off_counter) *off_counter = o;
  o += 256;
  return o;
}

}  // namespace knx

extern "C" size_t knx_sampler_workspace_size(int64_t rows, int64_t V) {
  if (rows < 0 || V <= 0) return 0;
  return knx::sampler_ws_layout(rows, V, nullptr, nullptr, nullptr, nullptr, nullptr);
}

namespace knx {
namespace {

// Self-conditioning copy for the shapes and alignments the stream kernel does not take (same rule
// and the same quotient: IEEE x / T).
__global__ void sc_cast_kernel(const float* __restrict__ x, int64_t rows, int64_t V, float temp,
                               int do_div, __nv_bfloat16* __restrict__ out,
                               const __nv_bfloat16* __restrict__ prev,
                               const uint8_t* __restrict__ finished, int64_t canvas_len) {
  pdl_wait_trigger();
  const int64_t n = rows * V;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / V;
    if (finished != nullptr && finished[r / canvas_len] != 0) {
      out[i] = prev[i];
    } else {
      const float q = do_div ? __fdiv_rn(x[i], temp) : x[i];
      out[i] = __ushort_as_bfloat16(static_cast<unsigned short>(bf16_bits(q)));
    }
  }
}

int sampler_run(const float* logits, int64_t rows, int64_t V, float temperature, int64_t seed,
                float* entropy, int64_t* samp, int64_t* amax, void* workspace,
                size_t workspace_bytes, cudaStream_t s, __nv_bfloat16* sc_out,
                const __nv_bfloat16* sc_prev, const uint8_t* finished, int64_t canvas_len) {
  if (rows < 0 || V <= 0 || V > 0x7fffffffLL || rows > (1LL << 31)) return KNX_E_INVALID;
  if (!(temperature > 0.f) || !isfinite(temperature)) return KNX_E_INVALID;
  if (!aligned(logits, 4)) return KNX_E_ALIGN;
  if (rows == 0) return KNX_OK;
  int nch = 0, ccols = 0;
  size_t o_ticket = 0, o_bound = 0, o_counter = 0;
  const size_t need = sampler_ws_layout(rows, V, &nch, &ccols, &o_ticket, &o_bound, &o_counter);
  if (workspace == nullptr || workspace_bytes < need) return KNX_E_WORKSPACE;
  if (!aligned(workspace, 256)) return KNX_E_ALIGN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  // row tickets, per-row Gumbel bounds and the work counter start from zero every call
  if (cudaMemsetAsync(ws + o_ticket, 0, o_counter + 256 - o_ticket, s) != cudaSuccess)
    return KNX_E_LAUNCH;
  const float rtemp = 1.0f / temperature;
  const int do_div = temperature != 1.0f;
  const int seed_is32 = (seed >= -2147483648LL && seed <= 2147483647LL) ? 1 : 0;
  const int want_g = samp != nullptr;
  const bool vec = (V % 4) == 0 && aligned(logits, 16);
  const int64_t items = rows * nch;
  const int64_t maxgrid = static_cast<int64_t>(num_sms()) * 3;
  const int grid = static_cast<int>(items < maxgrid ? items : maxgrid);
  Part* parts = reinterpret_cast<Part*>(ws);
  uint32_t* ticket = reinterpret_cast<uint32_t*>(ws + o_ticket);
  uint32_t* bound = reinterpret_cast<uint32_t*>(ws + o_bound);
  int* counter = reinterpret_cast<int*>(ws + o_counter);
  // the stream kernel writes the self-conditioning copy itself when both buffers allow 8-byte
  // stores; otherwise sc_cast_kernel does it after the sampler
  const bool sc_in_pass = sc_out != nullptr && aligned(sc_out, 8) &&
                          (sc_prev == nullptr || aligned(sc_prev, 8)) && vec && (ccols % 4) == 0;
  if (vec && (ccols % 4) == 0) {
    // streaming kernel: one persistent CTA per SM, static item assignment
    auto kern = sc_in_pass ? sampler_stream_kernel<true> : sampler_stream_kernel<false>;
    if (set_max_dyn_smem(reinterpret_cast<const void*>(kern), static_cast<int>(SX_SMEM)) != KNX_OK)
      return KNX_E_DEVICE;
    // quarter-row items (the workspace holds rows * nch >= rows * nch_s partials)
    const int nch_s = static_cast<int>((V + SX_CHUNK - 1) / SX_CHUNK);
    const int64_t sitems = rows * nch_s;
    const int64_t sms = num_sms();
    const int sgrid = static_cast<int>(sitems < sms ? sitems : sms);
    int* dev_err = counter + 1;  // workspace word next to the counter, zeroed above
    (void)launch_pdl(kern, sgrid, SX_THREADS, SX_SMEM, s, logits, rows, static_cast<int>(V),
                     temperature, rtemp, do_div, seed, seed_is32, want_g, nch_s, parts, bound,
                     dev_err, sc_in_pass ? sc_out : nullptr, sc_in_pass ? sc_prev : nullptr,
                     sc_in_pass ? finished : nullptr, static_cast<int>(canvas_len));
    if (cudaGetLastError() != cudaSuccess) return KNX_E_LAUNCH;
    (void)launch_pdl(row_merge_kernel, static_cast<unsigned>((rows + 127) / 128), 128, 0, s, parts,
                     rows, nch_s, entropy, samp, amax);
  } else if (vec) {
    (void)launch_pdl(sampler_kernel<true>, grid, SP_THREADS, 0, s, logits, rows,
                     static_cast<int>(V), temperature, rtemp, do_div, seed, seed_is32, want_g, nch,
                     ccols, parts, ticket, bound, counter, entropy, samp, amax);
  } else {
    (void)launch_pdl(sampler_kernel<false>, grid, SP_THREADS, 0, s, logits, rows,
                     static_cast<int>(V), temperature, rtemp, do_div, seed, seed_is32, want_g, nch,
                     ccols, parts, ticket, bound, counter, entropy, samp, amax);
  }
  if (sc_out != nullptr && !sc_in_pass) {
    if (cudaGetLastError() != cudaSuccess) return KNX_E_LAUNCH;
    const int64_t n = rows * V;
    const int64_t blocks = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
    (void)launch_pdl(sc_cast_kernel, static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, s,
                     logits, rows, V, temperature, do_div, sc_out, sc_prev, finished, canvas_len);
  }
  return launch_status();
}

}  // namespace
}  // namespace knx

extern "C" int knx_sampler_fused(const float* logits, int64_t rows, int64_t V, float temperature,
                                 int64_t seed, float* entropy, int64_t* samp, int64_t* amax,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  return knx::sampler_run(logits, rows, V, temperature, seed, entropy, samp, amax, workspace,
                          workspace_bytes, static_cast<cudaStream_t>(stream), nullptr, nullptr,
                          nullptr, 1);
}

extern "C" int knx_sampler_fused_sc(const float* logits, int64_t rows, int64_t V,
                                    float temperature, int64_t seed, float* entropy,
                                    int64_t* samp, int64_t* amax, void* sc_out,
                                    const void* sc_prev, const uint8_t* finished,
                                    int64_t canvas_len, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  using namespace knx;
  if (sc_out == nullptr || !aligned(sc_out, 2)) return sc_out == nullptr ? KNX_E_INVALID : KNX_E_ALIGN;
  if (finished != nullptr) {
    if (sc_prev == nullptr || canvas_len < 1 || rows % canvas_len != 0) return KNX_E_INVALID;
    if (!aligned(sc_prev, 2)) return KNX_E_ALIGN;
  }
  if (canvas_len > 0x7fffffffLL) return KNX_E_INVALID;
  return sampler_run(logits, rows, V, temperature, seed, entropy, samp, amax, workspace,
                     workspace_bytes, static_cast<cudaStream_t>(stream),
                     static_cast<__nv_bfloat16*>(sc_out), static_cast<const __nv_bfloat16*>(sc_prev),
                     finished, canvas_len > 0 ? canvas_len : 1);
}

extern "C" int knx_accept_stop(const float* entropy, const int64_t* cur, const int64_t* proposal,
                               int64_t B, int64_t L, float entropy_bound, uint8_t* mask,
                               int64_t* out, const int64_t* argmax, int64_t* history,
                               int stability_threshold, float confidence_threshold,
                               uint8_t* finished, void* stream) {
  using namespace knx;
  if (B < 0 || L <= 0 || L > 1024 || B > 65535 || stability_threshold < 0) return KNX_E_INVALID;
  if (finished && stability_threshold > 0 && (history == nullptr || argmax == nullptr))
    return KNX_E_INVALID;
  if (out && (cur == nullptr || proposal == nullptr)) return KNX_E_INVALID;
  if (B == 0) return KNX_OK;
  const int threads = static_cast<int>(((L + 31) / 32) * 32);
  (void)launch_pdl(accept_stop_kernel, static_cast<unsigned>(B), threads, 0,
                   static_cast<cudaStream_t>(stream), entropy, cur, proposal, static_cast<int>(B),
                   static_cast<int>(L), entropy_bound, mask, out, argmax, history,
                   stability_threshold, confidence_threshold, finished);
  return launch_status();
}
