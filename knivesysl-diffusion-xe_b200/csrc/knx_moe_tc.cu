// knx_moe_tc.cu — tcgen05 (5th-gen tensor core) grouped W4A16 GEMMs for the MoE layer.
//
// Same contract as the warp-MMA kernels in knx_moe.cu (gate_up+GELU into out2, down into out3,
// dense rows GEMM), different engine.  One persistent CTA per SM, warp-specialised:
//
//   warp 20      scheduler + weight producer: pulls (task, slice) work items from the counter,
//                publishes them in a 2-slot item ring (with the slice's scale/zero rows fetched by
//                1-D bulk copies), then streams the slice's packed nibbles with 2-D TMA loads
//                (64 B x rows boxes, 64-byte swizzle) into an 8-stage ring, 128 k per stage.
//   warp 21      activation producer: gathers the task's token rows (K-interleaved f16) with
//                cp.async straight into the UMMA 128-byte-swizzle K-major layout, 4-stage ring.
//   warps 0-15   dequant: thread = one weight row (= one TMEM lane); warps w, w+4, w+8, w+12
//                split each stage's 128 k in quarters.  Nibbles -> f16 pairs in registers (dequant8), tcgen05.st into a
//                TMEM A buffer (4 x 64 columns).
//   warp 22      MMA issuer (one thread): tcgen05.mma kind::f16, A from TMEM, B from shared memory
//                via a descriptor, D (fp32, 128 lanes x N tokens) in TMEM, double-buffered across
//                work items; tcgen05.commit releases A buffers, activation stages and D.
//   warps 16-19  epilogue: tcgen05.ld of D, tanh-GELU(gate) * up (gated) or plain f16 cast,
//                transposed through shared memory, coalesced row stores.
//
// The MMA is D[128 x N] += A[128 x 16] . B[N x 16]^T per k16 step, M = weight rows (64 gate + 64
// up, or 128 output rows), N = the task's tokens rounded up to 16.  Every barrier wait is bounded
// (2 s); on a timeout the kernel records KNX_DEV_TIMEOUT in the error word, all roles leave their
// loops, and the CTA releases its tensor memory before returning.
#include "knx_common.cuh"
#include "knx_internal.cuh"
#include "knx_sm100.cuh"

namespace knx {
namespace tc {

using namespace sm100;

constexpr int N_MAX = 64;                 // tokens per task (MMA N <= 64)
constexpr int BK = 128;                   // k per stage
constexpr int WROW = BK / 2;              // 64 bytes of nibbles per weight row per stage
constexpr int ROWS = 128;                 // MMA M
constexpr int SW = 8;                     // weight stages
constexpr int SA = 4;                     // activation stages
constexpr int NA = 4;                     // TMEM A buffers
constexpr int IR = 2;                     // work-item ring slots
constexpr int W_STAGE = ROWS * WROW;      // 8 KB
constexpr int A_KBLK = N_MAX * 128;       // one 64-k block: N_MAX rows x 128 B
constexpr int A_STAGE = 2 * A_KBLK;       // 16 KB
constexpr int A_COL0 = 0;                 // TMEM columns [0, 256): A buffers, 64 columns each
constexpr int D_COL0 = NA * 64;           // TMEM columns [256, 256 + 2*N_MAX): D buffers
constexpr int TMEM_COLS = 512;
constexpr int DQ_WARPS = 16;              // 4 per SM sub-partition; warp w: lanes 32*(w%4), k quarter w/4
constexpr int NUM_WARPS = DQ_WARPS + 4 + 3;
constexpr int NTHREADS = NUM_WARPS * 32;
constexpr int WARP_EPI0 = DQ_WARPS;       // warps 16-19: epilogue (lane quadrant = warp % 4)
constexpr int WARP_WPROD = DQ_WARPS + 4, WARP_APROD = DQ_WARPS + 5, WARP_MMA = DQ_WARPS + 6;
constexpr int ITEM_CONSUMERS = DQ_WARPS + 1 + 1 + 4;  // dequant, act producer, MMA, epilogue warps
constexpr int SZ_MAX = 40;                // scale/zero groups per row on this path

struct Item {
  int valid, e, cnt, slice;
  int slot0, npad, nvalid, pad;
};

struct Ctrl {
  uint64_t w_full[SW], w_empty[SW];
  uint64_t a_full[SA], a_empty[SA];
  uint64_t t_full[NA], t_empty[NA];  // TMEM A buffers
  uint64_t d_full[2], d_empty[2];
  uint64_t i_full[IR], i_empty[IR];
  uint64_t fin;          // MMA drain before tensor memory is released
  int epi_ok[4];         // epilogue warps' agreement flags (see the epilogue)
  Item items[IR];
  uint32_t tmem_base;
  int abort;
};

struct Params {
  const __half* act;          // activation rows (K-interleaved f16)
  int64_t act_stride;         // elements between rows
  const int32_t* sorted_pair;  // != null: act row of slot s = sorted_pair[s] / topk (GEMM1)
  int topk;
  const int32_t* offsets;     // [E+1] slot offsets (null: dense, slot = token)
  const int4* tasks;          // (expert, tok_start, count) or null (dense)
  const int32_t* ntasks;
  int dense_rows;
  int* work_counter;
  const __half* ws;           // scale [E, rows, ng]
  const __half* wz;           // zero  [E, rows, ng]
  int K;                      // contraction length
  int rows_per_expert;        // 2I (gated) or N (plain)
  int I;                      // gated: offset of the up rows
  int ng, gs;
  __half* out;                // gated: out2 [slots, I]; plain: [slots, N]
  int64_t out_stride;
  int nslices;
  int32_t* err;
};

// smem layout (from a 1024-aligned base): activation ring, weight ring, scale/zero slots, epilogue
constexpr int OFF_A = 0;
constexpr int OFF_W = OFF_A + SA * A_STAGE;
constexpr int OFF_SZ = OFF_W + SW * W_STAGE;
KNX_HOST_DEVINL size_t sz_slot_bytes(int ng) { return (static_cast<size_t>(512) * ng + 1023) & ~size_t(1023); }
constexpr int EPI_BYTES = 2 * 64 * N_MAX * 4 + N_MAX * (ROWS + 8) * 2;  // gate/up exchange + out tile
inline size_t smem_bytes(int ng) {
  return 1024 + OFF_SZ + IR * sz_slot_bytes(ng) + EPI_BYTES;
}

KNX_DEVINL void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }

KNX_DEVINL float gelu_tanh(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  const float th = 2.0f / (1.0f + expf(-2.0f * inner)) - 1.0f;
  return 0.5f * x * (1.0f + th);
}
KNX_DEVINL int perm_pos(int n) { return (n & ~7) + 2 * (n & 3) + ((n >> 2) & 1); }

template <bool GATED, bool ZINT>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const Params p) {
  pdl_wait_trigger();
  extern __shared__ uint8_t dsm_raw[];
  __shared__ Ctrl ctrl;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_ring = base + OFF_A;
  uint8_t* w_ring = base + OFF_W;
  const size_t szb = sz_slot_bytes(p.ng);
  uint8_t* sz_ring = base + OFF_SZ;
  uint8_t* epi = sz_ring + IR * szb;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nst = (p.K + BK - 1) / BK;

  if (tid == 0) {
    for (int s = 0; s < SW; ++s) { mbar_init(&ctrl.w_full[s], 1); mbar_init(&ctrl.w_empty[s], DQ_WARPS); }
    for (int s = 0; s < SA; ++s) { mbar_init(&ctrl.a_full[s], 32); mbar_init(&ctrl.a_empty[s], 1); }
    for (int b = 0; b < NA; ++b) { mbar_init(&ctrl.t_full[b], DQ_WARPS); mbar_init(&ctrl.t_empty[b], 1); }
    for (int d = 0; d < 2; ++d) { mbar_init(&ctrl.d_full[d], 1); mbar_init(&ctrl.d_empty[d], 4); }
    for (int i = 0; i < IR; ++i) {
      mbar_init(&ctrl.i_full[i], 1);
      mbar_init(&ctrl.i_empty[i], ITEM_CONSUMERS);
    }
    mbar_init(&ctrl.fin, 1);
    ctrl.abort = 0;
    fence_mbar_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(&ctrl.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == WARP_WPROD && lane == 0) prefetch_tensormap(&wmap);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl.tmem_base;
  volatile int* abort_flag = &ctrl.abort;
  auto fail = [&]() {
    *abort_flag = 1;
    if (p.err) atomicOr(p.err, KNX_DEV_TIMEOUT);
  };
  // bounded mbarrier wait; `backoff_ns` > 0 sleeps between polls (roles that wait long and
  // would otherwise take issue slots from the dequant warps)
  auto wait = [&](uint64_t* bar, uint32_t parity, uint32_t backoff_ns = 0) -> bool {
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity, 2000000000ull, backoff_ns)) {
      fail();
      return false;
    }
    return true;
  };

  if (warp == WARP_WPROD) {
    // ---------------------------------------------------------------- scheduler + weights
    if (lane == 0) {
      const int nwork = (p.tasks ? *p.ntasks : (p.dense_rows + N_MAX - 1) / N_MAX) * p.nslices;
      uint32_t wst = 0;
      for (int n = 0;; ++n) {
        const int slot = n % IR;
        if (!wait(&ctrl.i_empty[slot], ((n / IR) & 1) ^ 1)) break;
        const int wi = atomicAdd(p.work_counter, 1);
        Item it{};
        if (wi < nwork) {
          const int task = wi / p.nslices;
          it.slice = wi - task * p.nslices;
          int t0;
          if (p.tasks) {
            const int4 tk = p.tasks[task];
            it.e = tk.x; t0 = tk.y; it.cnt = tk.z;
          } else {
            it.e = 0; t0 = task * N_MAX; it.cnt = min(N_MAX, p.dense_rows - t0);
          }
          it.slot0 = (p.offsets ? p.offsets[it.e] : 0) + t0;
          it.npad = (it.cnt + 15) & ~15;
          it.nvalid = GATED ? ROWS : min(ROWS, p.rows_per_expert - it.slice * ROWS);
          it.valid = 1;
        }
        ctrl.items[slot] = it;
        if (!it.valid) {
          mbar_arrive(&ctrl.i_full[slot]);
          break;
        }
        // scale / zero rows of the slice -> slot (1-D bulk copies, 16-byte granules)
        uint8_t* szs = sz_ring + slot * szb;
        const int ng = p.ng;
        if (GATED) {
          const int64_t g0 = (static_cast<int64_t>(it.e) * p.rows_per_expert + it.slice * 64) * ng;
          const int64_t u0 = g0 + static_cast<int64_t>(p.I) * ng;
          const uint32_t b = 64u * ng * 2u;
          mbar_arrive_expect_tx(&ctrl.i_full[slot], 4 * b);
          bulk_load(szs + 0 * b, p.ws + g0, b, &ctrl.i_full[slot]);
          bulk_load(szs + 1 * b, p.wz + g0, b, &ctrl.i_full[slot]);
          bulk_load(szs + 2 * b, p.ws + u0, b, &ctrl.i_full[slot]);
          bulk_load(szs + 3 * b, p.wz + u0, b, &ctrl.i_full[slot]);
        } else {
          const int64_t r0 = (static_cast<int64_t>(it.e) * p.rows_per_expert + it.slice * ROWS) * ng;
          const uint32_t b = static_cast<uint32_t>(it.nvalid) * ng * 2u;
          mbar_arrive_expect_tx(&ctrl.i_full[slot], 2 * b);
          bulk_load(szs, p.ws + r0, b, &ctrl.i_full[slot]);
          bulk_load(szs + 256 * ng, p.wz + r0, b, &ctrl.i_full[slot]);
        }
        // packed weights, one stage = 128 k of all 128 rows
        for (int st = 0; st < nst; ++st, ++wst) {
          const int s = wst % SW;
          if (!wait(&ctrl.w_empty[s], ((wst / SW) & 1) ^ 1)) break;
          uint8_t* dst = w_ring + s * W_STAGE;
          mbar_arrive_expect_tx(&ctrl.w_full[s], W_STAGE);
          const int x = st * WROW;
          if (GATED) {
            const int y = it.e * p.rows_per_expert + it.slice * 64;
            tma_load_2d(dst, &wmap, &ctrl.w_full[s], x, y);
            tma_load_2d(dst + 64 * WROW, &wmap, &ctrl.w_full[s], x, y + p.I);
          } else {
            tma_load_2d(dst, &wmap, &ctrl.w_full[s], x, it.e * p.rows_per_expert + it.slice * ROWS);
          }
        }
        if (*abort_flag) break;
      }
    }
    __syncwarp();
  } else if (warp == WARP_APROD) {
    // ---------------------------------------------------------------- activation gather
    uint32_t ast = 0;
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      if (!wait(&ctrl.i_full[slot], (n / IR) & 1)) break;
      const Item it = ctrl.items[slot];
      if (!it.valid) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      // lane l copies the rows of tokens l and l + 32 (16-byte chunks straight into the swizzled
      // K-major layout: row t, chunk j -> block j/8, row group t/8, chunk (j%8) ^ (t%8))
      const __half* src0 = nullptr;
      const __half* src1 = nullptr;
      if (lane < it.cnt)
        src0 = p.act + (p.sorted_pair ? p.sorted_pair[it.slot0 + lane] / p.topk
                                      : static_cast<int64_t>(it.slot0 + lane)) * p.act_stride;
      if (lane + 32 < it.cnt)
        src1 = p.act + (p.sorted_pair ? p.sorted_pair[it.slot0 + lane + 32] / p.topk
                                      : static_cast<int64_t>(it.slot0 + lane + 32)) * p.act_stride;
      const uint32_t dst_row0 = (lane >> 3) * 1024 + (lane & 7) * 128;
      const uint32_t dst_row1 = ((lane + 32) >> 3) * 1024 + (lane & 7) * 128;
      bool ok = true;
      for (int st = 0; st < nst; ++st, ++ast) {
        const int s = ast % SA;
        if (!wait(&ctrl.a_empty[s], ((ast / SA) & 1) ^ 1, 32)) {
          ok = false;
          break;
        }
        uint8_t* dst = a_ring + s * A_STAGE;
        const int k0 = st * BK;
        const int kch = min(BK, p.K - k0) >> 3;  // 16-byte chunks per row this stage (16 or 8)
        if (src0) {
#pragma unroll 4
          for (int j = 0; j < kch; ++j)
            cp_async16(dst + (j >> 3) * A_KBLK + dst_row0 + (((j & 7) ^ (lane & 7)) << 4),
                       src0 + k0 + j * 8);
        }
        if (src1) {
#pragma unroll 4
          for (int j = 0; j < kch; ++j)
            cp_async16(dst + (j >> 3) * A_KBLK + dst_row1 + (((j & 7) ^ (lane & 7)) << 4),
                       src1 + k0 + j * 8);
        }
        cp_async_mbar_arrive_noinc(&ctrl.a_full[s]);
      }
      __syncwarp();
      if (!ok) break;
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
  } else if (warp < DQ_WARPS) {
    // ---------------------------------------------------------------- dequant -> TMEM
    const int q = warp & 3, kq = warp >> 2;  // lane quadrant, k quarter (32 k) of the stage
    const int row = 32 * q + lane;
    uint32_t wst = 0, tb = 0;
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      if (!wait(&ctrl.i_full[slot], (n / IR) & 1)) break;
      const Item it = ctrl.items[slot];
      if (!it.valid) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      const __half* szs = reinterpret_cast<const __half*>(sz_ring + slot * szb);
      const int ng = p.ng;
      const __half* srow;
      const __half* zrow;
      if (GATED) {
        srow = szs + (row < 64 ? 0 : 128 * ng) + (row & 63) * ng;
        zrow = srow + 64 * ng;
      } else {
        srow = szs + row * ng;
        zrow = szs + 128 * ng + row * ng;
      }
      const bool row_ok = row < it.nvalid;
      const int sw = (row >> 1) & 3;
      bool ok = true;
      for (int st = 0; st < nst; ++st, ++wst, ++tb) {
        const int ws = wst % SW, b = tb % NA;
        if (!wait(&ctrl.w_full[ws], (wst / SW) & 1) || !wait(&ctrl.t_empty[b], ((tb / NA) & 1) ^ 1)) {
          ok = false;
          break;
        }
        const int k0 = st * BK + kq * 32;
        if (k0 < p.K) {
          uint32_t v[16];
          if (row_ok) {
            const int grp = k0 / p.gs;
            const uint2 c = make_sz<ZINT>(srow[grp], zrow[grp]);
            const __half2 s2 = __low2half2(u32_as_h2(c.x)), cc = __high2half2(u32_as_h2(c.x));
            const __half2 s16 = __low2half2(u32_as_h2(c.y)), c16 = __high2half2(u32_as_h2(c.y));
            const uint4 u = lds128(smem_u32(w_ring + ws * W_STAGE + row * WROW) + ((kq ^ sw) << 4));
            const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t w4[4];
              dequant8<ZINT>(uu[i], s2, s16, cc, c16, w4);
              v[4 * i] = w4[0]; v[4 * i + 1] = w4[1]; v[4 * i + 2] = w4[2]; v[4 * i + 3] = w4[3];
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0u;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctrl.w_empty[ws]);  // weights of this stage consumed
          tmem_st16(tmem + ((32u * q) << 16) + A_COL0 + b * 64 + kq * 16, v);
          tmem_wait_st();
        } else {
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctrl.w_empty[ws]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.t_full[b]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
  } else if (warp == WARP_MMA) {
    // ---------------------------------------------------------------- tcgen05.mma issue
    if (lane == 0) {
      uint32_t ast = 0, tb = 0, dc = 0;
      for (int n = 0;; ++n) {
        const int slot = n % IR;
        if (!wait(&ctrl.i_full[slot], (n / IR) & 1)) break;
        const Item it = ctrl.items[slot];
        if (!it.valid) {
          mbar_arrive(&ctrl.i_empty[slot]);
          break;
        }
        const int db = dc & 1;
        if (!wait(&ctrl.d_empty[db], ((dc >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t idesc = idesc_f16_f32(ROWS, it.npad);
        const uint32_t d_tmem = tmem + D_COL0 + db * N_MAX;
        bool ok = true;
        for (int st = 0; st < nst; ++st, ++ast, ++tb) {
          const int s = ast % SA, b = tb % NA;
          if (!wait(&ctrl.a_full[s], (ast / SA) & 1) || !wait(&ctrl.t_full[b], (tb / NA) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fence_proxy_async_smem();
          const int nk = min(BK, p.K - st * BK) >> 4;
          const uint32_t a_base = smem_u32(a_ring + s * A_STAGE);
          for (int j = 0; j < nk; ++j) {
            const uint64_t bdesc = smem_desc_sw128_kmajor(a_base + (j >> 2) * A_KBLK + (j & 3) * 32);
            mma_f16_ts(d_tmem, tmem + A_COL0 + b * 64 + 8 * j, bdesc, idesc, (st | j) != 0);
          }
          mma_commit(&ctrl.t_empty[b]);
          mma_commit(&ctrl.a_empty[s]);
        }
        if (!ok) break;
        mma_commit(&ctrl.d_full[db]);
        ++dc;
        mbar_arrive(&ctrl.i_empty[slot]);
      }
      // drain: every issued MMA completes before the CTA releases tensor memory
      mma_commit(&ctrl.fin);
      mbar_wait(&ctrl.fin, 0);
    }
    __syncwarp();
  } else if (warp >= WARP_EPI0 && warp < WARP_EPI0 + 4) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const int et = tid - WARP_EPI0 * 32;  // 0..127
    float* xgate = reinterpret_cast<float*>(epi);                        // [N_MAX][64] fp32
    float* xup = xgate + 64 * N_MAX;                                     // [N_MAX][64] fp32
    __half* otile = reinterpret_cast<__half*>(epi + 2 * 64 * N_MAX * 4); // [N_MAX][ROWS + 8]
    constexpr int OT = ROWS + 8;
    uint32_t dc = 0;
    // The four epilogue warps meet at named barriers, which have no timeout; so after every
    // bounded mbarrier wait they first agree (through epi_ok) on whether all of them succeeded,
    // and leave together if not.
    auto agree = [&](bool ok) -> bool {
      if (lane == 0) ctrl.epi_ok[q] = ok ? 1 : 0;
      named_bar(1, 128);
      const bool all = ctrl.epi_ok[0] && ctrl.epi_ok[1] && ctrl.epi_ok[2] && ctrl.epi_ok[3];
      named_bar(1, 128);
      return all;
    };
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      if (!agree(wait(&ctrl.i_full[slot], (n / IR) & 1, 256))) break;
      const Item it = ctrl.items[slot];
      if (!it.valid) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      const int db = dc & 1;
      if (!agree(wait(&ctrl.d_full[db], (dc >> 1) & 1, 128))) break;
      tc_fence_after();
      // D (128 rows x npad tokens, fp32) -> shared memory, 16 columns at a time
#pragma unroll 1
      for (int c = 0; c < it.npad / 16; ++c) {
        uint32_t v[16];
        tmem_ld16(tmem + ((32u * q) << 16) + D_COL0 + db * N_MAX + c * 16, v);
        tmem_wait_ld();
        if (GATED) {
          float* xb = row < 64 ? xgate : xup;  // [N_MAX][64] fp32, token-major
#pragma unroll
          for (int i = 0; i < 16; ++i) xb[(c * 16 + i) * 64 + (row & 63)] = __uint_as_float(v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) otile[(c * 16 + i) * OT + row] = __float2half_rn(__uint_as_float(v[i]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl.d_empty[db]);
      ++dc;
      named_bar(1, 128);
      if (GATED) {
        for (int i = et; i < it.cnt * 64; i += 128) {
          const int t = i >> 6, nn = i & 63;
          otile[t * OT + perm_pos(nn)] =
              __float2half_rn(gelu_tanh(xgate[t * 64 + nn]) * xup[t * 64 + nn]);
        }
        named_bar(1, 128);
        for (int c = et; c < it.cnt * 8; c += 128) {
          const int t = c >> 3, ch = c & 7;
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(it.slot0 + t) * p.out_stride +
                                    it.slice * 64 + ch * 8) =
              *reinterpret_cast<const uint4*>(otile + t * OT + ch * 8);
        }
      } else {
        const int vch = it.nvalid >> 3;
        for (int c = et; c < it.cnt * vch; c += 128) {
          const int t = c / vch, ch = c - t * vch;
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(it.slot0 + t) * p.out_stride +
                                    it.slice * ROWS + ch * 8) =
              *reinterpret_cast<const uint4*>(otile + t * OT + ch * 8);
        }
      }
      named_bar(1, 128);
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
  }

  // teardown: every role has left its loop (normally or on abort); release tensor memory
  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace tc

// ------------------------------------------------------------------------------------------
// host side
namespace {

// cuTensorMapEncodeTiled is a driver entry point; it is resolved through the runtime so that the
// library itself does not link libcuda (and loads on machines without a driver).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool encode_weight_map(CUtensorMap* map, const uint8_t* q, int64_t total_rows, int64_t row_bytes,
                       int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(total_rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(tc::WROW), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(
      map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool GATED, bool ZINT>
int launch_tc(const tc::Params& p, const uint8_t* wq, int64_t total_rows, int64_t row_bytes,
              int64_t work_bound, cudaStream_t s) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = tc::smem_bytes(p.ng);
  if (!attr[dev & 63]) {
    if (cudaFuncSetAttribute(tc::tc_gemm_kernel<GATED, ZINT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(tc::smem_bytes(tc::SZ_MAX))) != cudaSuccess)
      return KNX_E_DEVICE;
    attr[dev & 63] = true;
  }
  CUtensorMap map;
  if (!encode_weight_map(&map, wq, total_rows, row_bytes, GATED ? 64 : tc::ROWS)) return KNX_E_DEVICE;
  const int sms = num_sms();
  const int grid = static_cast<int>(work_bound < sms ? (work_bound > 0 ? work_bound : 1) : sms);
  (void)launch_pdl(tc::tc_gemm_kernel<GATED, ZINT>, grid, tc::NTHREADS, smem, s, map, p);
  return launch_status();
}

}  // namespace

bool tc_supported(int64_t K, int gs, int ng, int64_t rows_per_expert, bool gated) {
  if (gs % 64 != 0 || ng > tc::SZ_MAX || (K % 64) != 0) return false;
  if (gated) return (rows_per_expert / 2) % 64 == 0;
  return rows_per_expert % tc::ROWS == 0;
}

int launch_tc_gateup(const __half* xp, const int32_t* sorted_pair, int topk, const int32_t* offsets,
                     const int4* tasks, const int32_t* ntasks, int* counter, const uint8_t* gu_q,
                     const __half* gu_s, const __half* gu_z, int E, int H, int I, int ng, int gs,
                     bool zint, __half* out2, int64_t max_tasks, int32_t* err, cudaStream_t s) {
  tc::Params p{};
  p.act = xp; p.act_stride = H; p.sorted_pair = sorted_pair; p.topk = topk; p.offsets = offsets;
  p.tasks = tasks; p.ntasks = ntasks; p.work_counter = counter; p.ws = gu_s; p.wz = gu_z;
  p.K = H; p.rows_per_expert = 2 * I; p.I = I; p.ng = ng; p.gs = gs; p.out = out2;
  p.out_stride = I; p.nslices = I / 64; p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_tc<true, true>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s)
              : launch_tc<true, false>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s);
}

int launch_tc_rows(const __half* act, int64_t act_stride, int K, const int32_t* offsets,
                   const int4* tasks, const int32_t* ntasks, int dense_rows, int* counter,
                   const uint8_t* wq, const __half* ws, const __half* wz, int E, int N, int ng,
                   int gs, bool zint, __half* out, int64_t out_stride, int64_t max_tasks,
                   int32_t* err, cudaStream_t s) {
  tc::Params p{};
  p.act = act; p.act_stride = act_stride; p.offsets = offsets; p.tasks = tasks; p.ntasks = ntasks;
  p.dense_rows = dense_rows; p.work_counter = counter; p.ws = ws; p.wz = wz; p.K = K;
  p.rows_per_expert = N; p.ng = ng; p.gs = gs; p.out = out; p.out_stride = out_stride;
  p.nslices = (N + tc::ROWS - 1) / tc::ROWS; p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_tc<false, true>(p, wq, int64_t(E) * N, K / 2, work, s)
              : launch_tc<false, false>(p, wq, int64_t(E) * N, K / 2, work, s);
}

}  // namespace knx
