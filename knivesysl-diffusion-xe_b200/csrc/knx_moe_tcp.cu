// knx_moe_tcp.cu — tcgen05 (5th-gen tensor core) grouped W4A16 GEMMs for large per-expert token
// counts (prefill chunks, batches of canvases).
//
// Same contract as the warp-MMA kernels in knx_moe.cu (gate_up+GELU into out2, down into out3,
// dense rows GEMM), different engine.  One MMA is D[128 x N] += A[128 x 16] . B[N x 16]^T with
//   M = the 128 tokens of one task (one expert's slots; the activations, gathered),
//   N = up to 256 weight rows of the expert (dequantised from the packed nibbles),
// so each packed weight row is dequantised once per 128 tokens and every instruction is the full
// M128 x N256 x K16 shape.  One persistent CTA per SM, warp-specialised:
//
//   warp 20      scheduler + weight producer: pulls (task, slice) work items from the counter,
//                publishes them in a 2-slot item ring, bulk-copies the item's scale / zero rows
//                into the item's shared-memory slot, then streams the slice's packed nibbles with
//                2-D TMA loads (32 B x 64 rows boxes, no swizzle) into a 4-stage ring, 64 k per
//                stage.
//   warps 21-22  activation producers: gather the task's token rows (K-interleaved f16) with
//                cp.async straight into the UMMA 128-byte-swizzle K-major layout (8 lanes per
//                128-byte row, 64 rows per warp; one warp's instruction stream was the limit),
//                4-stage ring.
//   warps 0-15   dequant: thread = (weight row, half of the stage's 64 k).  Nibbles -> f16 pairs
//                in registers (dequant8), stored into the B operand ring in the 128-byte-swizzle
//                K-major layout, 2 stages.  Scale / zero come from the item's slot.
//   warp 23      MMA issuer (one thread): tcgen05.mma kind::f16, A and B from shared memory through
//                descriptors, D (fp32, 128 token lanes x N columns) in TMEM, double-buffered across
//                work items (2 x 256 columns); tcgen05.commit releases the stages and D.
//   warps 16-19  epilogue: thread = token (TMEM lane).  tcgen05.ld of D; gated: gate column c and
//                up column c + N/2 sit in the same lane, so tanh-GELU(gate) * up needs no exchange;
//                plain: f16 cast.  Each warp stages 32 tokens x 64 columns in shared memory and
//                stores them as whole 128-byte row pieces.
//
// Work item (task, slice): gated slices hold gate rows [128 s, 128 s + h) and the matching up rows
// (h = min(128, I - 128 s), N = 2 h); plain slices hold rows [256 s, 256 s + N), N <= 256.  Token
// rows past the task's count load token 0's row again: their D rows are never stored, and rows of
// an MMA are independent.  Every barrier wait is bounded (2 s); on a timeout the
// kernel records KNX_DEV_TIMEOUT in the error word, all roles leave their loops, and the CTA
// releases its tensor memory before returning.
#include "knx_common.cuh"
#include "knx_internal.cuh"
#include "knx_sm100.cuh"

namespace knx {
namespace tcp {

using namespace sm100;

constexpr int TOKM = TC_TASK_TOKENS;      // tokens per task (MMA M = 128)
constexpr int NROWS = 256;                // weight rows per work item (MMA N <= 256)
constexpr int BK = 64;                    // k per stage
constexpr int WROW = BK / 2;              // 32 bytes of nibbles per weight row per stage
constexpr int BOX_ROWS = 64;              // rows per TMA box
constexpr int SW = 4;                     // packed weight stages
constexpr int SB = 2;                     // dequantised weight stages (MMA B operand)
constexpr int SA = 4;                     // activation stages (MMA A operand)
constexpr int SZ_MAX_NG = 24;             // scale groups per weight row on this path
constexpr int EPI_WARP_BYTES = 32 * 128;  // epilogue staging tile per warp: 32 tokens x 64 f16
constexpr int IR = 2;                     // work-item ring slots
constexpr int W_STAGE = NROWS * WROW;     // 8 KB
constexpr int B_STAGE = NROWS * 128;      // 32 KB: 256 rows x 64 f16
constexpr int A_STAGE = TOKM * 128;       // 16 KB: 128 rows x 64 f16
constexpr int D_COLS = 256;               // TMEM columns of one D buffer
constexpr int TMEM_COLS = 2 * D_COLS;
constexpr int DQ_WARPS = 16;
constexpr int EPI_WARPS = 4;
constexpr int WARP_EPI0 = DQ_WARPS;       // warps 16-19 (lane quadrant = warp % 4)
constexpr int A_WARPS = 2;                // activation producer warps
constexpr int WARP_WPROD = DQ_WARPS + EPI_WARPS, WARP_APROD0 = WARP_WPROD + 1;
constexpr int WARP_MMA = WARP_APROD0 + A_WARPS;
constexpr int NUM_WARPS = WARP_MMA + 1;
constexpr int NTHREADS = NUM_WARPS * 32;
constexpr int ITEM_CONSUMERS = DQ_WARPS + EPI_WARPS + A_WARPS + 1;  // + the MMA warp
constexpr int DQ_TPR = DQ_WARPS * 32 / NROWS;  // dequant threads per weight row
constexpr int DQ_WORDS = BK / 8 / DQ_TPR;       // 32-bit nibble words per thread per stage
static_assert(DQ_TPR * NROWS == DQ_WARPS * 32 && (DQ_TPR == 1 || DQ_TPR == 2), "dequant threads");
static_assert(TOKM == 128, "MMA M");
static_assert(WARP_EPI0 % 4 == 0, "epilogue warp e reads TMEM lane quadrant e % 4");

struct Item {
  int valid, e, cnt, slice;
  int slot0, nrows, pad0, pad1;
};

struct Ctrl {
  uint64_t w_full[SW], w_empty[SW];
  uint64_t b_full[SB], b_empty[SB];
  uint64_t a_full[SA], a_empty[SA];
  uint64_t d_full[2], d_empty[2];
  uint64_t i_full[IR], i_empty[IR];
  uint64_t sz_full[IR];  // the item's scale / zero rows have landed (dequant warps)
  uint64_t fin;  // MMA drain before tensor memory is released
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
  int K;                      // contraction length (multiple of 64)
  int rows_per_expert;        // 2I (gated) or N (plain)
  int I;                      // gated: offset of the up rows
  int ng, gs;
  __half* out;                // gated: out2 [slots, I]; plain: [slots, N]
  int64_t out_stride;
  int nslices;
  int32_t* err;
};

// smem layout (from a 1024-aligned base): activation ring, dequantised weight ring, packed ring
// and the scale / zero slots of the item ring: [s of the item's rows][z of the item's rows], f16,
// rows in B-operand order (gated: gate rows, then up rows)
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + SA * A_STAGE;
constexpr int OFF_W = OFF_B + SB * B_STAGE;
constexpr int OFF_SZ = OFF_W + SW * W_STAGE;
KNX_HOST_DEVINL int sz_slot_bytes(int ng) { return 2 * NROWS * ng * 2; }
// ... followed by the epilogue warps' staging tiles
inline size_t smem_bytes(int ng) {
  return 1024 + OFF_SZ + static_cast<size_t>(IR) * sz_slot_bytes(ng) + EPI_WARPS * EPI_WARP_BYTES;
}
// the largest configuration plus the static control block fits one CTA's 227 KB
static_assert(1024 + OFF_SZ + IR * 2 * NROWS * SZ_MAX_NG * 2 + EPI_WARPS * EPI_WARP_BYTES + 2048 <=
                  227 * 1024,
              "shared memory");


// f16x2 of two floats, low half = a
KNX_DEVINL void cp_async16_s(uint32_t saddr, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gmem) : "memory");
}

KNX_DEVINL uint32_t pack_h2(float a, float b) { return h2_as_u32(__floats2half2_rn(a, b)); }

template <bool GATED, bool ZINT>
__global__ void __launch_bounds__(NTHREADS, 1)
    tcp_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const Params p) {
  pdl_wait_trigger();
  extern __shared__ uint8_t dsm_raw[];
  __shared__ Ctrl ctrl;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t a_ring = smem_u32(base + OFF_A);
  const uint32_t b_ring = smem_u32(base + OFF_B);
  uint8_t* w_ring = base + OFF_W;
  uint8_t* sz_ring = base + OFF_SZ;
  const int szb = sz_slot_bytes(p.ng);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nst = p.K / BK;

  if (tid == 0) {
    for (int s = 0; s < SW; ++s) { mbar_init(&ctrl.w_full[s], 1); mbar_init(&ctrl.w_empty[s], DQ_WARPS); }
    for (int s = 0; s < SB; ++s) { mbar_init(&ctrl.b_full[s], DQ_WARPS); mbar_init(&ctrl.b_empty[s], 1); }
    for (int s = 0; s < SA; ++s) { mbar_init(&ctrl.a_full[s], 32 * A_WARPS); mbar_init(&ctrl.a_empty[s], 1); }
    for (int d = 0; d < 2; ++d) { mbar_init(&ctrl.d_full[d], 1); mbar_init(&ctrl.d_empty[d], EPI_WARPS); }
    for (int i = 0; i < IR; ++i) {
      mbar_init(&ctrl.i_full[i], 1);
      mbar_init(&ctrl.sz_full[i], 1);
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
      const int nwork = (p.tasks ? *p.ntasks : (p.dense_rows + TOKM - 1) / TOKM) * p.nslices;
      uint32_t wst = 0;
      for (int n = 0;; ++n) {
        const int slot = n % IR;
        if (!wait(&ctrl.i_empty[slot], ((n / IR) & 1) ^ 1, 64)) break;
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
            it.e = 0; t0 = task * TOKM; it.cnt = min(TOKM, p.dense_rows - t0);
          }
          it.slot0 = (p.offsets ? p.offsets[it.e] : 0) + t0;
          it.nrows = GATED ? 2 * min(NROWS / 2, p.I - it.slice * (NROWS / 2))
                           : min(NROWS, p.rows_per_expert - it.slice * NROWS);
          it.valid = 1;
        }
        ctrl.items[slot] = it;
        mbar_arrive(&ctrl.i_full[slot]);
        if (!it.valid) break;
        const int64_t erow = static_cast<int64_t>(it.e) * p.rows_per_expert;
        const int half = it.nrows >> 1;
        // scale / zero rows of the item -> its slot (1-D bulk copies; rows are whole 64-row
        // boxes, so every offset and size is a multiple of 128 bytes)
        {
          uint8_t* szs = sz_ring + slot * szb;
          const uint32_t zoff = static_cast<uint32_t>(it.nrows) * p.ng * 2;
          mbar_arrive_expect_tx(&ctrl.sz_full[slot], 2 * zoff);
          if (GATED) {
            const int64_t g0 = (erow + it.slice * (NROWS / 2)) * p.ng;
            const int64_t u0 = g0 + static_cast<int64_t>(p.I) * p.ng;
            const uint32_t b = static_cast<uint32_t>(half) * p.ng * 2;
            bulk_load(szs, p.ws + g0, b, &ctrl.sz_full[slot]);
            bulk_load(szs + b, p.ws + u0, b, &ctrl.sz_full[slot]);
            bulk_load(szs + zoff, p.wz + g0, b, &ctrl.sz_full[slot]);
            bulk_load(szs + zoff + b, p.wz + u0, b, &ctrl.sz_full[slot]);
          } else {
            const int64_t r0 = (erow + it.slice * NROWS) * p.ng;
            bulk_load(szs, p.ws + r0, zoff, &ctrl.sz_full[slot]);
            bulk_load(szs + zoff, p.wz + r0, zoff, &ctrl.sz_full[slot]);
          }
        }
        // packed weights: one stage = 64 k of the slice's rows, in boxes of 64 rows
        for (int st = 0; st < nst; ++st, ++wst) {
          const int s = wst % SW;
          if (!wait(&ctrl.w_empty[s], ((wst / SW) & 1) ^ 1)) break;
          uint8_t* dst = w_ring + s * W_STAGE;
          mbar_arrive_expect_tx(&ctrl.w_full[s], static_cast<uint32_t>(it.nrows) * WROW);
          const int x = st * WROW;
          if (GATED) {
            const int g0 = static_cast<int>(erow) + it.slice * (NROWS / 2);
            for (int b = 0; b < half; b += BOX_ROWS) {
              tma_load_2d(dst + b * WROW, &wmap, &ctrl.w_full[s], x, g0 + b);
              tma_load_2d(dst + (half + b) * WROW, &wmap, &ctrl.w_full[s], x, g0 + p.I + b);
            }
          } else {
            const int r0 = static_cast<int>(erow) + it.slice * NROWS;
            for (int b = 0; b < it.nrows; b += BOX_ROWS)
              tma_load_2d(dst + b * WROW, &wmap, &ctrl.w_full[s], x, r0 + b);
          }
        }
        if (*abort_flag) break;
      }
    }
    __syncwarp();
  } else if (warp >= WARP_APROD0 && warp < WARP_APROD0 + A_WARPS) {
    // ---------------------------------------------------------------- activation gather
    // A_WARPS warps split the 128 token rows; lane l of warp a copies 16-byte chunk (l % 8) of
    // rows 4 i + l / 8 for the warp's row groups i, straight into the swizzled K-major layout:
    // row t, chunk j -> (t / 8) * 1024 + (t % 8) * 128 + ((j ^ t % 8) * 16).  The lane's source
    // pointers are set once per item and advance by one stage each stage; rows past the task's
    // count copy token 0's row (their D rows are never stored).
    constexpr int AI = TOKM / 4 / A_WARPS;  // row groups (of four rows) per warp
    constexpr int AJ = TOKM / 32 / A_WARPS; // activation rows held per lane
    static_assert(AJ >= 1 && AI == 8 * AJ, "producer row mapping");
    const int aw = warp - WARP_APROD0;
    uint32_t ast = 0;
    const int rsub = lane >> 3, ch = lane & 7;
    // shared-memory offset of this lane's chunk of row group i (same for every stage)
    uint32_t doff[AI];
#pragma unroll
    for (int i = 0; i < AI; ++i) {
      const int t = 4 * (aw * AI + i) + rsub;
      doff[i] = (t >> 3) * 1024 + (t & 7) * 128 + ((ch ^ (t & 7)) << 4);
    }
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      if (!wait(&ctrl.i_full[slot], (n / IR) & 1, 64)) break;
      const Item it = ctrl.items[slot];
      if (!it.valid) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      // activation row of tokens 32 (aw * AJ + j) + lane
      int arow[AJ];
#pragma unroll
      for (int j = 0; j < AJ; ++j) {
        const int t = 32 * (aw * AJ + j) + lane;
        const int tt = t < it.cnt ? t : 0;
        arow[j] = p.sorted_pair ? p.sorted_pair[it.slot0 + tt] / p.topk : it.slot0 + tt;
      }
      const __half* src[AI];
#pragma unroll
      for (int i = 0; i < AI; ++i) {
        const int t = 4 * (aw * AI + i) + rsub;
        const int r = __shfl_sync(0xffffffffu, arow[i >> 3], t & 31);
        src[i] = p.act + static_cast<int64_t>(r) * p.act_stride + ch * 8;
      }
      bool ok = true;
      for (int st = 0; st < nst; ++st, ++ast) {
        const int s = ast % SA;
        if (!wait(&ctrl.a_empty[s], ((ast / SA) & 1) ^ 1, 32)) {
          ok = false;
          break;
        }
        const uint32_t dst = a_ring + s * A_STAGE;
#pragma unroll
        for (int i = 0; i < AI; ++i) {
          cp_async16_s(dst + doff[i], src[i]);
          src[i] += BK;
        }
        cp_async_mbar_arrive_noinc(&ctrl.a_full[s]);
      }
      __syncwarp();
      if (!ok) break;
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
  } else if (warp < DQ_WARPS) {
    // ---------------------------------------------------------------- dequant -> B ring
    const int row = tid / DQ_TPR, kh = tid % DQ_TPR;  // weight row of the item, part of the stage's k
    const int sw = row & 7;
    const int gstages = p.gs / BK;           // stages per scale group
    uint32_t wst = 0, bst = 0;
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      if (!wait(&ctrl.i_full[slot], (n / IR) & 1, 64)) break;
      const Item it = ctrl.items[slot];
      if (!it.valid) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      const bool row_ok = row < it.nrows;
      // this row's scale / zero in the item's slot (rows in B order)
      const uint32_t srow = smem_u32(sz_ring + slot * szb) + row * p.ng * 2;
      const uint32_t zrow = srow + it.nrows * p.ng * 2;
      if (!wait(&ctrl.sz_full[slot], (n / IR) & 1, 64)) break;
      __half2 s2 = __half2half2(__ushort_as_half(0)), s16 = s2, cc = s2, c16 = s2;
      const uint32_t wrow = smem_u32(w_ring) + row * WROW + kh * (WROW / DQ_TPR);
      const uint32_t brow = b_ring + (row >> 3) * 1024 + (row & 7) * 128;
      bool ok = true;
      int g = 0, gleft = 0;
      for (int st = 0; st < nst; ++st, ++wst, ++bst) {
        const int ws_ = wst % SW, bs = bst % SB;
        if (!wait(&ctrl.w_full[ws_], (wst / SW) & 1) ||
            !wait(&ctrl.b_empty[bs], ((bst / SB) & 1) ^ 1)) {
          ok = false;
          break;
        }
        uint4 u[DQ_WORDS / 4];
#pragma unroll
        for (int j = 0; j < DQ_WORDS / 4; ++j) u[j] = make_uint4(0u, 0u, 0u, 0u);
        if (row_ok) {
          if (gleft == 0) {  // first stage of a scale group
            const uint2 c = make_sz<ZINT>(lds16h(srow + 2 * g), lds16h(zrow + 2 * g));
            s2 = __low2half2(u32_as_h2(c.x)); cc = __high2half2(u32_as_h2(c.x));
            s16 = __low2half2(u32_as_h2(c.y)); c16 = __high2half2(u32_as_h2(c.y));
            ++g;
            gleft = gstages;
          }
          --gleft;
#pragma unroll
          for (int j = 0; j < DQ_WORDS / 4; ++j) u[j] = lds128(wrow + ws_ * W_STAGE + 16 * j);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.w_empty[ws_]);  // packed stage consumed
        if (row_ok) {
          const uint32_t dst = brow + bs * B_STAGE;
#pragma unroll
          for (int j = 0; j < DQ_WORDS / 4; ++j) {
            const uint32_t uu[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t w4[4];
              dequant8<ZINT>(uu[i], s2, s16, cc, c16, w4);
              const int chunk = kh * DQ_WORDS + 4 * j + i;  // 16-byte chunk (8 k) of the row
              sts128(dst + ((chunk ^ sw) << 4), w4[0], w4[1], w4[2], w4[3]);
            }
          }
        }
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.b_full[bs]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
  } else if (warp == WARP_MMA) {
    // ---------------------------------------------------------------- tcgen05.mma issue
    if (lane == 0) {
      uint32_t ast = 0, bst = 0, dc = 0;
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
        const uint32_t idesc = idesc_f16_f32(TOKM, it.nrows);
        const uint32_t d_tmem = tmem + db * D_COLS;
        bool ok = true;
        for (int st = 0; st < nst; ++st, ++ast, ++bst) {
          const int s = ast % SA, bs = bst % SB;
          if (!wait(&ctrl.a_full[s], (ast / SA) & 1) || !wait(&ctrl.b_full[bs], (bst / SB) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fence_proxy_async_smem();
          const uint32_t a_base = a_ring + s * A_STAGE, b_base = b_ring + bs * B_STAGE;
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            mma_f16_ss(d_tmem, smem_desc_sw128_kmajor(a_base + 32 * j),
                       smem_desc_sw128_kmajor(b_base + 32 * j), idesc, (st | j) != 0);
          mma_commit(&ctrl.a_empty[s]);
          mma_commit(&ctrl.b_empty[bs]);
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
  } else if (warp >= WARP_EPI0 && warp < WARP_EPI0 + EPI_WARPS) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const uint32_t lane_addr = (32u * q) << 16;
    const uint32_t stg = smem_u32(sz_ring + IR * szb) + q * EPI_WARP_BYTES;  // this warp's tile
    uint32_t dc = 0;
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      if (!wait(&ctrl.i_full[slot], (n / IR) & 1, 256)) break;
      const Item it = ctrl.items[slot];
      if (!it.valid) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      const int db = dc & 1;
      if (!wait(&ctrl.d_full[db], (dc >> 1) & 1, 128)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + lane_addr + db * D_COLS;
      // Output columns in blocks of 64: each thread (token) packs its 64 f16 into the warp's
      // 4 KB staging tile (row = token, 128-byte rows, 16-byte chunks XOR-swizzled by row), then
      // the warp stores the tile row-wise, four rows of 128 bytes per instruction.
      const int ncols = GATED ? (it.nrows >> 1) : it.nrows;
      const int colbase = GATED ? it.slice * (NROWS / 2) : it.slice * NROWS;
      const uint32_t srow = stg + lane * 128;
#pragma unroll 1
      for (int cb = 0; cb < ncols; cb += 64) {
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const int c = cb + 16 * sub;
          uint32_t w[8];
          if (GATED) {
            // gate column c, up column c + h; out2 channel 128 s + c, written in the
            // K-interleaved order the down GEMM reads: in each 8-group [c0, c4, c1, c5, c2, c6, c3, c7]
            uint32_t gv[16], uv[16];
            tmem_ld16(d_tmem + c, gv);
            tmem_ld16(d_tmem + ncols + c, uv);
            tmem_wait_ld();
            float r[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              r[i] = gelu_tanh(__uint_as_float(gv[i])) * __uint_as_float(uv[i]);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int i = 0; i < 4; ++i) w[4 * h + i] = pack_h2(r[8 * h + i], r[8 * h + i + 4]);
          } else {
            uint32_t v[16];
            tmem_ld16(d_tmem + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = pack_h2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          }
          sts128(srow + (((2 * sub) ^ (lane & 7)) << 4), w[0], w[1], w[2], w[3]);
          sts128(srow + (((2 * sub + 1) ^ (lane & 7)) << 4), w[4], w[5], w[6], w[7]);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + (lane >> 3), cc = lane & 7;
          const uint4 v = lds128(stg + rr * 128 + ((cc ^ (rr & 7)) << 4));
          const int t = 32 * q + rr;
          if (t < it.cnt)
            *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(it.slot0 + t) * p.out_stride +
                                      colbase + cb + 8 * cc) = v;
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ctrl.d_empty[db]);
        mbar_arrive(&ctrl.i_empty[slot]);
      }
      ++dc;
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

}  // namespace tcp

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

// packed weights [total_rows, row_bytes] u8; box = 32 bytes (64 k) x 64 rows, no swizzle
bool encode_weight_map(CUtensorMap* map, const uint8_t* q, int64_t total_rows, int64_t row_bytes) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(total_rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(tcp::WROW), static_cast<cuuint32_t>(tcp::BOX_ROWS)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(
      map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool GATED, bool ZINT>
int launch_tcp(const tcp::Params& p, const uint8_t* wq, int64_t total_rows, int64_t row_bytes,
               int64_t work_bound, cudaStream_t s) {
  // the scale / zero bulk copies need 16-byte aligned bases
  if ((reinterpret_cast<uintptr_t>(p.ws) & 15) || (reinterpret_cast<uintptr_t>(p.wz) & 15))
    return KNX_E_ALIGN;
  if (set_max_dyn_smem(reinterpret_cast<const void*>(tcp::tcp_gemm_kernel<GATED, ZINT>),
                       static_cast<int>(tcp::smem_bytes(tcp::SZ_MAX_NG))) != KNX_OK)
    return KNX_E_DEVICE;
  CUtensorMap map;
  if (!encode_weight_map(&map, wq, total_rows, row_bytes)) return KNX_E_DEVICE;
  const int sms = num_sms();
  const int grid = static_cast<int>(work_bound < sms ? (work_bound > 0 ? work_bound : 1) : sms);
  (void)launch_pdl(tcp::tcp_gemm_kernel<GATED, ZINT>, grid, tcp::NTHREADS, tcp::smem_bytes(p.ng), s,
                   map, p);
  return launch_status();
}

}  // namespace

// K a multiple of the stage, scale groups whole stages and at most SZ_MAX_NG of them (the item's
// scale / zero rows sit in shared memory), weight rows whole TMA boxes; the row
// indices of the tensor map (expert * rows + row) stay below 2^31.
bool tc_supported(int64_t K, int gs, int ng, int64_t rows_per_expert, bool gated) {
  if (K % tcp::BK != 0 || gs % tcp::BK != 0 || ng < 1 || ng > tcp::SZ_MAX_NG ||
      static_cast<int64_t>(ng) * gs != K)
    return false;
  if (gated) return (rows_per_expert / 2) % tcp::BOX_ROWS == 0 && rows_per_expert % 2 == 0;
  return rows_per_expert % tcp::BOX_ROWS == 0;
}

int launch_tc_gateup(const __half* xp, const int32_t* sorted_pair, int topk, const int32_t* offsets,
                     const int4* tasks, const int32_t* ntasks, int* counter, const uint8_t* gu_q,
                     const __half* gu_s, const __half* gu_z, int E, int H, int I, int ng, int gs,
                     bool zint, __half* out2, int64_t max_tasks, int32_t* err, cudaStream_t s) {
  if (static_cast<int64_t>(E) * 2 * I >= (int64_t(1) << 31)) return KNX_E_UNSUPPORTED;
  tcp::Params p{};
  p.act = xp; p.act_stride = H; p.sorted_pair = sorted_pair; p.topk = topk; p.offsets = offsets;
  p.tasks = tasks; p.ntasks = ntasks; p.work_counter = counter; p.ws = gu_s; p.wz = gu_z;
  p.K = H; p.rows_per_expert = 2 * I; p.I = I; p.ng = ng; p.gs = gs; p.out = out2;
  p.out_stride = I; p.nslices = (I + tcp::NROWS / 2 - 1) / (tcp::NROWS / 2); p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_tcp<true, true>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s)
              : launch_tcp<true, false>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s);
}

int launch_tc_rows(const __half* act, int64_t act_stride, int K, const int32_t* offsets,
                   const int4* tasks, const int32_t* ntasks, int dense_rows, int* counter,
                   const uint8_t* wq, const __half* ws, const __half* wz, int E, int N, int ng,
                   int gs, bool zint, __half* out, int64_t out_stride, int64_t max_tasks,
                   int32_t* err, cudaStream_t s) {
  if (static_cast<int64_t>(E) * N >= (int64_t(1) << 31)) return KNX_E_UNSUPPORTED;
  tcp::Params p{};
  p.act = act; p.act_stride = act_stride; p.offsets = offsets; p.tasks = tasks; p.ntasks = ntasks;
  p.dense_rows = dense_rows; p.work_counter = counter; p.ws = ws; p.wz = wz; p.K = K;
  p.rows_per_expert = N; p.ng = ng; p.gs = gs; p.out = out; p.out_stride = out_stride;
  p.nslices = (N + tcp::NROWS - 1) / tcp::NROWS; p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_tcp<false, true>(p, wq, int64_t(E) * N, K / 2, work, s)
              : launch_tcp<false, false>(p, wq, int64_t(E) * N, K / 2, work, s);
}

}  // namespace knx
