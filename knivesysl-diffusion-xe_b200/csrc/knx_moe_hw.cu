// knx_moe_hw.cu — warp-specialised grouped W4A16 GEMMs on the warp-level tensor-core path
// (mma.sync m16n8k16) for the small-token regime (<= 32 tokens per task).
//
// Why this shape (measured on B200): a tcgen05 M128 x K16 instruction costs ~108 ns whatever N
// is, which caps a weights-as-M tcgen05 GEMM at ~1.4 TB/s of nibbles when N (tokens) is small,
// while mma.sync has no such floor; and HBM only streams at full rate with >= ~128 KB of loads
// in flight per SM.  So:
//   * one persistent CTA per SM; a work item is (task of <= 32 tokens of one expert, slice of 256
//     weight rows) — gated: 128 gate rows + the matching 128 up rows;
//   * warp 16 (scheduler + weights): per item the slice's scale/zero rows by 1-D bulk copies, then
//     the packed nibbles by 2-D TMA (128-byte swizzle) in 32 KB stages (256 rows x 256 k) into a
//     ring of up to 4 stages (128 KB in flight);
//   * warp 17 (activations): per stage, one 1-D bulk copy per token of 256 k (512 B) gathered
//     by token id into a ring of 2-4 stages (rows padded to 576 B: conflict-free fragment loads);
//   * warps 0-15 (math): warp w owns one m16 row tile — gated: gate rows 8w..8w+7 on tile rows
//     0-7 and the matching up rows on tile rows 8-15, so each lane ends with gate and up of one
//     intermediate column; plain: rows 16w..16w+15 — over the full K.  Nibbles are dequantised in
//     registers into A fragments (dequant8: bit-identical to dequant_w4 for integer zero-points,
//     the reference kernel's f16 arithmetic otherwise) and multiplied with the B fragments of
//     the task's 1-4 n8 token tiles, so one dequantisation serves up to 32 tokens.  No split-K:
//     every output is one warp's fixed-order sum (deterministic), and a token's sum does not
//     depend on the other tokens of its task.
//   * GELU(gate) * up (gated) or the plain result: each warp stages its own 8 (gated) or 16
//     output columns per token in a private shared area and writes 16-byte chunks, so the math
//     warps never wait for one another; the gated output is written in the K-interleave the
//     down GEMM reads.
//   * gate_up -> down by task: gate_up's weight producer counts each finished item of a task
//     (after every math warp has released the slot, one GPU-scope fence), and the down kernel,
//     which does not wait for gate_up to finish, gathers a task's rows once its count is
//     complete.  Down's CTAs thus run on the SMs that gate_up's last items leave idle.
// All waits are bounded (2 s): on a timeout the kernel sets KNX_DEV_TIMEOUT and every role
// leaves at the next work-item boundary (each math warp decides by a warp vote); the producers
// wait (bounded) for their copies in flight before the CTA exits.
#include "knx_common.cuh"
#include "knx_internal.cuh"
#include "knx_sm100.cuh"

namespace knx {
namespace hw {

using namespace sm100;

constexpr int TOK = HW_TASK_TOKENS;      // tokens per task (32)
constexpr int NT = TOK / 8;              // n8 tiles per task
constexpr int BK = 256;                  // k per stage
constexpr int WROW = BK / 2;             // 128 bytes of nibbles per row per stage
constexpr int ROWS = 256;                // weight rows per item
constexpr int GROWS = ROWS / 2;          // gated: gate rows per item
constexpr int BOX_ROWS = 128;            // rows per TMA box
constexpr int SW_MAX = 4, SA_MAX = 4, IR = 2;
constexpr int W_STAGE = ROWS * WROW;     // 32 KB
constexpr int AROW = BK * 2 + 64;        // 576 B per token row per stage
constexpr int A_STAGE = TOK * AROW;      // 18 KB
constexpr int MATH_WARPS = 16;
constexpr int NUM_WARPS = MATH_WARPS + 2;
constexpr int NTHREADS = NUM_WARPS * 32;
constexpr int WARP_WPROD = MATH_WARPS, WARP_APROD = MATH_WARPS + 1;
constexpr int SZ_MAX = 32;               // groups per row
// per-warp output staging: 8 (gated) or 16 (plain) columns x 32 tokens of f16 per warp
constexpr int ot_bytes(bool gated) { return MATH_WARPS * TOK * (gated ? 8 : 16) * 2; }
constexpr size_t SMEM_LIMIT = 232448;    // 227 KB opt-in per block
constexpr size_t STATIC_RESERVE = 1024;  // Ctrl + alignment of the dynamic base

static_assert(NT == 4, "the math loop is written for 32-token tasks");
// Accumulator sets per n8 tile (1, 2 or 4).  One set: 18 warps put 5 on two SM sub-partitions,
// which caps a thread at 96 registers, and 4 token tiles x 2 sets spill there.
#ifndef KNX_HW_NACC
#define KNX_HW_NACC 1
#endif
constexpr int NACC = KNX_HW_NACC;
// The producers run stages ahead of the math warps and share their SM sub-partitions (warp 16
// with warps 0/4/8/12, warp 17 with 1/5/9/13): they back off between polls of their "empty"
// barriers instead of spinning, which would take issue slots from those math warps.
#ifndef KNX_HW_PROD_BACKOFF
#define KNX_HW_PROD_BACKOFF 256
#endif
constexpr uint32_t PROD_BACKOFF_NS = KNX_HW_PROD_BACKOFF;

struct Item {
  int valid, e, cnt, slice;
  int slot0, nvalid, task, pad;
};

struct Ctrl {
  uint64_t w_full[SW_MAX], w_empty[SW_MAX];
  uint64_t a_full[SA_MAX], a_empty[SA_MAX];
  uint64_t i_full[IR], i_empty[IR];
  Item items[IR];
  int abort;
};

struct Params {
  const __half* act;
  int64_t act_stride;
  const int32_t* sorted_pair;
  int topk;
  const int4* tasks;
  const int32_t* ntasks;
  int dense_rows;
  int* work_counter;
  const __half* ws;
  const __half* wz;
  int K, rows_per_expert, I, ng, gs;
  __half* out;
  int64_t out_stride;
  int nslices;
  int partial_last;  // the last slice has fewer valid rows than the others (scheduled last)
  int sw;  // weight ring depth (stages)
  int sa;  // activation ring depth (stages)
  int32_t* err;
  // Task readiness between the two GEMMs of a layer.  task_done (gated kernel only): incremented
  // once per finished item of a task, after all its output rows are written, and *items_done
  // once per finished item.  task_ready (plain kernel only; NULL = wait for the previous kernel):
  // a task's rows are gathered once task_ready[task] reaches ready_target (items per task), or
  // at once after *items_done has reached ready_target * tasks; the kernel then starts without
  // waiting for the previous kernel to finish.
  int* task_done;
  const int* task_ready;
  int* items_done;
  int ready_target;
};

KNX_HOST_DEVINL size_t sz_slot_bytes(int ng) { return static_cast<size_t>(ROWS) * ng * 4; }
inline size_t smem_bytes(bool gated, int ng, int sw, int sa) {
  return 1024 + static_cast<size_t>(sw) * W_STAGE + static_cast<size_t>(sa) * A_STAGE +
         ot_bytes(gated) + IR * sz_slot_bytes(ng);
}
// Ring depths that fit, in order of preference: at least 3 activation stages (their copies come
// from L2 but each is gathered token by token), then the deepest weight ring (it streams from
// HBM; 4 stages = 128 KB in flight).  Measured on the configs[1] gate_up: 3 + 3 beats 4 + 2.
inline bool ring_depths(bool gated, int ng, int& sw, int& sa) {
  static const int pref[][2] = {{4, 4}, {4, 3}, {3, 4}, {3, 3}, {4, 2}, {3, 2}, {2, 4}, {2, 3}, {2, 2}};
  for (const auto& c : pref) {
    sw = c[0];
    sa = c[1];
    if (smem_bytes(gated, ng, sw, sa) + STATIC_RESERVE <= SMEM_LIMIT) return true;
  }
  sw = sa = 0;
  return false;
}


// Dequant constants of one (row, group) as f16x2 broadcasts; the same values as make_sz (every
// operation below is exact or a single rounding of the exact result).
template <bool ZINT>
KNX_DEVINL void group_consts(__half s, __half z, __half2& s2, __half2& s16, __half2& c2,
                             __half2& c16) {
  // broadcast first, then one f16x2 operation per constant (each lane: the same single rounding)
  const __half2 k16 = __half2half2(__ushort_as_half(0x4c00u));
  const __half2 k1024 = __half2half2(__ushort_as_half(0x6400u));
  s2 = __half2half2(s);
  s16 = __hmul2(s2, __half2half2(__ushort_as_half(0x2c00u)));  // s / 16
  const __half2 z2 = __half2half2(z);
  c2 = ZINT ? __hadd2(z2, k1024) : z2;
  c16 = ZINT ? __hfma2(z2, k16, k1024) : __hmul2(z2, k16);
}

// One stage (256 k) of one warp's m16 tile: 8 k32 steps (jmax in the K tail), NTT n8 token
// tiles.  Scale-group boundaries are compile-time (GPJ k32 steps per group; GPJ = 8 also serves
// groups that span several stages): the steps of one group are unrolled, the groups are a loop
// (unrolling across groups lets the scheduler keep more steps in flight than 112 registers
// hold at 4 token tiles).
// wa: shared address of the lane's word of fragment row A in chunk 0 with the row's swizzle
// applied (stage base + row * 128 + (g << 4) + 4q): chunk j of the row is at wa ^ (j << 4).
// Fragment row B lies BOFF bytes further (same swizzle phase).
template <bool ZINT, int NTT, int GPJ, bool TAIL, int BOFF>
KNX_DEVINL void mma_stage(uint32_t wa, uint32_t ab, int jmax, int grp0,
                          uint32_t sA, uint32_t zA, uint32_t sB, uint32_t zB,
                          float (&acc)[NT][NACC][4]) {
  constexpr int UJ = NACC >= 2 ? NACC / 2 : 1;
  static_assert(GPJ % UJ == 0 || UJ == 1, "accumulator sets must repeat within a group");
#pragma unroll 1
  for (int j0 = 0; j0 < 8; j0 += GPJ) {
    if (TAIL && j0 >= jmax) break;
    __half2 sa2, sa16, ca2, ca16, sb2, sb16, cb2, cb16;
    const int grp = grp0 + j0 / GPJ;
    group_consts<ZINT>(lds16h(sA + 2 * grp), lds16h(zA + 2 * grp), sa2, sa16, ca2, ca16);
    group_consts<ZINT>(lds16h(sB + 2 * grp), lds16h(zB + 2 * grp), sb2, sb16, cb2, cb16);
#pragma unroll
    for (int jj = 0; jj < GPJ; ++jj) {
      const int j = j0 + jj;
      if (!TAIL || j < jmax) {
        const uint32_t aj = wa ^ static_cast<uint32_t>(j << 4);
        uint32_t fa[4], fb[4];
        dequant8<ZINT>(lds32(aj), sa2, sa16, ca2, ca16, fa);
        dequant8<ZINT>(lds32_at<BOFF>(aj), sb2, sb16, cb2, cb16, fb);
#pragma unroll
        for (int t = 0; t < NTT; ++t) {
          const uint4 b = lds128(ab + t * 8 * AROW + j * 64);
          // k16 halves into sets 2 * (jj % UJ) and +1 (NACC >= 2), both into set 0 (NACC 1)
          constexpr int S0 = NACC >= 2 ? 2 : 0, H1 = NACC >= 2 ? 1 : 0;
          mma_16816(acc[t][S0 * (jj % UJ)], fa[0], fb[0], fa[1], fb[1], b.x, b.y);
          mma_16816(acc[t][S0 * (jj % UJ) + H1], fa[2], fb[2], fa[3], fb[3], b.z, b.w);
        }
      }
    }
  }
}

template <bool GATED, bool ZINT, int GPJ>
__global__ void __launch_bounds__(NTHREADS, 1)
    hw_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const Params p) {
  // With per-task readiness the kernel runs alongside the tail of the previous one (its CTAs take
  // the SMs that kernel's CTAs leave): the activation rows are read only after their task's
  // count is complete, and the task list and counters were written before the previous kernel
  // started (they are read from L2 below).
  if (!GATED && p.task_ready) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  else pdl_wait_trigger();
  extern __shared__ uint8_t dsm_raw[];
  __shared__ Ctrl ctrl;
  // 1024-byte aligned base (the 128-byte swizzle needs it), by an offset from dsm_raw so that the
  // pointers derived from it stay recognisably shared
  uint8_t* base = dsm_raw + ((1024u - (smem_u32(dsm_raw) & 1023u)) & 1023u);
  const int sw = p.sw, sa = p.sa;
  uint8_t* w_ring = base;
  uint8_t* a_ring = base + sw * W_STAGE;
  const uint32_t ot = smem_u32(a_ring + sa * A_STAGE);  // output tile (shared address)
  uint8_t* sz_ring = a_ring + sa * A_STAGE + ot_bytes(GATED);
  const size_t szr = sz_slot_bytes(p.ng);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nst = (p.K + BK - 1) / BK;

  if (tid == 0) {
    for (int s = 0; s < sw; ++s) { mbar_init(&ctrl.w_full[s], 1); mbar_init(&ctrl.w_empty[s], MATH_WARPS); }
    for (int s = 0; s < sa; ++s) { mbar_init(&ctrl.a_full[s], 1); mbar_init(&ctrl.a_empty[s], MATH_WARPS); }
    for (int i = 0; i < IR; ++i) {
      mbar_init(&ctrl.i_full[i], 1);
      mbar_init(&ctrl.i_empty[i], MATH_WARPS + 1);
    }
    ctrl.abort = 0;
    fence_mbar_init();
  }
  if (warp == WARP_WPROD && lane == 0) prefetch_tensormap(&wmap);
  __syncthreads();
  volatile int* abort_flag = &ctrl.abort;
  auto wait = [&](uint64_t* bar, uint32_t parity, uint32_t backoff_ns = 0) -> bool {
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity, 2000000000ull, backoff_ns)) {
      *abort_flag = 1;
      if (p.err) atomicOr(p.err, KNX_DEV_TIMEOUT);
      return false;
    }
    return true;
  };

  if (warp == WARP_WPROD) {
    // ---------------------------------------------------------------- scheduler + weights
    if (lane == 0) {
      // the packed weights stream through once per task: evict them first, so that the
      // intermediates (out2 for the down GEMM, out3 for the combine) stay in L2
      const uint64_t wpol = l2_policy_evict_first();
      // the plain kernel may start before the previous kernel has finished (task_ready): its
      // task list is read from L2
      const int ntasks = p.tasks ? (GATED ? *p.ntasks : __ldcg(p.ntasks)) : 0;
      const int nwork = (p.tasks ? ntasks : (p.dense_rows + TOK - 1) / TOK) * p.nslices;
      uint32_t wst = 0;            // stages issued
      uint32_t wsl = 0, wph = 0;   // next ring slot and its phase parity
      int last_on_slot[IR];  // newest item per slot whose scale/zero copies were issued (-1: none)
      for (int i = 0; i < IR; ++i) last_on_slot[i] = -1;
      // gated kernel with task readiness: an item is counted once its slot's i_empty phase has
      // completed, i.e. every math warp has written its rows and arrived (release at CTA scope);
      // that wait acquires, and the GPU-scope fence here orders all those rows before the counts.
      // The producer, not a math warp, pays for the fence, after it has issued the next item's
      // first weight stage.
      auto count_done = [&](int task) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        fence_proxy_async_global();
        atomicAdd(p.task_done + task, 1);
        atomicAdd(p.items_done, 1);
      };
      for (int n = 0;; ++n) {
        const int slot = n % IR;
        if (!wait(&ctrl.i_empty[slot], ((n / IR) & 1) ^ 1, PROD_BACKOFF_NS)) break;
        // the item that last used this slot (n - IR), now finished, is counted below
        int done_task =
            (GATED && p.task_done && last_on_slot[slot] >= 0) ? ctrl.items[slot].task : -1;
        const int wi = atomicAdd(p.work_counter, 1);
        Item it{};
        if (wi < nwork) {
          // items of full slices first (task-major: a task's slices run together and share its
          // activations in L2), then the half-filled last slices of every task (gate_up with
          // I % 128 != 0), which are the cheapest items and so fill the tail of the grid
          const int nfull_sl = p.partial_last ? p.nslices - 1 : p.nslices;
          const int ntask = nwork / p.nslices;
          int task;
          if (wi < ntask * nfull_sl) {
            task = wi / nfull_sl;
            it.slice = wi - task * nfull_sl;
          } else {
            task = wi - ntask * nfull_sl;
            it.slice = nfull_sl;
          }
          if (p.tasks) {
            // (expert, first token, tokens, first slot)
            const int4 tk = GATED ? p.tasks[task] : __ldcg(p.tasks + task);
            it.e = tk.x; it.cnt = tk.z; it.slot0 = tk.w;
          } else {
            it.e = 0; it.slot0 = task * TOK; it.cnt = min(TOK, p.dense_rows - it.slot0);
          }
          it.task = task;
          it.nvalid = GATED ? min(GROWS, p.I - it.slice * GROWS)
                            : min(ROWS, p.rows_per_expert - it.slice * ROWS);
          it.valid = 1;
        }
        ctrl.items[slot] = it;
        if (!it.valid) {
          last_on_slot[slot] = -1;
          mbar_arrive(&ctrl.i_full[slot]);
          if (GATED && done_task >= 0) count_done(done_task);
          break;
        }
        last_on_slot[slot] = n;
        uint8_t* szs = sz_ring + slot * szr;
        const int ng = p.ng;
        // scale/zero rows (16-byte multiples): gated [s_gate | z_gate | s_up | z_up] regions of
        // 128 rows each, plain [s | z] regions of 256 rows each
        const uint32_t b = static_cast<uint32_t>(it.nvalid) * ng * 2u;
        if (GATED) {
          const int64_t g0 = (static_cast<int64_t>(it.e) * p.rows_per_expert + it.slice * GROWS) * ng;
          const int64_t u0 = g0 + static_cast<int64_t>(p.I) * ng;
          const uint32_t reg = GROWS * ng * 2u;
          mbar_arrive_expect_tx(&ctrl.i_full[slot], 4 * b);
          bulk_load(szs + 0 * reg, p.ws + g0, b, &ctrl.i_full[slot]);
          bulk_load(szs + 1 * reg, p.wz + g0, b, &ctrl.i_full[slot]);
          bulk_load(szs + 2 * reg, p.ws + u0, b, &ctrl.i_full[slot]);
          bulk_load(szs + 3 * reg, p.wz + u0, b, &ctrl.i_full[slot]);
        } else {
          const int64_t r0 = (static_cast<int64_t>(it.e) * p.rows_per_expert + it.slice * ROWS) * ng;
          const uint32_t reg = ROWS * ng * 2u;
          mbar_arrive_expect_tx(&ctrl.i_full[slot], 2 * b);
          bulk_load(szs, p.ws + r0, b, &ctrl.i_full[slot]);
          bulk_load(szs + reg, p.wz + r0, b, &ctrl.i_full[slot]);
        }
        for (int st = 0; st < nst; ++st, ++wst) {
          const int s = static_cast<int>(wsl);
          if (!wait(&ctrl.w_empty[s], wph ^ 1u, PROD_BACKOFF_NS)) break;
          if (++wsl == static_cast<uint32_t>(sw)) { wsl = 0; wph ^= 1u; }
          uint8_t* dst = w_ring + s * W_STAGE;
          mbar_arrive_expect_tx(&ctrl.w_full[s], W_STAGE);
          const int x = st * WROW;
          if (GATED) {
            const int y = it.e * p.rows_per_expert + it.slice * GROWS;
            tma_load_2d_hint(dst, &wmap, &ctrl.w_full[s], x, y, wpol);
            tma_load_2d_hint(dst + BOX_ROWS * WROW, &wmap, &ctrl.w_full[s], x, y + p.I, wpol);
          } else {
            const int y = it.e * p.rows_per_expert + it.slice * ROWS;
            tma_load_2d_hint(dst, &wmap, &ctrl.w_full[s], x, y, wpol);
            tma_load_2d_hint(dst + BOX_ROWS * WROW, &wmap, &ctrl.w_full[s], x, y + BOX_ROWS, wpol);
          }
          if (GATED && done_task >= 0) {
            count_done(done_task);
            done_task = -1;
          }
        }
        if (GATED && done_task >= 0) count_done(done_task);  // the stage loop gave up
        if (*abort_flag) break;
      }
      // the valid items posted after the last one counted above (the others were counted when
      // their slot was reused)
      if (GATED && p.task_done && !*abort_flag) {
        for (int i = 0; i < IR; ++i) {
          const int m = last_on_slot[i];
          if (m >= 0 && wait(&ctrl.i_empty[i], (m / IR) & 1, PROD_BACKOFF_NS))
            count_done(ctrl.items[i].task);
        }
      }
      // Copies already issued must land before the CTA exits (only pending after an abort): the
      // newest phase of every weight stage and of every item slot is waited for, bounded.
      for (uint32_t x = wst > static_cast<uint32_t>(sw) ? wst - sw : 0; x < wst; ++x)
        mbar_wait(&ctrl.w_full[x % sw], (x / sw) & 1);
      for (int i = 0; i < IR; ++i)
        if (last_on_slot[i] >= 0) mbar_wait(&ctrl.i_full[i], (last_on_slot[i] / IR) & 1);
    }
    __syncwarp();
  } else if (warp == WARP_APROD) {
    // ---------------------------------------------------------------- activation gather
    uint32_t ast = 0;            // stages issued
    uint32_t asl = 0, aph = 0;   // next ring slot and its phase parity
    int ready_task = -1;         // task whose rows are known to be written (task_ready)
    bool all_ready = false;      // every task's rows are written
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      // lane 0 waits and the warp follows its answer (a timeout is seen by every lane alike)
      bool got = true;
      if (lane == 0) got = wait(&ctrl.i_full[slot], (n / IR) & 1, PROD_BACKOFF_NS);
      if (!__shfl_sync(0xffffffffu, got, 0)) break;
      const Item it = ctrl.items[slot];
      if (!it.valid) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      if (!GATED && p.task_ready && !all_ready && it.task != ready_task) {
        // the task's rows are complete once every item of it has been counted (or every item
        // of every task): lane 0 waits (acquire), the warp barrier orders the lanes after it,
        // and each lane's proxy fence orders its bulk copies below after the rows
        bool rd = true, all = false;
        if (lane == 0) {
          all = ld_acquire_gpu(p.items_done) >= __ldcg(p.ntasks) * p.ready_target;
          rd = all || (!*abort_flag && wait_count_geq(p.task_ready + it.task, p.ready_target));
          if (!rd && !*abort_flag) {
            *abort_flag = 1;
            if (p.err) atomicOr(p.err, KNX_DEV_TIMEOUT);
          }
        }
        rd = __shfl_sync(0xffffffffu, rd, 0);
        all_ready = __shfl_sync(0xffffffffu, all, 0);
        __syncwarp();
        if (!rd) break;
        fence_proxy_async_global();
        ready_task = it.task;
      }
      const __half* src = nullptr;
      if (lane < it.cnt)
        src = p.act + (p.sorted_pair ? p.sorted_pair[it.slot0 + lane] / p.topk
                                     : static_cast<int64_t>(it.slot0 + lane)) * p.act_stride;
      bool ok = true;
      for (int st = 0; st < nst; ++st, ++ast) {
        const int s = static_cast<int>(asl);
        bool free_ = true;
        if (lane == 0) free_ = wait(&ctrl.a_empty[s], aph ^ 1u, PROD_BACKOFF_NS);
        if (!__shfl_sync(0xffffffffu, free_, 0)) {
          ok = false;
          break;
        }
        if (++asl == static_cast<uint32_t>(sa)) { asl = 0; aph ^= 1u; }
        const int k0 = st * BK;
        const uint32_t kb = static_cast<uint32_t>(min(BK, p.K - k0)) * 2u;
        if (lane == 0) mbar_arrive_expect_tx(&ctrl.a_full[s], kb * it.cnt);
        __syncwarp();
        if (src) bulk_load(a_ring + s * A_STAGE + lane * AROW, src + k0, kb, &ctrl.a_full[s]);
      }
      __syncwarp();
      if (!ok) break;
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
    // bulk copies already issued must land before the CTA exits (bounded)
    if (lane == 0)
      for (uint32_t x = ast > static_cast<uint32_t>(sa) ? ast - sa : 0; x < ast; ++x)
        mbar_wait(&ctrl.a_full[x % sa], (x / sa) & 1);
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- math warps
    const int g = lane >> 2, q = lane & 3;
    // smem rows of this lane's two fragment rows (tile rows g and g+8); both are = g (mod 8),
    // which the 128-byte swizzle uses: 16-byte chunk j of row r sits at chunk j ^ (r & 7)
    const int rA = GATED ? 8 * warp + g : 16 * warp + g;
    constexpr int BOFF = (GATED ? GROWS : 8) * WROW;  // row B = row A + GROWS (gated) or + 8
    const int first_row = GATED ? 8 * warp : 16 * warp;  // tile's first row (validity)
    // ring slots and phase parities, carried across items (no runtime divisions in the loop)
    uint32_t wsl = 0, wph = 0, asl = 0, aph = 0;
    const int spg = GPJ < 8 ? 1 : p.gs / BK;  // stages per scale group when groups span stages
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      const bool got = __all_sync(0xffffffffu, wait(&ctrl.i_full[slot], (n / IR) & 1, 64));
      const Item it = ctrl.items[slot];
      // each warp decides alone (no barrier among the math warps inside the loop); the vote
      // keeps the lanes of a warp together
      if (__any_sync(0xffffffffu, !got || !it.valid || *abort_flag)) {
        __syncwarp();
        if (lane == 0 && got) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      const uint32_t szs = smem_u32(sz_ring + slot * szr);
      const uint32_t ng2 = static_cast<uint32_t>(p.ng) * 2u;  // bytes per scale/zero row
      // shared addresses of the scale/zero rows of this lane's two fragment rows
      uint32_t sA, zA, sB, zB;
      if (GATED) {
        sA = szs + (8 * warp + g) * ng2;
        zA = sA + GROWS * ng2;
        sB = sA + 2 * GROWS * ng2;
        zB = sA + 3 * GROWS * ng2;
      } else {
        sA = szs + (16 * warp + g) * ng2;
        zA = sA + ROWS * ng2;
        sB = sA + 8 * ng2;
        zB = zA + 8 * ng2;
      }
      const bool active = first_row < it.nvalid;
      const int ntl = (it.cnt + 7) >> 3;
      // NACC independent accumulator sets per n8 tile (k16 half, j parity), added in a fixed
      // order at the end of the item
      float acc[NT][NACC][4];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int u = 0; u < NACC; ++u)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[t][u][i] = 0.f;
      int grp0 = 0, spg_left = spg;  // first scale group of the stage
      for (int st = 0; st < nst; ++st) {
        const int ws = static_cast<int>(wsl), as = static_cast<int>(asl);
        // mma.sync needs the whole warp: every lane follows the same answer
        const bool ready = __all_sync(0xffffffffu, wait(&ctrl.w_full[ws], wph) &&
                                                       wait(&ctrl.a_full[as], aph));
        if (ready && active) {
          const uint32_t wa = smem_u32(w_ring + ws * W_STAGE) + rA * WROW + (g << 4) + 4 * q;
          const uint32_t ab = smem_u32(a_ring + as * A_STAGE) + g * AROW + q * 16;
          const int jmax = min(8, (p.K - st * BK) >> 5);
          if (jmax == 8) {
            switch (ntl) {
              case 4: mma_stage<ZINT, 4, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, zA, sB, zB, acc); break;
              case 3: mma_stage<ZINT, 3, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, zA, sB, zB, acc); break;
              case 2: mma_stage<ZINT, 2, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, zA, sB, zB, acc); break;
              default: mma_stage<ZINT, 1, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, zA, sB, zB, acc);
            }
          } else {
            switch (ntl) {
              case 4: mma_stage<ZINT, 4, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, zA, sB, zB, acc); break;
              case 3: mma_stage<ZINT, 3, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, zA, sB, zB, acc); break;
              case 2: mma_stage<ZINT, 2, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, zA, sB, zB, acc); break;
              default: mma_stage<ZINT, 1, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, zA, sB, zB, acc);
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&ctrl.w_empty[ws]);
          mbar_arrive(&ctrl.a_empty[as]);
        }
        if (++wsl == static_cast<uint32_t>(sw)) { wsl = 0; wph ^= 1u; }
        if (++asl == static_cast<uint32_t>(sa)) { asl = 0; aph ^= 1u; }
        if (GPJ < 8) grp0 += 8 / GPJ;
        else if (--spg_left == 0) { ++grp0; spg_left = spg; }
      }
      float res[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float v = acc[t][0][i];
#pragma unroll
          for (int u = 1; u < NACC; ++u) v += acc[t][u][i];
          res[t][i] = v;
        }
      // ---- epilogue: each warp stages its own columns (gated: 8 per token, the K-interleave
      // inside the 8-group; plain: 16) in a private shared area, then writes 16-byte chunks
      constexpr int WCOLS = GATED ? 8 : 16;
      const uint32_t stg = ot + static_cast<uint32_t>(warp) * (TOK * WCOLS * 2);
      __syncwarp();  // this warp's reads of the previous item's staging are done
      if (active) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < ntl) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int tok = 8 * t + 2 * q + h;
              if (GATED) {
                const float v = gelu_tanh(res[t][h]) * res[t][2 + h];
                sts16h(stg + 2u * (tok * WCOLS + perm_pos(g)), __float2half_rn(v));
              } else {
                sts16h(stg + 2u * (tok * WCOLS + g), __float2half_rn(res[t][h]));
                sts16h(stg + 2u * (tok * WCOLS + 8 + g), __float2half_rn(res[t][2 + h]));
              }
            }
          }
        }
      }
      __syncwarp();
      if (active) {
        const int col0 = (GATED ? it.slice * GROWS : it.slice * ROWS) + first_row;
        for (int c = lane; c < it.cnt * (WCOLS / 8); c += 32) {
          const int t = GATED ? c : c >> 1, ch = GATED ? 0 : c & 1;
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(it.slot0 + t) * p.out_stride +
                                    col0 + ch * 8) = lds128(stg + 16u * c);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
  }
  __syncthreads();
}

}  // namespace hw

namespace {

using EncodeTiledFn2 = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool encode_map_hw(CUtensorMap* map, const uint8_t* q, int64_t total_rows, int64_t row_bytes) {
  static EncodeTiledFn2 fn = nullptr;
  if (fn == nullptr) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult r{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &r) != cudaSuccess ||
        r != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<EncodeTiledFn2>(f);
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(total_rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(hw::WROW), static_cast<cuuint32_t>(hw::BOX_ROWS)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool GATED, bool ZINT, int GPJ>
int launch_hw_g(const hw::Params& p, const CUtensorMap& map, int grid, cudaStream_t s) {
  if (set_max_dyn_smem(reinterpret_cast<const void*>(hw::hw_gemm_kernel<GATED, ZINT, GPJ>),
                       static_cast<int>(hw::SMEM_LIMIT - hw::STATIC_RESERVE)) != KNX_OK)
    return KNX_E_DEVICE;
  (void)launch_pdl(hw::hw_gemm_kernel<GATED, ZINT, GPJ>, grid, hw::NTHREADS,
                   hw::smem_bytes(GATED, p.ng, p.sw, p.sa), s, map, p);
  return launch_status();
}

template <bool GATED, bool ZINT>
int launch_hw(hw::Params p, const uint8_t* wq, int64_t total_rows, int64_t row_bytes,
              int64_t work_bound, cudaStream_t s) {
  if (!hw::ring_depths(GATED, p.ng, p.sw, p.sa)) return KNX_E_UNSUPPORTED;
  CUtensorMap map;
  if (!encode_map_hw(&map, wq, total_rows, row_bytes)) return KNX_E_DEVICE;
  const int sms = num_sms();
  const int grid = static_cast<int>(work_bound < sms ? (work_bound > 0 ? work_bound : 1) : sms);
  switch (p.gs) {
    case 32: return launch_hw_g<GATED, ZINT, 1>(p, map, grid, s);
    case 64: return launch_hw_g<GATED, ZINT, 2>(p, map, grid, s);
    case 128: return launch_hw_g<GATED, ZINT, 4>(p, map, grid, s);
    default: return launch_hw_g<GATED, ZINT, 8>(p, map, grid, s);  // gs % 256 == 0
  }
}

}  // namespace

bool hw_supported(int64_t K, int gs, int ng, int64_t rows_per_expert, bool gated) {
  // scale groups must not straddle a 256-k stage unless they cover whole stages
  if (!(gs == 32 || gs == 64 || gs == 128 || (gs > 0 && gs % 256 == 0))) return false;
  int sw, sa;
  if (ng > hw::SZ_MAX || (K % 64) != 0 || !hw::ring_depths(gated, ng, sw, sa)) return false;
  if (gated) return (rows_per_expert / 2) % 64 == 0;
  return rows_per_expert % 16 == 0;
}

int hw_gateup_items(int I) { return (I + hw::GROWS - 1) / hw::GROWS; }

int launch_hw_gateup(const __half* xp, const int32_t* sorted_pair, int topk, const int32_t* offsets,
                     const int4* tasks, const int32_t* ntasks, int* counter, const uint8_t* gu_q,
                     const __half* gu_s, const __half* gu_z, int E, int H, int I, int ng, int gs,
                     bool zint, __half* out2, int64_t max_tasks, int32_t* err, cudaStream_t s,
                     int* task_done, int* items_done) {
  if (task_done && !(items_done && tasks)) return KNX_E_INVALID;
  hw::Params p{};
  p.act = xp; p.act_stride = H; p.sorted_pair = sorted_pair; p.topk = topk;
  p.tasks = tasks; p.ntasks = ntasks; p.work_counter = counter; p.ws = gu_s; p.wz = gu_z;
  p.K = H; p.rows_per_expert = 2 * I; p.I = I; p.ng = ng; p.gs = gs; p.out = out2;
  p.out_stride = I; p.nslices = hw_gateup_items(I); p.err = err; p.task_done = task_done;
  p.items_done = items_done;
  p.partial_last = (I % hw::GROWS) != 0 && p.nslices > 1;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_hw<true, true>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s)
              : launch_hw<true, false>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s);
}

int launch_hw_rows(const __half* act, int64_t act_stride, int K, const int32_t* offsets,
                   const int4* tasks, const int32_t* ntasks, int dense_rows, int* counter,
                   const uint8_t* wq, const __half* ws, const __half* wz, int E, int N, int ng,
                   int gs, bool zint, __half* out, int64_t out_stride, int64_t max_tasks,
                   int32_t* err, cudaStream_t s, const int* task_ready, int* items_done,
                   int ready_target) {
  if (task_ready && !(items_done && tasks)) return KNX_E_INVALID;
  hw::Params p{};
  p.act = act; p.act_stride = act_stride; p.tasks = tasks; p.ntasks = ntasks;
  p.dense_rows = dense_rows; p.work_counter = counter; p.ws = ws; p.wz = wz; p.K = K;
  p.rows_per_expert = N; p.ng = ng; p.gs = gs; p.out = out; p.out_stride = out_stride;
  p.nslices = (N + hw::ROWS - 1) / hw::ROWS; p.err = err;
  p.task_ready = task_ready; p.items_done = items_done; p.ready_target = ready_target;
  p.partial_last = (N % hw::ROWS) != 0 && p.nslices > 1;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_hw<false, true>(p, wq, int64_t(E) * N, K / 2, work, s)
              : launch_hw<false, false>(p, wq, int64_t(E) * N, K / 2, work, s);
}

}  // namespace knx
