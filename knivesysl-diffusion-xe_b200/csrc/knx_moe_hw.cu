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
//     registers into A fragments and multiplied with the B fragments of the task's 1-4 n8 token
//     tiles, so one dequantisation serves up to 32 tokens.  No split-K: every output is one
//     warp's fixed-order sum (deterministic), and a token's sum does not depend on the other
//     tokens of its task.  Two dequantisation modes:
//       - exact (dequant8): A = (q - z) * s rounded to f16 once (integer zero-points,
//         bit-identical to dequant_w4) or the reference kernel's RN16(RN16(q - z) * s);
//         13-17 instructions per 8 nibbles;
//       - integer (dequant8_q, the default for scale groups of 32-128): A = q exactly, 9
//         instructions per 8 nibbles.  Each scale group accumulates into its own fp32
//         registers, which are scaled into the output by one FFMA per element, and the
//         zero-point term sum_g s_g z_g sum_{k in g} x_k is subtracted once per item (see
//         zero_point_term).  Nothing is rounded to f16 before the accumulators: this is the W4
//         arithmetic without the weight rounding of the other forms;
//   * warp 18 (integer mode only): the per-token group sums of the activations, from the same
//     activation ring, by MMAs with a ones matrix (16 tokens x 16 k per instruction), into a
//     per-item table the math warps read after their last stage.
//   * GELU(gate) * up (gated) or the plain result: each warp stages its own 8 (gated) or 16
//     output columns per token in a private shared area and writes 16-byte chunks, so the math
//     warps never wait for one another; the gated output is written in the K-interleave the
//     down GEMM reads.
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
constexpr int WARP_WPROD = MATH_WARPS, WARP_APROD = MATH_WARPS + 1, WARP_SUM = MATH_WARPS + 2;
constexpr int num_warps(bool iq) { return MATH_WARPS + (iq ? 3 : 2); }
constexpr int nthreads(bool iq) { return num_warps(iq) * 32; }
constexpr int SZ_MAX = 32;               // groups per row
// integer mode: per-item table of each token's group sums, negated and divided by 16, as f16
// hi and lo parts ([token][group], row stride 40 halves: the B-fragment loads of 8 tokens hit
// distinct banks)
constexpr int ASTR = 40;
constexpr int ASUM_LO = TOK * ASTR * 2;  // byte offset of the lo table
constexpr int ASUM_SLOT = 2 * ASUM_LO;   // 5 KB per item slot
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
  int slot0, nvalid, pad0, pad1;
};

struct Ctrl {
  uint64_t w_full[SW_MAX], w_empty[SW_MAX];
  uint64_t a_full[SA_MAX], a_empty[SA_MAX];
  uint64_t i_full[IR], i_empty[IR];
  uint64_t s_full[IR];  // integer mode: the item's group-sum table is written
  Item items[IR];
  int abort;
};

struct Params {
  const __half* act;
  int64_t act_stride;
  const int32_t* sorted_pair;
  int topk;
  const int32_t* offsets;
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
  int sw;  // weight ring depth (stages)
  int sa;  // activation ring depth (stages)
  int32_t* err;
};

KNX_HOST_DEVINL size_t sz_slot_bytes(int ng) { return static_cast<size_t>(ROWS) * ng * 4; }
inline size_t smem_bytes(bool gated, bool iq, int ng, int sw, int sa) {
  return 1024 + static_cast<size_t>(sw) * W_STAGE + static_cast<size_t>(sa) * A_STAGE +
         ot_bytes(gated) + IR * sz_slot_bytes(ng) + (iq ? IR * ASUM_SLOT : 0);
}
// Ring depths that fit, in order of preference: at least 3 activation stages (their copies come
// from L2 but each is gathered token by token), then the deepest weight ring (it streams from
// HBM; 4 stages = 128 KB in flight).  Measured on the configs[1] gate_up: 3 + 3 beats 4 + 2.
inline bool ring_depths(bool gated, bool iq, int ng, int& sw, int& sa) {
  static const int pref[][2] = {{4, 4}, {4, 3}, {3, 4}, {3, 3}, {4, 2}, {3, 2}, {2, 4}, {2, 3}, {2, 2}};
  for (const auto& c : pref) {
    sw = c[0];
    sa = c[1];
    if (smem_bytes(gated, iq, ng, sw, sa) + STATIC_RESERVE <= SMEM_LIMIT) return true;
  }
  sw = sa = 0;
  return false;
}

KNX_DEVINL float gelu_tanh(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  const float th = 2.0f / (1.0f + expf(-2.0f * inner)) - 1.0f;
  return 0.5f * x * (1.0f + th);
}
KNX_DEVINL int perm_pos(int n) { return (n & ~7) + 2 * (n & 3) + ((n >> 2) & 1); }

// Dequant constants of one (row, group) as f16x2 broadcasts; the same values as make_sz (every
// operation below is exact or a single rounding of the exact result).
template <bool ZINT>
KNX_DEVINL void group_consts(__half s, __half z, __half2& s2, __half2& s16, __half2& c2,
                             __half2& c16) {
  const __half k16 = __ushort_as_half(0x4c00u), k1024 = __ushort_as_half(0x6400u);
  const __half sh = __hmul(s, __ushort_as_half(0x2c00u));  // s / 16
  const __half c = ZINT ? __hadd(z, k1024) : z;
  const __half ch = ZINT ? __hfma(z, k16, k1024) : __hmul(z, k16);
  s2 = __half2half2(s);
  s16 = __half2half2(sh);
  c2 = __half2half2(c);
  c16 = __half2half2(ch);
}

// Integer mode: the 8 nibbles of one u32 as exact f16 values q in the four A-fragment registers
// of dequant8 (same k order).  Magic-number halves h = 1024 + q (low nibble) give q = h - 1024;
// h = 1024 + 16 q (high nibble) gives q = h / 16 - 64 in one fused multiply-add; both exact.
KNX_DEVINL void dequant8_q(uint32_t u, uint32_t (&w)[4]) {
  const uint32_t MAG = 0x64006400u;
  const __half2 m1024 = __half2half2(__ushort_as_half(0xe400u));   // -1024
  const __half2 r16 = __half2half2(__ushort_as_half(0x2c00u));     // 1/16
  const __half2 m64 = __half2half2(__ushort_as_half(0xd400u));     // -64
  const uint32_t p0 = lop3_and_or(u, 0x000F000Fu, MAG);
  const uint32_t p1 = lop3_and_or(u, 0x00F000F0u, MAG);
  const uint32_t u8 = u >> 8;
  const uint32_t p2 = lop3_and_or(u8, 0x000F000Fu, MAG);
  const uint32_t p3 = lop3_and_or(u8, 0x00F000F0u, MAG);
  w[0] = h2_as_u32(__hadd2(u32_as_h2(p0), m1024));
  w[1] = h2_as_u32(__hfma2(u32_as_h2(p1), r16, m64));
  w[2] = h2_as_u32(__hadd2(u32_as_h2(p2), m1024));
  w[3] = h2_as_u32(__hfma2(u32_as_h2(p3), r16, m64));
}

// D = A * B (no accumulator input): the first MMA of a scale group.
KNX_DEVINL void mma_16816_first(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// 16 s z of groups g0, g0 + 1 of one row as f16x2 hi + lo parts (hi = RN16(16 s z), lo =
// RN16(16 s z - hi): the fma forms the exact difference); groups >= ng are zero.
KNX_DEVINL void sz_split(uint32_t s_row, uint32_t z_row, int g0, int ng, uint32_t& hi,
                         uint32_t& lo) {
  const __half zero = __ushort_as_half(0);
  const __half s0 = g0 < ng ? lds16h(s_row + 2 * g0) : zero;
  const __half s1 = g0 + 1 < ng ? lds16h(s_row + 2 * g0 + 2) : zero;
  const __half z0 = g0 < ng ? lds16h(z_row + 2 * g0) : zero;
  const __half z1 = g0 + 1 < ng ? lds16h(z_row + 2 * g0 + 2) : zero;
  const __half2 s2 = __hmul2(__halves2half2(s0, s1), __half2half2(__ushort_as_half(0x4c00u)));
  const __half2 z2 = __halves2half2(z0, z1);
  const __half2 h = __hmul2(s2, z2);
  hi = h2_as_u32(h);
  lo = h2_as_u32(__hfma2(s2, z2, __hneg2(h)));
}

// Integer mode, once per item: acc[t] += sum_g (16 s z)[row][g] * (-asum[token][g] / 16) over
// the lane's rows (A operand: tile row g = row A, g + 8 = row B; k = the scale group) and token
// tiles (B operand: the group-sum table), as hi*hi + hi*lo + lo*hi: the products agree with the
// exact fp32 product of the two unsplit values to ~2^-22.  The scaling by 16 keeps both lo parts
// normal f16 numbers at the benchmark's value ranges.
// tab: shared address of the hi table entry of token g, group 2q (tile 0).
template <int NTT>
KNX_DEVINL void zero_point_term(uint32_t sA, uint32_t zA, uint32_t sB, uint32_t zB, int ng,
                                int q, uint32_t tab, float (&acc)[NT][NACC][4]) {
#pragma unroll 1
  for (int c = 0; c < ng; c += 16) {
    uint32_t ph[4], pl[4];
    sz_split(sA, zA, c + 2 * q, ng, ph[0], pl[0]);
    sz_split(sB, zB, c + 2 * q, ng, ph[1], pl[1]);
    sz_split(sA, zA, c + 2 * q + 8, ng, ph[2], pl[2]);
    sz_split(sB, zB, c + 2 * q + 8, ng, ph[3], pl[3]);
#pragma unroll
    for (int t = 0; t < NTT; ++t) {
      const uint32_t o = tab + static_cast<uint32_t>(t * 8 * ASTR * 2 + c * 2);
      const uint32_t bh0 = lds32(o), bh1 = lds32(o + 16);
      const uint32_t bl0 = lds32(o + ASUM_LO), bl1 = lds32(o + ASUM_LO + 16);
      mma_16816(acc[t][0], ph[0], ph[1], ph[2], ph[3], bh0, bh1);
      mma_16816(acc[t][0], ph[0], ph[1], ph[2], ph[3], bl0, bl1);
      mma_16816(acc[t][0], pl[0], pl[1], pl[2], pl[3], bh0, bh1);
    }
  }
}

// Integer mode: one stage (256 k) of one warp's m16 tile, GPJ k32 steps per scale group (1, 2
// or 4: groups never straddle a stage).  Every group's products accumulate in fresh fp32
// registers, then acc += s * group sum per element (s of the element's row).
template <int NTT, int GPJ, bool TAIL, int BOFF>
KNX_DEVINL void mma_stage_q(uint32_t wa, uint32_t ab, int jmax, int grp0, uint32_t sA,
                            uint32_t sB, float (&acc)[NT][NACC][4]) {
  static_assert(GPJ == 1 || GPJ == 2 || GPJ == 4, "integer mode: scale groups of 32-128");
#pragma unroll 1
  for (int j0 = 0; j0 < 8; j0 += GPJ) {
    if (TAIL && j0 >= jmax) break;
    const int grp = grp0 + j0 / GPJ;
    const float fsA = __half2float(lds16h(sA + 2 * grp));
    const float fsB = __half2float(lds16h(sB + 2 * grp));
    float part[NTT][4];
#pragma unroll
    for (int jj = 0; jj < GPJ; ++jj) {
      const uint32_t aj = wa ^ static_cast<uint32_t>((j0 + jj) << 4);
      uint32_t fa[4], fb[4];
      dequant8_q(lds32(aj), fa);
      dequant8_q(lds32_at<BOFF>(aj), fb);
#pragma unroll
      for (int t = 0; t < NTT; ++t) {
        const uint4 b = lds128(ab + t * 8 * AROW + (j0 + jj) * 64);
        if (jj == 0) mma_16816_first(part[t], fa[0], fb[0], fa[1], fb[1], b.x, b.y);
        else mma_16816(part[t], fa[0], fb[0], fa[1], fb[1], b.x, b.y);
        mma_16816(part[t], fa[2], fb[2], fa[3], fb[3], b.z, b.w);
      }
    }
#pragma unroll
    for (int t = 0; t < NTT; ++t) {
      acc[t][0][0] = fmaf(fsA, part[t][0], acc[t][0][0]);
      acc[t][0][1] = fmaf(fsA, part[t][1], acc[t][0][1]);
      acc[t][0][2] = fmaf(fsB, part[t][2], acc[t][0][2]);
      acc[t][0][3] = fmaf(fsB, part[t][3], acc[t][0][3]);
    }
  }
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

template <bool GATED, bool ZINT, bool IQ, int GPJ>
__global__ void __launch_bounds__(nthreads(IQ), 1)
    hw_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const Params p) {
  pdl_wait_trigger();
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
  uint8_t* asum_ring = sz_ring + IR * szr;  // integer mode only
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nst = (p.K + BK - 1) / BK;

  if (IQ) {
    // groups >= ng of the sum tables are never written and must read as zero
    for (int i = tid; i < IR * ASUM_SLOT / 16; i += nthreads(IQ))
      sts128(smem_u32(asum_ring) + 16u * i, 0u, 0u, 0u, 0u);
  }
  if (tid == 0) {
    // the group-sum warp (integer mode) consumes every activation stage and item like a math warp
    const uint32_t a_cons = MATH_WARPS + (IQ ? 1 : 0);
    for (int s = 0; s < sw; ++s) { mbar_init(&ctrl.w_full[s], 1); mbar_init(&ctrl.w_empty[s], MATH_WARPS); }
    for (int s = 0; s < sa; ++s) { mbar_init(&ctrl.a_full[s], 1); mbar_init(&ctrl.a_empty[s], a_cons); }
    for (int i = 0; i < IR; ++i) {
      mbar_init(&ctrl.i_full[i], 1);
      mbar_init(&ctrl.i_empty[i], a_cons + 1);
      mbar_init(&ctrl.s_full[i], 32);
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
      const int nwork = (p.tasks ? *p.ntasks : (p.dense_rows + TOK - 1) / TOK) * p.nslices;
      uint32_t wst = 0;            // stages issued
      uint32_t wsl = 0, wph = 0;   // next ring slot and its phase parity
      int last_on_slot[IR];  // newest item per slot whose scale/zero copies were issued (-1: none)
      for (int i = 0; i < IR; ++i) last_on_slot[i] = -1;
      for (int n = 0;; ++n) {
        const int slot = n % IR;
        if (!wait(&ctrl.i_empty[slot], ((n / IR) & 1) ^ 1, PROD_BACKOFF_NS)) break;
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
            it.e = 0; t0 = task * TOK; it.cnt = min(TOK, p.dense_rows - t0);
          }
          it.slot0 = (p.offsets ? p.offsets[it.e] : 0) + t0;
          it.nvalid = GATED ? min(GROWS, p.I - it.slice * GROWS)
                            : min(ROWS, p.rows_per_expert - it.slice * ROWS);
          it.valid = 1;
        }
        ctrl.items[slot] = it;
        if (!it.valid) {
          last_on_slot[slot] = -1;
          mbar_arrive(&ctrl.i_full[slot]);
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
            tma_load_2d(dst, &wmap, &ctrl.w_full[s], x, y);
            tma_load_2d(dst + BOX_ROWS * WROW, &wmap, &ctrl.w_full[s], x, y + p.I);
          } else {
            const int y = it.e * p.rows_per_expert + it.slice * ROWS;
            tma_load_2d(dst, &wmap, &ctrl.w_full[s], x, y);
            tma_load_2d(dst + BOX_ROWS * WROW, &wmap, &ctrl.w_full[s], x, y + BOX_ROWS);
          }
        }
        if (*abort_flag) break;
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
  } else if (IQ && warp == WARP_SUM) {
    // ---------------------------------------------------------------- activation group sums
    // D[16 tokens x 8] += A[16 tokens x 16 k] * ones: every column of D holds the tokens' sums.
    // Lane (g, q) feeds tokens g and g + 8 of a 16-token half with the 16 bytes it would load as
    // a B fragment (4 + 4 k of each), so two MMAs cover a 32-k step.
    const int g = lane >> 2, q = lane & 3;
    const uint32_t ones = 0x3C003C00u;  // f16x2 (1, 1)
    const int k32_per_group = p.gs >> 5;
    uint32_t asl = 0, aph = 0;
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      const bool got = __all_sync(0xffffffffu, wait(&ctrl.i_full[slot], (n / IR) & 1, 64));
      const Item it = ctrl.items[slot];
      if (__any_sync(0xffffffffu, !got || !it.valid || *abort_flag)) {
        __syncwarp();
        if (lane == 0 && got) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      const int nhalf = (it.cnt + 15) >> 4;  // 16-token halves of the task
      // this lane stores part (q & 1: lo, else hi) of token g (q < 2) or g + 8 (q >= 2)
      const uint32_t dst = smem_u32(asum_ring + slot * ASUM_SLOT) + ((q & 1) ? ASUM_LO : 0) +
                           static_cast<uint32_t>((g + ((q >> 1) << 3)) * ASTR * 2);
      float d[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) d[h][i] = 0.f;
      int grp = 0, left = k32_per_group;
      bool ok = true;
      for (int st = 0; st < nst; ++st) {
        const int as = static_cast<int>(asl);
        if (!__all_sync(0xffffffffu, wait(&ctrl.a_full[as], aph))) {
          ok = false;
          break;
        }
        const uint32_t ab = smem_u32(a_ring + as * A_STAGE) + g * AROW + q * 16;
        const int jmax = min(8, (p.K - st * BK) >> 5);
        for (int j = 0; j < jmax; ++j) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h < nhalf) {
              const uint4 x0 = lds128(ab + (2 * h) * 8 * AROW + j * 64);
              const uint4 x1 = lds128(ab + (2 * h + 1) * 8 * AROW + j * 64);
              mma_16816(d[h], x0.x, x1.x, x0.y, x1.y, ones, ones);
              mma_16816(d[h], x0.z, x1.z, x0.w, x1.w, ones, ones);
            }
          }
          if (--left == 0) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (h < nhalf) {
                // -sum / 16 as f16 hi + lo (an exact scaling; the zero-point term uses 16 s z)
                const float v = -0.0625f * ((q >> 1) ? d[h][2] : d[h][0]);
                const __half hi = __float2half_rn(v);
                const __half lo = __float2half_rn(v - __half2float(hi));
                sts16h(dst + static_cast<uint32_t>((16 * h * ASTR + grp) * 2), (q & 1) ? lo : hi);
              }
#pragma unroll
              for (int i = 0; i < 4; ++i) d[h][i] = 0.f;
            }
            ++grp;
            left = k32_per_group;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctrl.a_empty[as]);
        if (++asl == static_cast<uint32_t>(sa)) { asl = 0; aph ^= 1u; }
      }
      if (!ok) break;
      __syncwarp();
      mbar_arrive(&ctrl.s_full[slot]);  // every lane: each releases its own table entries
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
  } else if (warp < MATH_WARPS) {
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
          if (IQ) {
            if constexpr (IQ && GPJ <= 4) {
              if (jmax == 8) {
                switch (ntl) {
                  case 4: mma_stage_q<4, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, sB, acc); break;
                  case 3: mma_stage_q<3, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, sB, acc); break;
                  case 2: mma_stage_q<2, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, sB, acc); break;
                  default: mma_stage_q<1, GPJ, false, BOFF>(wa, ab, 8, grp0, sA, sB, acc);
                }
              } else {
                switch (ntl) {
                  case 4: mma_stage_q<4, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, sB, acc); break;
                  case 3: mma_stage_q<3, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, sB, acc); break;
                  case 2: mma_stage_q<2, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, sB, acc); break;
                  default: mma_stage_q<1, GPJ, true, BOFF>(wa, ab, jmax, grp0, sA, sB, acc);
                }
              }
            }
          } else if (jmax == 8) {
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
      if constexpr (IQ) {
        // the zero-point term, once the group-sum warp has written this item's table
        const bool sums = __all_sync(0xffffffffu, wait(&ctrl.s_full[slot], (n / IR) & 1));
        if (sums && active) {
          const uint32_t tab = smem_u32(asum_ring + slot * ASUM_SLOT) +
                               static_cast<uint32_t>((g * ASTR + 2 * q) * 2);
          switch (ntl) {
            case 4: zero_point_term<4>(sA, zA, sB, zB, p.ng, q, tab, acc); break;
            case 3: zero_point_term<3>(sA, zA, sB, zB, p.ng, q, tab, acc); break;
            case 2: zero_point_term<2>(sA, zA, sB, zB, p.ng, q, tab, acc); break;
            default: zero_point_term<1>(sA, zA, sB, zB, p.ng, q, tab, acc);
          }
        }
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

template <bool GATED, bool ZINT, bool IQ, int GPJ>
int launch_hw_g(const hw::Params& p, const CUtensorMap& map, int grid, cudaStream_t s) {
  if (set_max_dyn_smem(reinterpret_cast<const void*>(hw::hw_gemm_kernel<GATED, ZINT, IQ, GPJ>),
                       static_cast<int>(hw::SMEM_LIMIT - hw::STATIC_RESERVE)) != KNX_OK)
    return KNX_E_DEVICE;
  (void)launch_pdl(hw::hw_gemm_kernel<GATED, ZINT, IQ, GPJ>, grid, hw::nthreads(IQ),
                   hw::smem_bytes(GATED, IQ, p.ng, p.sw, p.sa), s, map, p);
  return launch_status();
}

template <bool GATED, bool ZINT, bool IQ>
int launch_hw(hw::Params p, const uint8_t* wq, int64_t total_rows, int64_t row_bytes,
              int64_t work_bound, cudaStream_t s) {
  if (!hw::ring_depths(GATED, IQ, p.ng, p.sw, p.sa)) return KNX_E_UNSUPPORTED;
  CUtensorMap map;
  if (!encode_map_hw(&map, wq, total_rows, row_bytes)) return KNX_E_DEVICE;
  const int sms = num_sms();
  const int grid = static_cast<int>(work_bound < sms ? (work_bound > 0 ? work_bound : 1) : sms);
  switch (p.gs) {
    case 32: return launch_hw_g<GATED, ZINT, IQ, 1>(p, map, grid, s);
    case 64: return launch_hw_g<GATED, ZINT, IQ, 2>(p, map, grid, s);
    case 128: return launch_hw_g<GATED, ZINT, IQ, 4>(p, map, grid, s);
    default:  // gs % 256 == 0: exact modes only (integer-mode groups never straddle a stage)
      if constexpr (IQ) return KNX_E_UNSUPPORTED;
      else return launch_hw_g<GATED, ZINT, false, 8>(p, map, grid, s);
  }
}

// The dequantisation mode of a call: integer (scale groups of 32-128) unless the caller asked
// for the exact forms; exact forms by the zero-point flag.
template <bool GATED>
int launch_hw_mode(const hw::Params& p, const uint8_t* wq, int64_t total_rows, int64_t row_bytes,
                   int64_t work_bound, int dq, cudaStream_t s) {
  if (dq == DQ_INTEGER && p.gs <= 128)
    return launch_hw<GATED, false, true>(p, wq, total_rows, row_bytes, work_bound, s);
  if (dq == DQ_EXACT_ZINT)
    return launch_hw<GATED, true, false>(p, wq, total_rows, row_bytes, work_bound, s);
  return launch_hw<GATED, false, false>(p, wq, total_rows, row_bytes, work_bound, s);
}

}  // namespace

bool hw_supported(int64_t K, int gs, int ng, int64_t rows_per_expert, bool gated) {
  // scale groups must not straddle a 256-k stage unless they cover whole stages
  if (!(gs == 32 || gs == 64 || gs == 128 || (gs > 0 && gs % 256 == 0))) return false;
  int sw, sa;
  if (ng > hw::SZ_MAX || (K % 64) != 0 || !hw::ring_depths(gated, gs <= 128, ng, sw, sa))
    return false;
  if (gated) return (rows_per_expert / 2) % 64 == 0;
  return rows_per_expert % 16 == 0;
}

int launch_hw_gateup(const __half* xp, const int32_t* sorted_pair, int topk, const int32_t* offsets,
                     const int4* tasks, const int32_t* ntasks, int* counter, const uint8_t* gu_q,
                     const __half* gu_s, const __half* gu_z, int E, int H, int I, int ng, int gs,
                     int dq, __half* out2, int64_t max_tasks, int32_t* err, cudaStream_t s) {
  hw::Params p{};
  p.act = xp; p.act_stride = H; p.sorted_pair = sorted_pair; p.topk = topk; p.offsets = offsets;
  p.tasks = tasks; p.ntasks = ntasks; p.work_counter = counter; p.ws = gu_s; p.wz = gu_z;
  p.K = H; p.rows_per_expert = 2 * I; p.I = I; p.ng = ng; p.gs = gs; p.out = out2;
  p.out_stride = I; p.nslices = (I + hw::GROWS - 1) / hw::GROWS; p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return launch_hw_mode<true>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, dq, s);
}

int launch_hw_rows(const __half* act, int64_t act_stride, int K, const int32_t* offsets,
                   const int4* tasks, const int32_t* ntasks, int dense_rows, int* counter,
                   const uint8_t* wq, const __half* ws, const __half* wz, int E, int N, int ng,
                   int gs, int dq, __half* out, int64_t out_stride, int64_t max_tasks,
                   int32_t* err, cudaStream_t s) {
  hw::Params p{};
  p.act = act; p.act_stride = act_stride; p.offsets = offsets; p.tasks = tasks; p.ntasks = ntasks;
  p.dense_rows = dense_rows; p.work_counter = counter; p.ws = ws; p.wz = wz; p.K = K;
  p.rows_per_expert = N; p.ng = ng; p.gs = gs; p.out = out; p.out_stride = out_stride;
  p.nslices = (N + hw::ROWS - 1) / hw::ROWS; p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return launch_hw_mode<false>(p, wq, int64_t(E) * N, K / 2, work, dq, s);
}

}  // namespace knx
