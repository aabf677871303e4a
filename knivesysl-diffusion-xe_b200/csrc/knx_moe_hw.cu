// knx_moe_hw.cu — warp-specialised grouped W4A16 GEMMs on the warp-level tensor-core path
// (mma.sync m16n8k16), the engine for the small-token regime (~16 tokens per expert), where it
// moves about twice as many weight-rows x k per cycle as tcgen05 (whose instructions cost ~128
// cycles each whatever N is).
//
// One persistent CTA per SM:
//   warps 0-15   math: dequantise nibbles in registers straight into A fragments (dequant8) and
//                issue m16n8k16 MMAs against the task's tokens (B fragments from shared memory).
//                Warp w owns two m16 row tiles (gated: 16 gate rows + the matching 16 up rows;
//                plain: 32 consecutive rows) and the k quarter w/4 of every 128-k stage; the four
//                quarters are summed through shared memory in fixed order at the end of a work
//                item (deterministic).
//   warp 16      scheduler + weight producer: work items from the counter, the slice's
//                scale/zero rows by 1-D bulk copies, packed nibbles by 2-D TMA (64-byte swizzle)
//                into an 8-stage ring; weight loads carry an L2 evict-first hint.
//   warp 17      activation producer: gathers the task's token rows (K-interleaved f16) with
//                cp.async into a 4-stage ring (rows padded to 320 B: conflict-free fragment
//                loads), with an L2 evict-last hint so the rows stay cached across slices.
// All waits are bounded (2 s); on a timeout the kernel sets KNX_DEV_TIMEOUT and every role leaves
// at the next work-item boundary (math warps agree through a named barrier first).
#include "knx_common.cuh"
#include "knx_internal.cuh"
#include "knx_sm100.cuh"

namespace knx {
namespace hw {

using namespace sm100;

constexpr int TOK = 32;                  // tokens per task
constexpr int NT = TOK / 8;              // n8 tiles
constexpr int BK = 128;                  // k per stage
constexpr int WROW = BK / 2;             // 64 bytes of nibbles per row per stage
constexpr int ROWS = 128;                // weight rows per item (gated: 64 gate + 64 up)
constexpr int SW = 8, SA = 4, IR = 2;
constexpr int W_STAGE = ROWS * WROW;     // 8 KB
constexpr int AROW = BK * 2 + 64;        // 320 B per token row per stage
constexpr int A_STAGE = TOK * AROW;      // 10 KB
constexpr int MATH_WARPS = 16;
constexpr int NUM_WARPS = MATH_WARPS + 2;
constexpr int NTHREADS = NUM_WARPS * 32;
constexpr int WARP_WPROD = MATH_WARPS, WARP_APROD = MATH_WARPS + 1;
constexpr int SZ_MAX = 32;
constexpr int OT = ROWS + 8;             // output tile row (halfs)

struct Item {
  int valid, e, cnt, slice;
  int slot0, nvalid, pad0, pad1;
};

struct Ctrl {
  uint64_t w_full[SW], w_empty[SW];
  uint64_t a_full[SA], a_empty[SA];
  uint64_t i_full[IR], i_empty[IR];
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
  int32_t* err;
};

// shared memory (from a 1024-aligned base)
constexpr int OFF_W = 0;
constexpr int OFF_A = OFF_W + SW * W_STAGE;
constexpr int OFF_RED = OFF_A + SA * A_STAGE;
constexpr int RED_BYTES = 3 * 4 * 32 * 32 * 4;   // k quarters 1..3 x 4 row pairs x 32 lanes x 32 f32
constexpr int OFF_OT = OFF_RED + RED_BYTES;
constexpr int OT_BYTES = TOK * OT * 2;
constexpr int OFF_SZ = OFF_OT + ((OT_BYTES + 1023) & ~1023);
KNX_HOST_DEVINL size_t sz_raw_bytes(int ng) { return (static_cast<size_t>(512) * ng + 127) & ~size_t(127); }
inline size_t smem_bytes(int ng) {
  return 1024 + OFF_SZ + IR * sz_raw_bytes(ng) + static_cast<size_t>(ROWS) * ng * 8;
}

KNX_DEVINL void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }
// Named barrier that also ORs a predicate over the participating threads: every thread gets the
// same answer, so warps that decide together whether to leave cannot disagree.
KNX_DEVINL bool bar_any(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %3, 0;\n\tbar.red.or.pred p, %1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(n), "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

KNX_DEVINL float gelu_tanh(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  const float th = 2.0f / (1.0f + expf(-2.0f * inner)) - 1.0f;
  return 0.5f * x * (1.0f + th);
}
KNX_DEVINL int perm_pos(int n) { return (n & ~7) + 2 * (n & 3) + ((n >> 2) & 1); }

KNX_DEVINL uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
KNX_DEVINL void cp_async16_hint(void* smem, const void* gmem, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(
                   smem_u32(smem)),
               "l"(gmem), "l"(pol));
}

template <bool GATED, bool ZINT>
__global__ void __launch_bounds__(NTHREADS, 1)
    hw_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const Params p) {
  extern __shared__ uint8_t dsm_raw[];
  __shared__ Ctrl ctrl;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_ring = base + OFF_W;
  uint8_t* a_ring = base + OFF_A;
  float* red = reinterpret_cast<float*>(base + OFF_RED);
  __half* otile = reinterpret_cast<__half*>(base + OFF_OT);
  const size_t szr = sz_raw_bytes(p.ng);
  uint8_t* sz_ring = base + OFF_SZ;
  uint2* sz2 = reinterpret_cast<uint2*>(sz_ring + IR * szr);  // [ROWS][ng]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nst = (p.K + BK - 1) / BK;

  if (tid == 0) {
    for (int s = 0; s < SW; ++s) { mbar_init(&ctrl.w_full[s], 1); mbar_init(&ctrl.w_empty[s], MATH_WARPS); }
    for (int s = 0; s < SA; ++s) { mbar_init(&ctrl.a_full[s], 32); mbar_init(&ctrl.a_empty[s], MATH_WARPS); }
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
      const int nwork = (p.tasks ? *p.ntasks : (p.dense_rows + TOK - 1) / TOK) * p.nslices;
      uint32_t wst = 0;
      int last_on_slot[IR];  // newest item per slot whose scale/zero copies were issued (-1: none)
      for (int i = 0; i < IR; ++i) last_on_slot[i] = -1;
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
            it.e = 0; t0 = task * TOK; it.cnt = min(TOK, p.dense_rows - t0);
          }
          it.slot0 = (p.offsets ? p.offsets[it.e] : 0) + t0;
          it.nvalid = GATED ? ROWS : min(ROWS, p.rows_per_expert - it.slice * ROWS);
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
      // Copies already issued must land before the CTA exits (only pending after an abort): the
      // newest phase of every weight stage and of every item slot is waited for, bounded.
      for (uint32_t x = wst > SW ? wst - SW : 0; x < wst; ++x)
        mbar_wait(&ctrl.w_full[x % SW], (x / SW) & 1);
      for (int i = 0; i < IR; ++i)
        if (last_on_slot[i] >= 0) mbar_wait(&ctrl.i_full[i], (last_on_slot[i] / IR) & 1);
    }
    __syncwarp();
  } else if (warp == WARP_APROD) {
    // ---------------------------------------------------------------- activation gather
    const uint64_t pol = policy_evict_last();
    uint32_t ast = 0;
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      if (!wait(&ctrl.i_full[slot], (n / IR) & 1, 64)) break;
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
        const int s = ast % SA;
        if (!wait(&ctrl.a_empty[s], ((ast / SA) & 1) ^ 1, 32)) {
          ok = false;
          break;
        }
        if (src) {
          uint8_t* dst = a_ring + s * A_STAGE + lane * AROW;
          const int k0 = st * BK;
          const int kch = min(BK, p.K - k0) >> 3;
#pragma unroll 4
          for (int j = 0; j < kch; ++j) cp_async16_hint(dst + j * 16, src + k0 + j * 8, pol);
        }
        cp_async_mbar_arrive_noinc(&ctrl.a_full[s]);
      }
      __syncwarp();
      if (!ok) break;
      if (lane == 0) mbar_arrive(&ctrl.i_empty[slot]);
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
  } else {
    // ---------------------------------------------------------------- math warps
    const int mp = warp & 3, kq = warp >> 2;
    const int g = lane >> 2, q = lane & 3;
    // two m16 row tiles: A = rows rA, rA+8; B = rows rB, rB+8
    const int rA = GATED ? 16 * mp + g : 32 * mp + g;
    const int rB = GATED ? 64 + 16 * mp + g : 32 * mp + 16 + g;
    const uint32_t chA = ((kq ^ ((rA >> 1) & 3)) << 4) + 4 * q;  // swizzled byte offset in the row
    const uint32_t chB = ((kq ^ ((rB >> 1) & 3)) << 4) + 4 * q;
    uint32_t wst = 0, ast = 0;
    for (int n = 0;; ++n) {
      const int slot = n % IR;
      const bool got = wait(&ctrl.i_full[slot], (n / IR) & 1, 64);
      const Item it = ctrl.items[slot];
      // all math warps leave together (the named barriers below need every one of them)
      if (bar_any(2, MATH_WARPS * 32, !got || !it.valid || *abort_flag)) {
        __syncwarp();
        if (lane == 0 && got) mbar_arrive(&ctrl.i_empty[slot]);
        break;
      }
      // per-item dequant constants {s, c, s/16, c16} for every (row, group)
      {
        const __half* szs = reinterpret_cast<const __half*>(sz_ring + slot * szr);
        const int ng = p.ng;
        for (int i = tid; i < ROWS * ng; i += MATH_WARPS * 32) {
          const int row = i / ng, grp = i - row * ng;
          const __half* srow;
          const __half* zrow;
          if (GATED) {
            srow = szs + (row < 64 ? 0 : 128 * ng) + (row & 63) * ng;
            zrow = srow + 64 * ng;
          } else {
            srow = szs + row * ng;
            zrow = szs + 128 * ng + row * ng;
          }
          sz2[i] = row < it.nvalid ? make_sz<ZINT>(srow[grp], zrow[grp]) : make_uint2(0u, 0u);
        }
      }
      named_bar(1, MATH_WARPS * 32);
      float accA[NT][4], accB[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) accA[t][i] = accB[t][i] = 0.f;
      const int ntl = (it.cnt + 7) >> 3;
      for (int st = 0; st < nst; ++st, ++wst, ++ast) {
        const int ws = wst % SW, as = ast % SA;
        const bool ready = wait(&ctrl.w_full[ws], (wst / SW) & 1) && wait(&ctrl.a_full[as], (ast / SA) & 1);
        const int k0 = st * BK + kq * 32;
        if (ready && k0 < p.K) {
          const int grp = k0 / p.gs;
          __half2 sA0, tA0, cA0, dA0, sA8, tA8, cA8, dA8, sB0, tB0, cB0, dB0, sB8, tB8, cB8, dB8;
          auto unpack = [&](uint2 v, __half2& s, __half2& s16, __half2& c, __half2& c16) {
            s = __low2half2(u32_as_h2(v.x));
            c = __high2half2(u32_as_h2(v.x));
            s16 = __low2half2(u32_as_h2(v.y));
            c16 = __high2half2(u32_as_h2(v.y));
          };
          unpack(sz2[rA * p.ng + grp], sA0, tA0, cA0, dA0);
          unpack(sz2[(rA + 8) * p.ng + grp], sA8, tA8, cA8, dA8);
          unpack(sz2[rB * p.ng + grp], sB0, tB0, cB0, dB0);
          unpack(sz2[(rB + 8) * p.ng + grp], sB8, tB8, cB8, dB8);
          const uint32_t wb = smem_u32(w_ring + ws * W_STAGE);
          uint32_t fA0[4], fA8[4], fB0[4], fB8[4];
          dequant8<ZINT>(lds32(wb + rA * WROW + chA), sA0, tA0, cA0, dA0, fA0);
          dequant8<ZINT>(lds32(wb + (rA + 8) * WROW + chA), sA8, tA8, cA8, dA8, fA8);
          dequant8<ZINT>(lds32(wb + rB * WROW + chB), sB0, tB0, cB0, dB0, fB0);
          dequant8<ZINT>(lds32(wb + (rB + 8) * WROW + chB), sB8, tB8, cB8, dB8, fB8);
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctrl.w_empty[ws]);  // nibbles consumed
          const uint32_t ab = smem_u32(a_ring + as * A_STAGE) + kq * 64 + q * 16;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < ntl) {
              const uint4 b = lds128(ab + (8 * t + g) * AROW);
              mma_16816(accA[t], fA0[0], fA8[0], fA0[1], fA8[1], b.x, b.y);
              mma_16816(accA[t], fA0[2], fA8[2], fA0[3], fA8[3], b.z, b.w);
              mma_16816(accB[t], fB0[0], fB8[0], fB0[1], fB8[1], b.x, b.y);
              mma_16816(accB[t], fB0[2], fB8[2], fB0[3], fB8[3], b.z, b.w);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctrl.a_empty[as]);
        } else {
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&ctrl.w_empty[ws]);
            mbar_arrive(&ctrl.a_empty[as]);
          }
        }
      }
      // ---- fixed-order split-K reduction over the four k quarters, epilogue, stores
      if (kq > 0) {
        float* r = red + ((kq - 1) * 4 + mp) * 32 * 32 + lane;
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            r[(t * 4 + i) * 32] = accA[t][i];
            r[(16 + t * 4 + i) * 32] = accB[t][i];
          }
      }
      named_bar(1, MATH_WARPS * 32);
      if (kq == 0) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < ntl) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float a = accA[t][i], b = accB[t][i];
#pragma unroll
              for (int k = 0; k < 3; ++k) {
                const float* r = red + (k * 4 + mp) * 32 * 32 + lane;
                a += r[(t * 4 + i) * 32];
                b += r[(16 + t * 4 + i) * 32];
              }
              const int tok = 8 * t + 2 * q + (i & 1);
              const int dr = (i & 2) ? 8 : 0;
              if (GATED) {
                otile[tok * OT + perm_pos(16 * mp + g + dr)] = __float2half_rn(gelu_tanh(a) * b);
              } else {
                otile[tok * OT + rA + dr] = __float2half_rn(a);
                otile[tok * OT + rB + dr] = __float2half_rn(b);
              }
            }
          }
        }
      }
      named_bar(1, MATH_WARPS * 32);
      if (GATED) {
        for (int c = tid; c < it.cnt * 8; c += MATH_WARPS * 32) {
          const int t = c >> 3, ch = c & 7;
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(it.slot0 + t) * p.out_stride +
                                    it.slice * 64 + ch * 8) =
              *reinterpret_cast<const uint4*>(otile + t * OT + ch * 8);
        }
      } else {
        const int vch = it.nvalid >> 3;
        for (int c = tid; c < it.cnt * vch; c += MATH_WARPS * 32) {
          const int t = c / vch, ch = c - t * vch;
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(it.slot0 + t) * p.out_stride +
                                    it.slice * ROWS + ch * 8) =
              *reinterpret_cast<const uint4*>(otile + t * OT + ch * 8);
        }
      }
      named_bar(1, MATH_WARPS * 32);
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

bool encode_map_hw(CUtensorMap* map, const uint8_t* q, int64_t total_rows, int64_t row_bytes,
                   int box_rows) {
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
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(hw::WROW), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool GATED, bool ZINT>
int launch_hw(const hw::Params& p, const uint8_t* wq, int64_t total_rows, int64_t row_bytes,
              int64_t work_bound, cudaStream_t s) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    if (cudaFuncSetAttribute(hw::hw_gemm_kernel<GATED, ZINT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(hw::smem_bytes(hw::SZ_MAX))) != cudaSuccess)
      return KNX_E_DEVICE;
    attr[dev & 63] = true;
  }
  CUtensorMap map;
  if (!encode_map_hw(&map, wq, total_rows, row_bytes, GATED ? 64 : hw::ROWS)) return KNX_E_DEVICE;
  const int sms = num_sms();
  const int grid = static_cast<int>(work_bound < sms ? (work_bound > 0 ? work_bound : 1) : sms);
  hw::hw_gemm_kernel<GATED, ZINT><<<grid, hw::NTHREADS, hw::smem_bytes(p.ng), s>>>(map, p);
  return launch_status();
}

}  // namespace

bool hw_supported(int64_t K, int gs, int ng, int64_t rows_per_expert, bool gated) {
  if (gs % 32 != 0 || ng > hw::SZ_MAX || (K % 64) != 0) return false;
  if (gated) return (rows_per_expert / 2) % 64 == 0;
  return rows_per_expert % hw::ROWS == 0;
}

int launch_hw_gateup(const __half* xp, const int32_t* sorted_pair, int topk, const int32_t* offsets,
                     const int4* tasks, const int32_t* ntasks, int* counter, const uint8_t* gu_q,
                     const __half* gu_s, const __half* gu_z, int E, int H, int I, int ng, int gs,
                     bool zint, __half* out2, int64_t max_tasks, int32_t* err, cudaStream_t s) {
  hw::Params p{};
  p.act = xp; p.act_stride = H; p.sorted_pair = sorted_pair; p.topk = topk; p.offsets = offsets;
  p.tasks = tasks; p.ntasks = ntasks; p.work_counter = counter; p.ws = gu_s; p.wz = gu_z;
  p.K = H; p.rows_per_expert = 2 * I; p.I = I; p.ng = ng; p.gs = gs; p.out = out2;
  p.out_stride = I; p.nslices = I / 64; p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_hw<true, true>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s)
              : launch_hw<true, false>(p, gu_q, int64_t(E) * 2 * I, H / 2, work, s);
}

int launch_hw_rows(const __half* act, int64_t act_stride, int K, const int32_t* offsets,
                   const int4* tasks, const int32_t* ntasks, int dense_rows, int* counter,
                   const uint8_t* wq, const __half* ws, const __half* wz, int E, int N, int ng,
                   int gs, bool zint, __half* out, int64_t out_stride, int64_t max_tasks,
                   int32_t* err, cudaStream_t s) {
  hw::Params p{};
  p.act = act; p.act_stride = act_stride; p.offsets = offsets; p.tasks = tasks; p.ntasks = ntasks;
  p.dense_rows = dense_rows; p.work_counter = counter; p.ws = ws; p.wz = wz; p.K = K;
  p.rows_per_expert = N; p.ng = ng; p.gs = gs; p.out = out; p.out_stride = out_stride;
  p.nslices = (N + hw::ROWS - 1) / hw::ROWS; p.err = err;
  const int64_t work = max_tasks * p.nslices;
  return zint ? launch_hw<false, true>(p, wq, int64_t(E) * N, K / 2, work, s)
              : launch_hw<false, false>(p, wq, int64_t(E) * N, K / 2, work, s);
}

}  // namespace knx
