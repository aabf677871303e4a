// knx_moe.cu — grouped W4A16 expert GEMMs for one MoE layer (gate_up + GELU, down), the
// fixed-order combine, and the dense W4A16 linear.
//
// Reference semantics: fused_moe_w4_v2.py:96-177 (GEMM kernels), :248-288 (combine),
// w4a16.py:63-108 (dense).  Weights are read in the pack_experts layout unchanged.
//
// Design (HBM-streaming regime, ~16 tokens per expert):
//   * weight-stationary "swap-AB" tiles: weight rows are the MMA M dimension (16 rows per
//     m16n8k16), tokens are the N dimension (8 per tile), so a task of <= 32 tokens wastes at most
//     7 columns; every weight byte is fetched from HBM and dequantised exactly once per task.
//   * nibbles are dequantised in registers straight into A fragments with the magic-number
//     trick (see dequant8 in knx_common.cuh); activations are kept in a K-interleaved copy so a
//     single 16-byte shared load yields both B fragments of a 32-k superstep.
//   * persistent CTAs pull (task, slice) work items from a device counter; the align kernel
//     orders tasks by token count (largest first) and resets the counters, so heavy experts start
//     first and the tail is short.  Each output element is produced by exactly one CTA with a
//     fixed summation order, so results are bit-identical run to run.
//   * a cp.async ring (weights XOR-swizzled, activations padded) keeps 3-4 stages in flight.
#include "knx_common.cuh"
#include "knx_internal.cuh"

namespace knx {

namespace {

constexpr int THREADS = 256;
constexpr int M_MAX = 32;       // tokens per task
constexpr int NT = M_MAX / 8;   // n8 tiles per task
constexpr int SZ_MAX_GROUPS = 56;  // H/gs (gate_up) and I/gs (down) limit

// GEMM1 (gate_up + GELU): slice = 64 gate rows + the matching 64 up rows, 256 k per stage.
constexpr int G1_ROWS = 64;
constexpr int G1_BK = 256;
constexpr int G1_STAGES = 4;
constexpr int G1_WROW = G1_BK / 2;                        // 128 B of nibbles per row per stage
constexpr int G1_WBYTES = 2 * G1_ROWS * G1_WROW;          // 16 KB
constexpr int G1_AROW = G1_BK * 2 + 64;                   // 576 B (padded) per token per stage
constexpr int G1_STAGE_BYTES = G1_WBYTES + M_MAX * G1_AROW;  // 34 KB

// GEMM2 (down, also the dense linear): slice = 128 output rows, 128 k per stage.
constexpr int G2_ROWS = 128;
constexpr int G2_BK = 128;
constexpr int G2_STAGES = 5;
constexpr int G2_WROW = G2_BK / 2;                        // 64 B
constexpr int G2_WBYTES = G2_ROWS * G2_WROW;              // 8 KB
constexpr int G2_AROW = G2_BK * 2 + 64;                   // 320 B
constexpr int G2_STAGE_BYTES = G2_WBYTES + M_MAX * G2_AROW;  // 18 KB
constexpr int G2_OROW = G2_ROWS * 2 + 16;                 // epilogue tile row (272 B)

// + raw scale/zero blocks (512*ng bytes) + per (row, group) dequant constants (128 rows x ng x 8 B)
inline size_t g1_smem(int ng) { return size_t(G1_STAGES) * G1_STAGE_BYTES + size_t(1536) * ng; }
inline size_t g2_smem(int ng) { return size_t(G2_STAGES) * G2_STAGE_BYTES + size_t(1536) * ng; }

KNX_DEVINL void unpack_sz(uint2 v, __half2& s, __half2& s16, __half2& c, __half2& c16) {
  s = __low2half2(u32_as_h2(v.x));
  c = __high2half2(u32_as_h2(v.x));
  s16 = __low2half2(u32_as_h2(v.y));
  c16 = __high2half2(u32_as_h2(v.y));
}


// ------------------------------------------------------------------------------------------
template <bool ZINT>
__global__ void __launch_bounds__(THREADS, 1)
    gateup_gelu_kernel(const __half* __restrict__ xp, const int32_t* __restrict__ sorted_pair,
                       int topk, const int32_t* __restrict__ offsets,
                       const int4* __restrict__ tasks, const int32_t* __restrict__ ntasks_ptr,
                       int* __restrict__ work_counter, const uint8_t* __restrict__ gu_q,
                       const __half* __restrict__ gu_s, const __half* __restrict__ gu_z, int H,
                       int I, int ng, int gs, __half* __restrict__ out2) {
  pdl_wait_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_tok[M_MAX];
  __shared__ int s_work;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int nslices = I / G1_ROWS;
  const int nwork = *ntasks_ptr * nslices;
  uint8_t* sz_raw = smem + G1_STAGES * G1_STAGE_BYTES;  // 4 blocks x 64*ng halfs
  uint2* sz2 = reinterpret_cast<uint2*>(sz_raw + 512 * ng);  // [128 rows][ng]
  const int rowbytes = H >> 1;
  const int nst = H / G1_BK;
  const int mt = warp & 3, kh = warp >> 2;
  const int r0 = 16 * mt + g;

  for (;;) {
    if (tid == 0) s_work = atomicAdd(work_counter, 1);
    __syncthreads();
    const int wi = s_work;
    if (wi >= nwork) break;
    const int task_id = wi / nslices, slice = wi - task_id * nslices;
    const int4 tk = tasks[task_id];
    const int e = tk.x, cnt = tk.z;
    const int slot0 = offsets[e] + tk.y;
    if (tid < M_MAX) s_tok[tid] = tid < cnt ? sorted_pair[slot0 + tid] / topk : 0;
    __syncthreads();
    const uint8_t* wg = gu_q + (static_cast<int64_t>(e) * 2 * I + slice * G1_ROWS) * rowbytes;
    const uint8_t* wu = wg + static_cast<int64_t>(I) * rowbytes;
    {  // scale/zero blocks for the whole slice: gate s, gate z, up s, up z (128*ng bytes each)
      const int64_t gb = (static_cast<int64_t>(e) * 2 * I + slice * G1_ROWS) * ng;
      const int64_t ub = gb + static_cast<int64_t>(I) * ng;
      const int chunks = 8 * ng;
      for (int c = tid; c < 4 * chunks; c += THREADS) {
        const int blk = c / chunks, cc = c - blk * chunks;
        const __half* src = ((blk & 1) ? gu_z : gu_s) + ((blk < 2) ? gb : ub) + cc * 8;
        cp_async16(sz_raw + blk * 128 * ng + cc * 16, src);
      }
    }
    auto load_stage = [&](int st, int buf) {
      uint8_t* W = smem + buf * G1_STAGE_BYTES;
      uint8_t* A = W + G1_WBYTES;
      const int kb = st * G1_WROW;
#pragma unroll
      for (int i = 0; i < (2 * G1_ROWS * G1_WROW / 16) / THREADS; ++i) {
        const int c = tid + i * THREADS;
        const int r = c >> 3, ch = c & 7;
        const uint8_t* src = (r < G1_ROWS ? wg + static_cast<int64_t>(r) * rowbytes
                                          : wu + static_cast<int64_t>(r - G1_ROWS) * rowbytes) +
                             kb + ch * 16;
        cp_async16(W + r * G1_WROW + ((ch ^ (r & 7)) << 4), src);
      }
      for (int c = tid; c < cnt * 32; c += THREADS) {
        const int t = c >> 5, ch = c & 31;
        cp_async16(A + t * G1_AROW + ch * 16,
                   xp + static_cast<int64_t>(s_tok[t]) * H + st * G1_BK + ch * 8);
      }
    };
#pragma unroll
    for (int s = 0; s < G1_STAGES - 1; ++s) {
      if (s < nst) load_stage(s, s);
      cp_async_commit();
    }

    float accg[NT][4], accu[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) accg[nt][i] = accu[nt][i] = 0.f;
    const int ntl = (cnt + 7) >> 3;

    for (int st = 0; st < nst; ++st) {
      cp_async_wait<G1_STAGES - 2>();
      __syncthreads();
      if (st == 0) {
        for (int i = tid; i < 2 * G1_ROWS * ng; i += THREADS) {
          const int row = i / ng, grp = i - row * ng;
          const int blk = row < G1_ROWS ? 0 : 2;
          const __half* rs = reinterpret_cast<const __half*>(sz_raw + blk * 128 * ng);
          const __half* rz = reinterpret_cast<const __half*>(sz_raw + (blk + 1) * 128 * ng);
          const int rr = row & (G1_ROWS - 1);
          sz2[row * ng + grp] = make_sz<ZINT>(rs[rr * ng + grp], rz[rr * ng + grp]);
        }
        __syncthreads();
      }
      {
        const int nx = st + G1_STAGES - 1;
        if (nx < nst) load_stage(nx, nx % G1_STAGES);
        cp_async_commit();
      }
      const uint32_t Wb = smem_u32(smem + (st % G1_STAGES) * G1_STAGE_BYTES);
      const uint32_t Ab = Wb + G1_WBYTES;
      const uint32_t wg0 = Wb + r0 * G1_WROW, wg8 = wg0 + 8 * G1_WROW;
      const uint32_t wu0 = Wb + (G1_ROWS + r0) * G1_WROW, wu8 = wu0 + 8 * G1_WROW;
      int cur = -1;
      __half2 sg0, tg0, cg0, dg0, sg8, tg8, cg8, dg8, su0, tu0, cu0, du0, su8, tu8, cu8, du8;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int ss = 4 * kh + j;
        const int grp = (st * G1_BK + ss * 32) / gs;
        if (grp != cur) {
          cur = grp;
          unpack_sz(sz2[r0 * ng + grp], sg0, tg0, cg0, dg0);
          unpack_sz(sz2[(r0 + 8) * ng + grp], sg8, tg8, cg8, dg8);
          unpack_sz(sz2[(G1_ROWS + r0) * ng + grp], su0, tu0, cu0, du0);
          unpack_sz(sz2[(G1_ROWS + r0 + 8) * ng + grp], su8, tu8, cu8, du8);
        }
        const uint32_t cho = ((ss ^ (r0 & 7)) << 4) + 4 * q;
        uint32_t fg0[4], fg8[4], fu0[4], fu8[4];
        dequant8<ZINT>(lds32(wg0 + cho), sg0, tg0, cg0, dg0, fg0);
        dequant8<ZINT>(lds32(wg8 + cho), sg8, tg8, cg8, dg8, fg8);
        dequant8<ZINT>(lds32(wu0 + cho), su0, tu0, cu0, du0, fu0);
        dequant8<ZINT>(lds32(wu8 + cho), su8, tu8, cu8, du8, fu8);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt < ntl) {
            const uint4 b = lds128(Ab + (8 * nt + g) * G1_AROW + ss * 64 + q * 16);
            mma_16816(accg[nt], fg0[0], fg8[0], fg0[1], fg8[1], b.x, b.y);
            mma_16816(accg[nt], fg0[2], fg8[2], fg0[3], fg8[3], b.z, b.w);
            mma_16816(accu[nt], fu0[0], fu8[0], fu0[1], fu8[1], b.x, b.y);
            mma_16816(accu[nt], fu0[2], fu8[2], fu0[3], fu8[3], b.z, b.w);
          }
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();

    // split-K reduction (warps 4-7 hold the second k half of each stage), GELU, f16 tile
    float* red = reinterpret_cast<float*>(smem);                         // 16 KB
    __half* otile = reinterpret_cast<__half*>(smem + 4 * NT * 8 * 32 * 4);  // [M_MAX][64]
    if (kh == 1) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          red[((mt * NT + nt) * 8 + i) * 32 + lane] = accg[nt][i];
          red[((mt * NT + nt) * 8 + 4 + i) * 32 + lane] = accu[nt][i];
        }
    }
    __syncthreads();
    if (kh == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt < ntl) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float gv = accg[nt][i] + red[((mt * NT + nt) * 8 + i) * 32 + lane];
            const float uv = accu[nt][i] + red[((mt * NT + nt) * 8 + 4 + i) * 32 + lane];
            const int n = r0 + ((i & 2) ? 8 : 0);
            const int t = 8 * nt + 2 * q + (i & 1);
            otile[t * G1_ROWS + perm_pos(n)] = __float2half_rn(gelu_tanh(gv) * uv);
          }
        }
      }
    }
    __syncthreads();
    for (int c = tid; c < cnt * 8; c += THREADS) {
      const int t = c >> 3, ch = c & 7;
      *reinterpret_cast<uint4*>(out2 + static_cast<int64_t>(slot0 + t) * I + slice * G1_ROWS +
                                ch * 8) =
          *reinterpret_cast<const uint4*>(otile + t * G1_ROWS + ch * 8);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------
// Generic "rows-by-slot" W4A16 GEMM used for the MoE down projection and the dense linear:
//   out[slot, n] = sum_k act[slot, k] * dequant(q[e, n, k]),   act in the K-interleave.
// tasks == nullptr: dense mode, task t = rows [32t, 32t+32) of expert 0, static striding.
template <bool ZINT>
__global__ void __launch_bounds__(THREADS, 2)
    rows_gemm_kernel(const __half* __restrict__ act, int64_t act_stride, int K,
                     const int32_t* __restrict__ offsets, const int4* __restrict__ tasks,
                     const int32_t* __restrict__ ntasks_ptr, int dense_rows,
                     int* __restrict__ work_counter, const uint8_t* __restrict__ wq,
                     const __half* __restrict__ ws, const __half* __restrict__ wz, int N, int ng,
                     int gs, __half* __restrict__ out, int64_t out_stride) {
  pdl_wait_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_work;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int nslices = (N + G2_ROWS - 1) / G2_ROWS;
  const int ntasks = tasks ? *ntasks_ptr : (dense_rows + M_MAX - 1) / M_MAX;
  const int nwork = ntasks * nslices;
  uint8_t* sz_raw = smem + G2_STAGES * G2_STAGE_BYTES;               // s block, z block
  uint2* sz2 = reinterpret_cast<uint2*>(sz_raw + 512 * ng);          // [128][ng]
  const int rowbytes = K >> 1;
  const int nst = (K + G2_BK - 1) / G2_BK;
  const int r0 = 16 * warp + g;
  const int swz = (g >> 1) & 3;

  for (int iter = 0;; ++iter) {
    int wi;
    if (work_counter) {
      if (tid == 0) s_work = atomicAdd(work_counter, 1);
      __syncthreads();
      wi = s_work;
    } else {
      wi = blockIdx.x + iter * gridDim.x;
    }
    if (wi >= nwork) break;
    const int task_id = wi / nslices, slice = wi - task_id * nslices;
    int e, t0, cnt;
    if (tasks) {
      const int4 tk = tasks[task_id];
      e = tk.x;
      t0 = tk.y;
      cnt = tk.z;
    } else {
      e = 0;
      t0 = task_id * M_MAX;
      cnt = min(M_MAX, dense_rows - t0);
    }
    const int slot0 = (offsets ? offsets[e] : 0) + t0;
    const int nvalid = min(G2_ROWS, N - slice * G2_ROWS);
    const int64_t row0 = static_cast<int64_t>(e) * N + slice * G2_ROWS;
    const uint8_t* wbase = wq + row0 * rowbytes;
    {
      const int nbytes = nvalid * ng * 2;
      const int chunks = (nbytes + 15) >> 4;
      for (int c = tid; c < 2 * chunks; c += THREADS) {
        const int blk = c / chunks, cc = c - blk * chunks;
        const uint8_t* src = reinterpret_cast<const uint8_t*>((blk ? wz : ws) + row0 * ng) + cc * 16;
        cp_async16(sz_raw + blk * 256 * ng + cc * 16, src, min(16, nbytes - cc * 16));
      }
    }
    auto load_stage = [&](int st, int buf) {
      uint8_t* W = smem + buf * G2_STAGE_BYTES;
      uint8_t* A = W + G2_WBYTES;
      const int k0 = st * G2_BK;
      const int kch = min(G2_BK, K - k0) >> 5;  // valid 16-byte weight chunks per row
#pragma unroll
      for (int i = 0; i < (G2_ROWS * G2_WROW / 16) / THREADS; ++i) {
        const int c = tid + i * THREADS;
        const int r = c >> 2, ch = c & 3;
        if (ch < kch) {
          const bool ok = r < nvalid;
          cp_async16(W + r * G2_WROW + ((ch ^ ((r >> 1) & 3)) << 4),
                     ok ? wbase + static_cast<int64_t>(r) * rowbytes + (k0 >> 1) + ch * 16 : wq,
                     ok ? 16 : 0);
        }
      }
      const int ach = kch * 4;  // 16-byte activation chunks per token
      for (int c = tid; c < cnt * ach; c += THREADS) {
        const int t = c / ach, ch = c - t * ach;
        cp_async16(A + t * G2_AROW + ch * 16,
                   act + static_cast<int64_t>(slot0 + t) * act_stride + k0 + ch * 8);
      }
    };
#pragma unroll
    for (int s = 0; s < G2_STAGES - 1; ++s) {
      if (s < nst) load_stage(s, s);
      cp_async_commit();
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
    const int ntl = (cnt + 7) >> 3;

    for (int st = 0; st < nst; ++st) {
      cp_async_wait<G2_STAGES - 2>();
      __syncthreads();
      if (st == 0) {
        const __half* rs = reinterpret_cast<const __half*>(sz_raw);
        const __half* rz = reinterpret_cast<const __half*>(sz_raw + 256 * ng);
        for (int i = tid; i < nvalid * ng; i += THREADS) sz2[i] = make_sz<ZINT>(rs[i], rz[i]);
        __syncthreads();
      }
      {
        const int nx = st + G2_STAGES - 1;
        if (nx < nst) load_stage(nx, nx % G2_STAGES);
        cp_async_commit();
      }
      const uint32_t Wb = smem_u32(smem + (st % G2_STAGES) * G2_STAGE_BYTES);
      const uint32_t Ab = Wb + G2_WBYTES;
      const uint32_t w0 = Wb + r0 * G2_WROW, w8 = w0 + 8 * G2_WROW;
      const int k0 = st * G2_BK;
      const int nss = min(G2_BK, K - k0) >> 5;
      const bool rows_ok = r0 < nvalid;  // r0 + 8 may still be out of range: garbage, not stored
      int cur = -1;
      __half2 s0, t0_, c0, d0, s8, t8, c8, d8;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < nss && rows_ok) {
          const int grp = (k0 + 32 * j) / gs;
          if (grp != cur) {
            cur = grp;
            unpack_sz(sz2[r0 * ng + grp], s0, t0_, c0, d0);
            unpack_sz((r0 + 8 < nvalid) ? sz2[(r0 + 8) * ng + grp] : make_uint2(0u, 0u), s8, t8,
                      c8, d8);
          }
          const uint32_t cho = ((j ^ swz) << 4) + 4 * q;
          uint32_t f0[4], f8[4];
          dequant8<ZINT>(lds32(w0 + cho), s0, t0_, c0, d0, f0);
          dequant8<ZINT>(lds32(w8 + cho), s8, t8, c8, d8, f8);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (nt < ntl) {
              const uint4 b = lds128(Ab + (8 * nt + g) * G2_AROW + j * 64 + q * 16);
              mma_16816(acc[nt], f0[0], f8[0], f0[1], f8[1], b.x, b.y);
              mma_16816(acc[nt], f0[2], f8[2], f0[3], f8[3], b.z, b.w);
            }
          }
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();
    __half* otile = reinterpret_cast<__half*>(smem);  // [M_MAX][G2_OROW bytes]
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (nt < ntl) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int n = r0 + ((i & 2) ? 8 : 0);
          const int t = 8 * nt + 2 * q + (i & 1);
          otile[t * (G2_OROW / 2) + n] = __float2half_rn(acc[nt][i]);
        }
      }
    }
    __syncthreads();
    const int vch = nvalid >> 3;  // N % 8 == 0
    for (int c = tid; c < cnt * vch; c += THREADS) {
      const int t = c / vch, ch = c - t * vch;
      *reinterpret_cast<uint4*>(out + static_cast<int64_t>(slot0 + t) * out_stride +
                                slice * G2_ROWS + ch * 8) =
          *reinterpret_cast<const uint4*>(otile + t * (G2_OROW / 2) + ch * 8);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------
// Fixed-order combine (fused_moe_w4_v2.py:248-263): y[t] = sum_{k in order} w[t,k]*out3[inv[t,k]],
// fp32 accumulate, one rounding to the output dtype.  Dropped pairs (inv < 0) contribute 0.
// y[t, 8 channels] = sum_{k in order} w[t,k] * f32(out3[inv[t*topk+k], 8 channels]).  TK > 0
// fixes topk at compile time so the TK row loads are all in flight before the sums (TK = 0: any
// topk, loop).  Same arithmetic and order in both forms.
template <typename TO, int TK>
__global__ void __launch_bounds__(256)
    combine_kernel(const __half* __restrict__ out3, const int32_t* __restrict__ inv,
                   const void* __restrict__ w, int w_dtype, int topk, int H,
                   TO* __restrict__ y) {
  pdl_wait_trigger();
  const int t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;  // 8-channel vector index
  if (v * 8 >= H) return;
  float acc[8] = {};
  auto add = [&](float wk, const uint4& raw) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      acc[2 * i] = fmaf(wk, f.x, acc[2 * i]);
      acc[2 * i + 1] = fmaf(wk, f.y, acc[2 * i + 1]);
    }
  };
  if constexpr (TK > 0) {
    uint4 raw[TK];
    float wk[TK];
#pragma unroll
    for (int k = 0; k < TK; ++k) {
      const int s = inv[static_cast<int64_t>(t) * TK + k];
      wk[k] = s < 0 ? 0.f : load_as_float(w, w_dtype, static_cast<int64_t>(t) * TK + k);
      raw[k] = s < 0 ? make_uint4(0, 0, 0, 0)
                     : *reinterpret_cast<const uint4*>(out3 + static_cast<int64_t>(s) * H + v * 8);
    }
#pragma unroll
    for (int k = 0; k < TK; ++k) {
      if (inv[static_cast<int64_t>(t) * TK + k] >= 0) add(wk[k], raw[k]);
    }
  } else {
    for (int k = 0; k < topk; ++k) {
      const int s = inv[static_cast<int64_t>(t) * topk + k];
      if (s < 0) continue;
      const float wk = load_as_float(w, w_dtype, static_cast<int64_t>(t) * topk + k);
      add(wk, *reinterpret_cast<const uint4*>(out3 + static_cast<int64_t>(s) * H + v * 8));
    }
  }
  TO o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<TO, __half>::value) {
      o[i] = __float2half_rn(acc[i]);
    } else {
      o[i] = __float2bfloat16_rn(acc[i]);
    }
  }
  *reinterpret_cast<uint4*>(y + static_cast<int64_t>(t) * H + v * 8) = *reinterpret_cast<uint4*>(o);
}

struct MoeWs {
  __half* xp;
  int32_t* counts;
  int32_t* offsets;
  int32_t* sorted_pair;
  int32_t* inv;
  int4* tasks;
  int32_t* ntasks;
  int32_t* counters;
  int n_counters;
  __half* out2;
  __half* out3;
  void* align_scratch;  // multi-CTA counting sort (N > ALIGN_MAX_PAIRS only)
  size_t bytes;
};

inline size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// The GEMM engine a call runs: an explicit flag, else the warp-specialised mma.sync kernels for
// small per-expert token counts and tcgen05 for large ones.  The switch point is the measured
// crossover of the two on B200 (MoE call with Zipf routing, H 2816, I 704): ws 297 / tc 317 us at
// 32 pairs per expert, ws 399 / tc 332 us at 48.
constexpr int64_t WS_MAX_TOKENS_PER_EXPERT = 36;
int engine_choice(int flags, int64_t tokens_per_expert) {
  if (flags & KNX_W4_WARP_MMA) return KNX_W4_WARP_MMA;
  if (flags & KNX_W4_WARP_WS) return KNX_W4_WARP_WS;
  if (flags & KNX_W4_TCGEN05) return KNX_W4_TCGEN05;
  return tokens_per_expert <= WS_MAX_TOKENS_PER_EXPERT ? KNX_W4_WARP_WS : KNX_W4_TCGEN05;
}

MoeWs carve_moe_ws(uint8_t* base, int64_t T, int64_t H, int64_t I, int E, int topk) {
  MoeWs w{};
  const int64_t N = T * topk;
  const int64_t max_tasks = (N + MIN_TASK_TOKENS - 1) / MIN_TASK_TOKENS + E;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + o : nullptr;
    o += up256(bytes);
    return p;
  };
  w.xp = reinterpret_cast<__half*>(take(size_t(T) * H * 2));
  w.counts = reinterpret_cast<int32_t*>(take(size_t(E) * 4));
  w.offsets = reinterpret_cast<int32_t*>(take(size_t(E + 1) * 4));
  w.sorted_pair = reinterpret_cast<int32_t*>(take(size_t(N) * 4));
  w.inv = reinterpret_cast<int32_t*>(take(size_t(N) * 4));
  w.tasks = reinterpret_cast<int4*>(take(size_t(max_tasks) * 16));
  w.ntasks = reinterpret_cast<int32_t*>(take(16));
  w.counters = reinterpret_cast<int32_t*>(take(size_t(gemm_counter_ints(max_tasks)) * 4));
  w.n_counters = static_cast<int>(gemm_counter_ints(max_tasks));
  w.out2 = reinterpret_cast<__half*>(take(size_t(N) * I * 2));
  w.out3 = reinterpret_cast<__half*>(take(size_t(N) * H * 2));
  w.align_scratch = N > ALIGN_MAX_PAIRS ? take(align_large_scratch_bytes(N, E)) : nullptr;
  w.bytes = o;
  return w;
}

bool set_smem_attrs() {
  const int m1 = static_cast<int>(g1_smem(SZ_MAX_GROUPS));
  const int m2 = static_cast<int>(g2_smem(SZ_MAX_GROUPS));
  return set_max_dyn_smem(reinterpret_cast<const void*>(gateup_gelu_kernel<true>), m1) == KNX_OK &&
         set_max_dyn_smem(reinterpret_cast<const void*>(gateup_gelu_kernel<false>), m1) == KNX_OK &&
         set_max_dyn_smem(reinterpret_cast<const void*>(rows_gemm_kernel<true>), m2) == KNX_OK &&
         set_max_dyn_smem(reinterpret_cast<const void*>(rows_gemm_kernel<false>), m2) == KNX_OK;
}

}  // namespace
// Engine of a call after the shape checks: tcgen05 / the warp-specialised mma.sync kernels where
// they support the shape, else the plain mma.sync kernels.
int moe_engine(int flags, int64_t tokens_per_expert, int64_t H, int64_t I, int gs_gu, int gs_dn) {
  const int ng1 = static_cast<int>(H / gs_gu), ng2 = static_cast<int>(I / gs_dn);
  const int eng = engine_choice(flags, tokens_per_expert);
  if (eng == KNX_W4_WARP_WS && hw_supported(H, gs_gu, ng1, 2 * I, true) &&
      hw_supported(I, gs_dn, ng2, H, false))
    return KNX_W4_WARP_WS;
  if (eng != KNX_W4_WARP_MMA && tc_supported(H, gs_gu, ng1, 2 * I, true) &&
      tc_supported(I, gs_dn, ng2, H, false))
    return KNX_W4_TCGEN05;
  return KNX_W4_WARP_MMA;
}

int engine_task_tokens(int eng) {
  return eng == KNX_W4_TCGEN05 ? TC_TASK_TOKENS : eng == KNX_W4_WARP_WS ? HW_TASK_TOKENS : M_MAX;
}

// gate_up + GELU then down over the task list (stage mark 2 between the two GEMMs).
int run_moe_gemms(const GemmArgs& a, int eng, int pc, cudaStream_t s) {
  const int tt = engine_task_tokens(eng);
  const int64_t max_tasks = (a.pairs + tt - 1) / tt + a.E;
  const int ng1 = static_cast<int>(a.H / a.gs_gu), ng2 = static_cast<int>(a.I / a.gs_dn);
  const int H = static_cast<int>(a.H), I = static_cast<int>(a.I);
  int st;
  if (eng == KNX_W4_TCGEN05) {
    st = launch_tc_gateup(a.xp, a.sorted_pair, a.topk, a.offsets, a.tasks, a.ntasks, a.counters,
                          a.gu_q, a.gu_s, a.gu_z, a.E, H, I, ng1, a.gs_gu, a.zint, a.out2,
                          max_tasks, a.err, s);
    if (st != KNX_OK) return st;
    prof::mark(pc, 2, s);
    return launch_tc_rows(a.out2, I, I, a.offsets, a.tasks, a.ntasks, 0, a.counters + 1, a.dn_q,
                          a.dn_s, a.dn_z, a.E, H, ng2, a.gs_dn, a.zint, a.out3, H, max_tasks,
                          a.err, s);
  }
  if (eng == KNX_W4_WARP_WS) {
    // gate_up counts the finished items of every task; down gathers a task's rows as soon as
    // all of its gate_up items are written, so its CTAs work on the SMs gate_up's tail frees
    int* ready = a.counters + GEMM_COUNTERS;
    st = launch_hw_gateup(a.xp, a.sorted_pair, a.topk, a.offsets, a.tasks, a.ntasks, a.counters,
                          a.gu_q, a.gu_s, a.gu_z, a.E, H, I, ng1, a.gs_gu, a.zint, a.out2,
                          max_tasks, a.err, s, ready, a.counters + 2);
    if (st != KNX_OK) return st;
    prof::mark(pc, 2, s);
    return launch_hw_rows(a.out2, I, I, a.offsets, a.tasks, a.ntasks, 0, a.counters + 1, a.dn_q,
                          a.dn_s, a.dn_z, a.E, H, ng2, a.gs_dn, a.zint, a.out3, H, max_tasks,
                          a.err, s, ready, a.counters + 2, hw_gateup_items(I));
  }
  if (!set_smem_attrs()) return KNX_E_DEVICE;
  const int sms = num_sms();
  {
    const int64_t work = max_tasks * (I / G1_ROWS);
    const int grid = static_cast<int>(work < sms ? work : sms);
    auto kern = a.zint ? gateup_gelu_kernel<true> : gateup_gelu_kernel<false>;
    (void)launch_pdl(kern, grid, THREADS, g1_smem(ng1), s, a.xp, a.sorted_pair, a.topk, a.offsets,
                     a.tasks, a.ntasks, a.counters, a.gu_q, a.gu_s, a.gu_z, H, I, ng1, a.gs_gu,
                     a.out2);
    st = launch_status();
    if (st != KNX_OK) return st;
  }
  prof::mark(pc, 2, s);
  {
    const int64_t work = max_tasks * ((H + G2_ROWS - 1) / G2_ROWS);
    const int grid = static_cast<int>(work < 2 * sms ? work : 2 * sms);
    auto kern = a.zint ? rows_gemm_kernel<true> : rows_gemm_kernel<false>;
    (void)launch_pdl(kern, grid, THREADS, g2_smem(ng2), s, a.out2, I, I, a.offsets, a.tasks,
                     a.ntasks, 0, a.counters + 1, a.dn_q, a.dn_s, a.dn_z, H, ng2, a.gs_dn, a.out3,
                     H);
    return launch_status();
  }
}

int launch_combine(const __half* out3, const int32_t* inv, const void* w, int w_dtype, int64_t T,
                   int topk, int64_t H, int out_dtype, void* out, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>((H / 8 + 255) / 256), static_cast<unsigned>(T));
  const int Hi = static_cast<int>(H);
  if (out_dtype == KNX_F16) {
    __half* o = static_cast<__half*>(out);
    if (topk == 8) (void)launch_pdl(combine_kernel<__half, 8>, grid, 256, 0, s, out3, inv, w,
                                    w_dtype, topk, Hi, o);
    else (void)launch_pdl(combine_kernel<__half, 0>, grid, 256, 0, s, out3, inv, w, w_dtype, topk,
                          Hi, o);
  } else {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
    if (topk == 8) (void)launch_pdl(combine_kernel<__nv_bfloat16, 8>, grid, 256, 0, s, out3, inv, w,
                                    w_dtype, topk, Hi, o);
    else (void)launch_pdl(combine_kernel<__nv_bfloat16, 0>, grid, 256, 0, s, out3, inv, w, w_dtype,
                          topk, Hi, o);
  }
  return launch_status();
}

}  // namespace knx



// ------------------------------------------------------------------------------------------
extern "C" size_t knx_moe_w4_workspace_size(int64_t T, int64_t H, int64_t I, int E, int topk) {
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || topk <= 0) return 0;
  return knx::carve_moe_ws(nullptr, T, H, I, E, topk).bytes;
}

extern "C" int knx_moe_w4(const void* hidden, const void* hidden_perm, int hidden_dtype,
                          const void* topk_ids, int ids_dtype, const void* topk_w, int w_dtype,
                          const uint8_t* gu_q, const void* gu_s, const void* gu_z,
                          const uint8_t* dn_q, const void* dn_s, const void* dn_z, int64_t T,
                          int64_t H, int64_t I, int E, int topk, int gs_gu, int gs_dn,
                          int flags, void* workspace, size_t workspace_bytes, void* out,
                          int32_t* err, void* stream) {
  using namespace knx;
  const bool zint = (flags & KNX_W4_INT_ZEROS) != 0;
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || topk <= 0 || topk > 16) return KNX_E_INVALID;
  if ((H % G1_BK) != 0 || (I % G1_ROWS) != 0 || H > (1 << 20) || I > (1 << 20))
    return KNX_E_UNSUPPORTED;
  if (gs_gu <= 0 || gs_dn <= 0 || (gs_gu % 32) != 0 || (gs_dn % 32) != 0 || (H % gs_gu) != 0 ||
      (I % gs_dn) != 0)
    return KNX_E_INVALID;
  const int ng1 = static_cast<int>(H / gs_gu), ng2 = static_cast<int>(I / gs_dn);
  if (ng1 > SZ_MAX_GROUPS || ng2 > SZ_MAX_GROUPS) return KNX_E_UNSUPPORTED;
  if (hidden_dtype != KNX_F16 && hidden_dtype != KNX_BF16) return KNX_E_INVALID;
  if (ids_dtype != KNX_I32 && ids_dtype != KNX_I64) return KNX_E_INVALID;
  if (w_dtype != KNX_F16 && w_dtype != KNX_BF16 && w_dtype != KNX_F32) return KNX_E_INVALID;
  if (E > ALIGN_MAX_EXPERTS || T * topk > (1LL << 30)) return KNX_E_UNSUPPORTED;
  if (!aligned(hidden, 16) || !aligned(out, 16) || (hidden_perm && !aligned(hidden_perm, 16)) ||
      !aligned(gu_q, 16) || !aligned(dn_q, 16) || !aligned(gu_s, 16) || !aligned(gu_z, 16) ||
      !aligned(dn_s, 16) || !aligned(dn_z, 16) || !aligned(workspace, 256))
    return KNX_E_ALIGN;
  if (T == 0) return KNX_OK;
  const size_t need = knx_moe_w4_workspace_size(T, H, I, E, topk);
  if (workspace == nullptr || workspace_bytes < need) return KNX_E_WORKSPACE;
  if (!set_smem_attrs()) return KNX_E_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  MoeWs w = carve_moe_ws(static_cast<uint8_t*>(workspace), T, H, I, E, topk);
  const __half* xp = static_cast<const __half*>(hidden_perm);
  int st;
  const int pc = prof::begin_call();
  prof::mark(pc, 0, s);
  if (!xp) {
    st = launch_permute(hidden, hidden_dtype, w.xp, T * H, s);
    if (st != KNX_OK) return st;
    xp = w.xp;
  }
  const int eng = moe_engine(flags, T * topk / E, H, I, gs_gu, gs_dn);
  // the per-task ready counts are used (and zeroed) by the ws engine only
  const int nc = eng == KNX_W4_WARP_WS ? w.n_counters : GEMM_COUNTERS;
  if (align_supported(T * topk, E)) {
    st = launch_align(topk_ids, ids_dtype, static_cast<int>(T), topk, E, 0,
                      engine_task_tokens(eng), w.counts, w.offsets, w.sorted_pair, w.inv, nullptr,
                      nullptr, nullptr, w.tasks, w.ntasks, w.counters, nc, err, s);
  } else {
    st = launch_align_large(topk_ids, ids_dtype, T * topk, E, w.counts, w.offsets, w.sorted_pair,
                            w.inv, w.align_scratch, err, s);
    if (st == KNX_OK)
      st = launch_tasks_from_offsets(w.offsets, E, engine_task_tokens(eng), w.tasks, w.ntasks,
                                     w.counters, nc, s);
  }
  if (st != KNX_OK) return st;
  prof::mark(pc, 1, s);
  GemmArgs ga{};
  ga.xp = xp; ga.sorted_pair = w.sorted_pair; ga.topk = topk; ga.offsets = w.offsets;
  ga.tasks = w.tasks; ga.ntasks = w.ntasks; ga.counters = w.counters;
  ga.gu_q = gu_q; ga.gu_s = static_cast<const __half*>(gu_s); ga.gu_z = static_cast<const __half*>(gu_z);
  ga.dn_q = dn_q; ga.dn_s = static_cast<const __half*>(dn_s); ga.dn_z = static_cast<const __half*>(dn_z);
  ga.E = E; ga.H = H; ga.I = I; ga.gs_gu = gs_gu; ga.gs_dn = gs_dn; ga.zint = zint;
  ga.out2 = w.out2; ga.out3 = w.out3; ga.pairs = T * topk; ga.err = err;
  st = run_moe_gemms(ga, eng, pc, s);
  if (st != KNX_OK) return st;
  prof::mark(pc, 3, s);
  st = launch_combine(w.out3, w.inv, topk_w, w_dtype, T, topk, H, hidden_dtype, out, s);
  prof::mark(pc, 4, s);
  return st;
}

extern "C" size_t knx_w4a16_workspace_size(int64_t M, int64_t K) {
  if (M < 0 || K <= 0) return 0;
  return knx::up256(size_t(M) * size_t(K) * 2) + 256;  // K-interleaved X + a work counter
}

extern "C" int knx_w4a16_linear(const void* X, const uint8_t* q, const void* s, const void* z,
                                int64_t M, int64_t N, int64_t K, int gs, int flags, void* Y,
                                void* workspace, size_t workspace_bytes, void* stream) {
  using namespace knx;
  if (M < 0 || N <= 0 || K <= 0 || (K % 64) != 0 || (N % 8) != 0 || gs <= 0 || (gs % 32) != 0 ||
      (K % gs) != 0 || M > (1 << 28) || N > (1 << 24) || K > (1 << 20))
    return KNX_E_INVALID;
  const int ng = static_cast<int>(K / gs);
  if (ng > SZ_MAX_GROUPS) return KNX_E_UNSUPPORTED;
  if (!aligned(X, 16) || !aligned(q, 16) || !aligned(s, 16) || !aligned(z, 16) ||
      !aligned(Y, 16) || !aligned(workspace, 16))
    return KNX_E_ALIGN;
  if ((K / 2) % 16 != 0) return KNX_E_ALIGN;
  if (M == 0) return KNX_OK;
  if (workspace == nullptr || workspace_bytes < knx_w4a16_workspace_size(M, K))
    return KNX_E_WORKSPACE;
  if (!set_smem_attrs()) return KNX_E_DEVICE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __half* xp = static_cast<__half*>(workspace);
  int rc = launch_permute(X, KNX_F16, xp, M * K, st);
  if (rc != KNX_OK) return rc;
  const bool zint = (flags & KNX_W4_INT_ZEROS) != 0;
  const int eng = engine_choice(flags, M);
  if (eng == KNX_W4_WARP_WS && hw_supported(K, gs, ng, N, false)) {
    int* counter = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + up256(size_t(M) * K * 2));
    if (cudaMemsetAsync(counter, 0, sizeof(int), st) != cudaSuccess) return KNX_E_LAUNCH;
    return launch_hw_rows(xp, K, static_cast<int>(K), nullptr, nullptr, nullptr,
                          static_cast<int>(M), counter, q, static_cast<const __half*>(s),
                          static_cast<const __half*>(z), 1, static_cast<int>(N), ng, gs, zint,
                          static_cast<__half*>(Y), N, (M + HW_TASK_TOKENS - 1) / HW_TASK_TOKENS,
                          nullptr, st);
  }
  if (eng != KNX_W4_WARP_MMA && tc_supported(K, gs, ng, N, false)) {
    int* counter = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + up256(size_t(M) * K * 2));
    if (cudaMemsetAsync(counter, 0, sizeof(int), st) != cudaSuccess) return KNX_E_LAUNCH;
    return launch_tc_rows(xp, K, static_cast<int>(K), nullptr, nullptr, nullptr,
                          static_cast<int>(M), counter, q, static_cast<const __half*>(s),
                          static_cast<const __half*>(z), 1, static_cast<int>(N), ng, gs, zint,
                          static_cast<__half*>(Y), N, (M + TC_TASK_TOKENS - 1) / TC_TASK_TOKENS,
                          nullptr, st);
  }
  const int64_t work = ((M + M_MAX - 1) / M_MAX) * ((N + G2_ROWS - 1) / G2_ROWS);
  const int sms = num_sms();
  const int grid = static_cast<int>(work < 2 * sms ? work : 2 * sms);
  auto kern = zint ? rows_gemm_kernel<true> : rows_gemm_kernel<false>;
  (void)launch_pdl(kern, grid, THREADS, g2_smem(ng), st, xp, K, static_cast<int>(K), nullptr,
                   nullptr, nullptr, static_cast<int>(M), nullptr, q, static_cast<const __half*>(s),
                   static_cast<const __half*>(z), static_cast<int>(N), ng, gs,
                   static_cast<__half*>(Y), N);
  return launch_status();
}
