// knx_internal.cuh — launch helpers shared between the translation units of libknx.so.
#pragma once
#include "knx_common.cuh"

namespace knx {

// Position of channel n inside the MoE K-interleave of its 8-group (the layout the down GEMM
// reads the gated intermediate in).
KNX_DEVINL int perm_pos(int n) { return (n & ~7) + 2 * (n & 3) + ((n >> 2) & 1); }

// tanh-form GELU of the gated epilogue, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
// (fused_moe_w4_v2.py:136-138), with tanh(y) = 1 - 2 / (1 + e^(2y)) from the fast exponential
// and division: ~1e-6 relative, far below the f16 rounding of GELU(gate) * up that follows.
KNX_DEVINL float gelu_tanh(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  const float th = 1.0f - __fdividef(2.0f, 1.0f + __expf(2.0f * inner));
  return 0.5f * x * (1.0f + th);
}

constexpr int64_t ALIGN_MAX_PAIRS = 32768;  // single-CTA counting sort limit (pairs)
constexpr int MAX_TASK_TOKENS = 128;        // largest task size the task-list builders accept
constexpr int ALIGN_MAX_EXPERTS = 256;

bool align_supported(int64_t N, int E);
size_t align_smem_bytes(int N, int E, int m_max);
int launch_align(const void* ids, int ids_dtype, int T, int topk, int E, int block_m, int m_max,
                 int32_t* counts, int32_t* offsets, int32_t* sorted_pair, int32_t* inv,
                 int32_t* sorted_rows, int32_t* expert_ids, int32_t* padded_inv, int4* tasks,
                 int32_t* ntasks, int32_t* work_counters, int n_work_counters, int32_t* err,
                 cudaStream_t stream, const int32_t* relabel = nullptr);
int launch_permute(const void* x, int dtype, __half* xp, int64_t elems, cudaStream_t stream);
// Counting sort for N > ALIGN_MAX_PAIRS (unpadded outputs only; scratch of
// align_large_scratch_bytes), and the task list from per-expert offsets (one CTA).
size_t align_large_scratch_bytes(int64_t N, int E);
int launch_align_large(const void* ids, int ids_dtype, int64_t N, int E, int32_t* counts,
                       int32_t* offsets, int32_t* sorted_pair, int32_t* inv, void* scratch,
                       int32_t* err, cudaStream_t s, const int32_t* relabel = nullptr);
int launch_tasks_from_offsets(const int32_t* offsets, int E, int m, int4* tasks, int32_t* ntasks,
                              int32_t* counters, int n_counters, cudaStream_t s);

// tcgen05 grouped W4A16 GEMMs (knx_moe_tcp.cu): MMA M = the tokens of one task
constexpr int TC_TASK_TOKENS = 128;  // tokens per task on the tcgen05 path
bool tc_supported(int64_t K, int gs, int ng, int64_t rows_per_expert, bool gated);
int launch_tc_gateup(const __half* xp, const int32_t* sorted_pair, int topk, const int32_t* offsets,
                     const int4* tasks, const int32_t* ntasks, int* counter, const uint8_t* gu_q,
                     const __half* gu_s, const __half* gu_z, int E, int H, int I, int ng, int gs,
                     bool zint, __half* out2, int64_t max_tasks, int32_t* err, cudaStream_t s);
int launch_tc_rows(const __half* act, int64_t act_stride, int K, const int32_t* offsets,
                   const int4* tasks, const int32_t* ntasks, int dense_rows, int* counter,
                   const uint8_t* wq, const __half* ws, const __half* wz, int E, int N, int ng,
                   int gs, bool zint, __half* out, int64_t out_stride, int64_t max_tasks,
                   int32_t* err, cudaStream_t s);

// warp-specialised mma.sync grouped W4A16 GEMMs (knx_moe_hw.cu), 32 tokens per task
constexpr int HW_TASK_TOKENS = 32;
constexpr int MIN_TASK_TOKENS = 16;  // smallest task size of any engine (sizes the task list)
bool hw_supported(int64_t K, int gs, int ng, int64_t rows_per_expert, bool gated);
// task_done (gate_up, may be NULL): one count per task, incremented once per finished item of
// the task (after its rows are written), and *items_done once per finished item;
// hw_gateup_items(I) items per task.
int hw_gateup_items(int I);
int launch_hw_gateup(const __half* xp, const int32_t* sorted_pair, int topk, const int32_t* offsets,
                     const int4* tasks, const int32_t* ntasks, int* counter, const uint8_t* gu_q,
                     const __half* gu_s, const __half* gu_z, int E, int H, int I, int ng, int gs,
                     bool zint, __half* out2, int64_t max_tasks, int32_t* err, cudaStream_t s,
                     int* task_done = nullptr, int* items_done = nullptr);
// task_ready (may be NULL): the down GEMM gathers a task's rows once task_ready[task] reaches
// ready_target (or *items_done reaches ready_target * tasks), instead of waiting for the whole
// previous kernel (programmatic dependent launch) before it starts; the other inputs must be
// complete before the previous kernel started.
int launch_hw_rows(const __half* act, int64_t act_stride, int K, const int32_t* offsets,
                   const int4* tasks, const int32_t* ntasks, int dense_rows, int* counter,
                   const uint8_t* wq, const __half* ws, const __half* wz, int E, int N, int ng,
                   int gs, bool zint, __half* out, int64_t out_stride, int64_t max_tasks,
                   int32_t* err, cudaStream_t s, const int* task_ready = nullptr,
                   int* items_done = nullptr, int ready_target = 0);

// The grouped expert GEMMs of one MoE layer over a task list (knx_moe.cu).
constexpr int GEMM_COUNTERS = 4;  // ints before the per-task ready counts in GemmArgs::counters
inline int64_t gemm_counter_ints(int64_t max_tasks) { return GEMM_COUNTERS + max_tasks; }
struct GemmArgs {
  const __half* xp;           // activation rows (K-interleaved f16)
  const int32_t* sorted_pair; // slot -> activation row * topk (+ k); NULL = row = slot
  int topk;
  const int32_t* offsets;     // [E + 1] slot offsets per expert
  const int4* tasks;          // (expert, first token in the expert, tokens, first slot)
  const int32_t* ntasks;
  int32_t* counters;          // GEMM_COUNTERS + max tasks ints, zero at entry: two work
                              // counters, the finished gate_up items, then (from GEMM_COUNTERS)
                              // one ready count per task
  const uint8_t* gu_q;
  const __half* gu_s;
  const __half* gu_z;
  const uint8_t* dn_q;
  const __half* dn_s;
  const __half* dn_z;
  int E;
  int64_t H, I;
  int gs_gu, gs_dn;
  bool zint;
  __half* out2;  // [pairs][I] f16 (K-interleaved)
  __half* out3;  // [pairs][H] f16
  int64_t pairs;
  int32_t* err;
};
int moe_engine(int flags, int64_t tokens_per_expert, int64_t H, int64_t I, int gs_gu, int gs_dn);
int engine_task_tokens(int eng);
int run_moe_gemms(const GemmArgs& a, int eng, int pc, cudaStream_t s);
int launch_combine(const __half* out3, const int32_t* inv, const void* w, int w_dtype, int64_t T,
                   int topk, int64_t H, int out_dtype, void* out, cudaStream_t s);

namespace prof {
int begin_call();                                  // -1 when stage recording is off
void mark(int call, int slot, cudaStream_t stream);  // record boundary `slot` of call `call`
}  // namespace prof

}  // namespace knx
