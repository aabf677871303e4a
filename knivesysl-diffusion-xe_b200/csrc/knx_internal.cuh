// knx_internal.cuh — launch helpers shared between the translation units of libknx.so.
#pragma once
#include "knx_common.cuh"

namespace knx {

constexpr int64_t ALIGN_MAX_PAIRS = 32768;  // single-CTA counting sort limit (pairs)
constexpr int ALIGN_MAX_EXPERTS = 256;

bool align_supported(int64_t N, int E);
size_t align_smem_bytes(int N, int E, int m_max);
int launch_align(const void* ids, int ids_dtype, int T, int topk, int E, int block_m, int m_max,
                 int32_t* counts, int32_t* offsets, int32_t* sorted_pair, int32_t* inv,
                 int32_t* sorted_rows, int32_t* expert_ids, int32_t* padded_inv, int4* tasks,
                 int32_t* ntasks, int32_t* work_counters, int n_work_counters, int32_t* err,
                 cudaStream_t stream);
int launch_permute(const void* x, int dtype, __half* xp, int64_t elems, cudaStream_t stream);

namespace prof {
int begin_call();                                  // -1 when stage recording is off
void mark(int call, int slot, cudaStream_t stream);  // record boundary `slot` of call `call`
}  // namespace prof

}  // namespace knx
