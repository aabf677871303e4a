/*
 * knx.h — C ABI of the B200 (sm_100a) kernels for the DiffusionGemma W4A16 MoE layer and the
 * block-diffusion sampler step.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA stream handle
 * (`cudaStream_t` passed as `void*`; NULL = legacy default stream). Nothing here allocates
 * device memory: callers pass outputs and, where a function needs scratch space, a workspace
 * whose size the matching `*_workspace_size` function reports (knx_sampler_fused_static keeps
 * its scratch inside the library instead). Every call is stream-ordered and never synchronises
 * the host.
 *
 * Return value: KNX_OK (0) or a negative KNX_E* status for host-detectable contract violations
 * (bad sizes, misaligned pointers, launch failures). Data-dependent problems found on the
 * device (for example an expert id outside [0, E]) are OR-ed as KNX_DEV_* bits into the
 * optional `err` device word; pass NULL to skip that reporting. Kernels never trap.
 *
 * Each declaration names the reference interface it replaces, as `file:line` inside the
 * reference project (SRSWTI/knivesysl-diffusion-xe, directory `kernels/`).
 */
#ifndef KNX_H_
#define KNX_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KNX_API __attribute__((visibility("default")))
#else
#define KNX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define KNX_OK 0
#define KNX_E_INVALID (-1)      /* bad size / dtype / flag combination                     */
#define KNX_E_ALIGN (-2)        /* pointer or stride violates the documented alignment      */
#define KNX_E_WORKSPACE (-3)    /* workspace NULL or smaller than *_workspace_size()        */
#define KNX_E_LAUNCH (-4)       /* cudaGetLastError() after a launch was not cudaSuccess     */
#define KNX_E_UNSUPPORTED (-5)  /* shape outside what the kernels were built for            */
#define KNX_E_DEVICE (-6)       /* device is not sm_100 or CUDA call failed                  */

/* device error bits (OR-ed into *err when err != NULL) */
#define KNX_DEV_BAD_EXPERT_ID 0x1 /* topk id < 0 or > E (id == E is the "dropped" sentinel) */
#define KNX_DEV_CAPACITY 0x2      /* a per-launch capacity bound was exceeded                */
#define KNX_DEV_TIMEOUT 0x4       /* a bounded on-chip wait gave up (protocol error); the call's
                                     outputs are invalid, the device and context stay usable  */

/* ---- dtypes ----------------------------------------------------------------------------- */
#define KNX_F16 0
#define KNX_BF16 1
#define KNX_F32 2
#define KNX_I32 3
#define KNX_I64 4

/* weight-format / engine flags */
#define KNX_W4_INT_ZEROS 0x1 /* all zero-points are integers in [0, 15] */
/* GEMM engine (at most one; none = automatic: the warp-specialised mma.sync kernels up to 36
 * (token, slot) pairs per expert on average, tcgen05 above that) */
#define KNX_W4_WARP_MMA 0x2  /* the plain mma.sync kernels (A/B runs) */
#define KNX_W4_WARP_WS 0x8   /* the warp-specialised mma.sync kernels (TMA-fed, 16 math warps) */
#define KNX_W4_TCGEN05 0x10  /* the tcgen05 kernels (128 tokens x 256 weight rows per MMA) */

KNX_API int knx_version(void);
/* 1 when the current device is a compute-capability 10.0 part (the only target). */
KNX_API int knx_device_ok(void);
KNX_API const char* knx_status_string(int status);

/* ---- RMSNorm ----------------------------------------------------------------------------
 * Replaces fused_rmsnorm (fused_rmsnorm.py:24-32, kernel fused_rmsnorm.py:10-21).
 * y[r,:] = x[r,:] * rsqrt(mean(x[r,:]^2) + eps) * w   (fp32 math; w may be NULL = no scale)
 * x, y: [rows, cols] contiguous in `dtype` (F16/BF16); w: [cols] in `w_dtype`.
 * flags & KNX_RMS_ROUND_BF16: round the fp32 result to bf16 before the final store in
 *   `dtype`, reproducing the reference kernel's bf16 store + .to(x.dtype) (fused_rmsnorm.py:21,32).
 * xperm (optional, F16 only): also writes y with the K-interleave used by the MoE GEMMs
 *   (see knx_moe_w4); pass NULL to skip. */
#define KNX_RMS_ROUND_BF16 0x1
KNX_API int knx_rmsnorm(const void* x, const void* w, int w_dtype, void* y, void* xperm, int64_t rows,
                int64_t cols, float eps, int dtype, int flags, void* stream);

/* ---- router ------------------------------------------------------------------------------
 * DiffusionGemma router (transformers, not vendored; consumer signature pack_experts.py:44,65):
 * logits = x . Wr^T (+ bias), p = softmax(logits), top-k by logit (ties -> lower expert id),
 * weights renormalised over the selected k.  x: f16 [T,H]; wr: f16 [E,H]; bias: f32 [E] or
 * NULL; logits_out: f32 [T,E] or NULL; ids: i32 [T,topk]; weights: f32 [T,topk].
 * Requires H % 256 == 0, E % 32 == 0, E <= 256, topk <= min(16, E).
 * workspace: >= knx_router_workspace_size(T, E) bytes (K-split partial logits). */
KNX_API size_t knx_router_workspace_size(int64_t T, int E);
KNX_API int knx_router_topk(const void* x, const void* wr, const float* bias, int64_t T, int64_t H, int E,
                    int topk, float* logits_out, int32_t* ids, float* weights, void* workspace,
                    size_t workspace_bytes, void* stream);

/* ---- RMSNorm + router in one launch ---------------------------------------------------------
 * knx_rmsnorm (x and w F16, `flags` as there) followed by knx_router_topk on its output, as one
 * kernel: y, xperm, logits_out, ids and weights are bit-identical to that pair.  No reference
 * counterpart of its own: it fuses the two calls above.  x, y, xperm: f16 [T,H];
 * norm_w: f16 [H]; wr: f16 [E,H]; bias: f32 [E] or NULL; logits_out: f32 [T,E] or NULL;
 * ids: i32 [T,topk]; weights: f32 [T,topk].  No workspace.  Returns KNX_E_UNSUPPORTED unless
 * E is 64 or 128 and H % 256 == 0 with H <= 3840 (then use the two calls). */
KNX_API int knx_rmsnorm_router_topk(const void* x, const void* norm_w, float eps, int flags,
                                    const void* wr, const float* bias, int64_t T, int64_t H, int E,
                                    int topk, void* y, void* xperm, float* logits_out,
                                    int32_t* ids, float* weights, void* stream);

/* ---- permutation (moe_align) ------------------------------------------------------------
 * Replaces moe_align (fused_moe_w4.py:15-51) and moe_align_cuda/_align_finalize
 * (fused_moe_w4_v2.py:32-74): a deterministic counting sort of the flat (token, slot) pairs
 * p = t*topk + k by expert, stable in p.  Outputs, all int32:
 *   counts[E]        pairs per expert (ids outside [0,E) are dropped and not counted)
 *   offsets[E+1]     exclusive prefix of counts (unpadded slot start per expert)
 *   sorted_pair[N]   pair index at each unpadded slot, N = T*topk (tail = N for dropped)
 *   inv[N]           unpadded slot of pair p (-1 for dropped pairs)
 * With block_m > 0 it also writes the reference's BM-padded form:
 *   sorted_rows[cap] (pad = N), expert_ids[max_blocks] (pad = E), padded_inv[N];
 *   cap = max_blocks*block_m, max_blocks = ceil(N/block_m) + E (fused_moe_w4.py:36-37).
 * Pass NULL for any output not wanted.  ids_dtype is KNX_I32 or KNX_I64. */
KNX_API int knx_moe_align(const void* topk_ids, int ids_dtype, int64_t T, int topk, int E, int block_m,
                  int32_t* counts, int32_t* offsets, int32_t* sorted_pair, int32_t* inv,
                  int32_t* sorted_rows, int32_t* expert_ids, int32_t* padded_inv, int32_t* err,
                  void* stream);

/* The same unpadded permutation (counts, offsets, sorted_pair, inv as above) for any pair count
 * up to 2^30, by a multi-CTA counting sort (knx_moe_align's single CTA holds T*topk <= 32768).
 * scratch: >= knx_moe_align_large_scratch_size(T*topk, E) bytes, 16-byte aligned. */
KNX_API size_t knx_moe_align_large_scratch_size(int64_t N, int E);
KNX_API int knx_moe_align_large(const void* topk_ids, int ids_dtype, int64_t T, int topk, int E,
                                int32_t* counts, int32_t* offsets, int32_t* sorted_pair, int32_t* inv,
                                void* scratch, size_t scratch_bytes, int32_t* err, void* stream);

/* The same unpadded permutation for relabelled experts: pair p counts as expert relabel[ids[p]]
 * (relabel: E int32 on the device, a permutation of 0..E-1; a label outside it is reported as
 * KNX_DEV_BAD_EXPERT_ID and the pair dropped).  Used by the expert-parallel layer so that
 * round-robin ownership of the labels spreads the load.  scratch as knx_moe_align_large when
 * T*topk > 32768 (else unused). */
KNX_API int knx_moe_align_relabeled(const void* topk_ids, int ids_dtype, int64_t T, int topk, int E,
                                    const int32_t* relabel, int32_t* counts, int32_t* offsets,
                                    int32_t* sorted_pair, int32_t* inv, void* scratch,
                                    size_t scratch_bytes, int32_t* err, void* stream);

/* ---- one W4A16 MoE layer ------------------------------------------------------------------
 * Replaces fused_moe_w4_v2 (fused_moe_w4_v2.py:319-371) and fused_moe_w4 (fused_moe_w4.py:104-128).
 * Weight buffers are the pack_experts layout, read unchanged (pack_experts.py:34-41, 87-106):
 *   gu_q u8 [E, 2I, H/2]   gu_s, gu_z f16 [E, 2I, H/gs_gu]   (rows [0,I) gate, [I,2I) up)
 *   dn_q u8 [E, H, I/2]    dn_s, dn_z f16 [E, H, I/gs_dn]
 *   nibble j of a row: byte j/2, low nibble for even j; w = (q - z) * s.
 * out[t,:] = sum_{k=0..topk-1, fixed order} w[t,k] * down_e(gelu_tanh(gate_e(x_t)) * up_e(x_t)),
 *   each pair's down output rounded to f16 before the fp32 weighted sum (fused_moe_w4_v2.py:248-263).
 * hidden/out: [T,H] in hidden_dtype (F16/BF16; hidden is used as f16 like the reference);
 * topk_ids: [T,topk] i32/i64; topk_w: [T,topk] F16/BF16/F32.
 * hidden_perm: optional f16 [T,H] copy of hidden already in the MoE K-interleave (as written by
 *   knx_rmsnorm's xperm); NULL = the layer builds it in its workspace.
 * flags & KNX_W4_INT_ZEROS: the caller guarantees every zero-point is an integer in [0,15] (what
 *   quantize_w4 writes, w4a16.py:27); weights are then dequantised bit-identically to dequant_w4
 *   (one rounding of (q - z) * s).  Without it any fp16 zero-point is accepted and weights are
 *   RN16(RN16(q - z) * s), the fp16 arithmetic of the reference kernel (fused_moe_w4_v2.py:126-128).
 * Contracts (fused_moe_w4_v2.py:325-328): H % 256 == 0, I % 64 == 0, gs_gu % 32 == 0 and
 *   divides H, gs_dn % 32 == 0 and divides I, H/gs_gu <= 56, I/gs_dn <= 56, topk <= 16,
 *   E <= 256, T*topk <= 2^30 (above 32768 pairs the permutation is a multi-CTA sort).
 * workspace: >= knx_moe_w4_workspace_size(T, H, I, E, topk) bytes, 256-byte aligned. */
KNX_API size_t knx_moe_w4_workspace_size(int64_t T, int64_t H, int64_t I, int E, int topk);
KNX_API int knx_moe_w4(const void* hidden, const void* hidden_perm, int hidden_dtype, const void* topk_ids,
               int ids_dtype, const void* topk_w, int w_dtype, const uint8_t* gu_q,
               const void* gu_s, const void* gu_z, const uint8_t* dn_q, const void* dn_s,
               const void* dn_z, int64_t T, int64_t H, int64_t I, int E, int topk, int gs_gu,
               int gs_dn, int flags, void* workspace, size_t workspace_bytes, void* out,
               int32_t* err, void* stream);

/* ---- expert parallelism (experts sharded over ranks, tokens data-parallel) ------------------
 * No counterpart in the reference (single-GPU only).  The host drives, between two NCCL
 * all-to-all exchanges: knx_moe_align on the global expert ids (the single-GPU slot order),
 * knx_gather_rows (dispatch rows in that order), knx_ep_layout + knx_moe_w4_grouped on each
 * expert rank, knx_gather_rows (rows back to receive order), knx_moe_combine on the source.
 * The result is bit-identical to knx_moe_w4 on one GPU when tokens_per_expert (the job-wide
 * average, which picks the engine) is the same.  The combine order follows
 * fused_moe_w4_v2.py:248-263.
 *
 * knx_gather_rows: dst[i, :] = src[idx[i] / div, :] for i < n (idx[i] < 0: a zero row);
 *   row_bytes % 16 == 0, src/dst 16-byte aligned.
 * knx_ep_layout: received rows arrive grouped by source s (rank order), then by local expert e,
 *   then in the source's slot order; recv_counts[s * El + e] (device int32) holds the counts.
 *   Writes offsets[El + 1] (slots per local expert, expert-major), rows[R] (slot -> received row)
 *   and inv[R] (received row -> slot), R = sum of recv_counts.  S <= 64, El <= 256.
 * knx_moe_w4_grouped: gate_up + GELU and down for R rows grouped by expert: slot i of expert e
 *   (offsets[e] <= i < offsets[e+1]) multiplies row rows[i] of xrows (f16, MoE K-interleave;
 *   rows NULL = row i); out3[i, :] f16.  Weights, group sizes and flags as knx_moe_w4 (E = the
 *   local expert count); tokens_per_expert picks the engine.
 * knx_moe_combine: out[t, :] = sum_{k fixed order} w[t,k] * out3[inv[t*topk+k], :] (inv < 0:
 *   skipped), as in knx_moe_w4. */
KNX_API int knx_gather_rows(const void* src, int64_t src_rows, int64_t row_bytes, const int32_t* idx,
                            int div, int64_t n, void* dst, void* stream);
KNX_API int knx_ep_layout(const int32_t* recv_counts, int S, int El, int64_t R, int32_t* offsets,
                          int32_t* rows, int32_t* inv, void* stream);
KNX_API size_t knx_moe_w4_grouped_workspace_size(int64_t R, int64_t H, int64_t I, int E);
KNX_API int knx_moe_w4_grouped(const void* xrows, const int32_t* rows, int64_t R,
                               const int32_t* offsets, const uint8_t* gu_q, const void* gu_s,
                               const void* gu_z, const uint8_t* dn_q, const void* dn_s,
                               const void* dn_z, int64_t H, int64_t I, int E, int gs_gu, int gs_dn,
                               int flags, int64_t tokens_per_expert, void* workspace,
                               size_t workspace_bytes, void* out3, int32_t* err, void* stream);
KNX_API int knx_moe_combine(const void* out3, const int32_t* inv, const void* topk_w, int w_dtype,
                            int64_t T, int topk, int64_t H, int out_dtype, void* out, void* stream);

/* ---- expert parallelism over NVLink, device-initiated -----------------------------------
 * The exchange of the expert-parallel layer by direct stores into peer memory (no host sync,
 * no collective library in the data path).  No reference counterpart: the reference has no
 * expert parallelism; these replace the two all-to-alls of the layer above.  Every rank holds a
 * region of the same layout mapped into all peers (e.g. torch symmetric memory): flags (world
 * uint32), cnt [world][E] int32, receive rows [r_cap][H] f16, return rows [n_cap][H] f16.
 * peer_* are device arrays of `world` pointers to those regions on each rank (index = rank).
 * E = El * world, world <= 8, E <= 256; rank r owns the experts e = el * world + r (local
 * expert el; round-robin sharding, see ep_moe.shard_experts(..., interleaved=True); when the
 * counting sort relabels the experts (knx_moe_align_relabeled), e is the label).  epoch: one more than the previous barrier's, the same
 * on every rank (each call below that takes one is a barrier).  err: KNX_DEV_TIMEOUT when a
 * barrier waited 2 s.
 *   knx_ep_p2p_counts    counts[E] of this rank's pairs (knx_moe_align) to every peer; barrier;
 *                        writes the plan (knx_ep_p2p_plan_ints ints).  plan[E .. E + El] are
 *                        the offsets of this rank's local experts in its receive rows.
 *   knx_ep_p2p_dispatch  pair rows of xp [T][H] in align order (sorted_pair, offsets) into the
 *                        owners' receive rows, at the slots the grouped GEMMs read (n_cap >=
 *                        T*topk: slots beyond offsets[E] are skipped).
 *   knx_ep_p2p_barrier   a barrier.
 *   knx_ep_p2p_return    result rows out3 [r_cap][H] (local, expert-major) into the sources'
 *                        return rows at their align slots (for knx_moe_combine there).
 *   knx_ep_p2p_dispatch_barrier, knx_ep_p2p_return_barrier
 *                        dispatch (return) followed by the barrier in one launch: the CTA that
 *                        finishes last runs the barrier.  arrive: one device uint32 per entry
 *                        point, zero before the first call, owned by this rank (left at zero
 *                        after every call).  Every rank takes the barrier even with no rows. */
KNX_API size_t knx_ep_p2p_plan_ints(int E, int El, int world);
KNX_API int knx_ep_p2p_counts(const int32_t* counts, int E, int El, int rank, int world,
                              int32_t* const* peer_cnt, uint32_t* const* peer_flags,
                              uint32_t epoch, int32_t* plan, int32_t* err, void* stream);
KNX_API int knx_ep_p2p_dispatch(const void* xp, int64_t H, int topk, const int32_t* sorted_pair,
                                const int32_t* offsets, int E, int El, const int32_t* plan,
                                void* const* peer_rows, int64_t n_cap, void* stream);
KNX_API int knx_ep_p2p_dispatch_barrier(const void* xp, int64_t H, int topk,
                                        const int32_t* sorted_pair, const int32_t* offsets, int E,
                                        int El, const int32_t* plan, void* const* peer_rows,
                                        int64_t n_cap, uint32_t* const* peer_flags, int rank,
                                        int world, uint32_t epoch, uint32_t* arrive, int32_t* err,
                                        void* stream);
KNX_API int knx_ep_p2p_return_barrier(const void* out3, int64_t H, int El, int world, int E,
                                      const int32_t* plan, void* const* peer_ret, int64_t r_cap,
                                      uint32_t* const* peer_flags, int rank, uint32_t epoch,
                                      uint32_t* arrive, int32_t* err, void* stream);
KNX_API int knx_ep_p2p_barrier(uint32_t* const* peer_flags, int rank, int world, uint32_t epoch,
                               int32_t* err, void* stream);
KNX_API int knx_ep_p2p_return(const void* out3, int64_t H, int El, int world, int E,
                              const int32_t* plan, void* const* peer_ret, int64_t r_cap,
                              void* stream);

/* ---- dense W4A16 linear -------------------------------------------------------------------
 * Replaces w4a16_linear (w4a16.py:96-108):  Y[M,N] = X[M,K] . dequant(q,s,z)^T, f16 out.
 * X: f16 [M,K] row-major; q u8 [N,K/2]; s,z f16 [N,K/gs].  K % 64 == 0, gs % 32 == 0, gs | K,
 * K/gs <= 56, N % 8 == 0.  flags: KNX_W4_INT_ZEROS as for knx_moe_w4.
 * workspace: >= knx_w4a16_workspace_size(M, K) bytes. */
KNX_API size_t knx_w4a16_workspace_size(int64_t M, int64_t K);
KNX_API int knx_w4a16_linear(const void* X, const uint8_t* q, const void* s, const void* z, int64_t M,
                     int64_t N, int64_t K, int gs, int flags, void* Y, void* workspace,
                     size_t workspace_bytes, void* stream);

/* ---- sampler ------------------------------------------------------------------------------
 * One streaming pass over fp32 logits [rows, V] that fuses, per row r:
 *   q = x / temperature (IEEE-rounded division; temperature == 1 leaves x unchanged)
 *   entropy[r] = logsumexp(q) - sum(q*exp(q-m))/sum(exp(q-m))  (fused_sampler_ops.py:22-40)
 *   samp[r]    = first argmax_c (q_c + g_c), g_c = -log(-log(clamp(u_c, 1e-10, 1-1e-7))),
 *                u_c = uniform(Philox4x32-10(key = seed + r, counter = (c,0,0,0)) word 0)
 *                exactly as Triton's tl.rand(seed + r, c) (fused_sampler_ops.py:54-81)
 *   amax[r]    = first argmax_c q_c
 * Any of entropy/samp/amax may be NULL.  V <= 2^31 - 1.
 * workspace: >= knx_sampler_workspace_size(rows, V) bytes. */
KNX_API size_t knx_sampler_workspace_size(int64_t rows, int64_t V);
KNX_API int knx_sampler_fused(const float* logits, int64_t rows, int64_t V, float temperature,
                      int64_t seed, float* entropy, int64_t* samp, int64_t* amax,
                      void* workspace, size_t workspace_bytes, void* stream);

/* knx_sampler_fused plus the denoising step's self-conditioning copy in the same pass over the
 * logits.  Replaces the end of the reference step (fast_sampler.py:103-109):
 *   processed = where(finished[:, None, None], self_conditioning_logits, processed)
 *   self_conditioning_logits = processed.to(bfloat16)
 * i.e. sc_out[r, :] = (finished && finished[r / canvas_len]) ? sc_prev[r, :] : bf16(x[r, :] / T),
 * with x / T the IEEE quotient the sampler uses and round-to-nearest-even (NaN -> 0x7FC0).
 * sc_out, sc_prev: bf16 [rows, V] (sc_prev may be sc_out itself); finished: one byte per canvas
 * of canvas_len rows (NULL: no canvas has finished; then sc_prev may be NULL).
 * entropy/samp/amax are bit-identical to knx_sampler_fused's.  With V % 4 == 0 and 8-byte aligned
 * bf16 buffers the copy is written by the sampling pass itself; otherwise one elementwise launch
 * follows it. */
KNX_API int knx_sampler_fused_sc(const float* logits, int64_t rows, int64_t V, float temperature,
                                 int64_t seed, float* entropy, int64_t* samp, int64_t* amax,
                                 void* sc_out, const void* sc_prev, const uint8_t* finished,
                                 int64_t canvas_len, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* knx_sampler_fused without a workspace argument, for callers that cannot allocate device memory
 * when they sample (FFI hosts without a CUDA allocator, serving loops whose device memory is
 * frozen after warm-up).  No counterpart in the reference: its sampler allocates its outputs and
 * temporaries through torch on every call.  Same outputs as knx_sampler_fused.
 * Scratch is a fixed KNX_SAMPLER_STATIC_SCRATCH_BYTES array inside the library, one per device:
 *   - calls needing more (knx_sampler_workspace_size(rows, V) > the limit; more than 3,969 rows
 *     at V = 262144) return KNX_E_WORKSPACE without launching anything;
 *   - the first call on a device looks the array up (cudaGetSymbolAddress with that device
 *     current); make it before any stream capture begins;
 *   - that address is kept for the life of the process: after cudaDeviceReset (or any other
 *     teardown of the device's primary context) it is stale, so do not call this entry point
 *     on that device again in the same process;
 *   - tickets/bounds/counter are zeroed in stream order by every call;
 *   - calls that can overlap in time on one device (other streams, unordered host threads) race
 *     on the shared scratch; calls in order on one stream are safe.
 * Allocates nothing (no cudaMalloc/cudaFree, no allocating library). */
#define KNX_SAMPLER_STATIC_SCRATCH_BYTES (1u << 20)
KNX_API int knx_sampler_fused_static(const float* logits, int64_t rows, int64_t V,
                                     float temperature, int64_t seed, float* entropy,
                                     int64_t* samp, int64_t* amax, void* stream);

/* Entropy-bound acceptance and the stable-and-confident stop test, one launch per batch.
 * Replaces _accept_canvas (fast_sampler.py:32-42) and _stop_call (fast_sampler.py:45-65).
 * entropy f32 [B,L]; cur, proposal, out i64 [B,L]; mask u8 [B,L] (1 = accepted):
 *   order = stable ascending sort of entropy; cum = running fp64 sum rounded to fp32;
 *   accepted = (cum - sorted_entropy) <= entropy_bound;  out = accepted ? proposal : cur.
 * Stop test (when finished != NULL): history i64 [S,B,L] of the last S argmax canvases
 *   (initialised to -1 by the caller), argmax i64 [B,L]:
 *   stable = S == 0 || all(history[s] == argmax); history rolls by one and stores argmax;
 *   confident = (fp64 sum of entropy / L, rounded to fp32) < confidence_threshold;
 *   finished[b] = stable && confident (u8).  L <= 1024. */
KNX_API int knx_accept_stop(const float* entropy, const int64_t* cur, const int64_t* proposal, int64_t B,
                    int64_t L, float entropy_bound, uint8_t* mask, int64_t* out,
                    const int64_t* argmax, int64_t* history, int stability_threshold,
                    float confidence_threshold, uint8_t* finished, void* stream);

/* ---- stage profiling (benchmarks) --------------------------------------------------------
 * knx_prof_start(max_calls): from now on knx_moe_w4 records a CUDA event at each of its stage
 * boundaries (prep = K-interleave copy + align, gate_up+GELU GEMM, down GEMM, combine) for up to
 * max_calls calls, without synchronising.  knx_prof_stop(stage_ms, n_stages, ncalls) waits for the
 * recorded events, writes the per-stage device time summed over the recorded calls and the number
 * of calls, and turns recording off.  Not thread-safe; meant for single-threaded benchmarks. */
#define KNX_PROF_STAGES 4
KNX_API int knx_prof_start(int max_calls);
KNX_API int knx_prof_stop(float* stage_ms, int n_stages, int* ncalls);

#ifdef __cplusplus
}
#endif
#endif /* KNX_H_ */
