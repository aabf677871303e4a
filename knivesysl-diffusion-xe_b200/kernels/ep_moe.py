"""ep_moe.py — the W4A16 MoE layer with its experts sharded over ranks (expert parallelism).

Rank r of N holds experts [r*E/N, (r+1)*E/N) and its own tokens (data-parallel canvases or a
slice of a prefill batch).  One layer is

    align (global expert ids: the single-GPU slot order, experts ascending then pair t*k+j)
    -> gather the pairs' activation rows in that order -> all-to-all (dispatch)
    -> re-slot the received rows expert-major -> grouped gate_up + GELU, down (local experts)
    -> rows back to receive order -> all-to-all (return)
    -> the fixed-order weighted combine of fused_moe_w4_v2.py:248-263 on the source rank.

Every pair's down output is computed by the same engine from the same activation row and weights
as on one GPU, and the returned rows reach the combine in the single-GPU slot order, so the output
is bit-identical to the single-GPU layer at any rank count.  The engine is chosen from the
job-wide tokens per expert, identically on every rank.  Two NCCL all-to-alls carry the rows; one
small all-to-all carries the per-expert counts, and their per-rank sums are read on the host once
per layer (all_to_all_single needs host split sizes).

The device steps come from an `ops` object: CudaOps runs the sm_100a kernels through libknx.so
(the only implementation shipped); tests substitute CPU stand-ins to check the host logic on gloo.
"""
import torch
import torch.distributed as dist

from _knx import (KNX_DEV_TIMEOUT, KNX_W4_INT_ZEROS, check, dtype_code, engine_flags, load, ptr,
                  require_device, stream_of, workspace, zero_flags)


class CudaOps:
    """The device steps on sm_100a (libknx.so)."""

    def align(self, ids, E, relabel=None):
        from fused_moe_w4 import moe_align_unpadded
        return moe_align_unpadded(ids, E, relabel)

    def gather_rows(self, src, idx, div, n):
        dev = require_device(src)
        dst = torch.empty((n,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
        row_bytes = src[0].numel() * src.element_size() if src.shape[0] else dst[0].numel() * dst.element_size()
        check(load().knx_gather_rows(ptr(src), src.shape[0], row_bytes, ptr(idx), int(div), n,
                                     ptr(dst), stream_of(dev)), "knx_gather_rows")
        return dst

    def layout(self, recv_counts, R):
        dev = require_device(recv_counts)
        S, El = recv_counts.shape
        i32 = dict(dtype=torch.int32, device=recv_counts.device)
        offsets = torch.empty(El + 1, **i32)
        rows = torch.empty(R, **i32)
        inv = torch.empty(R, **i32)
        check(load().knx_ep_layout(ptr(recv_counts.contiguous()), S, El, R, ptr(offsets), ptr(rows),
                                   ptr(inv), stream_of(dev)), "knx_ep_layout")
        return offsets, rows, inv

    def grouped(self, xrows, rows, offsets, weights, tokens_per_expert, flags):
        dev = require_device(xrows)
        gu_q, gu_s, gu_z, dn_q, dn_s, dn_z = weights
        R, H = xrows.shape
        El, twoI, _ = gu_q.shape
        I = twoI // 2
        out3 = torch.empty(R, H, dtype=torch.float16, device=xrows.device)
        lib = load()
        ws = workspace(dev, lib.knx_moe_w4_grouped_workspace_size(R, H, I, El), "ep_grouped")
        check(lib.knx_moe_w4_grouped(ptr(xrows), ptr(rows), R, ptr(offsets), ptr(gu_q), ptr(gu_s),
                                     ptr(gu_z), ptr(dn_q), ptr(dn_s), ptr(dn_z), H, I, El,
                                     H // gu_s.shape[-1], I // dn_s.shape[-1], flags,
                                     int(tokens_per_expert), ptr(ws), ws.numel(), ptr(out3), None,
                                     stream_of(dev)), "knx_moe_w4_grouped")
        return out3

    def grouped_rows(self, xrows, offsets, weights, tokens_per_expert, flags):
        """grouped() for rows already in slot order (row = slot); xrows: [R_cap, H]."""
        dev = require_device(xrows)
        gu_q, gu_s, gu_z, dn_q, dn_s, dn_z = weights
        R, H = xrows.shape
        El, twoI, _ = gu_q.shape
        I = twoI // 2
        out3 = torch.empty(R, H, dtype=torch.float16, device=xrows.device)
        lib = load()
        ws = workspace(dev, lib.knx_moe_w4_grouped_workspace_size(R, H, I, El), "ep_grouped")
        check(lib.knx_moe_w4_grouped(ptr(xrows), None, R, ptr(offsets), ptr(gu_q), ptr(gu_s),
                                     ptr(gu_z), ptr(dn_q), ptr(dn_s), ptr(dn_z), H, I, El,
                                     H // gu_s.shape[-1], I // dn_s.shape[-1], flags,
                                     int(tokens_per_expert), ptr(ws), ws.numel(), ptr(out3), None,
                                     stream_of(dev)), "knx_moe_w4_grouped")
        return out3

    def combine(self, out3, inv, w, T, out_dtype):
        dev = require_device(out3)
        H = out3.shape[1]
        tk = w.shape[1]
        y = torch.empty(T, H, dtype=out_dtype, device=w.device)
        check(load().knx_moe_combine(ptr(out3), ptr(inv), ptr(w), dtype_code(w.dtype), T, tk, H,
                                     dtype_code(out_dtype), ptr(y), stream_of(dev)),
              "knx_moe_combine")
        return y


class ExpertParallelMoE:
    """One W4A16 MoE layer over the ranks of `group`; this rank holds the local experts given.

    gu_q/gu_s/gu_z/dn_q/dn_s/dn_z: the pack_experts buffers of this rank's E_total / N experts
    (contiguous slices of the full [E_total, ...] tensors)."""

    def __init__(self, gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, E_total, group=None, ops=None,
                 engine=None, int_zeros=None):
        self.weights = (gu_q, gu_s, gu_z, dn_q, dn_s, dn_z)
        self.E = E_total
        self.group = group
        self.N = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        assert E_total % self.N == 0, f"{E_total} experts do not shard over {self.N} ranks"
        self.El = E_total // self.N
        assert gu_q.shape[0] == self.El, "local expert buffers must hold E_total / N experts"
        self.ops = ops or CudaOps()
        if int_zeros is None:
            flags = zero_flags(gu_z, dn_z) if gu_z.is_cuda else 0
        else:
            flags = KNX_W4_INT_ZEROS if int_zeros else 0
        self.flags = flags | engine_flags(engine)

    @torch.no_grad()
    def forward(self, x, topk_ids, topk_w, out_dtype=torch.float16, tokens_per_expert=None):
        """x: this rank's activation rows [T, H] (f16, MoE K-interleave on the device path);
        topk_ids/topk_w: [T, k].  tokens_per_expert: the job-wide (token, slot) pairs per expert
        (picks the GEMM engine; default: all-reduced from the ranks' T)."""
        N, El, E = self.N, self.El, self.E
        T, H = x.shape
        tk = topk_ids.shape[1]
        if tokens_per_expert is None:
            tot = torch.tensor([T * tk], dtype=torch.int64, device=x.device)
            if N > 1:
                dist.all_reduce(tot, group=self.group)
            tokens_per_expert = int(tot.item()) // E
        counts, offsets, sorted_pair, inv = self.ops.align(topk_ids, E)
        counts = counts.to(torch.int32)
        recv_counts = torch.empty_like(counts)
        if N > 1:
            dist.all_to_all_single(recv_counts, counts, group=self.group)
        else:
            recv_counts.copy_(counts)
        send_split = counts.view(N, El).sum(1)
        recv_split = recv_counts.view(N, El).sum(1)
        sizes = torch.cat([send_split, recv_split]).cpu().tolist()  # host split sizes
        send_split, recv_split = sizes[:N], sizes[N:]
        n_send, n_recv = sum(send_split), sum(recv_split)
        sendbuf = self.ops.gather_rows(x, sorted_pair, tk, n_send)
        if N > 1:
            recvbuf = torch.empty((n_recv, H), dtype=x.dtype, device=x.device)
            dist.all_to_all_single(recvbuf, sendbuf, recv_split, send_split, group=self.group)
        else:
            recvbuf = sendbuf
        loc_off, loc_rows, loc_inv = self.ops.layout(recv_counts.view(N, El), n_recv)
        out3_loc = self.ops.grouped(recvbuf, loc_rows, loc_off, self.weights, tokens_per_expert,
                                    self.flags)
        backbuf = self.ops.gather_rows(out3_loc, loc_inv, 1, n_recv)
        if N > 1:
            retbuf = torch.empty((n_send, H), dtype=out3_loc.dtype, device=x.device)
            dist.all_to_all_single(retbuf, backbuf, send_split, recv_split, group=self.group)
        else:
            retbuf = backbuf
        return self.ops.combine(retbuf, inv, topk_w.contiguous(), T, out_dtype)

    __call__ = forward


def shard_experts(gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, rank, world, interleaved=False, order=None):
    """This rank's experts of full pack_experts buffers: the contiguous slice
    [rank * E / world, (rank + 1) * E / world) (ExpertParallelMoE), or with interleaved=True the
    experts rank, rank + world, ... (P2PExpertParallelMoE).  order (with interleaved=True): the
    expert behind each label (balanced_relabel), so that this rank holds the experts labelled
    rank, rank + world, ..."""
    E = gu_q.shape[0]
    El = E // world
    if order is not None:
        if not interleaved:
            raise ValueError("order needs interleaved=True")
        idx = torch.as_tensor(list(order), dtype=torch.long)[rank::world].to(gu_q.device)
        return tuple(t.index_select(0, idx).contiguous() for t in (gu_q, gu_s, gu_z, dn_q, dn_s, dn_z))
    sl = slice(rank, E, world) if interleaved else slice(rank * El, (rank + 1) * El)
    return tuple(t[sl].contiguous() for t in (gu_q, gu_s, gu_z, dn_q, dn_s, dn_z))


def balanced_relabel(counts, world, task_tokens=32):
    """Labels for the experts so that round-robin ownership of the labels (rank r holds labels
    r, r + world, ...) balances the grouped-GEMM work: experts by descending task count
    (ceil(pairs / task_tokens); ties by expert id) go to the least loaded rank that still has room
    (E / world each; ties to the lower rank), and rank r's k-th expert gets label k * world + r.
    counts: pairs per expert over the whole job (e.g. measured on a calibration batch).
    -> (relabel, order): relabel[e] = label of expert e, order[label] = expert."""
    import math
    counts = [int(c) for c in counts]
    E = len(counts)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    cap = E // world
    load = [0] * world
    owned = [[] for _ in range(world)]
    for e in sorted(range(E), key=lambda e: (-math.ceil(counts[e] / task_tokens), e)):
        r = min((r for r in range(world) if len(owned[r]) < cap), key=lambda r: (load[r], r))
        owned[r].append(e)
        load[r] += math.ceil(counts[e] / task_tokens)
    relabel = [0] * E
    order = [0] * E
    for r in range(world):
        for k, e in enumerate(owned[r]):
            relabel[e] = k * world + r
            order[k * world + r] = e
    return relabel, order


class _P2PExchange:
    """One symmetric region per rank (torch symmetric memory, mapped into every peer) for the
    device-initiated exchange: flags | counts [world][E] | receive rows [r_cap][H] | return rows
    [n_cap][H].  Shared by every layer with the same group and sizes (layers run one after the
    other on the stream, and the barriers order each layer's use of the region after the last)."""

    _cache = {}

    @classmethod
    def get(cls, group, E, n_cap, H, device):
        key = (id(group), E, n_cap, H, str(device))
        ex = cls._cache.get(key)
        if ex is None:
            ex = cls._cache[key] = cls(group, E, n_cap, H, device)
        return ex

    def __init__(self, group, E, n_cap, H, device):
        import torch.distributed._symmetric_memory as symm_mem
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E, self.El, self.n_cap, self.H = E, E // self.world, n_cap, H
        self.r_cap = n_cap * self.world  # every pair of every rank could go to one owner
        al = lambda b: (b + 255) & ~255
        self.off_flags = 0
        self.off_cnt = al(64 * 4)
        self.off_rows = al(self.off_cnt + self.world * E * 4)
        self.off_ret = al(self.off_rows + self.r_cap * H * 2)
        total = al(self.off_ret + n_cap * H * 2)
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        if hasattr(symm_mem, "enable_symm_mem_for_group") and not symm_mem.is_symm_mem_enabled_for_group(grp.group_name):
            symm_mem.enable_symm_mem_for_group(grp.group_name)
        self.hdl = symm_mem.rendezvous(self.buf, grp)
        bases = [int(b) for b in self.hdl.buffer_ptrs]
        i64 = dict(dtype=torch.int64, device=device)
        self.peer_flags = torch.tensor([b + self.off_flags for b in bases], **i64)
        self.peer_cnt = torch.tensor([b + self.off_cnt for b in bases], **i64)
        self.peer_rows = torch.tensor([b + self.off_rows for b in bases], **i64)
        self.peer_ret = torch.tensor([b + self.off_ret for b in bases], **i64)
        self.rows = self.buf[self.off_rows:self.off_rows + self.r_cap * H * 2].view(torch.float16).view(self.r_cap, H)
        self.ret = self.buf[self.off_ret:self.off_ret + n_cap * H * 2].view(torch.float16).view(n_cap, H)
        self.plan = torch.empty(load().knx_ep_p2p_plan_ints(E, self.El, self.world), dtype=torch.int32,
                                device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        # arrival counters of the fused dispatch + barrier and return + barrier launches
        self.arrive = torch.zeros(2, dtype=torch.int32, device=device)
        self.epoch = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals

    def next_epoch(self):
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        return self.epoch


class P2PExpertParallelMoE(ExpertParallelMoE):
    """ExpertParallelMoE with the exchange done by the device over NVLink: the pairs' rows are
    stored straight into the owning ranks' memory and the results straight back (three
    device-side barriers per layer, two of them run by the last CTA of the copy launch before
    them), so no step of the layer waits for the host.  The local
    experts are rank, rank + world, ... (shard_experts(..., interleaved=True)), or with
    relabel the experts labelled so (shard_experts(..., interleaved=True, order=...) with the
    same balanced_relabel result): the router's ids are relabelled inside the counting sort.
    Needs every rank on one node with peer access, and the same token count T <= max_tokens on
    every rank.  The output is bit-identical to ExpertParallelMoE and to the single-GPU layer
    (relabelling moves experts between ranks; every expert sees the same rows in the same order)."""

    def __init__(self, gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, E_total, group=None, engine=None,
                 int_zeros=None, max_tokens=256, topk=8, relabel=None):
        super().__init__(gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, E_total, group=group, ops=CudaOps(),
                         engine=engine, int_zeros=int_zeros)
        H = gu_q.shape[2] * 2
        self.ex = _P2PExchange.get(group, E_total, max_tokens * topk, H, gu_q.device)
        self.relabel = (None if relabel is None else
                        torch.as_tensor(list(relabel), dtype=torch.int32).to(gu_q.device))
        # set to a list to get (stage name, CUDA event) marks recorded on the stream between
        # the layer's stages (benchmark breakdowns; records stop the kernels from overlapping)
        self.stage_events = None

    def _mark(self, name):
        if self.stage_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.stage_events.append((name, ev))

    @torch.no_grad()
    def forward(self, x, topk_ids, topk_w, out_dtype=torch.float16, tokens_per_expert=None):
        """x: this rank's activation rows [T, H] (f16, MoE K-interleave); topk_ids/topk_w:
        [T, k].  tokens_per_expert: the job-wide pairs per expert (engine choice); default
        T * k * world / E (every rank holds T tokens)."""
        ex, lib = self.ex, load()
        T, H = x.shape
        tk = topk_ids.shape[1]
        if T * tk > ex.n_cap:
            raise ValueError(f"{T} tokens x top-{tk} exceed the exchange capacity {ex.n_cap}")
        if tokens_per_expert is None:
            tokens_per_expert = T * tk * self.N // self.E
        dev = require_device(x)
        st = stream_of(dev)
        self._mark("start")
        counts, offsets, sorted_pair, inv = self.ops.align(topk_ids, self.E, self.relabel)
        counts = counts.to(torch.int32)
        E, El, world, rank = self.E, self.El, self.N, self.rank
        self._mark("align")
        check(lib.knx_ep_p2p_counts(ptr(counts), E, El, rank, world, ptr(ex.peer_cnt),
                                    ptr(ex.peer_flags), ex.next_epoch(), ptr(ex.plan), ptr(ex.err),
                                    st), "knx_ep_p2p_counts")
        self._mark("counts+barrier+plan")
        check(lib.knx_ep_p2p_dispatch_barrier(ptr(x.contiguous()), H, tk, ptr(sorted_pair),
                                              ptr(offsets), E, El, ptr(ex.plan), ptr(ex.peer_rows),
                                              T * tk, ptr(ex.peer_flags), rank, world,
                                              ex.next_epoch(), ptr(ex.arrive[0:1]), ptr(ex.err), st),
              "knx_ep_p2p_dispatch_barrier")
        self._mark("dispatch+barrier")
        recv_off = ex.plan[E:E + El + 1]
        out3 = self.ops.grouped_rows(ex.rows, recv_off, self.weights, tokens_per_expert, self.flags)
        self._mark("grouped_gemms")
        check(lib.knx_ep_p2p_return_barrier(ptr(out3), H, El, world, E, ptr(ex.plan),
                                            ptr(ex.peer_ret), ex.r_cap, ptr(ex.peer_flags), rank,
                                            ex.next_epoch(), ptr(ex.arrive[1:2]), ptr(ex.err), st),
              "knx_ep_p2p_return_barrier")
        self._mark("return+barrier")
        y = self.ops.combine(ex.ret[:T * tk], inv, topk_w.contiguous(), T, out_dtype)
        self._mark("combine")
        return y

    __call__ = forward

    def check_errors(self):
        """Read and clear the exchange's device error word (one host synchronisation).  Raises
        RuntimeError when a device-side barrier gave up because a peer did not arrive within
        2 s: every layer run through this exchange since the previous check may have returned
        invalid rows (after a failed counts barrier the plan is empty, so nothing is written
        into the peers and the GEMMs do nothing).  Call it where a sync is acceptable, e.g. once
        per denoising step; forward() itself never synchronises."""
        bad = int(self.ex.err.item())
        self.ex.err.zero_()
        if bad & KNX_DEV_TIMEOUT:
            raise RuntimeError("expert-parallel exchange: a device-side barrier timed out "
                               "(a peer rank did not arrive within 2 s)")
        return bad
