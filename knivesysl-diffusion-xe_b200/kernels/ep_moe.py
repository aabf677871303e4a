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

from _knx import (KNX_W4_INT_ZEROS, check, dtype_code, engine_flags, load, ptr, require_device,
                  stream_of, workspace, zero_flags)


class CudaOps:
    """The device steps on sm_100a (libknx.so)."""

    def align(self, ids, E):
        from fused_moe_w4 import moe_align_unpadded
        return moe_align_unpadded(ids, E)

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


def shard_experts(gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, rank, world):
    """This rank's contiguous expert slice of full pack_experts buffers."""
    E = gu_q.shape[0]
    El = E // world
    sl = slice(rank * El, (rank + 1) * El)
    return tuple(t[sl].contiguous() for t in (gu_q, gu_s, gu_z, dn_q, dn_s, dn_z))
