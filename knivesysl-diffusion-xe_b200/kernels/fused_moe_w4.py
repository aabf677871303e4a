"""fused_moe_w4.py — moe_align and the v1 entry point (drop-in for the reference module).

moe_align(topk_ids, block_m, E) returns exactly what the reference's torch version returns
(fused_moe_w4.py:15-51): (sorted_rows int64[cap], expert_ids int64[max_blocks], cap, inv
int64[Nexp]) with pad sentinels Nexp / E, dropped pairs (id == E) excluded and inv = 0 for them.
It is computed by one counting-sort launch instead of ~14 torch ops.

fused_moe_w4(hidden, exp, topk_ids, topk_w) runs the same sm_100a layer as fused_moe_w4_v2
(the activation must be tanh-GELU, which the kernel fuses).
"""
import torch

from _knx import check, dtype_code, load, ptr, require_device, stream_of, workspace

BLOCK_M = 64


@torch.no_grad()
def moe_align_raw(topk_ids, block_m, E):
    """int32 outputs of the counting sort in the reference's BM-padded form."""
    dev = require_device(topk_ids)
    T, tk = topk_ids.shape
    Nexp = T * tk
    max_blocks = (Nexp + block_m - 1) // block_m + E
    cap = max_blocks * block_m
    ids = topk_ids.contiguous()
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.long()
    i32 = dict(dtype=torch.int32, device=topk_ids.device)
    sorted_rows = torch.empty(cap, **i32)
    expert_ids = torch.empty(max_blocks, **i32)
    inv = torch.empty(Nexp, **i32)
    check(load().knx_moe_align(ptr(ids), dtype_code(ids.dtype), T, tk, E, block_m, None, None, None,
                               None, ptr(sorted_rows), ptr(expert_ids), ptr(inv), None,
                               stream_of(dev)), "knx_moe_align")
    return sorted_rows, expert_ids, cap, inv


@torch.no_grad()
def moe_align(topk_ids, block_m, E):
    sorted_rows, expert_ids, cap, inv = moe_align_raw(topk_ids, block_m, E)
    return sorted_rows.long(), expert_ids.long(), cap, inv.long()


@torch.no_grad()
def moe_align_unpadded(topk_ids, E, relabel=None):
    """(counts i32[E], offsets i32[E+1], sorted_pair i32[N], inv i32[N]): the unpadded stable
    permutation the GEMMs use (inv = -1 for dropped pairs).  relabel: optional int32 device
    tensor of E labels (a permutation of 0..E-1); pair p then counts as expert relabel[ids[p]]."""
    dev = require_device(topk_ids)
    T, tk = topk_ids.shape
    N = T * tk
    ids = topk_ids.contiguous()
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.long()
    i32 = dict(dtype=torch.int32, device=topk_ids.device)
    counts = torch.empty(E, **i32)
    offsets = torch.empty(E + 1, **i32)
    sorted_pair = torch.empty(N, **i32)
    inv = torch.empty(N, **i32)
    lib = load()
    if relabel is not None:
        if relabel.dtype != torch.int32 or relabel.numel() != E or relabel.device != topk_ids.device:
            raise ValueError("relabel must be an int32 tensor of E labels on the ids' device")
        nbytes = lib.knx_moe_align_large_scratch_size(N, E) if N > 32768 else 0
        scratch = workspace(dev, nbytes, "align_large") if nbytes else None
        check(lib.knx_moe_align_relabeled(ptr(ids), dtype_code(ids.dtype), T, tk, E,
                                          ptr(relabel.contiguous()), ptr(counts), ptr(offsets),
                                          ptr(sorted_pair), ptr(inv), ptr(scratch),
                                          scratch.numel() if scratch is not None else 0, None,
                                          stream_of(dev)), "knx_moe_align_relabeled")
    elif N <= 32768:
        check(lib.knx_moe_align(ptr(ids), dtype_code(ids.dtype), T, tk, E, 0, ptr(counts),
                                ptr(offsets), ptr(sorted_pair), ptr(inv), None, None, None, None,
                                stream_of(dev)), "knx_moe_align")
    else:  # more pairs than one CTA holds: the multi-CTA counting sort
        scratch = workspace(dev, lib.knx_moe_align_large_scratch_size(N, E), "align_large")
        check(lib.knx_moe_align_large(ptr(ids), dtype_code(ids.dtype), T, tk, E, ptr(counts),
                                      ptr(offsets), ptr(sorted_pair), ptr(inv), ptr(scratch),
                                      scratch.numel(), None, stream_of(dev)), "knx_moe_align_large")
    return counts, offsets, sorted_pair, inv


@torch.no_grad()
def fused_moe_w4(hidden, exp, topk_ids, topk_w):
    """One MoE layer, fused (same kernels as fused_moe_w4_v2)."""
    from fused_moe_w4_v2 import fused_moe_w4_v2
    return fused_moe_w4_v2(hidden, exp, topk_ids, topk_w)
