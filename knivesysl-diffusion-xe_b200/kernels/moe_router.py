"""moe_router.py — the DiffusionGemma MoE router on sm_100a.

route_topk(x, router_weight, top_k, bias=None) -> (ids i32[T,k], weights f32[T,k], logits f32[T,E])
  logits = x . Wr^T (+ bias); p = softmax(logits); top-k by logit, ties to the lower expert id;
  weights = p_top / sum(p_top).  This is the router behaviour consumed by experts.forward
  (pack_experts.py:44,65 of the reference); the model code itself lives in transformers.
"""
import torch

from _knx import (KNX_RMS_ROUND_BF16, check, load, ptr, require_device, stream_of,
                  workspace)


def route_topk(x, router_weight, top_k, bias=None, want_logits=True):
    dev = require_device(x)
    T, H = x.shape
    E = router_weight.shape[0]
    xh = x.contiguous().to(torch.float16)
    wr = router_weight.contiguous().to(torch.float16)
    b = bias.contiguous().float() if bias is not None else None
    ids = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    logits = torch.empty(T, E, dtype=torch.float32, device=x.device) if want_logits else None
    lib = load()
    ws = workspace(dev, lib.knx_router_workspace_size(T, E), "router")
    check(lib.knx_router_topk(ptr(xh), ptr(wr), ptr(b), T, H, E, int(top_k), ptr(logits), ptr(ids),
                              ptr(w), ptr(ws), ws.numel(), stream_of(dev)), "knx_router_topk")
    return ids, w, logits


KNX_E_UNSUPPORTED = -5
FUSED_MAX_TOKENS = 512


def rmsnorm_route_topk(x, norm_weight, eps, router_weight, top_k, bias=None, xperm=None,
                       round_bf16=True, want_logits=True):
    """fused_rmsnorm(x, norm_weight, eps, round_bf16, xperm) then route_topk on its output, as one
    launch where the shapes allow (f16 x and weights, E in {64, 128}, H % 256 == 0, H <= 3840)
    and the batch is a canvas (T <= FUSED_MAX_TOKENS: one cluster of 8 CTAs per 32 tokens, and
    only ~15 such clusters are resident at once on a B200); otherwise as the two calls.  Same
    bits either way.  -> (y, ids, weights, logits)."""
    import fused_rmsnorm
    dev = require_device(x)
    T, H = x.shape
    E = router_weight.shape[0]
    if (T <= FUSED_MAX_TOKENS and x.dtype == torch.float16 and norm_weight is not None
            and norm_weight.dtype == torch.float16 and router_weight.dtype == torch.float16):
        xc = x.contiguous()
        nw = norm_weight.contiguous()
        wr = router_weight.contiguous()
        b = bias.contiguous().float() if bias is not None else None
        y = torch.empty_like(xc)
        ids = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
        logits = torch.empty(T, E, dtype=torch.float32, device=x.device) if want_logits else None
        st = load().knx_rmsnorm_router_topk(ptr(xc), ptr(nw), float(eps),
                                            KNX_RMS_ROUND_BF16 if round_bf16 else 0, ptr(wr), ptr(b),
                                            T, H, E, int(top_k), ptr(y), ptr(xperm), ptr(logits),
                                            ptr(ids), ptr(w), stream_of(dev))
        if st != KNX_E_UNSUPPORTED:
            check(st, "knx_rmsnorm_router_topk")
            return y, ids, w, logits
    y = fused_rmsnorm.fused_rmsnorm(x, norm_weight, eps, round_bf16=round_bf16, xperm=xperm)
    ids, w, logits = route_topk(y, router_weight, top_k, bias=bias, want_logits=want_logits)
    return y, ids, w, logits
