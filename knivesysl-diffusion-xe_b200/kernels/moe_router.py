"""moe_router.py — the DiffusionGemma MoE router on sm_100a.

route_topk(x, router_weight, top_k, bias=None) -> (ids i32[T,k], weights f32[T,k], logits f32[T,E])
  logits = x . Wr^T (+ bias); p = softmax(logits); top-k by logit, ties to the lower expert id;
  weights = p_top / sum(p_top).  This is the router behaviour consumed by experts.forward
  (pack_experts.py:44,65 of the reference); the model code itself lives in transformers.
"""
import torch

from _knx import check, load, ptr, require_device, stream_of, workspace


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
