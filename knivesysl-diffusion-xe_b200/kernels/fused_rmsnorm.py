"""fused_rmsnorm.py — single-launch RMSNorm on sm_100a (drop-in for the reference module).

fused_rmsnorm(x, weight, eps) == x / sqrt(mean(x^2) + eps) * weight in fp32, stored through
bf16 and returned in x.dtype exactly like the reference kernel (fused_rmsnorm.py:10-32);
fused_rmsnorm(..., round_bf16=False) stores the fp32 result straight into x.dtype (the stock
DiffusionGemmaRMSNorm rounding, fused_rmsnorm.py:1-5).  patch_rmsnorms(model) rebinds every
DiffusionGemmaRMSNorm.forward (fused_rmsnorm.py:39-48).
"""
import torch

from _knx import (KNX_RMS_ROUND_BF16, check, dtype_code, load, ptr, require_device, stream_of)


def fused_rmsnorm(x, weight, eps, round_bf16=True, xperm=None):
    orig = x.shape
    dev = require_device(x)
    x2 = x.reshape(-1, orig[-1]).contiguous()
    rows, cols = x2.shape
    src = x2 if x2.dtype in (torch.float16, torch.bfloat16) else x2.to(torch.bfloat16)
    y = torch.empty_like(src)
    w = weight.contiguous() if weight is not None else None
    check(load().knx_rmsnorm(ptr(src), ptr(w), dtype_code(w.dtype) if w is not None else 0, ptr(y),
                             ptr(xperm), rows, cols, float(eps), dtype_code(src.dtype),
                             KNX_RMS_ROUND_BF16 if round_bf16 else 0, stream_of(dev)),
          "knx_rmsnorm")
    return y.reshape(orig).to(x.dtype)


def _fused_forward(self, x):
    return fused_rmsnorm(x, self.weight if getattr(self, "with_scale", True) else None, self.eps)


@torch.no_grad()
def patch_rmsnorms(model, verbose=True):
    from transformers.models.diffusion_gemma.modeling_diffusion_gemma import DiffusionGemmaRMSNorm
    n = 0
    for mod in model.modules():
        if isinstance(mod, DiffusionGemmaRMSNorm):
            mod.forward = _fused_forward.__get__(mod, mod.__class__)
            n += 1
    if verbose:
        print(f"[fused-rmsnorm] patched {n} RMSNorm modules -> single-kernel", flush=True)
    return n
