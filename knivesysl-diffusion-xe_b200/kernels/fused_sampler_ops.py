"""fused_sampler_ops.py — the sampler's streaming pass on sm_100a (drop-in for the reference).

fused_entropy(logits)              -> entropy of softmax(logits) per row, fp32 (nats)
gumbel_argmax_sample(logits, seed) -> (Gumbel-max sample, argmax), int64 per row
sample_step(logits, seed, temperature=1.0) -> (entropy, sample, argmax) from ONE pass that also
    applies the temperature (x / T), so the processed logits never have to be materialised.

Random stream: u = tl.rand(seed + row, col) of Triton (Philox4x32-10, first word, key = seed+row,
counter = col), clamped to [1e-10, 1-1e-7], g = -log(-log u) with this library's own
bit-reproducible log; sample = first argmax of x + g (fused_sampler_ops.py:54-81).
"""
import torch

from _knx import check, load, ptr, require_device, stream_of, workspace


def _run(logits, seed, temperature, want_h, want_s, want_a):
    x = logits.reshape(-1, logits.shape[-1])
    dev = require_device(x)
    if x.dtype != torch.float32:
        x = x.float()
    if not x.is_contiguous():
        x = x.contiguous()
    rows, V = x.shape
    h = torch.empty(rows, dtype=torch.float32, device=x.device) if want_h else None
    s = torch.empty(rows, dtype=torch.int64, device=x.device) if want_s else None
    a = torch.empty(rows, dtype=torch.int64, device=x.device) if want_a else None
    lib = load()
    ws = workspace(dev, lib.knx_sampler_workspace_size(rows, V), "sampler")
    check(lib.knx_sampler_fused(ptr(x), rows, V, float(temperature), int(seed), ptr(h), ptr(s),
                                ptr(a), ptr(ws), ws.numel(), stream_of(dev)), "knx_sampler_fused")
    shp = logits.shape[:-1]
    return (h.view(shp) if h is not None else None, s.view(shp) if s is not None else None,
            a.view(shp) if a is not None else None)


def fused_entropy(logits):
    """logits [..., V] -> entropy [...] fp32 (nats), one pass."""
    return _run(logits, 0, 1.0, True, False, False)[0]


def gumbel_argmax_sample(logits, seed):
    """logits [..., V] -> (sampled idx, argmax idx) int64 [...]."""
    _, s, a = _run(logits, seed, 1.0, False, True, True)
    return s, a


def sample_step(logits, seed, temperature=1.0):
    """(entropy, sample, argmax) of softmax(logits / temperature) in one streaming pass."""
    return _run(logits, seed, temperature, True, True, True)
