"""fused_sampler_ops.py — the sampler's streaming pass on sm_100a (drop-in for the reference).

fused_entropy(logits)              -> entropy of softmax(logits) per row, fp32 (nats)
gumbel_argmax_sample(logits, seed) -> (Gumbel-max sample, argmax), int64 per row
sample_step(logits, seed, temperature=1.0) -> (entropy, sample, argmax) from ONE pass that also
    applies the temperature (x / T), so the processed logits never have to be materialised.
sample_step_selfcond(logits, seed, temperature, sc_prev=None, finished=None)
    -> (entropy, sample, argmax, self_conditioning_logits): the same pass also writes the next
    step's bf16 self-conditioning logits, where(finished, sc_prev, x / T).to(bfloat16), in place
    of the reference step's separate where + cast over the logits (fast_sampler.py:103-109).

Random stream: u = tl.rand(seed + row, col) of Triton (Philox4x32-10, first word, key = seed+row,
counter = col), clamped to [1e-10, 1-1e-7], g = -log(-log u) with this library's own
bit-reproducible log; sample = first argmax of x + g (fused_sampler_ops.py:54-81).
"""
import torch

from _knx import check, load, ptr, require_device, stream_of, workspace


def _run(logits, seed, temperature, want_h, want_s, want_a, sc_out=None, sc_prev=None,
         finished=None):
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
    if sc_out is None:
        check(lib.knx_sampler_fused(ptr(x), rows, V, float(temperature), int(seed), ptr(h),
                                    ptr(s), ptr(a), ptr(ws), ws.numel(), stream_of(dev)),
              "knx_sampler_fused")
    else:
        canvas_len = rows // finished.numel() if finished is not None else 1
        check(lib.knx_sampler_fused_sc(ptr(x), rows, V, float(temperature), int(seed), ptr(h),
                                       ptr(s), ptr(a), ptr(sc_out), ptr(sc_prev), ptr(finished),
                                       canvas_len, ptr(ws), ws.numel(), stream_of(dev)),
              "knx_sampler_fused_sc")
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


def sample_step_selfcond(logits, seed, temperature=1.0, sc_prev=None, finished=None):
    """sample_step plus the next step's self-conditioning logits, written by the same pass:
    sc[r] = sc_prev[r] where the row's canvas has finished, else bf16(logits[r] / temperature).

    logits [B, L, V] (or [..., V]); sc_prev bf16 of the same shape (needed with `finished`);
    finished bool/uint8 [B] (one flag per canvas of L rows) or None.  Returns
    (entropy, sample, argmax, sc) with sc a new bf16 tensor shaped like logits."""
    V = logits.shape[-1]
    sc = torch.empty(logits.shape, dtype=torch.bfloat16, device=logits.device)
    fin = None
    if finished is not None:
        if sc_prev is None or sc_prev.shape != logits.shape or sc_prev.dtype != torch.bfloat16:
            raise ValueError("sample_step_selfcond: finished needs sc_prev, bf16, shaped like logits")
        rows = logits.numel() // V
        if rows % finished.numel() != 0:
            raise ValueError("sample_step_selfcond: rows must be a whole number of canvases")
        fin = finished.reshape(-1).to(torch.uint8).contiguous()
        sc_prev = sc_prev.contiguous()
    h, s, a = _run(logits, seed, temperature, True, True, True, sc_out=sc,
                   sc_prev=sc_prev if fin is not None else None, finished=fin)
    return h, s, a, sc
