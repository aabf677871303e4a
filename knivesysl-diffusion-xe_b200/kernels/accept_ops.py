"""accept_ops.py — entropy-bound acceptance and the stop test as one sm_100a launch.

accept_canvas(entropy, current, proposal, bound) -> (mask bool[B,L], canvas i64[B,L])
  stable ascending sort of the entropies, running sum (fp64, rounded to fp32 per prefix, as
  torch's CPU cumsum), accepted = cum - sorted <= bound, scattered back (fast_sampler.py:32-42).
accept_and_stop(...) additionally evaluates the stop test of fast_sampler.py:45-65 in the same
launch: stable = argmax canvas equals the last S canvases in `history` (which rolls), confident =
mean entropy < threshold.
"""
import torch

from _knx import check, load, ptr, require_device, stream_of


def _prep(entropy, current, proposal):
    h = entropy.reshape(-1, entropy.shape[-1]).float().contiguous()
    B, L = h.shape
    cur = current.reshape(B, L).long().contiguous()
    prop = proposal.reshape(B, L).long().contiguous()
    return h, cur, prop, B, L


def accept_canvas(entropy, current, proposal, bound):
    dev = require_device(entropy)
    h, cur, prop, B, L = _prep(entropy, current, proposal)
    mask = torch.empty(B, L, dtype=torch.uint8, device=h.device)
    out = torch.empty(B, L, dtype=torch.int64, device=h.device)
    check(load().knx_accept_stop(ptr(h), ptr(cur), ptr(prop), B, L, float(bound), ptr(mask),
                                 ptr(out), None, None, 0, 0.0, None, stream_of(dev)),
          "knx_accept_stop")
    return mask.bool().view(entropy.shape), out.view(current.shape)


def accept_and_stop(entropy, current, proposal, bound, argmax, history, confidence_threshold):
    """history: i64 [S,B,L] (S may be 0 -> pass None); returns (mask, canvas, finished bool[B])."""
    dev = require_device(entropy)
    h, cur, prop, B, L = _prep(entropy, current, proposal)
    mask = torch.empty(B, L, dtype=torch.uint8, device=h.device)
    out = torch.empty(B, L, dtype=torch.int64, device=h.device)
    fin = torch.empty(B, dtype=torch.uint8, device=h.device)
    S = 0 if history is None else history.shape[0]
    am = argmax.reshape(B, L).long().contiguous()
    check(load().knx_accept_stop(ptr(h), ptr(cur), ptr(prop), B, L, float(bound), ptr(mask),
                                 ptr(out), ptr(am), ptr(history), S, float(confidence_threshold),
                                 ptr(fin), stream_of(dev)), "knx_accept_stop")
    return mask.bool(), out, fin.bool()
