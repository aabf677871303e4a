"""pack_experts.py — the packed expert layout and the experts.forward replacements.

Layout (pack_experts.py:6,12,34-41,87-106 of the reference; the kernels read it unchanged):
  gu_q u8[E,2I,H/2]  gu_s/gu_z f16[E,2I,H/128]   gate rows [0,I), up rows [I,2I), group 128
  dn_q u8[E,H,I/2]   dn_s/dn_z f16[E,H,I/64]     down, group 64 (128 does not divide I = 704)
The six tensors are non-persistent buffers of the experts module (pack_experts.py:96-97).

Entry points, named as in the reference:
  pack_experts_module(exp, free_bf16=True, fused=True)  quantise one experts module in place and
      rebind its forward (fused: the sm_100a MoE layer; otherwise the per-expert loop below)
  pack_all_experts(model, free_bf16=True, verbose=True)  every DiffusionGemmaTextExperts module
  fused_experts_forward(self, hidden, top_k_index, top_k_weights)   the fused layer
  packed_experts_forward(self, hidden, top_k_index, top_k_weights)  per-expert dense W4A16 GEMMs,
      the reference's unfused semantics (pack_experts.py:44-62), kept for A/B checks
  dump_moe_stats()  report of the MOE_STATS=1 routing probe (pack_experts.py:20-29)
"""
import os

import torch

from w4a16 import quantize_w4, w4a16_linear

GU_GS, DN_GS = 128, 64
_BUFFERS = ("gu_q", "gu_s", "gu_z", "dn_q", "dn_s", "dn_z")


class _RoutingProbe:
    """MOE_STATS=1: per layer call, how many distinct experts the top-8/6/4/2 choices of all
    tokens touch (the bytes a layer must stream), and how many experts carry 80% of the routing."""

    CUTS = (8, 6, 4, 2)

    def __init__(self):
        self.calls = []  # (E, {k: distinct experts}, experts for 80% of the pairs)

    @torch.no_grad()
    def record(self, top_k_index, top_k_weights, E):
        # rank each token's choices by weight so that the first k columns are its top-k
        ranked = top_k_index.gather(-1, top_k_weights.argsort(dim=-1, descending=True))
        union = {k: int(ranked[:, :min(k, ranked.shape[1])].unique().numel()) for k in self.CUTS}
        load = torch.bincount(top_k_index.flatten(), minlength=E).float()
        share = load.sort(descending=True).values.cumsum(0) / load.sum().clamp(min=1)
        self.calls.append((E, union, int((share < 0.8).sum()) + 1))

    def report(self):
        if not self.calls:
            return
        n = len(self.calls)
        E = self.calls[0][0]
        avg = {k: sum(c[1][k] for c in self.calls) / n for k in self.CUTS}
        conc = sum(c[2] for c in self.calls) / n
        cuts = "  ".join(f"top-{k}={avg[k]:.0f}" for k in self.CUTS)
        print(f"\n=== MoE routing probe: {n} layer calls, {E} experts ===", flush=True)
        print(f"  distinct experts per call: {cuts}  (of {E})", flush=True)
        print(f"  experts carrying 80% of the routed pairs: {conc:.0f}/{E}", flush=True)


_PROBE = _RoutingProbe()


def dump_moe_stats():
    _PROBE.report()


@torch.no_grad()
def _pack_stack(W3d, gs):
    """[E, N, K] weights -> (q u8[E,N,K/2], s f16[E,N,K/gs], z f16[E,N,K/gs]).  Quantisation is
    per (row, group), so the experts' rows are packed as one [E*N, K] matrix."""
    E, N, K = W3d.shape
    q, s, z = quantize_w4(W3d.reshape(E * N, K).float(), gs)
    return q.reshape(E, N, K // 2), s.reshape(E, N, K // gs), z.reshape(E, N, K // gs)


def packed_experts_forward(self, hidden_states, top_k_index, top_k_weights):
    """Per-expert dense W4A16 GEMMs over the tokens routed to each expert, accumulated into the
    output in expert order (ids == num_experts are dropped), like the stock loop."""
    out = torch.zeros_like(hidden_states)
    E = self.num_experts
    flat = top_k_index.flatten()
    pairs = torch.argsort(flat, stable=True)        # pairs grouped by expert, in pair order
    counts = torch.bincount(flat, minlength=E + 1).tolist()
    k = top_k_index.shape[1]
    start = 0
    for e, n in enumerate(counts[:E]):
        if n == 0:
            continue
        p = pairs[start:start + n]
        start += n
        tok, slot = p // k, p % k
        gate_up = w4a16_linear(hidden_states[tok], self.gu_q[e], self.gu_s[e], self.gu_z[e],
                               BK=GU_GS)
        gate, up = gate_up.chunk(2, dim=-1)
        h = w4a16_linear(self.act_fn(gate) * up, self.dn_q[e], self.dn_s[e], self.dn_z[e],
                         BK=DN_GS)
        out.index_add_(0, tok, (h * top_k_weights[tok, slot, None]).to(out.dtype))
    return out


def fused_experts_forward(self, hidden_states, top_k_index, top_k_weights):
    """One fused MoE layer on sm_100a (gate_up + GELU, down, fixed-order combine)."""
    if os.environ.get("MOE_STATS"):
        _PROBE.record(top_k_index, top_k_weights, self.num_experts)
    from fused_moe_w4_v2 import fused_moe_w4_v2
    return fused_moe_w4_v2(hidden_states, self, top_k_index, top_k_weights)


@torch.no_grad()
def pack_experts_module(exp, free_bf16=True, fused=True):
    """Quantise one experts module in place: register the six packed buffers on the weights'
    device, optionally drop the bf16 weights, and rebind forward."""
    dev = exp.gate_up_proj.device
    packed = _pack_stack(exp.gate_up_proj.data, GU_GS) + _pack_stack(exp.down_proj.data, DN_GS)
    for name, t in zip(_BUFFERS, packed):
        exp.register_buffer(name, t.to(dev), persistent=False)
    if free_bf16:
        exp.gate_up_proj = None
        exp.down_proj = None
    forward = fused_experts_forward if fused else packed_experts_forward
    exp.forward = forward.__get__(exp, type(exp))
    return exp


@torch.no_grad()
def pack_all_experts(model, free_bf16=True, verbose=True):
    """Pack every DiffusionGemmaTextExperts module of `model`; returns how many were packed."""
    from transformers.models.diffusion_gemma.modeling_diffusion_gemma import (
        DiffusionGemmaTextExperts)
    mods = [m for m in model.modules() if isinstance(m, DiffusionGemmaTextExperts)]
    weights = sum(m.gate_up_proj.numel() + m.down_proj.numel() for m in mods)
    for m in mods:
        pack_experts_module(m, free_bf16)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    if verbose:
        gib = 2.0 ** 30
        print(f"[pack] {len(mods)} expert modules to W4 (gate_up group {GU_GS}, down group "
              f"{DN_GS}): {2 * weights / gib:.1f} GiB bf16 -> ~{weights / 2 / gib:.1f} GiB",
              flush=True)
    return len(mods)
