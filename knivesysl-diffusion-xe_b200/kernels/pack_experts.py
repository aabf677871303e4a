"""pack_experts.py — the packed expert layout and the experts.forward replacements.

Layout (pack_experts.py:6,12,34-41,87-106 of the reference, read unchanged by the kernels):
  gu_q u8[E,2I,H/2]  gu_s/gu_z f16[E,2I,H/128]   gate rows [0,I), up rows [I,2I), group 128
  dn_q u8[E,H,I/2]   dn_s/dn_z f16[E,H,I/64]     down, group 64 (128 does not divide I=704)

fused_experts_forward(self, hidden, top_k_index, top_k_weights) is what DiffusionGemma's
experts.forward is rebound to; packed_experts_forward is the per-expert reference loop
(pack_experts.py:44-62), kept for A/B checks.  MOE_STATS=1 keeps the routing probe.
"""
import collections
import os

import torch
import torch.nn.functional as F

from w4a16 import quantize_w4, w4a16_linear

GU_GS, DN_GS = 128, 64

_MOE_ACC = collections.defaultdict(list)


def dump_moe_stats():
    if not _MOE_ACC.get("u8"):
        return
    m = lambda x: sum(x) / len(x)
    E = _MOE_ACC["E"][0]
    print(f"\n=== MoE ROUTING PROBE (n={len(_MOE_ACC['u8'])} layer forwards, {E} experts) ===")
    print(f"  expert union per forward: top-8={m(_MOE_ACC['u8']):.0f} top-6={m(_MOE_ACC['u6']):.0f} "
          f"top-4={m(_MOE_ACC['u4']):.0f} top-2={m(_MOE_ACC['u2']):.0f} (of {E})")
    print(f"  experts holding 80% of routing mass: {m(_MOE_ACC['conc']):.0f}/{E}", flush=True)


@torch.no_grad()
def _pack_3d(W3d, gs):
    """W3d [E, N, K] -> stacked per-expert (qpacked, scale, zero)."""
    qs, ss, zs = [], [], []
    for e in range(W3d.shape[0]):
        q, s, z = quantize_w4(W3d[e].float(), gs)
        qs.append(q)
        ss.append(s)
        zs.append(z)
    return torch.stack(qs), torch.stack(ss), torch.stack(zs)


def packed_experts_forward(self, hidden_states, top_k_index, top_k_weights):
    """Per-expert loop with the dense W4A16 kernel (the reference's unfused path)."""
    final = torch.zeros_like(hidden_states)
    with torch.no_grad():
        expert_mask = F.one_hot(top_k_index, num_classes=self.num_experts).permute(2, 1, 0)
        expert_hit = torch.greater(expert_mask.sum(dim=(-1, -2)), 0).nonzero()
    for expert_idx in expert_hit:
        e = expert_idx[0]
        if e == self.num_experts:
            continue
        top_k_pos, token_idx = torch.where(expert_mask[e])
        cur = hidden_states[token_idx]
        gate_up = w4a16_linear(cur, self.gu_q[e], self.gu_s[e], self.gu_z[e], BK=GU_GS)
        gate, up = gate_up.chunk(2, dim=-1)
        h = self.act_fn(gate) * up
        h = w4a16_linear(h, self.dn_q[e], self.dn_s[e], self.dn_z[e], BK=DN_GS)
        h = h * top_k_weights[token_idx, top_k_pos, None]
        final.index_add_(0, token_idx, h.to(final.dtype))
    return final


def fused_experts_forward(self, hidden_states, top_k_index, top_k_weights):
    """One fused MoE layer on sm_100a (gate_up+GELU, down, fixed-order combine)."""
    if os.environ.get("MOE_STATS"):
        with torch.no_grad():
            order = top_k_weights.argsort(dim=-1, descending=True)
            tis = torch.gather(top_k_index, -1, order)
            tk = top_k_index.shape[1]
            for k, key in ((8, "u8"), (6, "u6"), (4, "u4"), (2, "u2")):
                _MOE_ACC[key].append(int(tis[:, :min(k, tk)].unique().numel()))
            hist = torch.bincount(top_k_index.reshape(-1), minlength=self.num_experts).float()
            cum = torch.cumsum(torch.sort(hist, descending=True).values, 0) / hist.sum().clamp(min=1)
            _MOE_ACC["conc"].append(int((cum < 0.8).sum()) + 1)
            _MOE_ACC["E"].append(self.num_experts)
    from fused_moe_w4_v2 import fused_moe_w4_v2
    return fused_moe_w4_v2(hidden_states, self, top_k_index, top_k_weights)


@torch.no_grad()
def pack_experts_module(exp, free_bf16=True, fused=True):
    """Pack one experts module in place: add the six packed buffers, bind the fused forward."""
    gu_q, gu_s, gu_z = _pack_3d(exp.gate_up_proj.data, GU_GS)
    dn_q, dn_s, dn_z = _pack_3d(exp.down_proj.data, DN_GS)
    dev = exp.gate_up_proj.device
    for nm, t in (("gu_q", gu_q), ("gu_s", gu_s), ("gu_z", gu_z), ("dn_q", dn_q), ("dn_s", dn_s),
                  ("dn_z", dn_z)):
        exp.register_buffer(nm, t.to(dev), persistent=False)
    if free_bf16:
        exp.gate_up_proj = None
        exp.down_proj = None
    fwd = fused_experts_forward if fused else packed_experts_forward
    exp.forward = fwd.__get__(exp, exp.__class__)
    return exp


@torch.no_grad()
def pack_all_experts(model, free_bf16=True, verbose=True):
    from transformers.models.diffusion_gemma.modeling_diffusion_gemma import DiffusionGemmaTextExperts
    n, gu_bits, dn_bits = 0, 0, 0
    for _, mod in model.named_modules():
        if isinstance(mod, DiffusionGemmaTextExperts):
            gu_bits += mod.gate_up_proj.numel()
            dn_bits += mod.down_proj.numel()
            pack_experts_module(mod, free_bf16)
            n += 1
    torch.cuda.empty_cache()
    if verbose:
        print(f"[pack] {n} expert modules -> W4 (gate_up gs{GU_GS}, down gs{DN_GS}); experts "
              f"{2 * (gu_bits + dn_bits) / 2**30:.1f}GiB bf16 -> ~{(gu_bits + dn_bits) / 2 / 2**30:.1f}GiB W4")
    return n
