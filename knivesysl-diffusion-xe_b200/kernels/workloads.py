"""workloads.py — seeded synthetic inputs with the shapes and distributions of the benchmark
configurations (no checkpoint or dataset is involved in any of them).

moe_weights(E, H, I, seed)       packed experts: nibbles uniform 0..15 (two per byte, low nibble
                                 = even k), fp16 scale ~U(0.002, 0.02), fp16 zero ~U(6, 9);
                                 gate_up groups of 128, down groups of 64
moe_inputs(T, H, E, topk, seed)  hidden f16 ~N(0,1), router weight f16 ~N(0, 0.02), RMSNorm
                                 weight f16 ~1+N(0, 0.1), the Zipf(s=1.1) router bias
zipf_bias(E, s, scale)           bias[e] = -scale * s * log(1 + e): log of a Zipf(s) pmf over
                                 expert ids, scaled so tokens-per-expert span ~0..80 at T=256
sampler_logits(rows, V, seed)    fp32 ~N(0, 3), 5% of rows with a single +15 spike
"""
import math

import torch

ZIPF_S = 1.1
ZIPF_SCALE = 0.3


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def moe_weights(E=128, H=2816, I=704, seed=0, device="cpu", gs_gu=128, gs_dn=64):
    g = _gen(seed, device)
    u8 = dict(dtype=torch.uint8, device=device)
    gu_q = torch.randint(0, 256, (E, 2 * I, H // 2), generator=g, **u8)
    dn_q = torch.randint(0, 256, (E, H, I // 2), generator=g, **u8)

    def sz(shape):
        s = (torch.rand(shape, generator=g, device=device) * 0.018 + 0.002).half()
        z = (torch.rand(shape, generator=g, device=device) * 3.0 + 6.0).half()
        return s, z
    gu_s, gu_z = sz((E, 2 * I, H // gs_gu))
    dn_s, dn_z = sz((E, H, I // gs_dn))
    return dict(gu_q=gu_q, gu_s=gu_s, gu_z=gu_z, dn_q=dn_q, dn_s=dn_s, dn_z=dn_z)


def zipf_bias(E=128, s=ZIPF_S, scale=ZIPF_SCALE, device="cpu"):
    e = torch.arange(E, dtype=torch.float32, device=device)
    return -scale * s * torch.log1p(e)


def moe_inputs(T=256, H=2816, E=128, seed=0, device="cpu"):
    g = _gen(seed + 1, device)
    hidden = torch.randn(T, H, generator=g, device=device).half()
    router_w = (torch.randn(E, H, generator=g, device=device) * 0.02).half()
    norm_w = (1.0 + 0.1 * torch.randn(H, generator=g, device=device)).half()
    return dict(hidden=hidden, router_w=router_w, norm_w=norm_w, bias=zipf_bias(E, device=device))


def random_routing(T, E, topk, seed=0, device="cpu"):
    """Uniform top-k routing (distinct experts per token) with softmax weights, as in the
    reference's own kernel tests (fused_moe_w4_v2.py:388-389)."""
    g = _gen(seed + 2, device)
    ids = torch.argsort(torch.rand(T, E, generator=g, device=device), dim=-1)[:, :topk]
    w = torch.softmax(torch.randn(T, topk, generator=g, device=device), -1)
    return ids, w


def sampler_logits(rows=256, V=262144, seed=0, device="cpu", spike_frac=0.05):
    g = _gen(seed + 3, device)
    x = torch.randn(rows, V, generator=g, device=device) * 3.0
    nspike = max(1, int(round(rows * spike_frac)))
    r = torch.randperm(rows, generator=g, device=device)[:nspike]
    c = torch.randint(0, V, (nspike,), generator=g, device=device)
    x[r, c] += 15.0
    return x


def temperature(step, max_steps=48, t_min=0.4, t_max=0.8):
    """T = t_min + (t_max - t_min) * remaining / max_steps with remaining = max_steps - step."""
    return t_min + (t_max - t_min) * (max_steps - step) / max_steps


def step_seed(s0, step):
    return (int(s0) ^ (int(step) * 0x9E3779B1)) & 0x7FFFFFFF


def moe_layer_bytes(counts, H=2816, I=704, gs_gu=128, gs_dn=64, T=256, E=128):
    """Algorithmic HBM bytes of one layer: packed weights + scale/zero of every touched expert,
    plus x read, y write and the router weight read."""
    per_expert = (2 * I * H // 2 + 2 * I * (H // gs_gu) * 2 * 2 + H * I // 2 +
                  H * (I // gs_dn) * 2 * 2)
    touched = int((counts > 0).sum())
    return touched * per_expert + 2 * T * H * 2 + E * H * 2


def moe_layer_flops(pairs, H=2816, I=704):
    return pairs * 2 * (H * 2 * I + I * H)
