"""load_w4_checkpoint.py — load a dg-w4a16-v1 checkpoint and bind the sm_100a kernels.

load_fast(ckpt, device="cuda", tier="turbo") and load_w4(ckpt, device) keep the reference's
contract (load_w4_checkpoint.py:30-129):
  * non-expert weights come from model*.safetensors; expert shards experts_*.safetensors are keyed
    by the layer index found in their first tensor name; encoder and decoder layer N share ONE
    loaded tensor (aliasing halves expert memory, load_w4_checkpoint.py:56-83);
  * every experts module gets gu_q/gu_s/gu_z/dn_q/dn_s/dn_z as non-persistent buffers and the
    fused forward; the generation config is loaded explicitly (early stop depends on it);
  * tier: "turbo" = fused sampler + RMSNorm kernels, "bitexact" = entropy dedup only, "off".
The model classes come from transformers (DiffusionGemma) and accelerate; load_expert_shards
needs neither and is what the expert-loading step itself runs.
"""
import json
import pathlib
import re

import torch

EXPERT_BUFS = ("gu_q", "gu_s", "gu_z", "dn_q", "dn_s", "dn_z")
_LAYER_RE = re.compile(r"\.layers\.(\d+)\.experts\.")


def load_expert_shards(ckpt, device="cuda"):
    """{layer index: {buffer name: tensor}} from experts_*.safetensors (first shard per layer
    wins, as in the reference); tensors are loaded once per layer."""
    from safetensors import safe_open
    from safetensors.torch import load_file
    ckpt = pathlib.Path(ckpt)
    shard_of = {}
    for f in sorted(ckpt.glob("experts_*.safetensors")):
        with safe_open(str(f), framework="pt") as h:
            k0 = next(iter(h.keys()))
        m = _LAYER_RE.search(k0)
        assert m, f"unrecognised expert tensor name {k0!r} in {f.name}"
        shard_of.setdefault(int(m.group(1)), (f, k0.rsplit(".", 1)[0]))
    out = {}
    for i, (f, src) in sorted(shard_of.items()):
        d = load_file(str(f), device=str(device))
        out[i] = {b: d[f"{src}.{b}"] for b in EXPERT_BUFS}
    return out


def bind_expert_buffers(modules_by_layer, shards):
    """Attach one loaded tensor set to every module of its layer (encoder and decoder alias)."""
    from pack_experts import fused_experts_forward
    missing = sorted(set(modules_by_layer) - set(shards))
    assert not missing, f"no expert shard for layer(s) {missing}"
    for i, mods in modules_by_layer.items():
        for _, mod in mods:
            mod.gate_up_proj = None
            mod.down_proj = None
            for b in EXPERT_BUFS:
                mod.register_buffer(b, shards[i][b], persistent=False)
            mod.forward = fused_experts_forward.__get__(mod, mod.__class__)


@torch.no_grad()
def load_w4(ckpt, device="cuda"):
    ckpt = pathlib.Path(ckpt).resolve()
    from accelerate import init_empty_weights
    from safetensors.torch import load_file
    from transformers import AutoConfig, AutoTokenizer, DiffusionGemmaForBlockDiffusion
    from transformers.models.diffusion_gemma.modeling_diffusion_gemma import DiffusionGemmaTextExperts
    from transformers.models.diffusion_gemma.generation_diffusion_gemma import (
        DiffusionGemmaGenerationConfig)
    assert (ckpt / "w4_meta.json").exists(), f"{ckpt} is not a dg-w4a16 checkpoint (no w4_meta.json)"
    cfg = AutoConfig.from_pretrained(str(ckpt))
    cfg._attn_implementation = "sdpa"
    with init_empty_weights(include_buffers=False):
        model = DiffusionGemmaForBlockDiffusion._from_config(cfg, torch_dtype=torch.bfloat16)
    sd = {}
    for f in sorted(ckpt.glob("model*.safetensors")):
        sd.update(load_file(str(f), device=str(device)))
    _, unexpected = model.load_state_dict(sd, strict=False, assign=True)
    model.tie_weights()
    assert not unexpected, f"unexpected keys: {unexpected[:5]}"
    by_layer = {}
    for name, mod in model.named_modules():
        if isinstance(mod, DiffusionGemmaTextExperts):
            m = re.search(r"\.layers\.(\d+)\.experts$", name)
            assert m, f"unrecognised experts module path: {name}"
            by_layer.setdefault(int(m.group(1)), []).append((name, mod))
    bind_expert_buffers(by_layer, load_expert_shards(ckpt, device))
    for n, p in model.named_parameters():
        assert not p.is_meta, f"param never materialised: {n}"
    model.generation_config = DiffusionGemmaGenerationConfig.from_pretrained(str(ckpt))
    assert model.generation_config.max_denoising_steps is not None, "generation_config failed to load"
    model.to(device).eval()
    tok = AutoTokenizer.from_pretrained(str(ckpt))
    meta = json.loads((ckpt / "w4_meta.json").read_text())
    print(f"[load_w4] {meta['format']} | {len(by_layer)} expert layers | device={device}", flush=True)
    return model, tok


@torch.no_grad()
def load_fast(ckpt, device="cuda", tier="turbo"):
    assert tier in ("turbo", "bitexact", "off"), f"unknown tier {tier!r}"
    model, tok = load_w4(ckpt, device)
    if tier != "off":
        import fast_sampler
        fast_sampler.install(parity=(tier == "turbo"))
        if tier == "turbo":
            from fused_rmsnorm import patch_rmsnorms
            patch_rmsnorms(model, verbose=False)
    print(f"[load_fast] tier={tier}", flush=True)
    return model, tok
