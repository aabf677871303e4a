"""load_w4_checkpoint.py — load a dg-w4a16-v1 checkpoint and bind the sm_100a kernels.

load_fast(ckpt, device="cuda", tier="turbo") and load_w4(ckpt, device) keep the reference's
contract (load_w4_checkpoint.py:30-129):
  * the checkpoint directory holds w4_meta.json, the non-expert weights (model*.safetensors) and
    one experts_*.safetensors shard per decoder-layer index; a shard is recognised by the layer
    index in its first tensor name, not by its file name or order;
  * the encoder and decoder experts modules of layer N share ONE loaded tensor set (inference is
    read-only; load_w4_checkpoint.py:56-83), and every experts module gets gu_q/gu_s/gu_z/
    dn_q/dn_s/dn_z as non-persistent buffers and the fused forward;
  * the generation config is read explicitly (the model is built from its config, which does not
    read it, and early stopping depends on it);
  * tier: "turbo" = fused sampler + RMSNorm kernels, "bitexact" = entropy reuse only, "off".
The model classes come from transformers (DiffusionGemma) and accelerate.  ExpertShards and
bind_expert_buffers, the expert-loading step itself, need neither.
"""
import json
import pathlib
import re

import torch

EXPERT_BUFS = ("gu_q", "gu_s", "gu_z", "dn_q", "dn_s", "dn_z")
_TENSOR_LAYER = re.compile(r"\.layers\.(\d+)\.experts\.")
_MODULE_LAYER = re.compile(r"\.layers\.(\d+)\.experts$")


class ExpertShards:
    """The experts_*.safetensors files of a checkpoint, indexed by layer.  For each layer the
    first file (in sorted name order) whose first tensor belongs to it is used; the tensor-name
    prefix of that file is kept to address its six buffers."""

    def __init__(self, ckpt):
        from safetensors import safe_open
        self.files = {}  # layer -> (path, prefix)
        for path in sorted(pathlib.Path(ckpt).glob("experts_*.safetensors")):
            with safe_open(str(path), framework="pt") as h:
                first = next(iter(h.keys()))
            m = _TENSOR_LAYER.search(first)
            if m is None:
                raise ValueError(f"{path.name}: {first!r} is not an experts tensor name")
            self.files.setdefault(int(m.group(1)), (path, first.rsplit(".", 1)[0]))

    def layers(self):
        return sorted(self.files)

    def load(self, layer, device):
        """{buffer name: tensor} of one layer, read once."""
        from safetensors.torch import load_file
        path, prefix = self.files[layer]
        tensors = load_file(str(path), device=str(device))
        return {b: tensors[f"{prefix}.{b}"] for b in EXPERT_BUFS}


def load_expert_shards(ckpt, device="cuda"):
    """{layer index: {buffer name: tensor}} for every expert shard of `ckpt`."""
    shards = ExpertShards(ckpt)
    return {layer: shards.load(layer, device) for layer in shards.layers()}


def experts_modules_by_layer(model, experts_cls):
    """{layer index: [(module path, module), ...]} of the model's experts modules (the encoder's
    and the decoder's of one index land in the same list)."""
    by_layer = {}
    for path, mod in model.named_modules():
        if isinstance(mod, experts_cls):
            m = _MODULE_LAYER.search(path)
            if m is None:
                raise ValueError(f"experts module at an unexpected path: {path}")
            by_layer.setdefault(int(m.group(1)), []).append((path, mod))
    return by_layer


def bind_expert_buffers(modules_by_layer, shards):
    """Give every module of a layer the same tensor set (encoder and decoder alias it), drop
    the bf16 projection placeholders, and bind the fused forward."""
    from pack_experts import fused_experts_forward
    absent = sorted(set(modules_by_layer) - set(shards))
    if absent:
        raise AssertionError(f"no expert shard for layer(s) {absent}")
    for layer, mods in modules_by_layer.items():
        tensors = shards[layer]
        for _, mod in mods:
            mod.gate_up_proj = None
            mod.down_proj = None
            for name in EXPERT_BUFS:
                mod.register_buffer(name, tensors[name], persistent=False)
            mod.forward = fused_experts_forward.__get__(mod, type(mod))


def _backbone(ckpt, device):
    """The model with every non-expert weight assigned from model*.safetensors (parameters are
    created on the meta device and replaced, buffers are real)."""
    from accelerate import init_empty_weights
    from safetensors.torch import load_file
    from transformers import AutoConfig, DiffusionGemmaForBlockDiffusion
    cfg = AutoConfig.from_pretrained(str(ckpt))
    cfg._attn_implementation = "sdpa"
    with init_empty_weights(include_buffers=False):
        model = DiffusionGemmaForBlockDiffusion._from_config(cfg, torch_dtype=torch.bfloat16)
    state = {}
    for path in sorted(ckpt.glob("model*.safetensors")):
        state.update(load_file(str(path), device=str(device)))
    _, unexpected = model.load_state_dict(state, strict=False, assign=True)
    model.tie_weights()
    if unexpected:
        raise AssertionError(f"unexpected keys: {unexpected[:5]}")
    return model


@torch.no_grad()
def load_w4(ckpt, device="cuda"):
    """(model, tokenizer) of a dg-w4a16-v1 checkpoint with the fused experts bound."""
    from transformers import AutoTokenizer
    from transformers.models.diffusion_gemma.generation_diffusion_gemma import (
        DiffusionGemmaGenerationConfig)
    from transformers.models.diffusion_gemma.modeling_diffusion_gemma import (
        DiffusionGemmaTextExperts)
    ckpt = pathlib.Path(ckpt).resolve()
    meta_file = ckpt / "w4_meta.json"
    if not meta_file.exists():
        raise AssertionError(f"{ckpt} is not a dg-w4a16 checkpoint (no w4_meta.json)")
    model = _backbone(ckpt, device)
    by_layer = experts_modules_by_layer(model, DiffusionGemmaTextExperts)
    bind_expert_buffers(by_layer, load_expert_shards(ckpt, device))
    meta_params = [n for n, p in model.named_parameters() if p.is_meta]
    if meta_params:
        raise AssertionError(f"parameters never loaded: {meta_params[:5]}")
    model.generation_config = DiffusionGemmaGenerationConfig.from_pretrained(str(ckpt))
    if model.generation_config.max_denoising_steps is None:
        raise AssertionError("generation config not loaded (max_denoising_steps is None)")
    model.to(device).eval()
    tok = AutoTokenizer.from_pretrained(str(ckpt))
    fmt = json.loads(meta_file.read_text())["format"]
    print(f"[load_w4] {fmt} | {len(by_layer)} expert layers | device={device}", flush=True)
    return model, tok


# tier -> (fast_sampler parity flag or None for no hooks, patch the RMSNorms)
_TIERS = {"turbo": (True, True), "bitexact": (False, False), "off": (None, False)}


@torch.no_grad()
def load_fast(ckpt, device="cuda", tier="turbo"):
    """load_w4 plus the sampler hooks and RMSNorm kernel of `tier` ("turbo": fused sampler and
    RMSNorm, a different Gumbel stream than the stock sampler; "bitexact": entropy reuse only,
    token-identical to the stock W4 model; "off": neither)."""
    if tier not in _TIERS:
        raise AssertionError(f"unknown tier {tier!r}")
    parity, norms = _TIERS[tier]
    model, tok = load_w4(ckpt, device)
    if parity is not None:
        import fast_sampler
        fast_sampler.install(parity=parity)
    if norms:
        from fused_rmsnorm import patch_rmsnorms
        patch_rmsnorms(model, verbose=False)
    print(f"[load_fast] tier={tier}", flush=True)
    return model, tok
