"""CPU tests of the host-side glue around the kernels: the denoising-step schedule (seed mixing
and temperature), the generation hooks of fast_sampler against stand-in transformers classes, the
expert-shard loader, and the expert packing helpers.  No GPU and no transformers install needed."""
import sys
import types

import pytest
import torch

from oracle import ref


# ------------------------------------------------------------------------------ step schedule
def _reference_seed(r, step_int):
    # fast_sampler.py:92 of the reference, transcribed as written there
    return (int(r) ^ (step_int * 0x9E3779B1)) & 0x7FFFFFFF


def _readme_temperature(t_min, t_max, remaining_steps, max_denoising_steps):
    # README.md:127-136 of the reference: the loop counts remaining_steps down from max to 1
    return t_min + (t_max - t_min) * remaining_steps / max_denoising_steps


@pytest.mark.parametrize("r", [0, 1, 1234, 2**31 - 2, 987654321])
def test_seed_mix_matches_reference_line(r):
    import fast_sampler
    import workloads
    for step in (0, 1, 2, 47, 48, 95, 1000, 2**20 + 3):
        want = _reference_seed(r, step)
        assert fast_sampler.mixed_seed(r, step) == want
        assert workloads.step_seed(r, step) == want
        assert ref.step_seed(r, step) == want
        assert 0 <= want < 2**31


def test_temperature_schedule_matches_readme_formula():
    import workloads
    t_min, t_max, n = 0.4, 0.8, 48
    got = [workloads.temperature(step, n, t_min, t_max) for step in range(n)]
    want = [_readme_temperature(t_min, t_max, n - step, n) for step in range(n)]
    assert got == want
    assert [ref.temperature(step, n, t_min, t_max) for step in range(n)] == want
    assert got[0] == pytest.approx(0.8)                    # first pass: remaining = 48
    assert got[-1] == pytest.approx(0.4 + 0.4 / 48)        # last pass: remaining = 1, not 0
    assert all(a > b for a, b in zip(got, got[1:]))


# ------------------------------------------------------------------------------ fast_sampler hooks
@pytest.fixture
def fake_generation(monkeypatch):
    """Stand-ins for transformers.models.diffusion_gemma.generation_diffusion_gemma."""
    mod = types.ModuleType("generation_diffusion_gemma")

    class EntropyBoundSampler:
        def accept_canvas(self, *a):
            return "stock accept"

    class StableAndConfidentStoppingCriteria:
        def __call__(self, *a, **k):
            return "stock stop"

    class DiffusionGemmaGenerationMixin:
        def _denoising_step(self, *a, **k):
            return "stock step"

    mod.EntropyBoundSampler = EntropyBoundSampler
    mod.StableAndConfidentStoppingCriteria = StableAndConfidentStoppingCriteria
    mod.DiffusionGemmaGenerationMixin = DiffusionGemmaGenerationMixin
    pkg = types.ModuleType("transformers.models.diffusion_gemma")
    pkg.generation_diffusion_gemma = mod
    for name, m in (("transformers.models.diffusion_gemma", pkg),
                    ("transformers.models.diffusion_gemma.generation_diffusion_gemma", mod)):
        monkeypatch.setitem(sys.modules, name, m)
    import fast_sampler
    yield mod
    fast_sampler.uninstall()


def test_install_uninstall_and_tier_guard(fake_generation):
    import fast_sampler
    G = fake_generation
    orig = (G.EntropyBoundSampler.accept_canvas, G.StableAndConfidentStoppingCriteria.__call__,
            G.DiffusionGemmaGenerationMixin._denoising_step)
    fast_sampler.install(parity=False)
    assert G.EntropyBoundSampler.accept_canvas is fast_sampler._accept_canvas
    assert G.StableAndConfidentStoppingCriteria.__call__ is fast_sampler._stop_call
    assert G.DiffusionGemmaGenerationMixin._denoising_step is orig[2]   # bit-exact tier
    fast_sampler.install(parity=False)                                   # same tier: no-op
    with pytest.raises(RuntimeError):
        fast_sampler.install(parity=True)                                # never a silent switch
    fast_sampler.uninstall()
    assert (G.EntropyBoundSampler.accept_canvas, G.StableAndConfidentStoppingCriteria.__call__,
            G.DiffusionGemmaGenerationMixin._denoising_step) == orig
    fast_sampler.install(parity=True)
    assert G.DiffusionGemmaGenerationMixin._denoising_step is fast_sampler._denoising_step_parity
    fast_sampler.uninstall()
    assert G.DiffusionGemmaGenerationMixin._denoising_step is orig[2]


def _stock_accept(entropy, cur, prop, bound):
    # the stock acceptance (fast_sampler.py:32-42 of the reference), transcribed
    sorted_h, sorted_idx = torch.sort(entropy, dim=-1, descending=False)
    cum = torch.cumsum(sorted_h, dim=-1)
    sel = cum - sorted_h <= bound
    mask = torch.scatter(input=torch.zeros_like(sel), dim=-1, index=sorted_idx, src=sel)
    return mask, torch.where(mask, prop, cur)


def _stock_stop(crit, argmax_canvas, entropy):
    # the stock stopping test (fast_sampler.py:45-65 of the reference), transcribed
    if crit.stability_threshold == 0:
        stable = torch.ones(argmax_canvas.shape[0], dtype=torch.bool)
    else:
        if crit.argmax_canvas_history is None:
            crit.argmax_canvas_history = torch.full(
                (crit.stability_threshold, argmax_canvas.shape[0], argmax_canvas.shape[1]), -1,
                dtype=argmax_canvas.dtype)
        stable = (crit.argmax_canvas_history == argmax_canvas[None, :, :]).all(dim=-1).all(dim=0)
        crit.argmax_canvas_history = torch.roll(crit.argmax_canvas_history, shifts=-1, dims=0)
        crit.argmax_canvas_history[-1] = argmax_canvas
    return stable & (torch.mean(entropy, dim=-1) < crit.confidence_threshold)


def test_bitexact_tier_accept_and_stop_match_stock(fake_generation):
    import fast_sampler
    fast_sampler.install(parity=False)
    g = torch.Generator().manual_seed(3)
    B, L, V = 2, 32, 50
    cur = torch.randint(0, V, (B, L), generator=g)
    prop = torch.randint(0, V, (B, L), generator=g)
    sampler = types.SimpleNamespace(entropy_bound=0.5)
    crit_a = types.SimpleNamespace(stability_threshold=2, argmax_canvas_history=None,
                                   confidence_threshold=3.5)
    crit_b = types.SimpleNamespace(stability_threshold=2, argmax_canvas_history=None,
                                   confidence_threshold=3.5)
    argmax = torch.randint(0, V, (B, L), generator=g)
    for step in range(4):
        logits = torch.randn(B, L, V, generator=g) * (0.2 + step)
        out = fast_sampler._accept_canvas(sampler, cur, prop, logits, step)
        h = torch.distributions.Categorical(logits=logits).entropy()
        mask, want = _stock_accept(h, cur, prop, 0.5)
        assert torch.equal(out, want) and torch.equal(sampler.accepted_token_mask, mask)
        if step == 2:
            argmax = argmax.clone()
            argmax[1, 0] += 1                     # canvas 1 changes once: unstable for 2 steps
        got = fast_sampler._stop_call(crit_a, argmax, logits)
        assert torch.equal(got, _stock_stop(crit_b, argmax, h))
        assert torch.equal(crit_a.argmax_canvas_history, crit_b.argmax_canvas_history)
    assert fast_sampler.stats() == {"hits": 4, "misses": 0}   # the stop test reused every entropy
    logits.add_(0)                                            # in place: the cache must miss
    fast_sampler._stop_call(crit_a, argmax, logits)
    assert fast_sampler.stats()["misses"] == 1


# ------------------------------------------------------------------------------ expert shards
def _write_shards(tmp_path, layers, E=2, H=64, I=32):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(1)
    made = {}
    for n, layer in enumerate(layers):
        prefix = f"model.decoder.layers.{layer}.experts"
        t = {"gu_q": torch.randint(0, 256, (E, 2 * I, H // 2), generator=g, dtype=torch.uint8),
             "gu_s": torch.rand(E, 2 * I, H // 32, generator=g).half(),
             "gu_z": torch.rand(E, 2 * I, H // 32, generator=g).half(),
             "dn_q": torch.randint(0, 256, (E, H, I // 2), generator=g, dtype=torch.uint8),
             "dn_s": torch.rand(E, H, I // 32, generator=g).half(),
             "dn_z": torch.rand(E, H, I // 32, generator=g).half()}
        # file names deliberately out of layer order: shards are keyed by tensor names
        save_file({f"{prefix}.{k}": v for k, v in t.items()},
                  str(tmp_path / f"experts_{len(layers) - n:03d}.safetensors"))
        made.setdefault(layer, t)
    return made


def test_expert_shards_are_keyed_by_layer_and_aliased(tmp_path):
    import load_w4_checkpoint as L
    # layer 1 appears twice: the first file in name order wins
    made = _write_shards(tmp_path, [3, 0, 1, 1])
    shards = L.load_expert_shards(tmp_path, device="cpu")
    assert sorted(shards) == [0, 1, 3]
    first_file_of_layer1 = L.ExpertShards(tmp_path).files[1][0].name
    assert first_file_of_layer1 == "experts_001.safetensors"      # the later-written copy
    for layer in (0, 3):
        for b in L.EXPERT_BUFS:
            assert torch.equal(shards[layer][b], made[layer][b])

    class Experts(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_up_proj = torch.nn.Parameter(torch.zeros(1))
            self.down_proj = torch.nn.Parameter(torch.zeros(1))
            self.num_experts = 2

    model = torch.nn.Module()
    model.encoder = torch.nn.Module()
    model.decoder = torch.nn.Module()
    model.encoder.layers = torch.nn.ModuleList([torch.nn.Module() for _ in range(4)])
    model.decoder.layers = torch.nn.ModuleList([torch.nn.Module() for _ in range(4)])
    for side in (model.encoder, model.decoder):
        for i in (0, 1, 3):
            side.layers[i].experts = Experts()
    by_layer = L.experts_modules_by_layer(model, Experts)
    assert sorted(by_layer) == [0, 1, 3] and all(len(v) == 2 for v in by_layer.values())
    L.bind_expert_buffers(by_layer, shards)
    for layer, mods in by_layer.items():
        (_, enc), (_, dec) = mods
        for b in L.EXPERT_BUFS:
            assert getattr(enc, b) is getattr(dec, b)                 # one tensor, two modules
            assert b not in enc.state_dict()                           # non-persistent
        assert enc.gate_up_proj is None and dec.down_proj is None
        assert enc.forward.__func__.__name__ == "fused_experts_forward"
    # a model layer without a shard is refused
    model.decoder.layers[2].experts = Experts()
    with pytest.raises(AssertionError):
        L.bind_expert_buffers(L.experts_modules_by_layer(model, Experts), shards)


# ------------------------------------------------------------------------------ packing
def test_pack_stack_equals_per_expert_quantize_and_module_binding():
    import pack_experts
    import w4a16
    g = torch.Generator().manual_seed(9)
    E, H, I = 3, 256, 64
    gate_up = torch.randn(E, 2 * I, H, generator=g) * 0.02
    down = torch.randn(E, H, I, generator=g) * 0.02
    q, s, z = pack_experts._pack_stack(gate_up, 128)
    for e in range(E):
        qe, se, ze = w4a16.quantize_w4(gate_up[e], 128)
        assert torch.equal(q[e], qe) and torch.equal(s[e], se) and torch.equal(z[e], ze)

    class Experts(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_up_proj = torch.nn.Parameter(gate_up.clone())
            self.down_proj = torch.nn.Parameter(down.clone())
            self.num_experts = E

    mod = pack_experts.pack_experts_module(Experts(), free_bf16=True, fused=False)
    assert mod.gu_q.shape == (E, 2 * I, H // 2) and mod.dn_s.shape == (E, H, I // 64)
    assert mod.gate_up_proj is None and mod.forward.__func__ is pack_experts.packed_experts_forward
    assert "gu_q" not in mod.state_dict()
    probe = pack_experts._RoutingProbe()
    ids = torch.tensor([[0, 1], [0, 2], [0, 1]])
    probe.record(ids, torch.tensor([[0.9, 0.1], [0.6, 0.4], [0.2, 0.8]]), E)
    E_, union, conc = probe.calls[0]
    assert union[2] == 3 and union[8] == 3 and conc == 2
