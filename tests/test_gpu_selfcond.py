"""The denoising step's self-conditioning copy written by the sampler pass (knx_sampler_fused_sc),
against the reference step's own arithmetic run by torch on the CPU:
    processed = where(finished[:, None, None], self_conditioning_logits, processed)
    self_conditioning_logits = processed.to(bfloat16)          (fast_sampler.py:103-109)
with processed = logits / T.  The copy must be bit-identical, and the sampling results must be
bit-identical to the pass without the copy."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(B, L, V, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B * L, V, generator=g) * 3.0
    # exact bf16 rounding ties (low 16 bits 0x8000, both parities of the kept bit) and values
    # whose rounding carries into the exponent
    ties = torch.tensor([0x3F808000, 0x3F818000, 0xC0A08000, 0x3F7FFFFF, 0x477FFFFF],
                        dtype=torch.int64).to(torch.int32).view(torch.float32)
    x[0, :ties.numel()] = ties
    x[-1, -ties.numel():] = ties
    prev = torch.randn(B * L, V, generator=g).bfloat16()
    return x, prev


def _bits(t):
    return t.contiguous().view(torch.int16)


@pytest.mark.parametrize("B,L,V,T", [(2, 64, 262144, 0.7), (3, 8, 4096, 1.0), (2, 5, 1003, 0.55)])
def test_selfcond_copy_matches_where_cast(cuda, B, L, V, T):
    import fused_sampler_ops
    x, prev = _case(B, L, V, seed=B * 1000 + V)
    finished = torch.zeros(B, dtype=torch.bool)
    finished[1] = True
    proc = x / T if T != 1.0 else x
    want = torch.where(finished.repeat_interleave(L)[:, None], prev, proc.to(torch.bfloat16))
    xd = x.view(B, L, V).to(cuda)
    pd = prev.view(B, L, V).to(cuda)
    for _ in range(2):  # twice in a row: nothing carries over between calls
        h, s, a, sc = fused_sampler_ops.sample_step_selfcond(xd, 123, T, pd, finished.to(cuda))
        assert sc.shape == (B, L, V) and sc.dtype == torch.bfloat16
        assert torch.equal(_bits(sc.cpu().view(-1, V)), _bits(want))
    h0, s0, a0 = fused_sampler_ops.sample_step(xd, 123, T)
    assert torch.equal(h.view(torch.int32), h0.view(torch.int32))
    assert torch.equal(s, s0) and torch.equal(a, a0)
    # no canvas finished: a plain cast
    _, _, _, sc2 = fused_sampler_ops.sample_step_selfcond(xd, 123, T)
    assert torch.equal(_bits(sc2.cpu().view(-1, V)), _bits(proc.to(torch.bfloat16)))


def test_selfcond_rejects_bad_arguments(cuda):
    import fused_sampler_ops
    x = torch.randn(2, 4, 256, device=cuda)
    with pytest.raises(ValueError):  # finished without the previous logits
        fused_sampler_ops.sample_step_selfcond(x, 1, 1.0, None, torch.zeros(2, dtype=torch.bool,
                                                                              device=cuda))
    with pytest.raises(ValueError):  # rows are not whole canvases
        fused_sampler_ops.sample_step_selfcond(x, 1, 1.0, torch.zeros_like(x, dtype=torch.bfloat16),
                                               torch.zeros(3, dtype=torch.bool, device=cuda))


def test_denoising_step_glue_writes_selfcond_from_the_pass(cuda):
    """fast_sampler._denoising_step_parity with stand-ins for the transformers objects (decoder,
    temperature processor, sampler, stopping test): with bf16 embeddings the returned
    self-conditioning logits are the reference step's where(finished, previous, processed) cast
    to bf16, and finished canvases keep their argmax."""
    from types import SimpleNamespace as NS

    import fast_sampler
    B, L, V, T = 2, 16, 4096, 0.6
    g = torch.Generator().manual_seed(7)
    raw = (torch.randn(B, L, V, generator=g) * 3.0).to(cuda)
    prev = torch.randn(B, L, V, generator=g).bfloat16().to(cuda)
    finished = torch.tensor([False, True], device=cuda)
    owner = NS(model=NS(decoder=NS(embed_tokens=NS(weight=torch.zeros(1, dtype=torch.bfloat16)))))
    sampler = NS(accept_canvas=lambda cur, den, logits, step: den,
                 renoise_canvas=lambda acc, step: acc)
    def stop(argmax_canvas, logits):  # confident canvases: mean entropy below a threshold
        return torch.distributions.Categorical(logits=logits.float()).entropy().mean(-1) < 2.0
    canvas = torch.zeros(B, L, dtype=torch.int64, device=cuda)
    old_argmax = torch.full((B, L), 7, dtype=torch.int64, device=cuda)
    _, new_argmax, sc, fin = fast_sampler._denoising_step_parity(
        owner, lambda **kw: NS(logits=raw), canvas, old_argmax, None, None, prev, None, None,
        finished.clone(), 3, sampler, lambda ids, logits, cur_step: logits / T, stop)
    # the stock step: where over the logits, stopping test on them, cast
    proc = torch.where(finished[:, None, None], prev, raw / T)
    want = proc.to(torch.bfloat16)
    fin_want = finished | stop(None, proc)
    assert sc.dtype == torch.bfloat16
    assert torch.equal(sc.view(torch.int16), want.view(torch.int16))
    assert torch.equal(new_argmax[1], old_argmax[1])
    assert torch.equal(new_argmax[0], (raw[0] / T).argmax(-1))
    assert torch.equal(fin, fin_want)
