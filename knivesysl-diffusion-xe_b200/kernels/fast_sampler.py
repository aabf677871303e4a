"""fast_sampler.py — DiffusionGemma denoising-step hooks on sm_100a (drop-in for the reference).

Public surface (the reference's, fast_sampler.py:113-143): install(parity=False), uninstall(),
stats().  install() replaces three methods of transformers' DiffusionGemma generation classes:

  EntropyBoundSampler.accept_canvas             entropy-bound acceptance (fast_sampler.py:32-42)
  StableAndConfidentStoppingCriteria.__call__   stable-and-confident stop (fast_sampler.py:45-65)
  DiffusionGemmaGenerationMixin._denoising_step only with parity=True (fast_sampler.py:68-110)

Two tiers, as in the reference:
  * bit-exact (parity=False): torch's own entropy chain; the stopping test reuses the entropy the
    acceptance step computed for the same logits tensor instead of recomputing it;
  * parity (parity=True): the step's sampling is ONE streaming pass over the processed logits
    (entropy, Gumbel-max sample and argmax together; optionally the bf16 self-conditioning copy),
    and acceptance runs on the sm_100a kernel.  The Gumbel stream differs from torch's
    multinomial, hence "parity", not bit-exact, with the stock generation.

The entropy reuse is keyed by the logits tensor's (data_ptr, _version): a tensor that was
replaced or written in place since misses the cache and is recomputed.
"""
import torch


class _EntropyCache:
    """The entropy most recently computed (or produced by the sampling pass) for one logits
    tensor, with hit / miss counters for stats()."""

    def __init__(self):
        self.reset()

    def reset(self):
        self.key = None
        self.value = None
        self.hits = 0
        self.misses = 0

    @staticmethod
    def _key(logits):
        return (logits.data_ptr(), logits._version)

    def put(self, logits, entropy):
        self.key = self._key(logits)
        self.value = entropy

    def get(self, logits):
        """The cached entropy of `logits` or None, counting the outcome."""
        if self.key is not None and self.key == self._key(logits):
            self.hits += 1
            return self.value
        self.misses += 1
        return None


_CACHE = _EntropyCache()
_TIER = {"parity": False}
_SAVED = {}  # (class name, attribute) -> the original attribute, while installed


def _generation_module():
    from transformers.models.diffusion_gemma import generation_diffusion_gemma
    return generation_diffusion_gemma


def _token_entropy(logits):
    """Per-position entropy of softmax(logits): the fused one-pass kernel in the parity tier,
    torch's Categorical chain (the stock computation) otherwise."""
    if _TIER["parity"]:
        from fused_sampler_ops import fused_entropy
        return fused_entropy(logits)
    return torch.distributions.Categorical(logits=logits).entropy()


def _entropy_bound_mask(entropy, bound):
    """Stock acceptance rule: positions sorted by entropy (ascending); a position is accepted
    while the entropy accumulated before it stays within `bound`."""
    h_sorted, order = torch.sort(entropy, dim=-1)
    before = torch.cumsum(h_sorted, dim=-1) - h_sorted
    return torch.zeros_like(entropy, dtype=torch.bool).scatter(-1, order, before <= bound)


def _accept_canvas(self, current_canvas, denoiser_canvas, logits, cur_step):
    entropy = _CACHE.get(logits) if _TIER["parity"] else None
    if entropy is None:
        entropy = _token_entropy(logits)
    _CACHE.put(logits, entropy)
    if _TIER["parity"]:
        from accept_ops import accept_canvas
        mask, accepted = accept_canvas(entropy, current_canvas, denoiser_canvas,
                                       self.entropy_bound)
        self.accepted_token_mask = mask
        return accepted
    self.accepted_token_mask = _entropy_bound_mask(entropy, self.entropy_bound)
    return torch.where(self.accepted_token_mask, denoiser_canvas, current_canvas)


def _stable_over_history(crit, argmax_canvas):
    """True per canvas when the last `stability_threshold` argmax canvases all equal this one;
    then this canvas enters the history (oldest dropped).  The history starts filled with -1."""
    depth = crit.stability_threshold
    if depth == 0:
        return torch.ones(argmax_canvas.shape[0], dtype=torch.bool, device=argmax_canvas.device)
    if crit.argmax_canvas_history is None:
        crit.argmax_canvas_history = torch.full((depth, *argmax_canvas.shape), -1,
                                                dtype=argmax_canvas.dtype,
                                                device=argmax_canvas.device)
    hist = crit.argmax_canvas_history
    stable = torch.eq(hist, argmax_canvas.unsqueeze(0)).flatten(2).all(-1).all(0)
    hist = hist.roll(-1, 0)
    hist[depth - 1] = argmax_canvas
    crit.argmax_canvas_history = hist
    return stable


def _stop_call(self, argmax_canvas, logits, **kwargs):
    stable = _stable_over_history(self, argmax_canvas)
    entropy = _CACHE.get(logits)
    if entropy is None:
        entropy = _token_entropy(logits)
    return stable & (entropy.mean(dim=-1) < self.confidence_threshold)


def mixed_seed(base, step):
    """Per-step Gumbel seed (fast_sampler.py:92): `base` (a draw from torch's CPU generator, so
    seeded runs reproduce) XOR the step index times the golden-ratio constant, kept to 31 bits."""
    return (int(base) ^ (int(step) * 0x9E3779B1)) & 0x7FFFFFFF


def _denoising_step_parity(self, decoder_forward, current_canvas, argmax_canvas, input_ids,
                           decoder_position_ids, self_conditioning_logits, mask_mapping,
                           past_key_values, finished_denoising, cur_step, sampler,
                           logits_processor, diffusion_stopping_criteria, **model_kwargs):
    """The stock step with its sampling block replaced by one fused pass (entropy + Gumbel-max +
    argmax).  With bf16 embeddings the same pass also writes the next self-conditioning logits,
    where(finished, previous, processed) in bf16, which the stock step builds with a where and a
    cast over the logits at its end (fast_sampler.py:103-109)."""
    from fused_sampler_ops import sample_step, sample_step_selfcond
    step_index = int(cur_step)
    cur_step = torch.tensor(cur_step, device=current_canvas.device, dtype=torch.int32)
    torch.compiler.cudagraph_mark_step_begin()
    out = decoder_forward(decoder_input_ids=current_canvas,
                          self_conditioning_logits=self_conditioning_logits,
                          decoder_attention_mask=mask_mapping, past_key_values=past_key_values,
                          decoder_position_ids=decoder_position_ids, **model_kwargs)
    processed = logits_processor(input_ids, out.logits, cur_step=cur_step)
    B, L = current_canvas.shape
    seed = mixed_seed(torch.randint(0, 2**31 - 1, (1,)).item(), step_index)
    emb_dtype = self.model.decoder.embed_tokens.weight.dtype
    copy_in_pass = (emb_dtype == torch.bfloat16 and torch.is_tensor(self_conditioning_logits)
                    and self_conditioning_logits.dtype == torch.bfloat16
                    and self_conditioning_logits.shape == processed.shape)
    if copy_in_pass:
        # the finished flags as they stand before this step's stopping test (the stock where)
        fin = finished_denoising if diffusion_stopping_criteria is not None else None
        entropy, samp, amax, sc_next = sample_step_selfcond(processed, seed, 1.0,
                                                            self_conditioning_logits, fin)
    else:
        entropy, samp, amax = sample_step(processed, seed)
    _CACHE.put(processed, entropy.view(B, L))
    proposal, new_argmax = samp.view(B, L), amax.view(B, L)
    accepted = sampler.accept_canvas(current_canvas, proposal, processed, cur_step).clone()
    new_canvas = sampler.renoise_canvas(accepted, cur_step).clone()
    if diffusion_stopping_criteria is not None:
        if copy_in_pass:
            # No finished.any() on the host (a device sync per step): the two B x L selects run
            # unconditionally, the copy above already holds the logits select, and the stopping
            # test sees the logits as sampled (a cache hit).  Its result is OR-ed into
            # `finished`, so what it says about canvases already finished changes nothing.
            keep = finished_denoising[:, None]
            new_argmax = torch.where(keep, argmax_canvas, new_argmax)
            new_canvas = torch.where(keep, current_canvas, new_canvas)
        elif finished_denoising.any():
            keep = finished_denoising[:, None]
            new_argmax = torch.where(keep, argmax_canvas, new_argmax)
            new_canvas = torch.where(keep, current_canvas, new_canvas)
            processed = torch.where(keep[..., None], self_conditioning_logits, processed)
        finished_denoising |= diffusion_stopping_criteria(new_argmax, processed)
    next_sc = sc_next if copy_in_pass else processed.to(emb_dtype)
    return new_canvas, new_argmax, next_sc, finished_denoising


# (class, attribute, replacement, parity tier only)
_HOOKS = (("EntropyBoundSampler", "accept_canvas", _accept_canvas, False),
          ("StableAndConfidentStoppingCriteria", "__call__", _stop_call, False),
          ("DiffusionGemmaGenerationMixin", "_denoising_step", _denoising_step_parity, True))


def install(parity=False):
    """Patch the generation classes.  Installing again with the same tier is a no-op; with the
    other tier it raises RuntimeError (uninstall() first), so a tier is never changed silently."""
    parity = bool(parity)
    if _SAVED:
        if parity != _TIER["parity"]:
            raise RuntimeError(f"fast_sampler is installed with parity={_TIER['parity']}; "
                               f"uninstall() it before install(parity={parity})")
        return
    gen = _generation_module()
    for cls_name, attr, fn, parity_only in _HOOKS:
        if parity_only and not parity:
            continue
        cls = getattr(gen, cls_name)
        _SAVED[(cls_name, attr)] = getattr(cls, attr)
        setattr(cls, attr, fn)
    _TIER["parity"] = parity
    _CACHE.reset()


def uninstall():
    """Restore every patched method (no-op when not installed)."""
    if not _SAVED:
        return
    gen = _generation_module()
    for (cls_name, attr), orig in list(_SAVED.items()):
        setattr(getattr(gen, cls_name), attr, orig)
    _SAVED.clear()
    _TIER["parity"] = False


def stats():
    """Entropy reuse counters since install(): {"hits": n, "misses": m}."""
    return {"hits": _CACHE.hits, "misses": _CACHE.misses}
