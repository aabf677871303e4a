"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own code.

Run where a checkout of the reference repository is available (read-only), passing its path
(or setting KNX_REFERENCE) — it is never needed at test time:

    python tests/golden/make_golden.py REF

The reference's Triton kernels are executed by Triton's CPU interpreter (TRITON_INTERPRET=1),
its pure-torch functions (quantize_w4, dequant_w4, moe_align) run as they are, and its
fast_sampler acceptance / stop functions run against a stand-in for the (absent) transformers
DiffusionGemma generation module, which they only need for class names.  Every fixture is
seeded, small, and saved as .npz next to this script.
"""
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KNX_REFERENCE", "")
if not REF or not os.path.isdir(os.path.join(REF, "kernels")):
    sys.exit("usage: make_golden.py REFERENCE_CHECKOUT  (or set KNX_REFERENCE)")
OUT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REF, "kernels"))


def save(name, **arrays):
    path = os.path.join(OUT, name)
    np.savez_compressed(path, **{k: (v.numpy() if torch.is_tensor(v) else np.asarray(v))
                                 for k, v in arrays.items()})
    print("wrote", path, {k: tuple(np.asarray(v).shape) for k, v in arrays.items()})


def gen_w4a16():
    import w4a16 as R
    # the interpreter has no GPU benchmarker: keep the first of the reference's own autotune
    # configs so the autotuner runs that one directly
    R._w4a16_kernel.configs = R._w4a16_kernel.configs[:1]
    g = torch.Generator().manual_seed(11)
    out = {}
    for tag, N, K, gs, M in (("g128", 64, 256, 128, 5), ("g64", 48, 192, 64, 3)):
        W = torch.randn(N, K, generator=g) * 0.02
        W[:, : K // 16] += torch.randn(N, K // 16, generator=g) * 0.15
        q, s, z = R.quantize_w4(W, gs)
        wdq = R.dequant_w4(q, s, z, gs)
        X = torch.randn(M, K, generator=g).half()
        Y = R.w4a16_linear(X, q, s, z, BK=gs)          # the reference Triton kernel (interpreted)
        out.update({f"{tag}_W": W, f"{tag}_q": q, f"{tag}_s": s, f"{tag}_z": z, f"{tag}_wdq": wdq,
                    f"{tag}_X": X, f"{tag}_Y": Y, f"{tag}_gs": np.int64(gs)})
    save("w4a16.npz", **out)


def gen_align():
    import fused_moe_w4 as R
    g = torch.Generator().manual_seed(12)
    out = {}
    for tag, T, tk, E, bm in (("a", 37, 8, 16, 4), ("b", 256, 8, 128, 32), ("c", 5, 2, 64, 16)):
        ids = torch.randint(0, E, (T, tk), generator=g)
        if tag == "a":
            ids[3, 1] = E          # dropped-pair sentinel
            ids[20, 7] = E
        sr, eids, cap, inv = R.moe_align(ids, bm, E)
        out.update({f"{tag}_ids": ids, f"{tag}_E": np.int64(E), f"{tag}_bm": np.int64(bm),
                    f"{tag}_sorted_rows": sr, f"{tag}_expert_ids": eids, f"{tag}_cap": np.int64(cap),
                    f"{tag}_inv": inv})
    save("moe_align.npz", **out)


def _gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


_gelu_tanh.__name__ = "gelu_pytorch_tanh"


def gen_moe():
    import fused_moe_w4 as V1
    import fused_moe_w4_v2 as V2
    from w4a16 import quantize_w4
    g = torch.Generator().manual_seed(13)
    out = {}
    for tag, T, H, I, E, tk in (("s", 12, 256, 64, 8, 4), ("m", 20, 512, 128, 6, 2)):
        gate_up = torch.randn(E, 2 * I, H, generator=g) * 0.02
        down = torch.randn(E, H, I, generator=g) * 0.02
        def pack(W3, gs):
            qs, ss, zs = zip(*[quantize_w4(W3[e], gs) for e in range(W3.shape[0])])
            return torch.stack(qs), torch.stack(ss), torch.stack(zs)
        gu_q, gu_s, gu_z = pack(gate_up, 128)
        dn_q, dn_s, dn_z = pack(down, 64)
        exp = types.SimpleNamespace(gu_q=gu_q, gu_s=gu_s, gu_z=gu_z, dn_q=dn_q, dn_s=dn_s,
                                    dn_z=dn_z, act_fn=_gelu_tanh, num_experts=E)
        hs = (torch.randn(T, H, generator=g) * 0.5).half()
        ids = torch.randint(0, E, (T, tk), generator=g)
        wts = torch.softmax(torch.randn(T, tk, generator=g), -1).half()
        y2 = V2.fused_moe_w4_v2(hs, exp, ids, wts)     # Triton kernels, interpreted
        y1 = V1.fused_moe_w4(hs, exp, ids, wts)
        out.update({f"{tag}_hidden": hs, f"{tag}_ids": ids, f"{tag}_w": wts, f"{tag}_gu_q": gu_q,
                    f"{tag}_gu_s": gu_s, f"{tag}_gu_z": gu_z, f"{tag}_dn_q": dn_q,
                    f"{tag}_dn_s": dn_s, f"{tag}_dn_z": dn_z, f"{tag}_y_v2": y2, f"{tag}_y_v1": y1})
    save("moe_layer.npz", **out)


def gen_rmsnorm():
    import fused_rmsnorm as R
    g = torch.Generator().manual_seed(14)
    out = {}
    for tag, rows, cols, dt in (("f16", 5, 2816, torch.float16), ("bf16", 3, 256, torch.bfloat16)):
        x = (torch.randn(rows, cols, generator=g) * 0.7).to(dt)
        w = (1.0 + 0.1 * torch.randn(cols, generator=g)).to(dt)
        y = R.fused_rmsnorm(x, w, 1e-6)
        out.update({f"{tag}_x": x.float(), f"{tag}_w": w.float(), f"{tag}_y": y.float()})
    save("rmsnorm.npz", **out)


def gen_sampler():
    import triton
    import triton.language as tl
    import fused_sampler_ops as R

    @triton.jit
    def _rand_kernel(Out, V, seed, BLOCK: tl.constexpr):
        row = tl.program_id(0)
        offs = tl.arange(0, BLOCK)
        u = tl.rand(seed + row, offs)
        tl.store(Out + row * V + offs, u, mask=offs < V)

    g = torch.Generator().manual_seed(15)
    out = {}
    # raw tl.rand stream (the Triton function the reference calls), incl. the i32 seed wrap
    for tag, seed in (("r0", 1234), ("r1", 2**31 - 2), ("r2", 0)):
        u = torch.empty(3, 256)
        _rand_kernel[(3,)](u, 256, seed, BLOCK=256)
        out[f"{tag}_u"] = u
        out[f"{tag}_seed"] = np.int64(seed)
    for tag, rows, V, seed in (("s0", 4, 5000, 1234), ("s1", 3, 4097, 2**31 - 2),
                               ("s2", 2, 8192, 987654321)):
        x = torch.randn(rows, V, generator=g) * 3
        x[0, 17] += 15.0
        h = R.fused_entropy(x)
        samp, amax = R.gumbel_argmax_sample(x, seed)
        out.update({f"{tag}_x": x, f"{tag}_seed": np.int64(seed), f"{tag}_h": h,
                    f"{tag}_samp": samp, f"{tag}_amax": amax})
    save("sampler.npz", **out)


def gen_accept():
    # fast_sampler imports transformers' DiffusionGemma generation module only for class names;
    # give it a stand-in with those attributes so the reference functions can run as written.
    mod = types.ModuleType("transformers.models.diffusion_gemma.generation_diffusion_gemma")
    for name in ("EntropyBoundSampler", "StableAndConfidentStoppingCriteria",
                 "DiffusionGemmaGenerationMixin"):
        setattr(mod, name, type(name, (), {}))
    pkg = types.ModuleType("transformers.models.diffusion_gemma")
    pkg.generation_diffusion_gemma = mod
    sys.modules["transformers.models.diffusion_gemma"] = pkg
    sys.modules["transformers.models.diffusion_gemma.generation_diffusion_gemma"] = mod
    import fast_sampler as R
    g = torch.Generator().manual_seed(16)
    out = {}
    for tag, L, scale, bound in (("a", 256, 0.02, 0.1), ("b", 256, 0.002, 0.1), ("c", 64, 0.5, 2.0)):
        logits = torch.randn(1, L, 50, generator=g) / scale
        H = torch.distributions.Categorical(logits=logits).entropy()
        cur = torch.randint(0, 1000, (1, L), generator=g)
        prop = torch.randint(0, 1000, (1, L), generator=g)
        sampler = types.SimpleNamespace(entropy_bound=bound)
        res = R._accept_canvas(sampler, cur, prop, logits, 0)
        crit = types.SimpleNamespace(stability_threshold=2, argmax_canvas_history=None,
                                     confidence_threshold=0.005)
        am = logits.argmax(-1)
        f1 = R._stop_call(crit, am, logits)
        f2 = R._stop_call(crit, am, logits)
        f3 = R._stop_call(crit, am, logits)
        out.update({f"{tag}_H": H, f"{tag}_cur": cur, f"{tag}_prop": prop,
                    f"{tag}_bound": np.float64(bound), f"{tag}_mask": sampler.accepted_token_mask,
                    f"{tag}_out": res, f"{tag}_argmax": am,
                    f"{tag}_stop": torch.stack([f1, f2, f3])})
    save("accept.npz", **out)


if __name__ == "__main__":
    torch.manual_seed(0)
    gen_w4a16()
    gen_align()
    gen_rmsnorm()
    gen_sampler()
    gen_accept()
    gen_moe()
