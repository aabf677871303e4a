"""Pin the CPU oracle: every restated function against fixtures produced by the reference's own
code (tests/golden/make_golden.py) and against published known-answer vectors."""
import numpy as np
import pytest
import torch

from conftest import assert_close_fp16, golden
from oracle import ref


# Published Philox4x32-10 known-answer vectors (Random123 kat_vectors; Salmon et al. SC'11).
PHILOX_KAT = [
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
    ((0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff), (0xffffffff, 0xffffffff),
     (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
    ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
     (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1)),
]


@pytest.mark.parametrize("ctr,key,expect", PHILOX_KAT)
def test_philox_known_answers(ctr, key, expect):
    assert tuple(ref.philox4x32_10(ctr, key)) == expect


def test_uniform_stream_matches_triton_tl_rand():
    g = golden("sampler.npz")
    for tag in ("r0", "r1", "r2"):
        seed = int(g[f"{tag}_seed"])
        u = g[f"{tag}_u"]
        rows, V = u.shape
        lib = ref.clib()
        import ctypes
        key = (ctypes.c_uint32 * 2)()
        lib.oracle_row_key.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
        lib.oracle_uniform.argtypes = [ctypes.c_uint32]
        lib.oracle_uniform.restype = ctypes.c_float
        lib.oracle_philox_w0.argtypes = [ctypes.c_uint32, ctypes.c_void_p]
        lib.oracle_philox_w0.restype = ctypes.c_uint32
        mine = np.empty_like(u)
        for r in range(rows):
            lib.oracle_row_key(seed, r, key)
            for c in range(V):
                mine[r, c] = lib.oracle_uniform(lib.oracle_philox_w0(c, key))
        assert np.array_equal(mine.view(np.uint32), u.view(np.uint32)), tag


def test_oracle_log_accuracy():
    lib = ref.clib()
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.uniform(1e-10, 1.0, 20000), rng.uniform(1e-7, 30.0, 20000),
                         np.float32([1.0, 0.5, 2.0, 1.1920929e-07, 23.02585])]).astype(np.float32)
    got = np.array([lib.oracle_log(float(x)) for x in xs], dtype=np.float32)
    exact = np.log(xs.astype(np.float64))
    ulp = np.spacing(np.abs(exact).astype(np.float32)).astype(np.float64)
    err_ulp = np.abs(got.astype(np.float64) - exact) / np.maximum(ulp, 1e-45)
    assert err_ulp.max() <= 3.0, err_ulp.max()  # faithful to ~2 ulp; bit-identity CPU/GPU is what matters


def test_markstein_division_is_ieee_for_schedule_temperatures():
    lib = ref.clib()
    for step in range(0, 48, 7):
        T = np.float32(ref.temperature(step, 48, 0.4, 0.8))
        assert lib.oracle_markstein_mismatches(float(T), 200000, 77 + step) == 0


def test_gumbel_argmax_matches_reference_kernel():
    g = golden("sampler.npz")
    for tag in ("s0", "s1", "s2"):
        x = torch.from_numpy(g[f"{tag}_x"])
        samp, amax = ref.gumbel_argmax(x, int(g[f"{tag}_seed"]))
        assert np.array_equal(amax.numpy(), g[f"{tag}_amax"]), tag
        assert np.array_equal(samp.numpy(), g[f"{tag}_samp"]), tag


def test_entropy_matches_reference_kernel():
    g = golden("sampler.npz")
    for tag in ("s0", "s1", "s2"):
        h = ref.entropy(torch.from_numpy(g[f"{tag}_x"]))
        want = torch.from_numpy(g[f"{tag}_h"])
        rel = ((h - want).abs().max() / want.abs().max()).item()
        assert rel < 1e-5, (tag, rel)


def test_moe_align_matches_reference():
    g = golden("moe_align.npz")
    for tag in ("a", "b", "c"):
        sr, eids, cap, inv = ref.moe_align(g[f"{tag}_ids"], int(g[f"{tag}_bm"]), int(g[f"{tag}_E"]))
        assert cap == int(g[f"{tag}_cap"])
        assert np.array_equal(sr, g[f"{tag}_sorted_rows"]), tag
        assert np.array_equal(eids, g[f"{tag}_expert_ids"]), tag
        assert np.array_equal(inv, g[f"{tag}_inv"]), tag


def test_moe_align_unpadded_is_padded_order_compacted():
    g = golden("moe_align.npz")
    for tag in ("a", "b", "c"):
        ids, E = g[f"{tag}_ids"], int(g[f"{tag}_E"])
        counts, offsets, sp, inv = ref.moe_align_unpadded(ids, E)
        sr = g[f"{tag}_sorted_rows"]
        N = ids.size
        assert np.array_equal(sp[sp < N], sr[sr < N])
        assert np.array_equal(np.bincount(ids.reshape(-1)[ids.reshape(-1) < E], minlength=E), counts)
        ok = inv >= 0
        assert np.array_equal(sp[inv[ok]], np.nonzero(ok)[0])


def test_quant_dequant_match_reference():
    g = golden("w4a16.npz")
    for tag in ("g128", "g64"):
        gs = int(g[f"{tag}_gs"])
        q, s, z = ref.quantize_w4(torch.from_numpy(g[f"{tag}_W"]), gs)
        assert np.array_equal(q.numpy(), g[f"{tag}_q"])
        assert np.array_equal(s.numpy(), g[f"{tag}_s"])
        assert np.array_equal(z.numpy(), g[f"{tag}_z"])
        w = ref.dequant_w4(q, s, z, gs)
        assert np.array_equal(w.numpy(), g[f"{tag}_wdq"])


def test_dense_linear_oracle_matches_reference_kernel():
    g = golden("w4a16.npz")
    for tag in ("g128", "g64"):
        gs = int(g[f"{tag}_gs"])
        W = ref.dequant_w4(torch.from_numpy(g[f"{tag}_q"]), torch.from_numpy(g[f"{tag}_s"]),
                           torch.from_numpy(g[f"{tag}_z"]), gs)
        y = (torch.from_numpy(g[f"{tag}_X"]).float() @ W.float().T).half()
        assert_close_fp16(y, torch.from_numpy(g[f"{tag}_Y"]), what=tag)


def test_moe_layer_oracle_matches_reference_v2():
    g = golden("moe_layer.npz")
    for tag in ("s", "m"):
        t = {k[len(tag) + 1:]: torch.from_numpy(v) for k, v in g.items() if k.startswith(tag + "_")}
        y = ref.moe_layer(t["hidden"], t["gu_q"], t["gu_s"], t["gu_z"], t["dn_q"], t["dn_s"],
                          t["dn_z"], t["ids"], t["w"])
        assert_close_fp16(y, t["y_v2"], what=f"{tag} vs v2")
        assert_close_fp16(y, t["y_v1"], what=f"{tag} vs v1")


def test_rmsnorm_oracle_matches_reference_kernel():
    g = golden("rmsnorm.npz")
    for tag, dt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
        x = torch.from_numpy(g[f"{tag}_x"]).to(dt)
        w = torch.from_numpy(g[f"{tag}_w"]).to(dt)
        y = ref.rmsnorm(x, w, 1e-6, round_bf16=True)
        want = torch.from_numpy(g[f"{tag}_y"])
        assert_close_fp16(y, want, what=tag)
        # Triton's CPU interpreter casts fp32 -> bf16 by truncation (the GPU rounds to nearest),
        # so the fixture equals the oracle's fp32 result truncated to bf16, bit for bit.
        xf = x.float()
        y32 = (xf / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).numpy()
        rz = torch.from_numpy((y32.view(np.uint32) & 0xFFFF0000).view(np.float32))
        assert torch.equal(rz.to(dt).float(), want), tag


def test_accept_and_stop_match_reference():
    g = golden("accept.npz")
    for tag in ("a", "b", "c"):
        H = torch.from_numpy(g[f"{tag}_H"])
        mask, out = ref.accept_canvas(H, torch.from_numpy(g[f"{tag}_cur"]),
                                      torch.from_numpy(g[f"{tag}_prop"]), float(g[f"{tag}_bound"]))
        assert np.array_equal(mask.numpy(), g[f"{tag}_mask"]), tag
        assert np.array_equal(out.numpy(), g[f"{tag}_out"]), tag
        am = torch.from_numpy(g[f"{tag}_argmax"])
        hist = torch.full((2,) + tuple(am.shape), -1, dtype=am.dtype)
        got = []
        for _ in range(3):
            f, hist = ref.stop_test(am, hist, H, 0.005)
            got.append(f)
        assert np.array_equal(torch.stack(got).numpy(), g[f"{tag}_stop"]), tag


def test_kperm_is_the_interleave():
    x = torch.arange(16)
    assert ref.kperm(x).tolist() == [0, 4, 1, 5, 2, 6, 3, 7, 8, 12, 9, 13, 10, 14, 11, 15]


def test_router_oracle_tie_break_and_renorm():
    logits = torch.tensor([[1.0, 3.0, 3.0, 0.5, 3.0]])
    ids, w, _ = ref.router_topk(None, None, None, 2, logits=logits)
    assert ids.tolist() == [[1, 2]]
    assert abs(w.sum().item() - 1.0) < 1e-6
