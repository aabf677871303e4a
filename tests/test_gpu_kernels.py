"""GPU parity tests: every sm_100a kernel through libknx.so against the CPU oracle (and, where a
fixture exists, against the reference's own outputs).  Tolerances are the north-star ones:
integers / indices / masks bit-exact; fp16 outputs |d| <= 2e-3 + 1e-2 |ref|; entropy 1e-4 rel."""
import numpy as np
import pytest
import torch

from conftest import assert_close_fp16, golden
from oracle import ref

pytestmark = pytest.mark.gpu


def _to(d, dev):
    return {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in d.items()}


# ------------------------------------------------------------------------------ RMSNorm
@pytest.mark.parametrize("rows,cols,dt,has_w", [
    (256, 2816, torch.float16, True), (7, 2816, torch.bfloat16, True), (33, 256, torch.float16, False),
    (5, 8192, torch.float16, True), (1, 64, torch.bfloat16, True)])
def test_rmsnorm_vs_oracle(cuda, rows, cols, dt, has_w):
    import fused_rmsnorm
    g = torch.Generator().manual_seed(rows * 31 + cols)
    x = (torch.randn(rows, cols, generator=g) * 0.8).to(dt)
    w = (1 + 0.1 * torch.randn(cols, generator=g)).to(dt) if has_w else None
    for rb in (True, False):
        y = fused_rmsnorm.fused_rmsnorm(x.to(cuda), w.to(cuda) if w is not None else None, 1e-6,
                                        round_bf16=rb)
        want = ref.rmsnorm(x, w, 1e-6, round_bf16=rb)
        assert y.dtype == dt
        assert_close_fp16(y, want, what=f"rmsnorm rb={rb}")


def test_rmsnorm_golden_and_kperm(cuda):
    import _knx
    import fused_rmsnorm
    gd = golden("rmsnorm.npz")
    x = torch.from_numpy(gd["f16_x"]).half()
    w = torch.from_numpy(gd["f16_w"]).half()
    xp = torch.empty_like(x, device=cuda)
    y = fused_rmsnorm.fused_rmsnorm(x.to(cuda), w.to(cuda), 1e-6, xperm=xp)
    assert_close_fp16(y, torch.from_numpy(gd["f16_y"]), what="vs reference")
    assert torch.equal(xp.cpu(), ref.kperm(y.cpu()))


# ------------------------------------------------------------------------------ align
@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_moe_align_matches_reference_golden(cuda, tag):
    import fused_moe_w4
    gd = golden("moe_align.npz")
    ids = torch.from_numpy(gd[f"{tag}_ids"]).to(cuda)
    sr, eids, cap, inv = fused_moe_w4.moe_align(ids, int(gd[f"{tag}_bm"]), int(gd[f"{tag}_E"]))
    assert cap == int(gd[f"{tag}_cap"])
    assert np.array_equal(sr.cpu().numpy(), gd[f"{tag}_sorted_rows"])
    assert np.array_equal(eids.cpu().numpy(), gd[f"{tag}_expert_ids"])
    assert np.array_equal(inv.cpu().numpy(), gd[f"{tag}_inv"])


@pytest.mark.parametrize("T,tk,E,skew", [(256, 8, 128, True), (1, 8, 128, False), (7, 2, 16, True),
                                         (4096, 8, 128, True), (100, 8, 256, False)])
def test_moe_align_unpadded_exact(cuda, T, tk, E, skew):
    import fused_moe_w4
    g = torch.Generator().manual_seed(T + E)
    if skew:   # heavy skew: most pairs on expert 3
        ids = torch.where(torch.rand(T, tk, generator=g) < 0.6, torch.full((T, tk), 3),
                          torch.randint(0, E, (T, tk), generator=g))
    else:
        ids = torch.randint(0, E, (T, tk), generator=g)
    ids[0, 0] = E  # one dropped pair
    for dt in (torch.int64, torch.int32):
        c, o, sp, inv = fused_moe_w4.moe_align_unpadded(ids.to(dt).to(cuda), E)
        rc, ro, rsp, rinv = ref.moe_align_unpadded(ids.numpy(), E)
        assert np.array_equal(c.cpu().numpy(), rc)
        assert np.array_equal(o.cpu().numpy(), ro)
        assert np.array_equal(sp.cpu().numpy(), rsp)
        assert np.array_equal(inv.cpu().numpy(), rinv)


# ------------------------------------------------------------------------------ MoE layer
@pytest.mark.parametrize("tag", ["s", "m"])
def test_moe_layer_vs_reference_golden(cuda, tag):
    import fused_moe_w4_v2
    gd = golden("moe_layer.npz")
    t = {k[len(tag) + 1:]: torch.from_numpy(v) for k, v in gd.items() if k.startswith(tag + "_")}
    d = _to(t, cuda)
    y = fused_moe_w4_v2.moe_forward(d["hidden"], d["gu_q"], d["gu_s"], d["gu_z"], d["dn_q"],
                                    d["dn_s"], d["dn_z"], d["ids"], d["w"])
    assert_close_fp16(y, t["y_v2"], what="vs reference v2 kernel")
    want = ref.moe_layer(t["hidden"], t["gu_q"], t["gu_s"], t["gu_z"], t["dn_q"], t["dn_s"],
                         t["dn_z"], t["ids"], t["w"])
    assert_close_fp16(y, want, what="vs oracle")


def _moe_case(T, E, H, I, tk, seed, skew=None):
    import workloads
    W = workloads.moe_weights(E, H, I, seed=seed)
    g = torch.Generator().manual_seed(seed + 5)
    hidden = torch.randn(T, H, generator=g).half()
    ids, w = workloads.random_routing(T, E, tk, seed=seed)
    if skew == "one":
        ids[:, 0] = 1          # every token hits expert 1 (count T > task size: chunked tasks)
    elif skew == "drop":
        ids[::3, -1] = E       # dropped pairs (reference sentinel)
    return W, hidden, ids, w


@pytest.mark.parametrize("engine", ["tc", "ws", "mma"])
@pytest.mark.parametrize("T,E,H,I,tk,skew", [
    (256, 128, 2816, 704, 8, None),       # configs[0] shapes
    (1, 128, 2816, 704, 8, None), (7, 16, 512, 128, 4, None), (33, 8, 256, 64, 2, "one"),
    (100, 32, 768, 192, 8, "drop"), (300, 4, 256, 64, 2, "one")])
def test_moe_layer_vs_oracle(cuda, T, E, H, I, tk, skew, engine):
    import fused_moe_w4_v2
    W, hidden, ids, w = _moe_case(T, E, H, I, tk, seed=T + E, skew=skew)
    Wd = _to(W, cuda)
    y = fused_moe_w4_v2.moe_forward(hidden.to(cuda), Wd["gu_q"], Wd["gu_s"], Wd["gu_z"], Wd["dn_q"],
                                    Wd["dn_s"], Wd["dn_z"], ids.to(cuda), w.to(cuda), engine=engine)
    want = ref.moe_layer(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"], W["dn_z"],
                         ids, w)
    assert_close_fp16(y, want, what=f"moe {engine} T={T} E={E} H={H}")


def test_moe_engines_agree_and_are_deterministic(cuda):
    import fused_moe_w4_v2
    W, hidden, ids, w = _moe_case(256, 128, 2816, 704, 8, seed=21)
    Wd = _to(W, cuda)
    args = (Wd["gu_q"], Wd["gu_s"], Wd["gu_z"], Wd["dn_q"], Wd["dn_s"], Wd["dn_z"])
    ys = {}
    for eng in ("tc", "ws", "mma"):
        a = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *args, ids.to(cuda), w.to(cuda), engine=eng)
        b = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *args, ids.to(cuda), w.to(cuda), engine=eng)
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), eng
        ys[eng] = a
    assert_close_fp16(ys["tc"], ys["mma"], what="tc vs mma")
    assert_close_fp16(ys["ws"], ys["mma"], what="ws vs mma")


def test_moe_integer_zeros_exact_dequant(cuda):
    """quantize_w4 packs (integer zero-points): both engines dequantise bit-identically to
    dequant_w4, so the layer matches the oracle at the unscaled fp16 tolerance too."""
    import fused_moe_w4_v2
    import workloads
    E, H, I, T, tk = 8, 512, 128, 48, 4
    g = torch.Generator().manual_seed(5)
    packs = {}
    for nm, (N_, K_, gs_) in {"gu": (2 * I, H, 128), "dn": (H, I, 64)}.items():
        qs, ss, zs = zip(*[ref.quantize_w4(torch.randn(N_, K_, generator=g) * 0.02, gs_)
                           for _ in range(E)])
        packs[nm] = (torch.stack(qs), torch.stack(ss), torch.stack(zs))
    hidden = (torch.randn(T, H, generator=g) * 0.5).half()
    ids, w = workloads.random_routing(T, E, tk, seed=5)
    want = ref.moe_layer(hidden, *packs["gu"], *packs["dn"], ids, w)
    for eng in ("tc", "ws", "mma"):
        y = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *[t.to(cuda) for t in packs["gu"]],
                                        *[t.to(cuda) for t in packs["dn"]], ids.to(cuda),
                                        w.to(cuda), engine=eng)
        assert_close_fp16(y, want, what=eng)


def test_moe_layer_dtypes_and_bit_identical_reruns(cuda):
    import fused_moe_w4_v2
    W, hidden, ids, w = _moe_case(64, 16, 512, 128, 8, seed=9)
    Wd = _to(W, cuda)
    args = (Wd["gu_q"], Wd["gu_s"], Wd["gu_z"], Wd["dn_q"], Wd["dn_s"], Wd["dn_z"])
    base = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *args, ids.to(cuda), w.to(cuda))
    for _ in range(3):
        again = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *args, ids.to(cuda), w.to(cuda))
        assert torch.equal(base.view(torch.int16), again.view(torch.int16))
    # int32 ids, f16 / bf16 / f32 weights: same result up to the weight rounding
    for wd in (torch.float16, torch.bfloat16):
        y = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *args, ids.int().to(cuda), w.to(wd).to(cuda))
        want = ref.moe_layer(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                             W["dn_z"], ids, w.to(wd).float())
        assert_close_fp16(y, want, what=str(wd))
    yb = fused_moe_w4_v2.moe_forward(hidden.bfloat16().to(cuda), *args, ids.to(cuda), w.to(cuda))
    assert yb.dtype == torch.bfloat16
    want = ref.moe_layer(hidden.bfloat16(), W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                         W["dn_z"], ids, w)
    assert_close_fp16(yb, want, what="bf16 hidden")


def test_moe_exp_object_api(cuda):
    import types
    import fused_moe_w4
    import fused_moe_w4_v2
    W, hidden, ids, w = _moe_case(16, 8, 256, 64, 2, seed=3)
    Wd = _to(W, cuda)
    act = lambda x: torch.nn.functional.gelu(x, approximate="tanh")
    act.__name__ = "gelu_pytorch_tanh"
    exp = types.SimpleNamespace(act_fn=act, num_experts=8, **Wd)
    y1 = fused_moe_w4_v2.fused_moe_w4_v2(hidden.to(cuda), exp, ids.to(cuda), w.to(cuda))
    y0 = fused_moe_w4.fused_moe_w4(hidden.to(cuda), exp, ids.to(cuda), w.to(cuda))
    assert torch.equal(y0, y1)
    # the reference's MOE_NS down layout is accepted (converted back once)
    exp2 = types.SimpleNamespace(act_fn=act, num_experts=8, **Wd)
    exp2.dn_q = fused_moe_w4_v2.preshuffle_T_dn(Wd["dn_q"])
    exp2.dn_ns = True
    y2 = fused_moe_w4_v2.fused_moe_w4_v2(hidden.to(cuda), exp2, ids.to(cuda), w.to(cuda))
    assert torch.equal(y1, y2)


# ------------------------------------------------------------------------------ dense linear
@pytest.mark.parametrize("tag", ["g128", "g64"])
def test_w4a16_linear_vs_reference_golden(cuda, tag):
    import w4a16
    gd = golden("w4a16.npz")
    gs = int(gd[f"{tag}_gs"])
    Y = w4a16.w4a16_linear(torch.from_numpy(gd[f"{tag}_X"]).to(cuda),
                           torch.from_numpy(gd[f"{tag}_q"]).to(cuda),
                           torch.from_numpy(gd[f"{tag}_s"]).to(cuda),
                           torch.from_numpy(gd[f"{tag}_z"]).to(cuda), BK=gs)
    assert_close_fp16(Y, torch.from_numpy(gd[f"{tag}_Y"]), what=tag)


@pytest.mark.parametrize("engine", ["tc", "ws", "mma"])
@pytest.mark.parametrize("N,K,M", [(2816, 2816, 256), (1408, 2816, 64), (2816, 704, 64),
                                   (4096, 2816, 256), (200, 256, 3), (1408, 2816, 130),
                                   # 24 scale groups: the tcgen05 engine's largest shared-memory
                                   # configuration; 25: past it (another engine takes the shape)
                                   (512, 3072, 256), (192, 3200, 129)])
def test_w4a16_linear_killtest_shapes(cuda, N, K, M, engine):
    import w4a16
    gs = 128 if K % 128 == 0 else 64
    g = torch.Generator().manual_seed(N + K)
    Wt = torch.randn(N, K, generator=g) * 0.02
    Wt[:, : K // 40] += torch.randn(N, K // 40, generator=g) * 0.15
    q, s, z = ref.quantize_w4(Wt, gs)
    X = torch.randn(M, K, generator=g).half()
    Y = w4a16.w4a16_linear(X.to(cuda), q.to(cuda), s.to(cuda), z.to(cuda), BK=gs, engine=engine)
    want = (X.float() @ ref.dequant_w4(q, s, z, gs).float().T).half()
    assert_close_fp16(Y, want, what=f"{N}x{K}@{M}")


def test_quantize_on_gpu_matches_oracle(cuda):
    import w4a16
    Wt = torch.randn(96, 512, generator=torch.Generator().manual_seed(2)) * 0.05
    q, s, z = w4a16.quantize_w4(Wt.to(cuda), 128)
    rq, rs, rz = ref.quantize_w4(Wt, 128)
    assert torch.equal(q.cpu(), rq) and torch.equal(s.cpu(), rs) and torch.equal(z.cpu(), rz)
    assert torch.equal(w4a16.dequant_w4(q, s, z, 128).cpu(), ref.dequant_w4(rq, rs, rz, 128))


# ------------------------------------------------------------------------------ router
def test_router_topk_exact_given_logits(cuda):
    import moe_router
    import workloads
    inp = workloads.moe_inputs(256, 2816, 128, seed=0)
    ids, w, logits = moe_router.route_topk(inp["hidden"].to(cuda), inp["router_w"].to(cuda), 8,
                                           bias=inp["bias"].to(cuda))
    lg = logits.cpu()
    want_logits = inp["hidden"].float() @ inp["router_w"].float().T + inp["bias"]
    assert (lg - want_logits).abs().max().item() < 1e-3
    rid, rw, _ = ref.router_topk(None, None, None, 8, logits=lg)
    assert torch.equal(ids.cpu(), rid)
    assert (w.cpu() - rw).abs().max().item() < 1e-6
    counts = torch.bincount(ids.cpu().flatten().long(), minlength=128)
    assert counts.max().item() > 40    # the Zipf bias skews routing


@pytest.mark.parametrize("T,H,E,rb,with_bias", [(256, 2816, 128, True, True),
                                                 (100, 2816, 128, False, True),
                                                 (7, 1024, 64, True, False),
                                                 (513, 2816, 128, True, True),
                                                 (33, 3840, 64, False, True)])
def test_fused_rmsnorm_router_bit_identical_to_two_calls(cuda, T, H, E, rb, with_bias):
    """knx_rmsnorm_router_topk (one clustered launch) against knx_rmsnorm + knx_router_topk:
    y, the K-interleaved copy, logits, ids and weights all bit for bit."""
    import ctypes
    import _knx
    import fused_rmsnorm
    import moe_router
    import workloads
    inp = workloads.moe_inputs(T, H, E, seed=T + H, device=cuda)
    bias = inp["bias"] if with_bias else None
    xp1 = torch.empty(T, H, dtype=torch.float16, device=cuda)
    y1 = fused_rmsnorm.fused_rmsnorm(inp["hidden"], inp["norm_w"], 1e-6, round_bf16=rb, xperm=xp1)
    ids1, w1, lg1 = moe_router.route_topk(y1, inp["router_w"], 8, bias=bias)
    # the one-launch path itself (not the two-call fallback of rmsnorm_route_topk)
    lib = _knx.load()
    y2 = torch.empty(T, H, dtype=torch.float16, device=cuda)
    xp2 = torch.empty_like(xp1)
    ids2 = torch.empty(T, 8, dtype=torch.int32, device=cuda)
    w2 = torch.empty(T, 8, dtype=torch.float32, device=cuda)
    lg2 = torch.empty(T, E, dtype=torch.float32, device=cuda)
    vp = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    st = lib.knx_rmsnorm_router_topk(vp(inp["hidden"]), vp(inp["norm_w"]), 1e-6,
                                     _knx.KNX_RMS_ROUND_BF16 if rb else 0, vp(inp["router_w"]),
                                     vp(bias), T, H, E, 8, vp(y2), vp(xp2), vp(lg2), vp(ids2),
                                     vp(w2), _knx.stream_of(cuda.index or 0))
    assert st == 0, st
    torch.cuda.synchronize()
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    assert torch.equal(xp1.view(torch.int16), xp2.view(torch.int16))
    assert torch.equal(lg1.view(torch.int32), lg2.view(torch.int32))
    assert torch.equal(ids1, ids2)
    assert torch.equal(w1.view(torch.int32), w2.view(torch.int32))


def test_fused_rmsnorm_router_unsupported_shape_falls_back(cuda):
    import moe_router
    import workloads
    inp = workloads.moe_inputs(64, 1024, 256, seed=5, device=cuda)  # E = 256: two-call path
    y, ids, w, lg = moe_router.rmsnorm_route_topk(inp["hidden"], inp["norm_w"], 1e-6,
                                                  inp["router_w"], 8, bias=inp["bias"])
    assert ids.shape == (64, 8) and torch.isfinite(w).all()


# ------------------------------------------------------------------------------ sampler
@pytest.mark.parametrize("tag", ["s0", "s1", "s2"])
def test_sampler_vs_reference_golden(cuda, tag):
    import fused_sampler_ops
    gd = golden("sampler.npz")
    x = torch.from_numpy(gd[f"{tag}_x"]).to(cuda)
    h = fused_sampler_ops.fused_entropy(x)
    s, a = fused_sampler_ops.gumbel_argmax_sample(x, int(gd[f"{tag}_seed"]))
    assert np.array_equal(a.cpu().numpy(), gd[f"{tag}_amax"])
    assert np.array_equal(s.cpu().numpy(), gd[f"{tag}_samp"])
    want = torch.from_numpy(gd[f"{tag}_h"])
    assert ((h.cpu() - want).abs() / want.abs().max()).max().item() < 1e-4


@pytest.mark.parametrize("rows,V,step", [(8, 262144, 0), (8, 262144, 47), (5, 100003, 20),
                                         (3, 4096, 5), (2, 1, 0)])
def test_sampler_step_vs_oracle(cuda, rows, V, step):
    import fused_sampler_ops
    import workloads
    x = workloads.sampler_logits(rows, V, seed=rows + V, spike_frac=0.3)
    T = np.float32(workloads.temperature(step))
    seed = workloads.step_seed(1234, step)
    h, s, a = fused_sampler_ops.sample_step(x.to(cuda), seed, float(T))
    rs, ra = ref.gumbel_argmax(x, seed, temperature=float(T))
    assert np.array_equal(a.cpu().numpy(), ra.numpy())
    assert np.array_equal(s.cpu().numpy(), rs.numpy())
    rh = ref.entropy(x / torch.tensor(T), dtype=torch.float64)
    assert ((h.cpu().double() - rh).abs() <= 1e-4 * rh.abs() + 1e-7).all()
    # determinism
    h2, s2, a2 = fused_sampler_ops.sample_step(x.to(cuda), seed, float(T))
    assert torch.equal(h, h2) and torch.equal(s, s2) and torch.equal(a, a2)


def test_sampler_full_size_properties(cuda):
    """configs[2] size: argmax exact for all 256 rows; samples exact on a subset (oracle time)."""
    import fused_sampler_ops
    import workloads
    x = workloads.sampler_logits(256, 262144, seed=0, device="cuda")
    T = np.float32(workloads.temperature(10))
    seed = workloads.step_seed(1234, 10)
    h, s, a = fused_sampler_ops.sample_step(x, seed, float(T))
    q = x / torch.tensor(T, device=cuda)
    assert torch.equal(a, q.argmax(-1))
    rows = [0, 1, 77, 255]
    assert seed + 255 < 2**31          # per-row keys: the row's Philox key is seed + row
    for r in rows:
        r_s, _ = ref.gumbel_argmax(x[r:r + 1].cpu(), seed + r, temperature=float(T))
        assert s[r].item() == r_s[0].item()
    rh = ref.entropy(q.cpu(), dtype=torch.float64)
    assert ((h.cpu().double() - rh).abs() <= 1e-4 * rh.abs() + 1e-7).all()


@pytest.mark.parametrize("V,step", [(262144, 0), (262144, 30), (262144, 47), (4099, 30)])
def test_sampler_masked_and_infinite_rows(cuda, V, step):
    """Rows that bound or index handling could get wrong, on the streaming path (V = 262144) and
    the generic one (V = 4099): masked (-inf) rows, a fully masked row (index 0, as the
    reference's scan keeps its initial index), +inf entries (the first wins), NaN entries, a far
    spike and ties."""
    import fused_sampler_ops
    import workloads
    g = torch.Generator().manual_seed(step + 11)
    x = torch.randn(8, V, generator=g) * 3.0
    x[1][torch.rand(V, generator=g) < 0.99] = -float("inf")     # 99% masked
    x[2][:] = -float("inf")
    x[2][[5, (3 * V) // 4]] = torch.tensor([1.0, 2.0])           # two finite columns
    x[3][[V // 250, V // 2 + 7]] = float("inf")                  # +inf twice: the first wins
    x[4][:] = -float("inf")                                      # fully masked row
    x[5][3] += 40.0                                              # one far spike
    x[6][:] = 1.0                                                # all equal
    x[7][[7, V // 3, V - 1]] = float("nan")
    T = np.float32(workloads.temperature(step))
    seed = workloads.step_seed(1234, step)
    h, s, a = fused_sampler_ops.sample_step(x.to(cuda), seed, float(T))
    rs, ra = ref.gumbel_argmax(x, seed, temperature=float(T))
    assert np.array_equal(s.cpu().numpy(), rs.numpy())
    assert np.array_equal(a.cpu().numpy(), ra.numpy())
    assert s[3].item() == V // 250 and s[4].item() == 0 and a[4].item() == 0
    # entropy of the finite entries (rows with -inf entries: the reference's x * e term is
    # -inf * 0 = NaN there, this library leaves masked entries out of the sum)
    q = x.double() / float(T)
    for r in (0, 1, 2, 5, 6):
        qr = q[r][torch.isfinite(q[r])]
        p = torch.softmax(qr, 0)
        want = -(p * torch.log_softmax(qr, 0)).sum().item()
        assert abs(h[r].item() - want) <= 1e-4 * abs(want) + 1e-6, (r, h[r].item(), want)
    assert h[4].item() == 0.0


# ------------------------------------------------------------------------------ accept / stop
@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_accept_stop_vs_reference_golden(cuda, tag):
    import accept_ops
    gd = golden("accept.npz")
    H = torch.from_numpy(gd[f"{tag}_H"]).to(cuda)
    cur = torch.from_numpy(gd[f"{tag}_cur"]).to(cuda)
    prop = torch.from_numpy(gd[f"{tag}_prop"]).to(cuda)
    mask, out = accept_ops.accept_canvas(H, cur, prop, float(gd[f"{tag}_bound"]))
    assert np.array_equal(mask.cpu().numpy(), gd[f"{tag}_mask"])
    assert np.array_equal(out.cpu().numpy(), gd[f"{tag}_out"])
    am = torch.from_numpy(gd[f"{tag}_argmax"]).to(cuda)
    hist = torch.full((2,) + tuple(am.shape), -1, dtype=torch.int64, device=cuda)
    got = []
    for _ in range(3):
        _, _, fin = accept_ops.accept_and_stop(H, cur, prop, float(gd[f"{tag}_bound"]), am, hist,
                                               0.005)
        got.append(fin.cpu())
    assert np.array_equal(torch.stack(got).numpy(), gd[f"{tag}_stop"])


def test_accept_ties_and_batches_vs_oracle(cuda):
    import accept_ops
    g = torch.Generator().manual_seed(4)
    H = torch.rand(3, 256, generator=g) * 0.01
    H[0, 10:20] = 0.003          # ties: stable order by position
    H[1] = 0.0005                # all equal
    cur = torch.randint(0, 99, (3, 256), generator=g)
    prop = torch.randint(0, 99, (3, 256), generator=g)
    mask, out = accept_ops.accept_canvas(H.to(cuda), cur.to(cuda), prop.to(cuda), 0.1)
    rm, ro = ref.accept_canvas(H, cur, prop, 0.1)
    assert torch.equal(mask.cpu(), rm) and torch.equal(out.cpu(), ro)


def test_align_large_matches_unpadded_reference(cuda):
    """More pairs than one CTA holds: the multi-CTA counting sort gives the same stable
    permutation (experts ascending, pairs ascending within an expert; bad ids dropped)."""
    import fused_moe_w4
    g = torch.Generator().manual_seed(77)
    for T, tk, E in ((4608, 8, 128), (20000, 8, 256), (5000, 7, 64)):
        ids = torch.randint(0, E, (T, tk), generator=g, dtype=torch.int32)
        ids[3, 2] = E  # dropped
        counts, offsets, sp, inv = fused_moe_w4.moe_align_unpadded(ids.to(cuda), E)
        flat = ids.flatten().long()
        valid = flat < E
        order = torch.argsort(torch.where(valid, flat, torch.full_like(flat, E)), stable=True)
        nv = int(valid.sum())
        assert torch.equal(counts.cpu().long(), torch.bincount(flat[valid], minlength=E))
        assert torch.equal(sp.cpu()[:nv].long(), order[:nv])
        assert (sp.cpu()[nv:] == T * tk).all()
        want_inv = torch.full((T * tk,), -1, dtype=torch.long)
        want_inv[order[:nv]] = torch.arange(nv)
        assert torch.equal(inv.cpu().long(), want_inv)


def test_moe_layer_large_batch_matches_small_batches(cuda):
    """A 4608-token layer (36864 pairs, multi-CTA permutation) equals the same tokens run as
    256-token layers, row for row, with the same engine."""
    import fused_moe_w4_v2
    import workloads
    W = workloads.moe_weights(128, 2816, 704, seed=61, device=cuda)
    args = (W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"], W["dn_z"])
    T = 4608
    g = torch.Generator(device=cuda).manual_seed(62)
    hidden = (torch.randn(T, 2816, generator=g, device=cuda) * 0.5).half()
    ids, w = workloads.random_routing(T, 128, 8, seed=63, device=cuda)
    for eng in ("ws", "tc"):
        big = fused_moe_w4_v2.moe_forward(hidden, *args, ids, w, engine=eng)
        parts = [fused_moe_w4_v2.moe_forward(hidden[i:i + 256], *args, ids[i:i + 256],
                                             w[i:i + 256], engine=eng) for i in range(0, T, 256)]
        assert torch.equal(big.view(torch.int16), torch.cat(parts).view(torch.int16)), eng
