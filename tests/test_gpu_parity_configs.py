"""GPU parity at the benchmark configurations themselves (not only at reduced shapes):

* configs[1] end to end: the one-launch RMSNorm + router (Zipf-biased logits, up to ~80 pairs
  on the hottest expert, so its tokens span several tasks) feeding the MoE layer, against the
  CPU oracle stage by stage;
* the 18,432-token expert-parallel batch on one GPU (tcgen05 engine, 4,000+ pairs on
  the hottest expert), checked against the oracle on the hottest and a cold expert;
* the sampler at 256 x 262,144, every row's sampled token at three temperatures of
  the schedule;
* every engine at the configs[0] shape against the oracle and against the W4 arithmetic with
  unrounded weights in float64 (how far each is from the exact math, beside the reference's own
  torch path).
"""
import os

import numpy as np
import pytest
import torch

from conftest import assert_close_fp16
from oracle import ref

pytestmark = pytest.mark.gpu


def _threads():
    return max(1, len(os.sched_getaffinity(0)))


def _near_tie_rows(logits, topk, ulps=4):
    """Rows whose top-(k+1) sorted logits have two neighbours closer than `ulps` fp32 ulps: there
    the ordered top-k list depends on the last bits of the logits."""
    lg = logits.numpy().astype(np.float32)
    srt = -np.sort(-lg, axis=1)[:, :topk + 1]
    gaps = srt[:, :-1].astype(np.float64) - srt[:, 1:].astype(np.float64)
    ulp = np.spacing(np.abs(srt[:, :-1])).astype(np.float64)
    return (gaps < ulps * ulp).any(axis=1)


def test_configs1_pipeline_end_to_end(cuda):
    """RMSNorm -> router (Zipf bias) -> 128-expert top-8 MoE at T=256, the bench's own calls."""
    import fused_moe_w4_v2
    import moe_router
    import workloads
    torch.set_num_threads(_threads())
    T, H, I, E, K = 256, 2816, 704, 128, 8
    inp = workloads.moe_inputs(T, H, E, seed=0)
    W = workloads.moe_weights(E, H, I, seed=100)
    d = {k: v.to(cuda) for k, v in inp.items()}
    xp = torch.empty(T, H, dtype=torch.float16, device=cuda)
    y_norm, ids, w, logits = moe_router.rmsnorm_route_topk(d["hidden"], d["norm_w"], 1e-6,
                                                           d["router_w"], K, bias=d["bias"],
                                                           xperm=xp)
    Wd = {k: v.to(cuda) for k, v in W.items()}
    args = (Wd["gu_q"], Wd["gu_s"], Wd["gu_z"], Wd["dn_q"], Wd["dn_s"], Wd["dn_z"])
    y = fused_moe_w4_v2.moe_forward(y_norm, *args, ids, w, hidden_perm=xp)
    # RMSNorm (the reference kernel's bf16 store, then the f16 cast) and its interleaved copy
    want_norm = ref.rmsnorm(inp["hidden"], inp["norm_w"], 1e-6, round_bf16=True)
    assert_close_fp16(y_norm, want_norm, what="cfg1 rmsnorm")
    assert torch.equal(xp.cpu(), ref.kperm(y_norm.cpu()))
    # router: ids bit-exact given the kernel's logits
    lg = logits.cpu()
    rid, rw, _ = ref.router_topk(None, None, None, K, logits=lg)
    assert torch.equal(ids.cpu(), rid)
    assert (w.cpu() - rw).abs().max().item() < 1e-6
    # ... and from the oracle's own fp32 logits: any row that differs must be a near tie
    lo = y_norm.cpu().float() @ inp["router_w"].float().T + inp["bias"]
    assert (lg - lo).abs().max().item() < 1e-3
    oid, _, _ = ref.router_topk(None, None, None, K, logits=lo)
    differ = (oid != ids.cpu()).any(dim=1).numpy()
    ties = _near_tie_rows(lo, K)
    print(f"cfg1 router: {int(differ.sum())} of {T} rows differ from the ids of fp32-oracle "
          f"logits; {int(ties.sum())} rows have a top-{K + 1} gap under 4 ulp")
    assert not (differ & ~ties).any(), np.nonzero(differ & ~ties)
    counts = torch.bincount(ids.cpu().flatten().long(), minlength=E)
    assert counts.max().item() > 32          # the hottest expert spans several 32-token tasks
    # MoE on the kernel's normalised input and routing
    want = ref.moe_layer(y_norm.cpu(), W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                         W["dn_z"], ids.cpu(), w.cpu())
    assert_close_fp16(y, want, what="cfg1 layer (default engine)")
    again = fused_moe_w4_v2.moe_forward(y_norm, *args, ids, w, hidden_perm=xp)
    assert torch.equal(y.view(torch.int16), again.view(torch.int16))


def test_configs4_prefill_sampled_experts(cuda):
    """18,432 tokens (8 canvases + one 16,384-token prefill chunk), Zipf routing, the engine the
    bench runs (tcgen05 at ~1,150 pairs per expert); the oracle checks the hottest expert (all
    its pairs) and a cold one, with every other pair dropped on both sides."""
    import fused_moe_w4_v2
    import moe_router
    import workloads
    torch.set_num_threads(_threads())
    T, H, I, E, K = 18432, 2816, 704, 128, 8
    inp = workloads.moe_inputs(T, H, E, seed=4, device=cuda)
    x, ids, w, _ = moe_router.rmsnorm_route_topk(inp["hidden"], inp["norm_w"], 1e-6,
                                                 inp["router_w"], K, bias=inp["bias"],
                                                 want_logits=False)
    counts = torch.bincount(ids.flatten().long(), minlength=E).cpu()
    hot = int(counts.argmax())
    pos = torch.nonzero(counts > 0).flatten()
    cold = int(pos[counts[pos].argmin()])
    assert counts[hot] > 4000, counts[hot]
    # one kept pair per row, weight 1: the output row is that pair's down output itself, so the
    # comparison is per pair (a sum of several rounded pairs can cancel to near zero)
    keep = ids == hot                          # top-k ids of a row are distinct
    keep = keep | ((ids == cold) & ~keep.any(dim=1, keepdim=True))
    ids_f = torch.where(keep, ids, torch.full_like(ids, E))   # E = the reference's dropped id
    w_f = keep.float()
    W = workloads.moe_weights(E, H, I, seed=7, device=cuda)
    y = fused_moe_w4_v2.moe_forward(x, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                                    W["dn_z"], ids_f, w_f)
    Wc = {k: v.cpu() for k, v in W.items()}
    want = ref.moe_layer(x.cpu(), Wc["gu_q"], Wc["gu_s"], Wc["gu_z"], Wc["dn_q"], Wc["dn_s"],
                         Wc["dn_z"], ids_f.cpu(), w_f.cpu())
    rows = keep.any(dim=1).cpu()
    n_hot = int((ids_f == hot).sum())
    assert n_hot == int(counts[hot])           # every pair of the hottest expert is checked
    assert_close_fp16(y.cpu()[rows], want[rows],
                      what=f"cfg4 tc per pair, expert {hot} ({n_hot} pairs) + expert {cold}")
    assert (y.cpu()[~rows] == 0).all()


@pytest.mark.parametrize("step", [0, 24, 47])
def test_configs2_sampler_all_rows(cuda, step):
    """256 x 262,144 at T = 0.8, 0.6 and 0.408 (steps 0, 24, 47): every row's Gumbel sample and
    argmax bit-exact against the C oracle, entropy within 1e-4 of float64."""
    import fused_sampler_ops
    import workloads
    x = workloads.sampler_logits(256, 262144, seed=0, device="cuda")
    T = np.float32(workloads.temperature(step))
    seed = workloads.step_seed(1234, step)
    h, s, a = fused_sampler_ops.sample_step(x, seed, float(T))
    xc = x.cpu()
    rs, ra = ref.gumbel_argmax(xc, seed, temperature=float(T), nthreads=_threads())
    assert torch.equal(a.cpu(), ra)
    assert torch.equal(s.cpu(), rs), int((s.cpu() != rs).sum())
    rh = ref.entropy(xc / torch.tensor(T), dtype=torch.float64)
    assert ((h.cpu().double() - rh).abs() <= 1e-4 * rh.abs() + 1e-7).all()


def _moe_layer_unrounded(hidden, W, ids, w, gs_gu=128, gs_dn=64):
    """The oracle's layer with float64 weights (q - z) * s that are never rounded to f16; the
    intermediate f16 roundings of the reference (gate_up output, down output) are kept."""
    def deq(q, s, z, gs):
        N, Kh = q.shape
        codes = torch.stack((q & 0xF, q >> 4), dim=-1).reshape(N, 2 * Kh).double()
        codes = codes.reshape(N, -1, gs)
        return ((codes - z.double()[..., None]) * s.double()[..., None]).reshape(N, -1)
    T, H = hidden.shape
    tk = ids.shape[1]
    E, twoI, _ = W["gu_q"].shape
    I = twoI // 2
    x = hidden.double()
    out3 = torch.zeros(T * tk, H, dtype=torch.float16)
    for e in range(E):
        t_idx, j_idx = torch.where(ids == e)
        if t_idx.numel() == 0:
            continue
        gu = x[t_idx] @ deq(W["gu_q"][e], W["gu_s"][e], W["gu_z"][e], gs_gu).T
        act = (ref.gelu_tanh(gu[:, :I]) * gu[:, I:]).half().double()
        out3[t_idx * tk + j_idx] = (act @ deq(W["dn_q"][e], W["dn_s"][e], W["dn_z"][e], gs_dn).T).half()
    o3 = out3.float().view(T, tk, H)
    valid = (ids >= 0) & (ids < E)
    y = torch.zeros(T, H)
    for j in range(tk):
        y = y + torch.where(valid[:, j, None], w[:, j, None].float() * o3[:, j], torch.zeros(()))
    return y.to(hidden.dtype)


def test_engines_vs_unrounded_w4_arithmetic(cuda):
    """configs[0] shapes: every engine's rms distance to the W4 arithmetic with unrounded
    weights is within 10% of the reference torch path's own (which rounds each dequantised
    weight to f16); all engines bit-identical run to run."""
    import fused_moe_w4_v2
    import workloads
    torch.set_num_threads(_threads())
    T, E, H, I, tk = 256, 128, 2816, 704, 8
    W = workloads.moe_weights(E, H, I, seed=T + E)
    g = torch.Generator().manual_seed(T + E + 5)
    hidden = torch.randn(T, H, generator=g).half()
    ids, w = workloads.random_routing(T, E, tk, seed=T + E)
    Wd = {k: v.to(cuda) for k, v in W.items()}
    args = (Wd["gu_q"], Wd["gu_s"], Wd["gu_z"], Wd["dn_q"], Wd["dn_s"], Wd["dn_z"])
    truth = _moe_layer_unrounded(hidden, W, ids, w).float()
    want = ref.moe_layer(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"], W["dn_z"],
                         ids, w).float()
    rms = lambda a: (a - truth).pow(2).mean().sqrt().item()
    e_ref = rms(want)
    for eng in ("ws", "tc", "mma"):
        y = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *args, ids.to(cuda), w.to(cuda),
                                        engine=eng)
        y2 = fused_moe_w4_v2.moe_forward(hidden.to(cuda), *args, ids.to(cuda), w.to(cuda),
                                         engine=eng)
        assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
        e = rms(y.cpu().float())
        print(f"rms distance to the unrounded W4 arithmetic: {eng} {e:.3e}, reference torch "
              f"path {e_ref:.3e}")
        assert e <= 1.10 * e_ref, (eng, e, e_ref)


def test_ws_large_activations_and_scales(cuda):
    """The warp-specialised dense W4A16 GEMM with activations up to 60 and scales up to 0.05,
    zero-points up to 15 (outputs in the thousands, still inside the f16 range)."""
    import w4a16
    g = torch.Generator().manual_seed(8)
    M, N, K, gs = 40, 256, 1024, 128
    X = (torch.randn(M, K, generator=g) * 20).clamp(-60, 60).half()
    X[3] = 30.0                                     # one row of constant large activations
    q = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    s = (torch.rand(N, K // gs, generator=g) * 0.049 + 0.001).half()
    z = (torch.rand(N, K // gs, generator=g) * 15).half()
    want = X.double() @ ref.dequant_w4(q, s, z, gs).double().T
    assert want.abs().max().item() < 60000
    Y = w4a16.w4a16_linear(X.to(cuda), q.to(cuda), s.to(cuda), z.to(cuda), BK=gs, engine="ws")
    assert_close_fp16(Y, want.half(), what="w4a16 ws large activations")
