"""fused_moe_w4_v2.py — one W4A16 MoE layer on sm_100a (drop-in for the reference module).

fused_moe_w4_v2(hidden, exp, topk_ids, topk_w) keeps the reference contract
(fused_moe_w4_v2.py:319-371):
  * exp carries the pack_experts buffers gu_q/gu_s/gu_z (gate_up, group 128) and dn_q/dn_s/dn_z
    (down, group 64); hidden [T,H] f16/bf16 is used as f16; the result has hidden.dtype;
  * the activation is tanh-GELU fused into the first GEMM's epilogue (checked once per module);
  * the top-k combine runs in fixed k order in fp32 with every pair's down output rounded to f16
    first, so the output is bit-identical run to run (no atomics anywhere).
The whole layer is five stream-ordered launches (K-interleave copy, counting-sort align, gate_up
+GELU GEMM, down GEMM, combine), never synchronises the host and is CUDA-graph capturable.

moe_align_cuda(topk_ids, block_m, E) mirrors fused_moe_w4_v2.py:46-74 on the same kernel as
knx_moe_align (int32 outputs: a_row[cap], expert_ids[nblk], cap, inv[Nexp]).
"""
import os

import torch

from _knx import (KNX_DEV_BAD_EXPERT_ID, KNX_DEV_TIMEOUT, KNX_W4_INT_ZEROS, check, dtype_code, engine_flags, load,
                  ptr, require_device, stream_of, workspace, zero_flags)

# Module globals named as in the reference (which tunes its Triton launches with them).  Here they
# describe the plain mma.sync engine (engine="mma") only; the default engines take other tiles:
# "ws" 128 gate + 128 up (gate_up) or 256 (down) weight rows per work item and 256 k per stage,
# "tc" 128 tokens x 256 weight rows per MMA.  No engine uses BM-padded blocks: tasks are expert
# token chunks (at most 32 tokens for "ws" and "mma", 128 for "tc").
BM_V2 = 32
G1 = dict(BN=64, BK=256, stages=4)   # mma gate_up+GELU: 64 gate + 64 up rows per CTA tile
G2 = dict(BN=128, BK=128, stages=5)  # mma down: 128 output rows per CTA tile

_TANH_GELU_NAMES = ("gelu_pytorch_tanh", "gelu_new", "gelu_tanh", "quick_gelu_tanh")


def hidden_device(exp):
    """Device of the module's packed buffers (scales first), CPU when it has none."""
    t = next((getattr(exp, b) for b in ("gu_s", "gu_q") if getattr(exp, b, None) is not None),
             None)
    return t.device if t is not None else "cpu"


def _act_name(fn):
    return None if fn is None else (getattr(fn, "__name__", None) or type(fn).__name__)


def _is_tanh_gelu(fn, device):
    """By name (any name containing "gelu" passes, as in the reference), else by value on four
    probe points against 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    name = _act_name(fn)
    if name in _TANH_GELU_NAMES or "gelu" in str(name).lower():
        return True
    if fn is None:
        return False
    x = torch.tensor([-1.0, 0.0, 0.5, 2.0], device=device)
    want = 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x.pow(3))))
    return bool(torch.allclose(fn(x).float(), want, atol=1e-3))


def _check_act(exp):
    """The gate_up epilogue computes tanh-GELU; a module whose act_fn is something else (or
    missing) is refused once, with AssertionError (fused_moe_w4_v2.py:291-308)."""
    fn = getattr(exp, "act_fn", None)
    if not _is_tanh_gelu(fn, hidden_device(exp)):
        raise AssertionError(f"fused_moe_w4_v2 computes tanh-GELU but this module's act_fn is "
                             f"{_act_name(fn)!r}")
    exp._act_checked = True
    return True


def unshuffle_T_dn(ns, BK=64):
    """Inverse of the reference's MOE_NS repack (fused_moe_w4_v2.py:187-197): [E,K/2,N] -> the
    standard [E,N,K/2] pack.  The sm_100a kernels read only the standard layout."""
    E_, Kh, N = ns.shape
    K = 2 * Kh
    packed = ns.transpose(1, 2).contiguous().reshape(E_, N, K // BK, BK // 2)
    lo, hi = packed & 0xF, packed >> 4                     # codes k0..k31, k32..k63 of a chunk
    codes = torch.cat((lo, hi), dim=-1).reshape(E_, N, K)
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).contiguous()


def preshuffle_T_dn(qpacked, BK=64):
    """The reference's MOE_NS repack (kept for API parity; the kernels do not need it)."""
    E_, N, Kh = qpacked.shape
    K = 2 * Kh
    codes = torch.stack((qpacked & 0xF, qpacked >> 4), dim=-1).reshape(E_, N, K)
    c = codes.reshape(E_, N, K // BK, BK)
    ns = (c[..., : BK // 2] | (c[..., BK // 2:] << 4)).reshape(E_, N, Kh)
    return ns.transpose(1, 2).contiguous()


def enable_ns_down(exp):
    """No-op on sm_100a, kept for API parity: the down GEMM reads the standard pack (its limit
    is instruction issue, not the layout's access pattern), so the preshuffled layout is not
    installed (returns exp unchanged, dn_ns stays False)."""
    exp.dn_ns = False
    return exp


def _standard_dn(exp):
    if getattr(exp, "dn_ns", False):      # someone installed the reference's NS pack: undo once
        exp.dn_q = unshuffle_T_dn(exp.dn_q)
        exp.dn_ns = False
    return exp.dn_q


def _err_word(dev):
    if os.environ.get("MOE_VALIDATE") == "1":
        return torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
    return None


def moe_forward(hidden, gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, topk_ids, topk_w, hidden_perm=None,
                out=None, int_zeros=None, engine=None):
    """Raw entry: one MoE layer from explicit buffers (see knx_moe_w4 in include/knx.h).
    int_zeros: True/False to state whether the zero-points are integers in [0, 15]; None checks
    once per tensor (see _knx.zero_flags).  engine: see _knx.engine_flags."""
    dev = require_device(hidden)
    T, H = hidden.shape
    tk = topk_ids.shape[1]
    E, twoI, _ = gu_q.shape
    I = twoI // 2
    assert H % 256 == 0, f"hidden dim {H} must be divisible by 256"
    assert I % 64 == 0, f"expert intermediate {I} must be divisible by 64"
    gs_gu = H // gu_s.shape[-1]
    gs_dn = I // dn_s.shape[-1]
    hidden = hidden.contiguous()
    ids = topk_ids.contiguous()
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.long()
    w = topk_w.contiguous()
    if out is None:
        out = torch.empty_like(hidden)
    if int_zeros is None:
        flags = zero_flags(gu_z, dn_z)
    else:
        flags = KNX_W4_INT_ZEROS if int_zeros else 0
    flags |= engine_flags(engine)
    lib = load()
    nbytes = lib.knx_moe_w4_workspace_size(T, H, I, E, tk)
    ws = workspace(dev, nbytes, "moe")
    err = _err_word(dev)
    check(lib.knx_moe_w4(ptr(hidden), ptr(hidden_perm), dtype_code(hidden.dtype), ptr(ids),
                         dtype_code(ids.dtype), ptr(w), dtype_code(w.dtype), ptr(gu_q), ptr(gu_s),
                         ptr(gu_z), ptr(dn_q), ptr(dn_s), ptr(dn_z), T, H, I, E, tk, gs_gu, gs_dn,
                         flags, ptr(ws), ws.numel(), ptr(out), ptr(err), stream_of(dev)),
          "knx_moe_w4")
    if err is not None:
        bad = int(err.item())
        assert not (bad & KNX_DEV_BAD_EXPERT_ID), f"moe: expert ids must be in [0,{E}]"
        assert not (bad & KNX_DEV_TIMEOUT), "moe: a bounded on-chip wait timed out"
    return out


@torch.no_grad()
def fused_moe_w4_v2(hidden, exp, topk_ids, topk_w):
    assert getattr(exp, "_act_checked", False) or _check_act(exp), "unsupported activation"
    return moe_forward(hidden, exp.gu_q, exp.gu_s, exp.gu_z, _standard_dn(exp), exp.dn_s, exp.dn_z,
                       topk_ids, topk_w)


@torch.no_grad()
def moe_align_cuda(topk_ids, block_m, E):
    """(a_row i32[cap], expert_ids i32[nblk], cap, inv i32[Nexp]) — fused_moe_w4_v2.py:46-74
    semantics with pad row T and pad block E, via the counting-sort kernel."""
    from fused_moe_w4 import moe_align_raw
    sorted_rows, expert_ids, _, inv = moe_align_raw(topk_ids, block_m, E)
    T, tk = topk_ids.shape
    Nexp = T * tk
    mx = Nexp + E * (block_m - 1)               # the reference's capacity bound for this path
    if Nexp < E:
        mx = min(Nexp * block_m, mx)
    nblk = (mx + block_m - 1) // block_m
    cap = nblk * block_m
    sorted_rows, expert_ids = sorted_rows[:cap], expert_ids[:nblk]
    a_row = torch.where(sorted_rows < Nexp, sorted_rows // tk, torch.full_like(sorted_rows, T))
    return a_row, expert_ids, cap, inv
