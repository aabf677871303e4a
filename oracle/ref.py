"""Torch/numpy CPU restatement of the reference hot path — TEST INFRASTRUCTURE ONLY.

Functions (reference file:line in the reference project's kernels/ directory):
  dequant_w4            w4a16.py:35-48       fp32 (q - z) * s, one rounding to f16
  quantize_w4           w4a16.py:19-32
  moe_align             fused_moe_w4.py:15-51 (stable argsort, BM padding, sentinels)
  moe_align_unpadded    same order without BM padding (what the kernels use)
  moe_layer             fused_moe_w4_v2.py:319-371 via pack_experts.py:44-62 semantics:
                        per expert F.linear on dequantised f16 weights (fp32 accumulate),
                        tanh-GELU (fused_moe_w4_v2.py:136-138) -> f16, down -> f16 per pair,
                        fixed-k-order fp32 combine (fused_moe_w4_v2.py:248-263)
  rmsnorm               fused_rmsnorm.py:10-32 (bf16 store) / stock chain fused_rmsnorm.py:1-5
  router_topk           DiffusionGemma router as specified: softmax -> top-k -> renormalise
  entropy               fast_sampler.py:29 (torch Categorical entropy)
  gumbel_argmax         fused_sampler_ops.py:54-93 (C restatement in sampler_oracle.c)
  accept_canvas         fast_sampler.py:32-42 (stable sort; torch CPU cumsum = fp64 prefix)
  stop_test             fast_sampler.py:45-65
"""
import ctypes
import math
import pathlib

import numpy as np
import torch

from . import build_oracle

_HERE = pathlib.Path(__file__).resolve().parent
_clib = None


def clib():
    global _clib
    if _clib is None:
        path = build_oracle.build()
        lib = ctypes.CDLL(str(path))
        vp, i64, f32, u32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_uint32
        lib.oracle_gumbel_argmax.argtypes = [vp, i64, i64, f32, i64, vp, vp, ctypes.c_int]
        lib.oracle_gumbel_noise.argtypes = [i64, i64, i64, vp]
        lib.oracle_philox4x32_10.argtypes = [vp, vp, vp]
        lib.oracle_log.argtypes = [f32]
        lib.oracle_log.restype = f32
        lib.oracle_gumbel.argtypes = [u32]
        lib.oracle_gumbel.restype = f32
        lib.oracle_markstein_mismatches.argtypes = [f32, i64, u32]
        lib.oracle_markstein_mismatches.restype = i64
        _clib = lib
    return _clib


# ---------------------------------------------------------------------------------- W4 format
def quantize_w4(W, group_size=128):
    N, K = W.shape
    Wg = W.float().reshape(N, K // group_size, group_size)
    wmin, wmax = Wg.min(-1).values, Wg.max(-1).values
    scale = (wmax - wmin).clamp(min=1e-8) / 15.0
    zero = (-wmin / scale).round().clamp(0, 15)
    q = (Wg / scale[..., None] + zero[..., None]).round().clamp(0, 15).to(torch.uint8).reshape(N, K)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous(), scale.half(), zero.half()


def dequant_w4(qpacked, scale, zero, group_size):
    """[..., N, K/2] -> f16 [..., N, K]."""
    *lead, N, Kh = qpacked.shape
    K = 2 * Kh
    lo = (qpacked & 0xF).float()
    hi = (qpacked >> 4).float()
    q = torch.stack((lo, hi), dim=-1).reshape(*lead, N, K // group_size, group_size)
    W = (q - zero.float()[..., None]) * scale.float()[..., None]
    return W.reshape(*lead, N, K).half()


# ---------------------------------------------------------------------------------- permutation
def moe_align(topk_ids, block_m, E):
    """Reference moe_align (fused_moe_w4.py:15-51) restated with numpy; returns int64 arrays
    (sorted_rows[cap], expert_ids[max_blocks], cap, inv[Nexp])."""
    ids = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    Nexp = ids.size
    flat = np.minimum(ids, E)
    valid = flat < E
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat[valid], minlength=E)[:E]
    nblk = (counts + block_m - 1) // block_m
    max_blocks = (Nexp + block_m - 1) // block_m + E
    cap = max_blocks * block_m
    cum = np.cumsum(nblk)
    expert_ids = np.searchsorted(cum, np.arange(max_blocks), side="right").astype(np.int64)
    sorted_rows = np.full(cap, Nexp, dtype=np.int64)
    inv = np.zeros(Nexp, dtype=np.int64)
    blk_start = (cum - nblk) * block_m
    rank = np.zeros(E, dtype=np.int64)
    for p in order:
        e = flat[p]
        if e >= E:
            continue
        d = blk_start[e] + rank[e]
        rank[e] += 1
        sorted_rows[d] = p
        inv[p] = d
    return sorted_rows, expert_ids, cap, inv


def moe_align_unpadded(topk_ids, E):
    """Stable counting sort without padding: counts[E], offsets[E+1], sorted_pair[N] (tail = N),
    inv[N] (-1 for ids outside [0, E))."""
    ids = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    N = ids.size
    ok = (ids >= 0) & (ids < E)
    counts = np.bincount(ids[ok], minlength=E)[:E].astype(np.int64)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    key = np.where(ok, ids, E)
    order = np.argsort(key, kind="stable")
    nvalid = int(ok.sum())
    sorted_pair = np.full(N, N, dtype=np.int64)
    sorted_pair[:nvalid] = order[:nvalid]
    inv = np.full(N, -1, dtype=np.int64)
    inv[order[:nvalid]] = np.arange(nvalid)
    return counts, offsets, sorted_pair, inv


# ---------------------------------------------------------------------------------- MoE layer
def gelu_tanh(x):
    inner = 0.7978845608028654 * (x + 0.044715 * x * x * x)
    return 0.5 * x * (1.0 + (2.0 / (1.0 + torch.exp(-2.0 * inner)) - 1.0))


def moe_layer(hidden, gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, topk_ids, topk_w, gs_gu=128, gs_dn=64,
              out_dtype=None, return_pairs=False, dense=None):
    """One MoE layer on CPU.  Per pair p = t*k + j with expert e: out3[p] = f16(down_e(
    f16(gelu(gate_e(x_t)) * up_e(x_t)))); y[t] = sum_j w[t,j] * f32(out3[p]) in j order.
    dense: optional list of (gate_up, down) fp32 weights per expert, dequantised beforehand
    (dense_experts), used instead of dequantising inside the call."""
    T, H = hidden.shape
    tk = topk_ids.shape[1]
    E, twoI, _ = gu_q.shape
    I = twoI // 2
    x = hidden.half().float()
    ids = topk_ids.long()
    w = topk_w.float()
    out3 = torch.zeros(T * tk, H, dtype=torch.float16)
    for e in range(E):
        t_idx, j_idx = torch.where(ids == e)
        if t_idx.numel() == 0:
            continue
        if dense is not None:
            Wgu, Wdn = dense[e]
        else:
            Wgu = dequant_w4(gu_q[e], gu_s[e], gu_z[e], gs_gu).float()
            Wdn = dequant_w4(dn_q[e], dn_s[e], dn_z[e], gs_dn).float()
        gu = x[t_idx] @ Wgu.T
        act = (gelu_tanh(gu[:, :I]) * gu[:, I:]).half().float()
        o = (act @ Wdn.T).half()
        out3[t_idx * tk + j_idx] = o
    y = torch.zeros(T, H, dtype=torch.float32)
    o3 = out3.float().view(T, tk, H)
    valid = (ids >= 0) & (ids < E)
    for j in range(tk):
        y = y + torch.where(valid[:, j, None], w[:, j, None] * o3[:, j], torch.zeros(()))
    y = y.to(out_dtype or hidden.dtype)
    return (y, out3) if return_pairs else y


def dense_experts(gu_q, gu_s, gu_z, dn_q, dn_s, dn_z, gs_gu=128, gs_dn=64):
    """Every expert's weights dequantised once to fp32 (moe_layer(..., dense=...))."""
    return [(dequant_w4(gu_q[e], gu_s[e], gu_z[e], gs_gu).float(),
             dequant_w4(dn_q[e], dn_s[e], dn_z[e], gs_dn).float()) for e in range(gu_q.shape[0])]


# ---------------------------------------------------------------------------------- RMSNorm
def rmsnorm(x, w, eps, round_bf16=True):
    xf = x.float()
    y = xf / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if w is not None:
        y = y * w.float()
    if round_bf16:
        y = y.to(torch.bfloat16)
    return y.to(x.dtype)


def kperm(x):
    """The kernels' K-interleave of the last dim: position 2*(i%4)+i//4 of each 8-group holds i."""
    shp = x.shape
    g = x.reshape(*shp[:-1], shp[-1] // 8, 2, 4)      # [.., grp, i//4, i%4]
    return g.transpose(-1, -2).reshape(shp)


# ---------------------------------------------------------------------------------- router
def router_topk(x, wr, bias, topk, logits=None):
    """logits (given or x.wr^T + bias in fp32) -> ids (stable: larger logit, then lower id),
    renormalised softmax weights."""
    if logits is None:
        logits = x.float() @ wr.float().T
        if bias is not None:
            logits = logits + bias.float()
    order = torch.from_numpy(np.argsort(-logits.numpy(), axis=-1, kind="stable"))
    ids = order[:, :topk]
    p = torch.softmax(logits.double(), dim=-1)
    pt = torch.gather(p, 1, ids)
    w = (pt / pt.sum(-1, keepdim=True)).float()
    return ids.int(), w, logits


# ---------------------------------------------------------------------------------- sampler
def entropy(logits, dtype=torch.float32):
    """torch Categorical entropy (fast_sampler.py:29); dtype=float64 gives the accurate value."""
    return torch.distributions.Categorical(logits=logits.to(dtype)).entropy()


def gumbel_argmax(logits, seed, temperature=1.0, nthreads=8):
    x = np.ascontiguousarray(logits.detach().cpu().float().numpy())
    rows, V = x.shape
    samp = np.empty(rows, dtype=np.int64)
    amax = np.empty(rows, dtype=np.int64)
    clib().oracle_gumbel_argmax(x.ctypes.data, rows, V, float(temperature), int(seed),
                                samp.ctypes.data, amax.ctypes.data, int(nthreads))
    return torch.from_numpy(samp), torch.from_numpy(amax)


def gumbel_noise(rows, V, seed):
    g = np.empty((rows, V), dtype=np.float32)
    clib().oracle_gumbel_noise(rows, V, int(seed), g.ctypes.data)
    return torch.from_numpy(g)


def philox4x32_10(ctr, key):
    c = (ctypes.c_uint32 * 4)(*ctr)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    clib().oracle_philox4x32_10(c, k, o)
    return list(o)


def temperature(step, max_steps, t_min, t_max):
    """README.md:127-136: T = t_min + (t_max - t_min) * remaining / max_steps, remaining = 48..1."""
    remaining = max_steps - step
    return t_min + (t_max - t_min) * remaining / max_steps


def step_seed(s0, step):
    """fast_sampler.py:92 seed mixing."""
    return (int(s0) ^ (int(step) * 0x9E3779B1)) & 0x7FFFFFFF


def accept_canvas(H, cur, prop, bound):
    """Stable ascending sort, fp64 running sum rounded to fp32 per prefix, (cum - h) <= bound."""
    H = H.float()
    B, L = H.shape
    mask = torch.zeros(B, L, dtype=torch.bool)
    for b in range(B):
        h = H[b].numpy()
        order = np.argsort(h, kind="stable")
        hs = h[order]
        cum = np.cumsum(hs.astype(np.float64)).astype(np.float32)
        sel = (cum - hs) <= np.float32(bound)
        mask[b, torch.from_numpy(order)] = torch.from_numpy(sel)
    return mask, torch.where(mask, prop.long(), cur.long())


def stop_test(argmax, history, H, confidence_threshold):
    """Returns (finished bool[B], new history); history [S,B,L] or None for S = 0."""
    B, L = argmax.shape
    if history is None or history.shape[0] == 0:
        stable = torch.ones(B, dtype=torch.bool)
        newh = history
    else:
        stable = (history == argmax[None]).all(-1).all(0)
        newh = torch.roll(history, shifts=-1, dims=0).clone()
        newh[-1] = argmax
    mean = torch.from_numpy((H.double().sum(-1) / L).float().numpy())
    return stable & (mean < np.float32(confidence_threshold)), newh
