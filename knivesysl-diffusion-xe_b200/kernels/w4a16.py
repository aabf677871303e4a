"""w4a16.py — packed 4-bit weight / 16-bit activation format and the dense W4A16 linear.

Same API as the reference module (w4a16.py:19-108):
  quantize_w4(W, group_size)      -> (qpacked u8[N,K/2], scale f16[N,K/gs], zero f16[N,K/gs])
  dequant_w4(q, s, z, group_size) -> W f16[N,K]      (the fp16 reference weight)
  w4a16_linear(X, q, s, z, BK)    -> Y f16[M,N] = X . dequant(q,s,z)^T   (sm_100a kernel)

Format (w4a16.py:19-32): asymmetric group quantisation along K; per (row, group)
  scale = max(w_max - w_min, 1e-8) / 15,  zero = clamp(round(-w_min/scale), 0, 15),
  q = clamp(round(w/scale + zero), 0, 15),  w ~= (q - zero) * scale;
two nibbles per byte, the even k in the low nibble.
"""
import torch

from _knx import (KNX_W4_INT_ZEROS, check, engine_flags, load, ptr, require_device, stream_of,
                  workspace, zero_flags)

GS = 128  # default group size along K


@torch.no_grad()
def quantize_w4(W, group_size=GS):
    """W[N,K] float -> (qpacked uint8[N,K//2], scale fp16[N,K//gs], zero fp16[N,K//gs])."""
    N, K = W.shape
    assert K % group_size == 0, "K must be divisible by the group size"
    Wg = W.float().reshape(N, K // group_size, group_size)
    lo = Wg.amin(-1)
    hi = Wg.amax(-1)
    # tensor divisors keep the division IEEE-exact on every device (a CUDA tensor divided by a
    # Python scalar is a multiply by the reciprocal), so CPU and GPU packs are bit-identical
    scale = (hi - lo).clamp(min=1e-8) / torch.full_like(hi, 15.0)
    zero = torch.round(-lo / scale).clamp(0, 15)
    q = torch.round(Wg / scale[..., None] + zero[..., None]).clamp(0, 15).to(torch.uint8)
    q = q.reshape(N, K)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()
    return packed, scale.to(torch.float16).contiguous(), zero.to(torch.float16).contiguous()


@torch.no_grad()
def dequant_w4(qpacked, scale, zero, group_size=GS):
    """qpacked[N,K//2] -> fp16 W[N,K] = (q - zero) * scale computed in fp32, rounded once."""
    N, Kh = qpacked.shape
    K = 2 * Kh
    q = torch.stack((qpacked & 0xF, qpacked >> 4), dim=-1).reshape(N, K).float()
    q = q.reshape(N, K // group_size, group_size)
    W = (q - zero.float()[..., None]) * scale.float()[..., None]
    return W.reshape(N, K).to(torch.float16)


def w4a16_linear(X, qpacked, scale, zero, BK=GS, int_zeros=None, engine=None):
    """Y[M,N] = X[M,K] @ dequant(qpacked)[N,K].T, fp16 out; reads the packed nibbles directly.

    BK is the group size (the reference ties its K tile to it).  Requirements: K % 64 == 0,
    BK % 32 == 0, K % BK == 0, N % 8 == 0, K / BK <= 56.  Integer zero-points (quantize_w4's)
    dequantise exactly like dequant_w4; other fp16 zero-points as RN16(RN16(q - z) * s)."""
    M, K = X.shape
    N = qpacked.shape[0]
    assert K % BK == 0, "K must be divisible by BK (== group size)"
    dev = require_device(X)
    Xc = X.contiguous().to(torch.float16)
    q = qpacked.contiguous()
    s = scale.contiguous().to(torch.float16)
    z = zero.contiguous().to(torch.float16)
    Y = torch.empty(M, N, device=X.device, dtype=torch.float16)
    if int_zeros is None:
        flags = zero_flags(z)
    else:
        flags = KNX_W4_INT_ZEROS if int_zeros else 0
    flags |= engine_flags(engine)
    lib = load()
    nbytes = lib.knx_w4a16_workspace_size(M, K)
    ws = workspace(dev, nbytes, "w4a16")
    check(lib.knx_w4a16_linear(ptr(Xc), ptr(q), ptr(s), ptr(z), M, N, K, int(BK), flags, ptr(Y),
                               ptr(ws), ws.numel(), stream_of(dev)), "knx_w4a16_linear")
    return Y
