"""_knx.py — ctypes binding of libknx.so (the sm_100a kernels behind include/knx.h).

The library is loaded from ../lib/libknx.so next to this package directory.  There is no CPU
or PyTorch fallback: if the library is missing or the device is not an sm_100 part, every entry
point raises.  Build it with `python build.py` in the package root (nvcc only, no GPU needed).

Helpers here own the per-(device, stream) workspace caches: a workspace is a grow-only uint8
tensor reused by calls on the same stream (stream order makes reuse safe); calls on other
streams get their own.
"""
import ctypes
import os
import pathlib
import threading

import torch

PKG = pathlib.Path(__file__).resolve().parent.parent
LIB_PATH = pathlib.Path(os.environ.get("KNX_LIB", PKG / "lib" / "libknx.so"))

KNX_F16, KNX_BF16, KNX_F32, KNX_I32, KNX_I64 = 0, 1, 2, 3, 4
KNX_RMS_ROUND_BF16 = 0x1
KNX_DEV_BAD_EXPERT_ID = 0x1
KNX_DEV_TIMEOUT = 0x4
KNX_SAMPLER_STATIC_SCRATCH_BYTES = 1 << 20  # include/knx.h
KNX_W4_INT_ZEROS = 0x1
KNX_W4_WARP_MMA = 0x2
KNX_W4_WARP_WS = 0x8
KNX_W4_TCGEN05 = 0x10
_ENGINES = {"auto": 0, "tc": KNX_W4_TCGEN05, "mma": KNX_W4_WARP_MMA, "ws": KNX_W4_WARP_WS}


def engine_flags(engine=None):
    """Engine selection flags for the W4A16 GEMMs: "auto" (the default: the warp-specialised
    mma.sync kernels up to 36 tokens per expert, tcgen05 above), "ws", "tc" (tcgen05) or "mma"
    (the plain mma.sync kernels); `engine` or the KNX_ENGINE environment variable chooses."""
    engine = engine or os.environ.get("KNX_ENGINE", "auto")
    if engine not in _ENGINES:
        raise ValueError(f"unknown engine {engine!r}")
    return _ENGINES[engine]

_c = ctypes
_vp, _i64, _i32, _f32, _sz = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_float, _c.c_size_t

_SIGS = {
    "knx_version": (_i32, []),
    "knx_device_ok": (_i32, []),
    "knx_status_string": (_c.c_char_p, [_i32]),
    "knx_rmsnorm": (_i32, [_vp, _vp, _i32, _vp, _vp, _i64, _i64, _f32, _i32, _i32, _vp]),
    "knx_router_workspace_size": (_sz, [_i64, _i32]),
    "knx_router_topk": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "knx_ep_p2p_plan_ints": (_sz, [_i32, _i32, _i32]),
    "knx_ep_p2p_counts": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _c.c_uint32, _vp, _vp, _vp]),
    "knx_ep_p2p_dispatch": (_i32, [_vp, _i64, _i32, _vp, _vp, _i32, _i32, _vp, _vp, _i64, _vp]),
    "knx_ep_p2p_barrier": (_i32, [_vp, _i32, _i32, _c.c_uint32, _vp, _vp]),
    "knx_ep_p2p_return": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _i64, _vp]),
    "knx_ep_p2p_dispatch_barrier": (_i32, [_vp, _i64, _i32, _vp, _vp, _i32, _i32, _vp, _vp, _i64,
                                           _vp, _i32, _i32, _c.c_uint32, _vp, _vp, _vp]),
    "knx_ep_p2p_return_barrier": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _i64, _vp, _i32,
                                         _c.c_uint32, _vp, _vp, _vp]),
    "knx_rmsnorm_router_topk": (_i32, [_vp, _vp, _f32, _i32, _vp, _vp, _i64, _i64, _i32, _i32,
                                       _vp, _vp, _vp, _vp, _vp, _vp]),
    "knx_moe_align": (_i32, [_vp, _i32, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                             _vp, _vp]),
    "knx_moe_align_large_scratch_size": (_sz, [_i64, _i32]),
    "knx_moe_align_large": (_i32, [_vp, _i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _sz, _vp,
                                   _vp]),
    "knx_moe_align_relabeled": (_i32, [_vp, _i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp,
                                       _sz, _vp, _vp]),
    "knx_moe_w4_workspace_size": (_sz, [_i64, _i64, _i64, _i32, _i32]),
    "knx_moe_w4": (_i32, [_vp, _vp, _i32, _vp, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp,
                          _i64, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp, _vp,
                          _vp]),
    "knx_w4a16_workspace_size": (_sz, [_i64, _i64]),
    "knx_w4a16_linear": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp, _vp, _sz,
                                _vp]),
    "knx_sampler_workspace_size": (_sz, [_i64, _i64]),
    "knx_sampler_fused": (_i32, [_vp, _i64, _i64, _f32, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "knx_sampler_fused_static": (_i32, [_vp, _i64, _i64, _f32, _i64, _vp, _vp, _vp, _vp]),
    "knx_sampler_fused_sc": (_i32, [_vp, _i64, _i64, _f32, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _i64, _vp, _sz, _vp]),
    "knx_accept_stop": (_i32, [_vp, _vp, _vp, _i64, _i64, _f32, _vp, _vp, _vp, _vp, _i32, _f32,
                               _vp, _vp]),
    "knx_gather_rows": (_i32, [_vp, _i64, _i64, _vp, _i32, _i64, _vp, _vp]),
    "knx_ep_layout": (_i32, [_vp, _i32, _i32, _i64, _vp, _vp, _vp, _vp]),
    "knx_moe_w4_grouped_workspace_size": (_sz, [_i64, _i64, _i64, _i32]),
    "knx_moe_w4_grouped": (_i32, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                  _i32, _i32, _i32, _i32, _i64, _vp, _sz, _vp, _vp, _vp]),
    "knx_moe_combine": (_i32, [_vp, _vp, _vp, _i32, _i64, _i32, _i64, _i32, _vp, _vp]),
    "knx_prof_start": (_i32, [_i32]),
    "knx_prof_stop": (_i32, [_vp, _i32, _vp]),
}

PROF_STAGES = ("prep", "gate_up_gelu", "down", "combine")


def prof_start(max_calls):
    check(load().knx_prof_start(int(max_calls)), "knx_prof_start")


def prof_stop():
    """-> ({stage: summed ms}, ncalls) for the knx_moe_w4 calls since prof_start."""
    ms = (ctypes.c_float * len(PROF_STAGES))()
    n = ctypes.c_int(0)
    check(load().knx_prof_stop(ms, len(PROF_STAGES), ctypes.byref(n)), "knx_prof_stop")
    return dict(zip(PROF_STAGES, list(ms))), n.value

_lib = None
_lock = threading.Lock()


def load():
    """Load libknx.so and bind every C-ABI symbol (raises if the library is absent)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"libknx.so not found at {LIB_PATH}; run `python build.py` in {PKG}")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols():
    return sorted(_SIGS)


_dev_checked = {}


def require_device(t):
    """The kernels exist for sm_100a only: refuse anything else loudly."""
    if not t.is_cuda:
        raise RuntimeError("knx kernels need CUDA tensors (no CPU fallback exists)")
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    ok = _dev_checked.get(idx)
    if ok is None:
        ok = torch.cuda.get_device_capability(idx) == (10, 0)
        _dev_checked[idx] = ok
    if not ok:
        raise RuntimeError(f"knx kernels are built for sm_100a only; device {idx} is "
                           f"sm_{''.join(map(str, torch.cuda.get_device_capability(idx)))}")
    return idx


def check(status, what):
    if status != 0:
        msg = load().knx_status_string(status).decode()
        raise RuntimeError(f"{what} failed: status {status} ({msg})")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(device_index):
    return ctypes.c_void_p(torch.cuda.current_stream(device_index).cuda_stream)


def dtype_code(dt):
    return {torch.float16: KNX_F16, torch.bfloat16: KNX_BF16, torch.float32: KNX_F32,
            torch.int32: KNX_I32, torch.int64: KNX_I64}[dt]


def zero_flags(*zeros):
    """KNX_W4_INT_ZEROS when every zero-point tensor holds integers in [0, 15] (quantize_w4's
    output): the kernels then dequantise bit-identically to dequant_w4.  The check runs once per
    tensor object and version (one device sync at first use) and is cached on the tensor."""
    flag = KNX_W4_INT_ZEROS
    for z in zeros:
        c = getattr(z, "_knx_zint", None)
        if c is None or c[0] != z._version:
            ok = bool(((z == torch.round(z)) & (z >= 0) & (z <= 15)).all())
            c = (z._version, ok)
            try:
                z._knx_zint = c
            except (AttributeError, RuntimeError):
                pass
        if not c[1]:
            flag = 0
    return flag


_ws = {}


def workspace(device_index, nbytes, purpose):
    """Grow-only uint8 workspace per (device, current stream, purpose), 256-byte aligned."""
    key = (device_index, torch.cuda.current_stream(device_index).cuda_stream, purpose)
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=f"cuda:{device_index}")
        _ws[key] = buf
    return buf
