"""The C-ABI library loads on a machine without a GPU, exports every symbol include/knx.h
declares, and rejects contract violations on the host before touching the device."""
import ctypes
import re

import pytest

import _knx
from conftest import REPO


def header_symbols():
    text = (REPO / "include" / "knx.h").read_text()
    return sorted(set(re.findall(r"KNX_API\s+[\w\s\*]+?\b(knx_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _knx.load()
    declared = header_symbols()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_knx.exported_symbols())


def test_integration_stubs_match_the_signature_table():
    """The ctypes stubs a maintainer of the reference would copy from INTEGRATION.md declare the
    same argument types as the library's own binding table."""
    types = {"vp": ctypes.c_void_p, "i64": ctypes.c_int64, "i32": ctypes.c_int,
             "f32": ctypes.c_float, "sz": ctypes.c_size_t}
    text = (REPO / "INTEGRATION.md").read_text()
    stubs = re.findall(r"lib\.(knx_\w+)\.argtypes = \[([^\]]*)\]", text)
    assert len(stubs) >= 15
    for name, args in stubs:
        got = [types[a.strip()] for a in args.replace("\n", " ").split(",") if a.strip()]
        assert got == list(_knx._SIGS[name][1]), name


def test_status_strings_and_version():
    lib = _knx.load()
    assert lib.knx_version() > 0
    assert lib.knx_status_string(0) == b"ok"
    assert b"workspace" in lib.knx_status_string(-3)


def test_workspace_sizes_are_host_only_and_monotone():
    lib = _knx.load()
    a = lib.knx_moe_w4_workspace_size(256, 2816, 704, 128, 8)
    b = lib.knx_moe_w4_workspace_size(512, 2816, 704, 128, 8)
    assert 0 < a < b
    assert a % 256 == 0
    assert lib.knx_sampler_workspace_size(256, 262144) > 256 * 8 * 32
    assert lib.knx_router_workspace_size(256, 128) >= 4 * 256 * 128 * 4
    assert lib.knx_w4a16_workspace_size(64, 2816) >= 64 * 2816 * 2


@pytest.mark.parametrize("H,I,gs_gu,gs_dn,expect", [
    (2816 + 8, 704, 128, 64, -5),   # H % 256 != 0
    (2816, 700, 128, 64, -5),       # I % 64 != 0
    (2816, 704, 100, 64, -1),       # group size not a multiple of 32
    (2816, 704, 128, 48, -1),
])
def test_moe_contract_violations_rejected_on_host(H, I, gs_gu, gs_dn, expect):
    lib = _knx.load()
    st = lib.knx_moe_w4(None, None, 0, None, 4, None, 2, None, None, None, None, None, None,
                        256, H, I, 128, 8, gs_gu, gs_dn, 0, None, 0, None, None, None)
    assert st == expect


def test_sampler_and_accept_reject_bad_arguments():
    lib = _knx.load()
    assert lib.knx_sampler_fused(None, 4, 100, 0.0, 1, None, None, None, None, 0, None) == -1
    assert lib.knx_sampler_fused(None, 4, 100, 1.0, 1, None, None, None, None, 0, None) == -3
    assert lib.knx_accept_stop(None, None, None, 1, 2048, 0.1, None, None, None, None, 0, 0.0,
                               None, None) == -1


def test_sampler_selfcond_rejects_bad_arguments_on_host():
    """knx_sampler_fused_sc checks its self-conditioning arguments before touching the device
    (the addresses below are never dereferenced)."""
    lib = _knx.load()
    f = lib.knx_sampler_fused_sc
    sc, prev, fin = 4096, 8192, 12288
    # no output buffer
    assert f(None, 4, 100, 1.0, 1, None, None, None, None, None, None, 1, None, 0, None) == -1
    # finished flags without the previous logits, or rows that are not whole canvases
    assert f(None, 4, 100, 1.0, 1, None, None, None, sc, None, fin, 2, None, 0, None) == -1
    assert f(None, 4, 100, 1.0, 1, None, None, None, sc, prev, fin, 3, None, 0, None) == -1
    # bf16 buffers must be 2-byte aligned
    assert f(None, 4, 100, 1.0, 1, None, None, None, sc + 1, None, None, 1, None, 0, None) == -2
    # valid arguments reach the workspace check, which fails without touching the device
    assert f(None, 4, 100, 1.0, 1, None, None, None, sc, prev, fin, 2, None, 0, None) == -3


def test_ep_exchange_rejects_bad_arguments_on_host():
    """The NVLink exchange entry points check their arguments before any launch (the pointers
    below are never dereferenced): world and rank ranges, the expert split, row widths and
    alignment, and the fused copy-and-barrier forms' arrival counter."""
    lib = _knx.load()
    fl, cnt, x = 4096, 8192, 12288
    # world beyond 8, rank outside the world, E not El * world
    assert lib.knx_ep_p2p_counts(None, 128, 16, 0, 9, None, None, 1, None, None, None) == -1
    assert lib.knx_ep_p2p_counts(None, 128, 64, 2, 2, None, None, 1, None, None, None) == -1
    assert lib.knx_ep_p2p_counts(None, 128, 60, 0, 2, None, None, 1, None, None, None) == -1
    assert lib.knx_ep_p2p_barrier(fl, 2, 2, 1, None, None) == -1
    # dispatch + barrier: H not a multiple of 8, no arrival counter, misaligned rows
    d = lib.knx_ep_p2p_dispatch_barrier
    assert d(x, 2817, 8, None, None, 128, 64, None, None, 2048, fl, 0, 2, 1, cnt, None, None) == -1
    assert d(x, 2816, 8, None, None, 128, 64, None, None, 2048, fl, 0, 2, 1, None, None, None) == -1
    assert d(x, 2816, 8, None, None, 128, 64, None, None, 2048, fl, 2, 2, 1, cnt, None, None) == -1
    assert d(x + 8, 2816, 8, None, None, 128, 64, None, None, 2048, fl, 0, 2, 1, cnt, None,
             None) == -2
    # return + barrier: world beyond 8, El * world beyond 256 experts, no arrival counter
    r = lib.knx_ep_p2p_return_barrier
    assert r(x, 2816, 16, 9, 144, None, None, 4096, fl, 0, 1, cnt, None, None) == -1
    assert r(x, 2816, 200, 2, 400, None, None, 4096, fl, 0, 1, cnt, None, None) == -1
    assert r(x, 2816, 64, 2, 128, None, None, 4096, fl, 0, 1, None, None, None) == -1


def test_relabeled_align_rejects_bad_arguments_on_host():
    """knx_moe_align_relabeled needs its table and a supported id type and expert count, and
    the multi-CTA size needs its scratch (checked before any launch)."""
    lib = _knx.load()
    f = lib.knx_moe_align_relabeled
    ids, tab = 4096, 8192
    assert f(ids, _knx.KNX_I32, 256, 8, 128, None, None, None, None, None, None, 0, None, None) == -1
    assert f(ids, _knx.KNX_F16, 256, 8, 128, tab, None, None, None, None, None, 0, None, None) == -1
    assert f(ids, _knx.KNX_I32, 256, 8, 512, tab, None, None, None, None, None, 0, None, None) == -1
    # 8192 tokens x top-8 needs the multi-CTA sort and its scratch
    assert f(ids, _knx.KNX_I32, 8192, 8, 128, tab, None, None, None, None, None, 0, None,
             None) == -3
    assert f(ids, _knx.KNX_I32, 0, 8, 128, tab, None, None, None, None, None, 0, None, None) == 0
