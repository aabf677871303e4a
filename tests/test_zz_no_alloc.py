"""knx_sampler_fused_static (the sampler entry point that allocates nothing: its scratch is a
fixed array inside libknx.so) against knx_sampler_fused with a caller workspace, through the C ABI.

Named to be collected last, so that it runs both after every other GPU test in one process and,
as `pytest tests/test_zz_no_alloc.py`, alone in a fresh process."""
import ctypes

import pytest
import torch

import _knx

pytestmark = pytest.mark.gpu

ROWS, V = 256, 262144


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _run_workspace(lib, x, temperature, seed, stream):
    rows, v = x.shape
    ws = torch.empty(lib.knx_sampler_workspace_size(rows, v), dtype=torch.uint8, device=x.device)
    h = torch.empty(rows, dtype=torch.float32, device=x.device)
    s = torch.empty(rows, dtype=torch.int64, device=x.device)
    a = torch.empty(rows, dtype=torch.int64, device=x.device)
    _knx.check(lib.knx_sampler_fused(_vp(x), rows, v, temperature, seed, _vp(h), _vp(s), _vp(a),
                                     _vp(ws), ws.numel(), stream), "knx_sampler_fused")
    return h, s, a


def _run_static(lib, x, temperature, seed, stream, out):
    rows, v = x.shape
    h, s, a = out
    _knx.check(lib.knx_sampler_fused_static(_vp(x), rows, v, temperature, seed, _vp(h), _vp(s),
                                            _vp(a), stream), "knx_sampler_fused_static")


def test_static_scratch_sampler_matches_workspace_entry(cuda):
    import workloads
    lib = _knx.load()
    stream = _knx.stream_of(cuda.index or 0)
    xs = [workloads.sampler_logits(ROWS, V, seed=s, device=cuda) for s in (3, 4)]
    cases = [(xs[0], 0.8, 1234), (xs[1], 0.55, 1235)]
    outs = [(torch.empty(ROWS, dtype=torch.float32, device=cuda),
             torch.empty(ROWS, dtype=torch.int64, device=cuda),
             torch.empty(ROWS, dtype=torch.int64, device=cuda)) for _ in cases]
    # two calls in a row on one stream, no synchronisation between them
    for (x, temp, seed), out in zip(cases, outs):
        _run_static(lib, x, temp, seed, stream, out)
    torch.cuda.synchronize()
    for (x, temp, seed), (h, s, a) in zip(cases, outs):
        hw, sw, aw = _run_workspace(lib, x, temp, seed, stream)
        torch.cuda.synchronize()
        # the same kernel runs on both paths: entropy within the sampler tolerance (1e-4 rel),
        # sampled and argmax indices exact
        assert torch.allclose(h, hw, rtol=1e-4, atol=1e-7), (temp, (h - hw).abs().max().item())
        assert torch.equal(s, sw), temp
        assert torch.equal(a, aw), temp


def test_static_scratch_sampler_rejects_oversize_without_launch(cuda):
    lib = _knx.load()
    cap = _knx.KNX_SAMPLER_STATIC_SCRATCH_BYTES
    assert lib.knx_sampler_workspace_size(3969, V) <= cap < lib.knx_sampler_workspace_size(3970, V)
    x = torch.zeros(1, 16, dtype=torch.float32, device=cuda)  # never read: rejected on the host
    st = lib.knx_sampler_fused_static(_vp(x), 3970, V, 1.0, 0, None, None, None,
                                      _knx.stream_of(cuda.index or 0))
    assert st == -3  # KNX_E_WORKSPACE
