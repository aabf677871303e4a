"""Test configuration: the `gpu` marker, import paths, shared fixtures.

CPU tests (`-m "not gpu"`) check the oracle against the golden fixtures made from the reference,
the host-side logic and the C ABI surface.  GPU tests (`-m gpu`) are the parity tests proper:
they call the sm_100a kernels through libknx.so and compare with the oracle.
"""
import os
import pathlib
import sys

import numpy as np
import pytest
import torch

REPO = pathlib.Path(__file__).resolve().parent.parent
PKG = REPO / "knivesysl-diffusion-xe_b200"
for p in (str(PKG / "kernels"), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and libknx.so")


def golden(name):
    return dict(np.load(GOLDEN / name))


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def assert_close_fp16(out, ref, rtol=1e-2, atol=2e-3, what=""):
    """The north-star tolerance for fp16 outputs: |out - ref| <= atol + rtol * |ref|."""
    o = out.float().cpu()
    r = ref.float().cpu()
    err = (o - r).abs()
    bound = atol + rtol * r.abs()
    bad = (err > bound).sum().item()
    assert bad == 0, (f"{what}: {bad}/{err.numel()} elements outside atol={atol} rtol={rtol}; "
                      f"max err {err.max().item():.3e}")
