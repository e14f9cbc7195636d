import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def rel_err(got: torch.Tensor, ref: torch.Tensor):
    """(max-abs, mean-abs) of got - ref relative to the RMS of ref."""
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    rms = r.pow(2).mean().sqrt().clamp_min(1e-30)
    d = (g - r).abs()
    return (d.max() / rms).item(), (d.mean() / rms).item()


# The tolerance for bf16 outputs: max-abs <= 2e-2 and mean-abs <= 2e-3 of the output RMS
BF16_MAX = 2e-2
BF16_MEAN = 2e-3


def assert_bf16_close(got, ref, name="", max_tol=BF16_MAX, mean_tol=BF16_MEAN):
    mx, mn = rel_err(got, ref)
    assert mx <= max_tol and mn <= mean_tol, f"{name}: max-abs/rms={mx:.3e} mean-abs/rms={mn:.3e}"


def assert_ulp_close(got, ref, name="", ulps=2, max_frac=1e-3, mean_tol=BF16_MEAN):
    """Element-wise bf16 check for intermediate tensors that pass through chains of
    bf16 roundings: at most ``max_frac`` of the elements may differ by more than
    ``ulps`` bf16 ulps of their magnitude, and the mean-abs error stays within
    ``mean_tol`` of the RMS."""
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    mag = torch.maximum(g.abs(), r.abs()).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
    bad = (g - r).abs() > ulps * ulp
    frac = bad.float().mean().item()
    _, mn = rel_err(got, ref)
    assert frac <= max_frac and mn <= mean_tol, f"{name}: {frac:.2e} of elements beyond {ulps} ulp, mean-abs/rms={mn:.3e}"
