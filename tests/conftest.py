import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def reference_path(allow_checkout: bool = True):
    """Directory from which the SparkDiffusion reference imports: ``SPARKDIFFUSION_REF``,
    the installed copy ``baseline/_ref``, or (CPU tests in the build container only,
    ``allow_checkout``) the read-only source checkout; None when none exists (the GPU box
    has only the installed copy)."""
    cands = [os.environ.get("SPARKDIFFUSION_REF", ""), os.path.join(ROOT, "baseline", "_ref")]
    if allow_checkout:
        cands.append("/root/reference")
    for p in cands:
        if p and os.path.isdir(os.path.join(p, "sparkdiffusion", "networks")):
            return p
    return None


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


def assert_bf16_close(got, ref, name="", max_tol=BF16_MAX, mean_tol=BF16_MEAN, ulp_floor=False, steps=1.0):
    """max-abs <= ``max_tol`` and mean-abs <= ``mean_tol`` of the RMS of ``ref``.

    ``ulp_floor``: for a bf16 result checked against an fp32 (unrounded) oracle,
    each element may instead differ by one bf16 rounding step (ulp) of its own
    magnitude where that step exceeds ``max_tol`` of the RMS: an output whose
    largest elements sit ~6x above its RMS cannot be represented in bf16 closer
    than that (one step is then up to ~4e-2 of the RMS).  ``steps`` widens the
    per-element floor to that many steps (results that pass through several
    bf16 roundings, e.g. gradients)."""
    if not ulp_floor:
        mx, mn = rel_err(got, ref)
        assert mx <= max_tol and mn <= mean_tol, f"{name}: max-abs/rms={mx:.3e} mean-abs/rms={mn:.3e}"
        return
    worst, mx, mn = bf16_bound_ratio(got, ref, max_tol, steps)
    assert worst <= 1.0 and mn <= mean_tol, (f"{name}: max-abs/rms={mx:.3e} ({worst:.2f} of the per-element bound "
                                             f"max({max_tol:g}*rms, {steps:g} bf16 step)), mean-abs/rms={mn:.3e}")


def bf16_bound_ratio(got, ref, max_tol=BF16_MAX, steps=1.0):
    """(worst element's |got - ref| over its bound max(``max_tol`` * RMS,
    ``steps`` bf16 steps of the element), max-abs / RMS, mean-abs / RMS)."""
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    rms = r.pow(2).mean().sqrt().clamp_min(1e-30)
    d = (g - r).abs()
    step = torch.exp2(torch.floor(torch.log2(r.abs().clamp_min(1e-30))) - 7)
    bound = torch.maximum(max_tol * rms, steps * step)
    return (d / bound).max().item(), (d.max() / rms).item(), (d.mean() / rms).item()


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
