"""Comparison with recorded outputs of the reference's own GPU path.

The fixtures ``tests/golden/ref_b200_*.pt`` hold what SparkDiffusion's fused
RoLa inference path (Triton + cuBLAS, sparkdiffusion/ops/fused_kernel/) produced
on a B200 for the seeded configurations: its LUT in ``torch.topk`` order, its
bf16 pooled scores of the top blocks of every row, and sampled rows of its
outputs.  This module measures this build's LUT and outputs against them; it
is used by the GPU tests and by ``bench.py``'s parity report, never on the
forward path.

Selection policy difference: the reference scores the pooled blocks in bf16
(fused_sparse_attn.py:181), this build in fp32, so where the reference's bf16
scores of two blocks at the k-th boundary are equal or one bf16 step apart the
two selections may keep different blocks.  ``selection_report`` classifies
every mismatching row by the reference's own scores: ``tie`` (the swapped
blocks' bf16 scores are equal), ``boundary`` (within ``boundary_ulps`` bf16
steps of each other at the k-th score) or ``unexplained``.
"""

from __future__ import annotations

import os

import torch

HEAD_DIM = 128
GOLDEN_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tests", "golden")


def load_fixture(name: str) -> dict | None:
    """``ref_b200_<name>.pt`` from tests/golden, or None when it is absent."""
    path = os.path.join(GOLDEN_DIR, f"ref_b200_{name}.pt")
    return torch.load(path) if os.path.exists(path) else None


def bf16_ulp(v: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |v| (8 significant bits)."""
    a = v.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def rel_err(got: torch.Tensor, ref: torch.Tensor, mask: torch.Tensor | None = None) -> tuple[float, float]:
    """(max-abs, mean-abs) of got - ref relative to the RMS of ref (over ``mask`` if given)."""
    g, r = got.float().cpu(), ref.float().cpu()
    rms = r.pow(2).mean().sqrt().clamp_min(1e-30)
    d = (g - r).abs()
    if mask is not None:
        d = d[mask]
    return (d.max() / rms).item(), (d.mean() / rms).item()


def worst_of_bound(got: torch.Tensor, ref: torch.Tensor, mask: torch.Tensor | None = None,
                   max_tol: float = 2e-2, steps: float = 1.0) -> float:
    """Largest |got - ref| over the per-element bound max(max_tol * RMS(ref),
    ``steps`` bf16 steps of the reference element): two bf16 results of the same
    value can sit a rounding step apart, and for an element several times the RMS
    that step alone exceeds 2e-2 of the RMS.  <= 1 means every element is within it."""
    g, r = got.float().cpu(), ref.float().cpu()
    rms = r.pow(2).mean().sqrt().clamp_min(1e-30)
    ratio = (g - r).abs() / torch.maximum(max_tol * rms, steps * bf16_ulp(r))
    if mask is not None:
        ratio = ratio[mask]
    return ratio.max().item()


def selection_report(lut: torch.Tensor, fx: dict, heads: int, boundary_ulps: float = 2,
                     B: int = 1) -> tuple[dict, torch.Tensor]:
    """Per-row set agreement of this build's ``lut`` (``[B*H, NB, k]``, rows in
    (batch, head) order) with the fixture's LUT, which holds heads 0..heads-1 of
    every batch element in the same order.  Returns the report and the
    ``[B*heads, NB]`` agreement mask."""
    ref = fx["lut"].long()
    _, NB, k = ref.shape
    mine = lut.detach().cpu().long().reshape(B, -1, NB, k)[:, :heads].reshape(B * heads, NB, k)
    vals, idx = fx["score_vals"].float(), fx["score_idx"].long()
    agree = (torch.sort(mine, -1).values == torch.sort(ref, -1).values).all(-1)
    rep = {"rows": int(agree.numel()), "agree": int(agree.sum()), "tie": 0, "boundary": 0, "unexplained": 0,
           "max_gap_ulps": 0.0}
    for h, m in zip(*torch.nonzero(~agree, as_tuple=True)):
        h, m = int(h), int(m)
        s_mine, s_ref = set(mine[h, m].tolist()), set(ref[h, m].tolist())
        pos = {j: p for p, j in enumerate(idx[h, m].tolist())}
        row = vals[h, m]
        if any(j not in pos for j in s_mine - s_ref):
            rep["unexplained"] += 1  # a kept block the reference scored far below its k-th
            continue
        hi = max(row[pos[j]] for j in s_ref - s_mine)
        lo = min(row[pos[j]] for j in s_mine - s_ref)
        gap = float((hi - lo) / bf16_ulp(row[k - 1]))
        rep["max_gap_ulps"] = max(rep["max_gap_ulps"], gap)
        if gap == 0:
            rep["tie"] += 1
        elif gap <= boundary_ulps:
            rep["boundary"] += 1
        else:
            rep["unexplained"] += 1
    rep["agree_frac"] = rep["agree"] / rep["rows"]
    return rep, agree


def sample_heads(t_tok_major: torch.Tensor, fx: dict, B: int, L: int, H: int, heads: int) -> torch.Tensor:
    """Token-major ``[B, L, H*D]`` -> ``[B, heads, S, D]`` on the fixture's token rows."""
    tok = fx["tokens"].long().to(t_tok_major.device)
    return t_tok_major.reshape(B, L, H, HEAD_DIM)[:, tok, :heads].permute(0, 2, 1, 3).float().cpu()


def sample_out(out: torch.Tensor, fx: dict, B: int, L: int, heads: int) -> torch.Tensor:
    """``[B, L, H*D]`` -> ``[B, S, heads*D]`` on the fixture's token rows."""
    tok = fx["tokens"].long().to(out.device)
    return out.reshape(B, L, -1)[:, tok, : heads * HEAD_DIM].float().cpu()


def agree_mask(agree: torch.Tensor, fx: dict, heads: int, blk: int) -> torch.Tensor:
    """``[B, S, heads*D]`` mask of sampled output elements whose query block's kept sets agree."""
    a = agree.reshape(-1, heads, agree.shape[-1])[:, :, fx["tokens"].long() // blk].transpose(1, 2)  # [B, S, heads]
    return a[..., None].expand(-1, -1, -1, HEAD_DIM).reshape(a.shape[0], -1, heads * HEAD_DIM)


def output_parity(out: torch.Tensor, lut: torch.Tensor, fx: dict, B: int, L: int, H: int, blk: int) -> dict:
    """Selection report plus the gated output's error against the reference's on
    the sampled rows of the query blocks whose kept sets agree."""
    heads = fx["config"]["H"]
    rep, agree = selection_report(lut, fx, heads, B=B)
    got, mask = sample_out(out, fx, B, L, heads), agree_mask(agree, fx, heads, blk)
    mx, mn = rel_err(got, fx["out"], mask)
    return {"heads": heads, "lut_rows": rep["rows"], "lut_agree": rep["agree"], "lut_tie": rep["tie"],
            "lut_boundary": rep["boundary"], "lut_unexplained": rep["unexplained"],
            "out_max_rel": mx, "out_mean_rel": mn,
            "out_worst_of_bound": worst_of_bound(got, fx["out"], mask, steps=2.0),
            "sampled_tokens": int(fx["tokens"].numel())}
