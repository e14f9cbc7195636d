"""The benchmark configurations C1..C5 and their seeded synthetic inputs.

There is no dataset on this path: every configuration is a random-init RoLa
attention layer on synthetic activations with the shapes of Wan 2.1/2.2 video
latents.  Seeds: ``torch.Generator`` seed 0 for the tensors, seed 1 for the
per-block offsets.
"""

from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    grid: tuple  # latent (T, H, W) token grid
    blk: int
    topk: int
    rank: int
    dtype: torch.dtype
    from_x: bool  # True: start from hidden states x and a QKV weight; False: from q/k/v
    layers: int = 1
    head_dim: int = 128

    @property
    def L(self) -> int:
        return self.grid[0] * self.grid[1] * self.grid[2]

    @property
    def NB(self) -> int:
        return (self.L + self.blk - 1) // self.blk

    @property
    def dim(self) -> int:
        return self.H * self.head_dim

    @property
    def reference_topk_ratio(self) -> float:
        """Ratio that makes the reference's int(ratio*NB) equal ``topk``."""
        return (self.topk + 0.5) / self.NB

    def attn_flops(self) -> float:
        """Selected-block attention FLOPs 4*D*sum(rows*cols) over valid tokens
        (uniform-approximation-free only for a given LUT; see ``attn_flops_lut``)."""
        return 4.0 * self.head_dim * self.B * self.H * self.L * self.topk * self.blk

    def prologue_flops(self) -> float:
        return 6.0 * self.B * self.L * self.dim * self.dim if self.from_x else 0.0

    def scaled(self, *, H: int | None = None, grid: tuple | None = None, B: int | None = None) -> "Workload":
        """Same recipe with fewer heads / tokens (parity tests)."""
        g = grid or self.grid
        nb = (g[0] * g[1] * g[2] + self.blk - 1) // self.blk
        return dataclasses.replace(self, H=H or self.H, grid=g, B=B or self.B, topk=min(self.topk, nb),
                                   name=f"{self.name}-scaled")


C1 = Workload("C1 CPU fp32 plumbing", 1, 12, (6, 16, 16), 64, 6, 16, torch.float32, False)
C2 = Workload("C2 Wan2.1-1.3B 480P 0.90", 1, 12, (21, 30, 52), 128, 26, 64, torch.bfloat16, False)
C3 = Workload("C3 Wan2.1-14B 480P 0.90", 1, 40, (21, 30, 52), 128, 26, 64, torch.bfloat16, True)
C4 = Workload("C4 Wan2.1-14B 720P 0.97", 1, 40, (21, 45, 80), 128, 18, 64, torch.bfloat16, True)
C5 = Workload("C5 Wan2.2-14B 480P 0.95 CFG", 2, 40, (21, 30, 52), 128, 13, 64, torch.bfloat16, True, layers=40)
ALL = {"C1": C1, "C2": C2, "C3": C3, "C4": C4, "C5": C5}


def attn_flops_lut(lut: torch.Tensor, L: int, blk: int, D: int = 128) -> float:
    """Exact selected-block FLOPs 4*D*sum_{b,h,m} rows(m)*sum_{j in LUT} cols(j)."""
    nb = (L + blk - 1) // blk
    sizes = torch.full((nb,), blk, dtype=torch.float64)
    sizes[-1] = L - (nb - 1) * blk
    lut = lut.reshape(-1, nb, lut.shape[-1]).long().cpu()
    cols = sizes[lut].sum(-1)  # [BH, NBq]
    return float(4.0 * D * (cols * sizes[None, :]).sum())


def make_inputs(wl: Workload, device="cpu", seed: int = 0) -> dict:
    """Seeded synthetic inputs for one layer of ``wl`` (all in ``wl.dtype``).

    q/k/v mode (C1, C2): q, k, v ~ N(0,1) plus a per-block N(0,1) offset shared
    by the tokens of a block, followed (in the layer) by qk-RMSNorm with unit
    weight; x ~ N(0,1) feeds the gate.  x mode (C3-C5): x ~ N(0,1) and a fused
    QKV weight [3*dim, dim] ~ N(0, 0.02), no bias.  Low-rank factors
    ~ N(0, 1/sqrt(head_dim)); gate weight ~ N(0, 0.02); gate bias -1.946.
    """
    dt = wl.dtype
    B, L, dim, D = wl.B, wl.L, wl.dim, wl.head_dim
    g = torch.Generator(device=device).manual_seed(seed)
    g1 = torch.Generator(device=device).manual_seed(seed + 1)

    def randn(*shape, gen=g, std=1.0):
        return (torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std)

    out: dict = {}
    if wl.from_x:
        out["x"] = randn(B, L, dim).to(dt)
        out["w_qkv"] = randn(3 * dim, dim, std=0.02).to(dt)
        out["b_qkv"] = None
    else:
        q = randn(B, L, dim)
        k = randn(B, L, dim)
        v = randn(B, L, dim)
        out["x"] = randn(B, L, dim).to(dt)
        nb = wl.NB
        for name, t in (("q_raw", q), ("k_raw", k), ("v_raw", v)):
            off = randn(B, nb, dim, gen=g1)
            off = off.repeat_interleave(wl.blk, dim=1)[:, :L]
            out[name] = (t + off).to(dt)
    out["norm_wq"] = torch.ones(dim, device=device, dtype=dt)
    out["norm_wk"] = torch.ones(dim, device=device, dtype=dt)
    out["proj_q"] = randn(wl.rank, D, std=1.0 / math.sqrt(D)).to(dt)
    out["proj_k"] = randn(wl.rank, D, std=1.0 / math.sqrt(D)).to(dt)
    out["gate_w"] = randn(1, D, std=0.02).to(dt)
    out["gate_b"] = torch.full((1, wl.H, 1, 1), -1.946, device=device, dtype=torch.float32)
    return out
