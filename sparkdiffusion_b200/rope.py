"""Wan 3D RoPE angles and the cos/sin tables shared by all layers of a forward.

Host-side table preparation (once per forward, shared by every block, as the
reference does through ``rope_cache``):

* ``wan_rope_freqs`` restates ``VideoRopePosition3DEmb.generate_embeddings``
  (sparkdiffusion/networks/wan2pt1.py:45-137);
* ``prepare_cos_sin`` restates fused_qkv_rope.py:37-50 (interleaved fp32);
* ``prepare_lowrank_cos_sin`` restates fused_lowrank.py:254-267 (angles cast
  to the data dtype before cos/sin), without the power-of-two padding that only
  served Triton.
"""

from __future__ import annotations

import torch


def wan_rope_freqs(T: int, H: int, W: int, head_dim: int = 128, theta: float = 10000.0,
                   device: torch.device | str | None = None) -> torch.Tensor:
    """Raw angles ``[T*H*W, head_dim // 2]`` fp32 in (t h w) token order."""
    dim_h = head_dim // 6 * 2
    dim_t = head_dim - 2 * dim_h
    seq = torch.arange(max(H, W, T), device=device).float()
    spatial = torch.arange(0, dim_h, 2, device=device)[: dim_h // 2].float() / dim_h
    temporal = torch.arange(0, dim_t, 2, device=device)[: dim_t // 2].float() / dim_t
    h_freqs = 1.0 / (theta ** spatial)
    w_freqs = 1.0 / (theta ** spatial)
    t_freqs = 1.0 / (theta ** temporal)
    ft = torch.outer(seq[:T], t_freqs)
    fh = torch.outer(seq[:H], h_freqs)
    fw = torch.outer(seq[:W], w_freqs)
    out = torch.cat(
        [
            ft[:, None, None, :].expand(T, H, W, -1),
            fh[None, :, None, :].expand(T, H, W, -1),
            fw[None, None, :, :].expand(T, H, W, -1),
        ],
        dim=-1,
    )
    return out.reshape(T * H * W, -1).float().contiguous()


def prepare_cos_sin(freqs: torch.Tensor, L: int, D: int) -> torch.Tensor:
    """Interleaved ``[L, D]`` fp32 table (cos0, sin0, cos1, sin1, ...)."""
    f = freqs[:L, : D // 2]
    cos = torch.cos(f).to(torch.float32)
    sin = torch.sin(f).to(torch.float32)
    return torch.stack([cos, sin], dim=-1).reshape(L, D).contiguous()


def prepare_lowrank_cos_sin(freqs: torch.Tensor, L: int, rank: int, dtype: torch.dtype):
    """(cos, sin, rope_dim): ``[L, rope_dim]`` tables in ``dtype``."""
    rope_dim = min(rank // 2, freqs.shape[-1])
    f = freqs[:L, :rope_dim].to(dtype)
    return torch.cos(f).contiguous(), torch.sin(f).contiguous(), rope_dim
