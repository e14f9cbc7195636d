"""Training path of the RoLa layer on the B200 kernels.

The reference trains ``WanSelfAttentionRoLa`` through its non-fused forward
(sparkdiffusion/networks/wan_rola_attention.py:452-559): eager q/k/v
projections, ``WanRMSNorm`` (wan2pt1.py:188-206), ``rope_apply``
(wan2pt1.py:156-185), the low-rank branch (``_lowrank_attn``,
wan_rola_attention.py:329-391) and the gated fusion in PyTorch, and the
block-sparse softmax attention from the external SLA package:
``get_block_map`` for the selection and ``_attention.apply`` for the forward
and backward (wan_rola_attention.py:293-327).  Here the selection runs on the
B200 selection kernels and the attention's forward (with the row
log-sum-exp) and backward on the tcgen05 kernels (``BlockSparseAttention``);
the eager parts stay eager PyTorch, as in the reference.  There is no
fallback: the attention raises without the CUDA library.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib, ops


def select_blocks(q: torch.Tensor, k: torch.Tensor, topk_ratio: float, blk: int):
    """Block selection of ``q, k [B, H, L, 128]`` (post-RoPE, bf16): mean
    pooling, smooth-K centre, fp32 scores, top-k with ties toward the lower
    index — the semantics of the reference's ``get_block_map``
    (fused_sparse_attn.py:179-198 restates it for the fused path).  Returns
    ``(lut [B*H, NB, topk], topk, paired)``; ``paired`` is the block-64 table
    the attention kernels take (None for block 128)."""
    B, H, L, _ = q.shape
    NB = (L + blk - 1) // blk
    topk = ops.topk_count(topk_ratio, NB)
    with torch.no_grad():
        pq = ops.mean_pool(q, blk)
        pk = ops.mean_pool(k, blk, center=ops.smooth_k_center(k, blk))
        lut = ops.block_select(pq, pk, topk)
        paired = None
        if blk == 64:
            paired = torch.empty(B * H, (NB + 1) // 2, 2 * topk + 1, device=q.device, dtype=torch.int32)
            _lib.call("rola_b200_pair_blocks", ops._ptr(lut), B * H, NB, topk, ops._ptr(paired), ops._stream())
    return lut, topk, paired


class BlockSparseAttention(torch.autograd.Function):
    """o = block-sparse softmax attention of ``q, k, v [B, H, L, 128]`` (bf16)
    over the selection ``lut``; backward on the B200 kernels.  The counterpart
    of SLA's ``_attention.apply(q, k, v, sparse_map, lut, real_topk, BLKQ,
    BLKK)`` (wan_rola_attention.py:320-321)."""

    @staticmethod
    def forward(ctx, q, k, v, lut, paired, blk: int, topk: int):
        o, lse = ops.sparse_attention_fwd_lse(q, k, v, lut if blk == 128 else paired, blk, topk)
        ctx.save_for_backward(q, k, v, o, lse, lut, paired if paired is not None else lut)
        ctx.blk, ctx.topk = blk, topk
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, lut, paired = ctx.saved_tensors
        dq, dk, dv = ops.sparse_attention_bwd(q, k, v, o, do, lut, paired if ctx.blk == 64 else None, lse, ctx.blk,
                                              ctx.topk)
        return dq, dk, dv, None, None, None, None


def sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, topk_ratio: float, blkq: int,
                     blkk: int) -> torch.Tensor:
    """The reference's ``_sparse_attn`` (wan_rola_attention.py:293-327) on the
    B200 kernels: ``q, k, v [B, H, L, 128]`` -> ``o [B, H, L, 128]`` in the
    input dtype, differentiable in q, k and v."""
    if blkq != blkk or blkq not in (64, 128):
        raise ValueError("the B200 attention kernels support blkq == blkk in (64, 128)")
    if not q.is_cuda:
        raise RuntimeError("the B200 training path runs on CUDA tensors only")
    dt = q.dtype
    qb, kb, vb = (t.to(torch.bfloat16) for t in (q, k, v))
    lut, topk, paired = select_blocks(qb.detach(), kb.detach(), topk_ratio, blkq)
    o = BlockSparseAttention.apply(qb, kb, vb, lut, paired, blkq, topk)
    return o.to(dt)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``WanRMSNorm.forward`` (wan2pt1.py:200-206): fp32 normalisation, cast back, times the weight."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).type_as(x) * weight


def rope_apply(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """``rope_apply`` (wan2pt1.py:156-185): interleaved pairs rotated in fp32 by
    the raw angles ``freqs [L, D/2]``; ``x [B, L, H, D]``."""
    B, L, H, D = x.shape
    f = freqs[:L].reshape(L, D // 2)
    c = torch.cos(f).float()[None, :, None, :]
    s = torch.sin(f).float()[None, :, None, :]
    xf = x.float()
    e, o = xf[..., 0::2], xf[..., 1::2]
    return torch.stack([e * c - o * s, e * s + o * c], dim=-1).flatten(-2).to(x.dtype)


def rope_rank(x: torch.Tensor, freqs: torch.Tensor, rank: int) -> torch.Tensor:
    """Truncated interleaved RoPE of the low-rank features ``x [B, H, L, rank]``
    (``_apply_rope_rank``, wan_rola_attention.py:329-364): angles cast to the
    data dtype, the first ``min(rank/2, D/2)`` pairs rotated, the rest unchanged."""
    L = x.shape[2]
    rd = min(rank // 2, freqs.shape[-1])
    f = freqs[:L, :rd].to(x.dtype)
    c, s = torch.cos(f), torch.sin(f)
    x1, x2 = x[..., : 2 * rd].unflatten(-1, (-1, 2)).unbind(-1)
    rot = torch.stack([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).flatten(-2)
    if 2 * rd < rank:
        rot = torch.cat([rot, x[..., 2 * rd:]], dim=-1)
    return rot


def lowrank_attention(layer, qn: torch.Tensor, kn: torch.Tensor, v: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """``_lowrank_attn`` (wan_rola_attention.py:366-391) over ``[B, H, L, D]``:
    SiLU projections to the rank, truncated RoPE, O = Q_lr (K_lr^T V), RMS-normed."""
    q_lr = rope_rank(F.silu(layer.proj_q(qn)), freqs, layer.rola_rank)
    k_lr = rope_rank(F.silu(layer.proj_k(kn)), freqs, layer.rola_rank)
    out = q_lr @ (k_lr.transpose(-2, -1) @ v)
    return F.rms_norm(out, [out.shape[-1]])


def training_attention_core(layer, x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """The reference's non-fused forward up to (not including) ``self.o``
    (wan_rola_attention.py:481-545): differentiable in x and every parameter."""
    b, s, _ = x.shape
    n, d = layer.num_heads, layer.head_dim
    q = layer.q(x)
    k = layer.k(x)
    if layer.qk_norm:
        q = rms_norm(q, layer.norm_q.weight, layer.norm_q.eps)
        k = rms_norm(k, layer.norm_k.weight, layer.norm_k.eps)
    q = q.view(b, s, n, d)
    k = k.view(b, s, n, d)
    v = layer.v(x).view(b, s, n, d)
    q_rope = rope_apply(q, freqs)
    k_rope = rope_apply(k, freqs)
    v_bhld = v.transpose(1, 2)
    o_s = sparse_attention(q_rope.transpose(1, 2), k_rope.transpose(1, 2), v_bhld, layer.rola_topk_ratio,
                           layer.rola_blkq, layer.rola_blkk)
    o_l = lowrank_attention(layer, q.transpose(1, 2), k.transpose(1, 2), v_bhld, freqs)
    x_bhld = x.view(b, s, n, d).transpose(1, 2)
    gate = torch.sigmoid(layer.gate_proj(x_bhld) + layer.gate_bias)
    o_s_scale = (o_s.pow(2).mean(dim=-1, keepdim=True) + 1e-5).sqrt()
    fused = o_s.float() / o_s_scale.float() + gate * o_l.float()
    out_bhld = (fused * o_s_scale.float()).to(o_l.dtype)
    return out_bhld.transpose(1, 2).reshape(b, s, n * d)


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Dense softmax attention of ``q, k, v [B, H, L, 128]``, differentiable:
    the block-sparse kernels with every 128-token key block selected."""
    if not q.is_cuda:
        raise RuntimeError("the B200 training path runs on CUDA tensors only")
    B, H, L, _ = q.shape
    NB = (L + 127) // 128
    lut = ops._full_lut(B * H, NB, q.device)
    dt = q.dtype
    o = BlockSparseAttention.apply(*(t.to(torch.bfloat16) for t in (q, k, v)), lut, None, 128, NB)
    return o.to(dt)


def dense_training_forward(layer, x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """``WanSelfAttention.forward``'s differentiable route (wan2pt1.py:313-328)
    with the attention on the B200 kernels: projections, ``WanRMSNorm``, ``rope_apply``,
    dense attention, ``self.o``."""
    b, s, _ = x.shape
    n, d = layer.num_heads, layer.head_dim
    q, k = layer.q(x), layer.k(x)
    if layer.qk_norm:
        q = rms_norm(q, layer.norm_q.weight, layer.norm_q.eps)
        k = rms_norm(k, layer.norm_k.weight, layer.norm_k.eps)
    q = rope_apply(q.view(b, s, n, d), freqs)
    k = rope_apply(k.view(b, s, n, d), freqs)
    v = layer.v(x).view(b, s, n, d)
    o = dense_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return layer.o(o.transpose(1, 2).reshape(b, s, n * d))
