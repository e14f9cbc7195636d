"""``torch.ops.rola_b200.*``: the B200 kernels as PyTorch custom operators.

The Wan inference entry points compile the whole model
(``torch.compile(model, ...)``, sparkdiffusion/utils/inference_optimization.py:122).
Each op here is opaque to Dynamo/Inductor: its real implementation launches
librola_b200 kernels through the C ABI (``ops``), and a fake (meta) kernel
gives output shapes and dtypes for tracing, so a compiled graph holds one node
per op instead of tracing into ctypes calls on ``data_ptr()``.  The drop-in
layers call these ops.

Ops (inputs and layouts as in ``ops``; outputs are new tensors):

* ``qkv_gemm(x2d, w, bias?) -> [M, N]`` bf16 (the QKV projection and ``self.o``);
* ``attention_core(x, w_qkv, b_qkv?, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq?,
  norm_wk?, proj_q, proj_k, gate_w, gate_b, num_heads, topk, eps, blk=128, w_scale?) -> [B, L, H*D]``
  (``w_scale`` given: ``w_qkv`` is float8_e4m3fn, the reference's FP8 mode)
  bf16: ``fused_forward`` minus ``self.o`` (wan_rola_attention.py:414-446);
* ``block_select(pooled_q, pooled_k, topk) -> [B*H, NBq, topk]`` int32;
* ``fused_sparse_attn(q, k, v, topk_ratio, blkq, blkk, num_heads) -> [B, H, L, D]``
  (fused_sparse_attn.py:151-215);
* ``dense_attention(q, k, v, num_heads) -> [B, H, L, D]``.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops

BF16 = torch.bfloat16
Tensor = torch.Tensor


@torch.library.custom_op("rola_b200::qkv_gemm", mutates_args=())
def qkv_gemm(x2d: Tensor, w: Tensor, bias: Optional[Tensor]) -> Tensor:
    return ops.qkv_gemm(x2d, w, bias)


@qkv_gemm.register_fake
def _(x2d, w, bias):
    return x2d.new_empty(x2d.shape[0], w.shape[0], dtype=BF16)


@torch.library.custom_op("rola_b200::attention_core", mutates_args=())
def attention_core(x: Tensor, w_qkv: Tensor, b_qkv: Optional[Tensor], cos_sin: Tensor, lr_cos: Tensor,
                   lr_sin: Tensor, rope_dim: int, norm_wq: Optional[Tensor], norm_wk: Optional[Tensor],
                   proj_q: Tensor, proj_k: Tensor, gate_w: Tensor, gate_b: Tensor, num_heads: int, topk: int,
                   eps: float, blk: int = 128, w_scale: Optional[Tensor] = None) -> Tensor:
    return ops.rola_attention_core(x, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq, norm_wk, proj_q,
                                   proj_k, gate_w, gate_b, num_heads, blk, topk, eps, w_scale=w_scale)


@attention_core.register_fake
def _(x, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq, norm_wk, proj_q, proj_k, gate_w, gate_b,
      num_heads, topk, eps, blk=128, w_scale=None):
    return x.new_empty(x.shape, dtype=BF16)


@torch.library.custom_op("rola_b200::block_select", mutates_args=())
def block_select(pooled_q: Tensor, pooled_k: Tensor, topk: int) -> Tensor:
    return ops.block_select(pooled_q, pooled_k, topk)


@block_select.register_fake
def _(pooled_q, pooled_k, topk):
    B, H, NBq, _ = pooled_q.shape
    return pooled_q.new_empty(B * H, NBq, topk, dtype=torch.int32)


@torch.library.custom_op("rola_b200::fused_sparse_attn", mutates_args=())
def fused_sparse_attn(q: Tensor, k: Tensor, v: Tensor, topk_ratio: float, blkq: int, blkk: int,
                      num_heads: int) -> Tensor:
    return ops.fused_sparse_attn(q, k, v, topk_ratio, blkq, blkk, num_heads)


@fused_sparse_attn.register_fake
def _(q, k, v, topk_ratio, blkq, blkk, num_heads):
    BH, L, D = q.shape
    return v.new_empty(BH // num_heads, num_heads, L, D)


@torch.library.custom_op("rola_b200::dense_attention", mutates_args=())
def dense_attention(q: Tensor, k: Tensor, v: Tensor, num_heads: int) -> Tensor:
    return ops.dense_attention(q, k, v, num_heads)


@dense_attention.register_fake
def _(q, k, v, num_heads):
    BH, L, D = q.shape
    return v.new_empty(BH // num_heads, num_heads, L, D)
