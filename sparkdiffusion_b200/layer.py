"""Drop-in RoLa self-attention layer backed by the B200 kernels.

``WanSelfAttentionRoLaB200`` has the constructor signature, parameter names
and shapes of the reference's ``WanSelfAttentionRoLa``
(sparkdiffusion/networks/wan_rola_attention.py:209-287), so RoLa checkpoints
load into it, and the forward contract of the sparse-attention plugin
interface: ``forward(x [B, L, dim], seq_lens, freqs [L, D/2], rope_cache=None)
-> [B, L, dim]`` (sparse_attn_registry.py:16-18, wan2pt1.py:468-472).  It is
registered as ``"rola_b200"``.

Inference runs the fused B200 path (the reference's fused path has the same
gating, wan_rola_attention.py:467-477).  Under autograd (training, or an input
that requires grad) the forward takes the reference's non-fused training
route instead (``train.training_attention_core``): eager projections, norm,
RoPE, low-rank branch and gate, with the block-sparse attention's forward and
backward on the tcgen05 kernels in place of the external SLA package.  CPU
tensors raise instead of falling back.  The inference kernels are reached
through the custom operators ``torch.ops.rola_b200.*`` (``torch_ops``), so
``torch.compile`` of a model holding these layers captures each as one opaque
node (meta tensors run the operators' shape functions only).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops, torch_ops  # noqa: F401  (torch_ops registers torch.ops.rola_b200.*)
from .registry import register_sparse_attn
from .rope import prepare_cos_sin, prepare_lowrank_cos_sin


class RMSNormWeight(nn.Module):
    """Holds ``weight [dim]`` like ``WanRMSNorm`` (wan2pt1.py:188-206); the
    normalisation itself runs inside the fused prologue kernel."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def reset_parameters(self):
        self.weight.data.fill_(1.0)


@register_sparse_attn("rola_b200", sparse_param_names=["proj_q", "proj_k", "gate_proj", "gate_bias"])
class WanSelfAttentionRoLaB200(nn.Module):
    def __init__(self, dim: int, num_heads: int, qk_norm: bool = True, eps: float = 1e-6,
                 rola_topk_ratio: float = 0.1, rola_rank: int = 64, rola_blkq: int = 128, rola_blkk: int = 128,
                 attn_precision: str = "bf16"):
        super().__init__()
        assert dim % num_heads == 0
        if attn_precision not in ("bf16", "int8"):
            raise ValueError(f"attn_precision must be bf16/int8, got {attn_precision!r}")
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.qk_norm = qk_norm
        self.eps = eps
        self.rola_topk_ratio = rola_topk_ratio
        self.rola_rank = rola_rank
        self.rola_blkq = rola_blkq
        self.rola_blkk = rola_blkk
        self.attn_precision = attn_precision
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        if qk_norm:
            self.norm_q = RMSNormWeight(dim, eps=eps)
            self.norm_k = RMSNormWeight(dim, eps=eps)
        else:
            self.norm_q = nn.Identity()
            self.norm_k = nn.Identity()
        h, r = self.head_dim, rola_rank
        self.proj_q = nn.Linear(h, r, bias=False)
        self.proj_k = nn.Linear(h, r, bias=False)
        self.gate_proj = nn.Linear(h, 1, bias=False)
        self.gate_bias = nn.Parameter(torch.full((1, num_heads, 1, 1), -1.946))
        self.init_weights()
        self._layer_name = "RoLaB200"
        self._use_fused_inference = True
        self._pg = None
        self._qkv_cache = None
        self._o_cache = None

    def init_weights(self):
        """Re-apply the RoLa-specific init after WanModel's xavier pass
        (wan_rola_attention.py:278-287)."""
        nn.init.kaiming_uniform_(self.proj_q.weight, a=math.sqrt(5))
        nn.init.kaiming_uniform_(self.proj_k.weight, a=math.sqrt(5))
        nn.init.zeros_(self.gate_proj.weight)
        self.gate_bias.data.fill_(-1.946)

    def set_context_parallel_group(self, process_group, ranks, stream):
        """Receives the sequence-parallel group (wan2pt1.py:942-960); with more
        than one rank the forward runs the Ulysses sequence<->head exchange."""
        del ranks, stream
        self._pg = process_group

    def _fused_qkv(self):
        if torch.compiler.is_compiling():  # traced: no data pointers, the concatenation is part of the graph
            return (torch.cat([self.q.weight, self.k.weight, self.v.weight], 0).to(torch.bfloat16),
                    torch.cat([self.q.bias, self.k.bias, self.v.bias], 0).to(torch.bfloat16))
        key = tuple((p.data_ptr(), p._version) for p in (self.q.weight, self.k.weight, self.v.weight,
                                                         self.q.bias, self.k.bias, self.v.bias))
        if self._qkv_cache is None or self._qkv_cache[0] != key:
            w = torch.cat([self.q.weight, self.k.weight, self.v.weight], 0).to(torch.bfloat16).contiguous()
            b = torch.cat([self.q.bias, self.k.bias, self.v.bias], 0).to(torch.bfloat16).contiguous()
            self._qkv_cache = (key, w, b)
        return self._qkv_cache[1], self._qkv_cache[2]

    @staticmethod
    def _is_fp8(mod) -> bool:
        """The reference's FP8Linear (sparkdiffusion/ops/quantization/fp8_linear.py:134-155): e4m3
        ``weight_fp8 [out, in]`` and fp32 ``w_scale_t [1, out]`` buffers instead of ``weight``."""
        return hasattr(mod, "weight_fp8") and hasattr(mod, "w_scale_t")

    def _fp8_qkv(self):
        """(w_fp8 [3*dim, dim], w_scale [3*dim], bias) when q/k/v were converted to
        FP8Linear (prequantize_qkv / convert_dit_linears_to_fp8), else None."""
        mods = (self.q, self.k, self.v)
        if not all(self._is_fp8(m) for m in mods):
            if any(self._is_fp8(m) for m in mods):
                raise ValueError("q, k and v must all be FP8Linear or all nn.Linear")
            return None
        biases = [getattr(m, "bias", None) for m in mods]

        def build():
            w8 = torch.cat([m.weight_fp8.view(torch.uint8) for m in mods], 0).view(torch.float8_e4m3fn)
            ws = torch.cat([m.w_scale_t.reshape(-1).float() for m in mods], 0)
            b = None if any(t is None for t in biases) else torch.cat(biases, 0).to(torch.bfloat16)
            return w8, ws, b

        if torch.compiler.is_compiling():
            return build()
        key = tuple(t.data_ptr() for m in mods for t in (m.weight_fp8, m.w_scale_t))
        if self._qkv_cache is None or self._qkv_cache[0] != key:
            self._qkv_cache = (key, *build())
        return self._qkv_cache[1:]

    def _autograd_route(self, x: torch.Tensor) -> bool:
        """The reference trains through its non-fused forward whenever autograd
        records (wan_rola_attention.py:467-477); so does this layer."""
        return torch.is_grad_enabled() and (self.training or x.requires_grad)

    def attention_core(self, x: torch.Tensor, freqs: torch.Tensor, rope_cache=None) -> torch.Tensor:
        """Everything of the forward except the output projection."""
        if x.device.type == "cpu":
            raise RuntimeError("WanSelfAttentionRoLaB200 runs on CUDA tensors only")
        if self.attn_precision != "bf16":
            raise ValueError("the B200 path implements attn_precision='bf16'")
        if self.rola_blkq != self.rola_blkk or self.rola_blkq not in (64, 128):
            raise ValueError("the B200 attention kernel supports rola_blkq == rola_blkk in (64, 128)")
        B, L, dim = x.shape
        if L < max(self.rola_blkq, self.rola_blkk):
            raise ValueError("sequence shorter than one block")
        if self._autograd_route(x):
            if self._pg is not None and torch.distributed.get_world_size(self._pg) > 1:
                raise RuntimeError("the sequence-parallel route of WanSelfAttentionRoLaB200 is inference-only")
            from .train import training_attention_core
            return training_attention_core(self, x, freqs)
        x = x.to(torch.bfloat16).contiguous()
        D = self.head_dim
        if rope_cache is not None and rope_cache[0] is not None:
            cos_sin = rope_cache[0]
        else:
            cos_sin = prepare_cos_sin(freqs, freqs.shape[0], D)
        if rope_cache is not None and rope_cache[1] is not None:
            lr_cos, lr_sin, rope_dim = rope_cache[1][0], rope_cache[1][1], rope_cache[1][2]
        else:
            lr_cos, lr_sin, rope_dim = prepare_lowrank_cos_sin(freqs, freqs.shape[0], self.rola_rank, torch.bfloat16)
        fp8 = self._fp8_qkv()
        if fp8 is not None:
            w_qkv, w_scale, b_qkv = fp8
        else:
            (w_qkv, b_qkv), w_scale = self._fused_qkv(), None
        nwq = self.norm_q.weight if self.qk_norm else None
        nwk = self.norm_k.weight if self.qk_norm else None
        if self._pg is not None and torch.distributed.get_world_size(self._pg) > 1:
            if w_scale is not None:
                raise ValueError("the sequence-parallel route takes bf16 q/k/v projections")
            from .ulysses import ulysses_rola_attention
            return ulysses_rola_attention(self, x, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, nwq, nwk)
        blk = self.rola_blkq
        NB = (L + blk - 1) // blk
        topk = ops.topk_count(self.rola_topk_ratio, NB)
        return torch.ops.rola_b200.attention_core(x, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, nwq, nwk,
                                                  self.proj_q.weight, self.proj_k.weight, self.gate_proj.weight,
                                                  self.gate_bias, self.num_heads, topk, self.eps, blk, w_scale)

    def _o_weight(self):
        """bf16 copy of the output projection for the tcgen05 GEMM (cached like the QKV weight)."""
        if torch.compiler.is_compiling():
            return self.o.weight.to(torch.bfloat16), self.o.bias.to(torch.bfloat16)
        key = (self.o.weight.data_ptr(), self.o.weight._version, self.o.bias.data_ptr(), self.o.bias._version)
        if self._o_cache is None or self._o_cache[0] != key:
            self._o_cache = (key, self.o.weight.to(torch.bfloat16).contiguous(),
                             self.o.bias.to(torch.bfloat16).contiguous())
        return self._o_cache[1], self._o_cache[2]

    def forward(self, x: torch.Tensor, seq_lens: torch.Tensor, freqs: torch.Tensor, rope_cache=None) -> torch.Tensor:
        del seq_lens
        out = self.attention_core(x, freqs, rope_cache)
        if self._autograd_route(x):
            return self.o(out)  # wan_rola_attention.py:552
        B, L, dim = out.shape
        if self._is_fp8(self.o):
            # FP8Linear output projection: per-token quantization of the attention output
            xq, xs = ops.quantize_rows_e4m3(out.reshape(B * L, dim))
            y = ops.qkv_gemm_fp8(xq, xs, self.o.weight_fp8, self.o.w_scale_t, getattr(self.o, "bias", None))
            return y.view(B, L, dim).to(x.dtype)
        if dim % 256 == 0:
            # self.o (wan_rola_attention.py:447) on the same persistent tcgen05 GEMM as the QKV projection
            w, b = self._o_weight()
            y = torch.ops.rola_b200.qkv_gemm(out.reshape(B * L, dim), w, b).view(B, L, dim)
            return y.to(self.o.weight.dtype)
        return F.linear(out.to(self.o.weight.dtype), self.o.weight, self.o.bias)


class WanSelfAttentionB200(nn.Module):
    """Dense self-attention of the Wan DiT on the B200 kernels: the fused
    inference path of ``WanSelfAttention.forward`` (wan2pt1.py:221-324) — one
    QKV GEMM, the streaming qk-RMSNorm + RoPE pass, dense attention (the
    block-sparse kernel with every key block selected) and the output
    projection on the same GEMM.  Same parameter names and shapes (q, k, v, o,
    norm_q, norm_k) as the reference layer, so its checkpoints load unchanged.
    Under autograd the reference's differentiable route (wan2pt1.py:313-328) runs,
    with the attention's forward and backward on the tcgen05 kernels (every
    key block selected)."""

    def __init__(self, dim: int, num_heads: int, qk_norm: bool = True, eps: float = 1e-6):
        super().__init__()
        assert dim % num_heads == 0
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.qk_norm = qk_norm
        self.eps = eps
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        self.norm_q = RMSNormWeight(dim, eps=eps) if qk_norm else nn.Identity()
        self.norm_k = RMSNormWeight(dim, eps=eps) if qk_norm else nn.Identity()
        self._layer_name = "DenseB200"
        self._qkv_cache = None
        self._o_cache = None
        self.init_weights()

    def init_weights(self):
        """Same init as the reference layer (wan2pt1.py:247-262)."""
        std = 1.0 / math.sqrt(self.dim)
        for lin in (self.q, self.k, self.v, self.o):
            torch.nn.init.trunc_normal_(lin.weight, std=std)
            lin.bias.data.zero_()
        if self.qk_norm:
            self.norm_q.reset_parameters()
            self.norm_k.reset_parameters()

    _fused_qkv = WanSelfAttentionRoLaB200._fused_qkv
    _o_weight = WanSelfAttentionRoLaB200._o_weight

    def forward(self, x: torch.Tensor, seq_lens: torch.Tensor, freqs: torch.Tensor, rope_cache=None) -> torch.Tensor:
        del seq_lens
        if not x.is_cuda:
            raise RuntimeError("WanSelfAttentionB200 runs on CUDA tensors only")
        if self.head_dim != 128 or self.dim % 256 != 0:
            raise ValueError("the B200 path needs head_dim 128 and an even head count")
        B, L, dim = x.shape
        H = self.num_heads
        if torch.is_grad_enabled() and (self.training or x.requires_grad):
            from .train import dense_training_forward
            return dense_training_forward(self, x, freqs)
        x = x.to(torch.bfloat16).contiguous()
        if rope_cache is not None and rope_cache[0] is not None:
            cos_sin = rope_cache[0].to(torch.float32).contiguous()
        else:
            cos_sin = prepare_cos_sin(freqs, freqs.shape[0], self.head_dim).to(torch.float32).contiguous()
        w_qkv, b_qkv = self._fused_qkv()
        ssq = torch.empty(B * L, 3 * dim // 256, device=x.device, dtype=torch.float32)
        qkv = ops.qkv_gemm(x.reshape(B * L, dim), w_qkv, b_qkv, ssq).view(B, L, 3 * dim)
        bf = torch.bfloat16
        q_rope = torch.empty(B, L, dim, device=x.device, dtype=bf)
        k_rope = torch.empty_like(q_rope)
        nwq = ops._bf16_vec(self.norm_q.weight, dim, "norm_q") if self.qk_norm else None
        nwk = ops._bf16_vec(self.norm_k.weight, dim, "norm_k") if self.qk_norm else None
        from . import _lib

        _lib.call("rola_b200_qk_norm_rope", ops._ptr(qkv), ops._ptr(qkv[..., dim:]), 3 * dim,
                  ops._ptr(ssq if self.qk_norm else None), ssq.shape[-1] if self.qk_norm else 0, None,
                  ops._ptr(nwq), ops._ptr(nwk), ops._ptr(cos_sin), None, None, B, L, H, 128, self.eps,
                  ops._ptr(q_rope), ops._ptr(k_rope), None, None, None, None, None, ops._stream())
        out = torch.empty(B, L, dim, device=x.device, dtype=bf)
        tok = (L * dim, 128, dim)  # (b, h, t) strides of the token-major [B, L, H*D] tensors
        ops.dense_attention_strided(q_rope, k_rope, qkv[..., 2 * dim:], B, L, H, tok, (L * 3 * dim, 128, 3 * dim),
                                    out, tok)
        w, b = self._o_weight()
        y = ops.qkv_gemm(out.reshape(B * L, dim), w, b).view(B, L, dim)
        return y.to(self.o.weight.dtype)
