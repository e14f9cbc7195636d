"""The dense self-attention layer on the B200 kernels (``layer.WanSelfAttentionB200``,
the fused path of ``WanSelfAttention.forward``, sparkdiffusion/networks/wan2pt1.py:282-324):
QKV projection, qk-RMSNorm + RoPE, dense attention (the block-sparse kernel with
every key block kept) and the output projection.

Checked stage by stage against the oracle: the layer's projections to the bf16
ulp, attention from the GPU's roped q/k and v against the oracle's recurrence
(per-element bound: 2e-2 of the RMS or one bf16 step of the element), and the
output projection of the GPU's attention output.  A ragged tail block (600 tokens).
"""

import pytest
import torch

from conftest import assert_bf16_close, assert_ulp_close
from oracle import rola_oracle as orc
from sparkdiffusion_b200 import _lib, ops
from sparkdiffusion_b200.rope import prepare_cos_sin, wan_rope_freqs

pytestmark = pytest.mark.gpu


def test_dense_layer_matches_oracle_by_stage():
    from sparkdiffusion_b200.layer import WanSelfAttentionB200

    torch.manual_seed(3)
    grid = (3, 10, 20)
    L, dim, H = grid[0] * grid[1] * grid[2], 512, 4
    layer = WanSelfAttentionB200(dim, H, True, 1e-6)
    with torch.no_grad():
        layer.norm_q.weight.uniform_(0.5, 1.5)
        layer.norm_k.weight.uniform_(0.5, 1.5)
        for lin in (layer.q, layer.k, layer.v, layer.o):
            lin.bias.normal_(0.0, 0.02)
    layer = layer.to(torch.bfloat16).cuda().eval()
    x = (torch.randn(1, L, dim) * 0.5).to(torch.bfloat16)
    freqs = wan_rope_freqs(*grid)
    with torch.no_grad():
        y = layer(x.cuda(), torch.tensor([L]), freqs.cuda())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert y.shape == (1, L, dim) and y.dtype == torch.bfloat16

    # the same stages through the ops the layer runs, keeping the intermediates
    w = {n: getattr(layer, n) for n in ("q", "k", "v", "o")}
    cos_sin = prepare_cos_sin(freqs, L, 128)
    with torch.no_grad():
        q, k, v = ops.fused_qkv_gemm_rope(x.cuda(), w["q"], w["k"], w["v"], freqs.cuda(), layer.norm_q.weight,
                                          layer.norm_k.weight, H, 128)
        o = ops.dense_attention(q, k, v, num_heads=H)  # [B, H, L, D]
        o_tok = o.permute(0, 2, 1, 3).reshape(1, L, dim).contiguous()
        y2 = ops.qkv_gemm(o_tok.view(L, dim), w["o"].weight, w["o"].bias).view(1, L, dim)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), y2.cpu()), "the layer and its stages run the same kernels"

    # projections + norm + RoPE to the bf16 ulp
    cpu = {n: (m.weight.detach().cpu(), m.bias.detach().cpu()) for n, m in w.items()}
    raw = [orc.qkv_linear(x, *cpu[n]) for n in ("q", "k", "v")]
    q_rope, k_rope, v_ref, _, _ = orc.qkv_epilogue(*raw, cos_sin, layer.norm_q.weight.detach().cpu(),
                                                   layer.norm_k.weight.detach().cpu(), H, 1e-6)
    assert_ulp_close(q.cpu().view(1, H, L, 128), q_rope.reshape(1, H, L, 128), "q_rope")
    assert_ulp_close(k.cpu().view(1, H, L, 128), k_rope.reshape(1, H, L, 128), "k_rope")
    # dense attention from the GPU's own q/k/v
    NB = (L + 127) // 128
    lut = torch.arange(NB, dtype=torch.int32).expand(H, NB, NB).reshape(1, H, NB, NB)
    o_ref = orc.sparse_attn_lut(q.cpu().view(1, H, L, 128), k.cpu().view(1, H, L, 128),
                                v.cpu().view(1, H, L, 128), lut, 128, 128, out_dtype=torch.float32)
    assert_bf16_close(o.cpu(), o_ref, "dense attention", ulp_floor=True)
    # output projection of the GPU's attention output
    y_ref = orc.qkv_linear(o_tok.cpu(), *cpu["o"], out_dtype=torch.float32)
    assert_bf16_close(y.cpu().view(L, dim).float(), y_ref.view(L, dim), "output projection", ulp_floor=True)
