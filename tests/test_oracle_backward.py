"""CPU pin of the oracle's training section: the written-out gradient of the
block-sparse attention equals torch.autograd of the forward restatement, and
the forward restatement with a LUT equals the reference-pinned online-softmax
restatement ``sparse_attn_lut`` (fp32, no bf16 rounding)."""

import math

import torch

from conftest import bf16_bound_ratio
from oracle import rola_oracle as orc


def _lut(BH, NB, k, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randperm(NB, generator=g)[:k].sort().values for _ in range(BH * NB)]).reshape(
        BH, NB, k).int()


def test_backward_formula_matches_autograd():
    torch.manual_seed(0)
    for blk, L, k in ((128, 600, 2), (64, 300, 3)):
        B, H, D = 1, 2, 128
        q, k4, v = (torch.randn(B, H, L, D, dtype=torch.float64, requires_grad=True) for _ in range(3))
        lut = _lut(B * H, (L + blk - 1) // blk, k, seed=blk)
        o, _ = orc.block_sparse_attention(q, k4, v, lut, blk, blk)
        do = torch.randn_like(o)
        o.backward(do)
        dq, dk, dv = orc.block_sparse_attention_backward(q.detach(), k4.detach(), v.detach(), lut, do, blk, blk)
        for got, ref in ((dq, q.grad), (dk, k4.grad), (dv, v.grad)):
            assert torch.allclose(got, ref, rtol=1e-10, atol=1e-10)


def test_forward_matches_online_softmax_restatement():
    torch.manual_seed(1)
    B, H, L, D, blk = 1, 2, 600, 128, 128
    q, k, v = (torch.randn(B, H, L, D) for _ in range(3))
    lut = _lut(B * H, (L + blk - 1) // blk, 2, seed=3)
    o, lse2 = orc.block_sparse_attention(q, k, v, lut, blk, blk, dtype=torch.float64)
    ref = orc.sparse_attn_lut(q, k, v, lut, blk, blk, out_dtype=torch.float32)
    assert (o.float() - ref).abs().max().item() < 1e-4
    # lse2 is log2 of the softmax denominator in units of D^-1/2 log2(e)
    s = (q.double() @ k.double().transpose(-1, -2)) * D ** -0.5
    mask = orc.block_mask(lut, L, blk, blk).reshape(B, H, L, L)
    den = torch.where(mask, s.exp(), torch.zeros_like(s)).sum(-1)
    assert torch.allclose(lse2, den.log() / math.log(2), rtol=1e-9, atol=1e-9)


def test_staged_rounding_distance_on_a_two_key_softmax():
    """The bf16 materialisation points of a flash-style backward (delta from the
    rounded forward output; P and dS rounded before their MMAs) move the
    gradient furthest where a softmax runs over two keys: a 2-row key block
    (L = 130, block 128) selected alone by the other query block.  There
    dS = P1 P2 (dP1 - dP2) cancels.  This pins how far the staged algorithm
    itself sits from the exact gradient, the distance that the GPU test's
    exact-gradient check scales its bound by."""
    g = torch.Generator().manual_seed(0)
    L, blk = 130, 128
    q, k, v, do = (torch.randn(1, 1, L, 128, generator=g).to(torch.bfloat16) for _ in range(4))
    lut = torch.tensor([[[1], [0]]], dtype=torch.int32)  # each query block selects the other key block
    exact = orc.block_sparse_attention_backward(q, k, v, lut, do, blk, blk)
    o_fwd = orc.sparse_attn_lut(q, k, v, lut, blk, blk)
    staged = orc.block_sparse_attention_backward(q, k, v, lut, do, blk, blk, round_dtype=torch.bfloat16, o_fwd=o_fwd)
    worst = {n: bf16_bound_ratio(s, e, 2e-2, 4.0) for n, s, e in zip(("dq", "dk", "dv"), staged, exact)}
    # beyond one bound somewhere (the reason for the relative check), within a few everywhere
    assert max(w[0] for w in worst.values()) > 1.0, worst
    for name, (w, _, mean) in worst.items():
        assert w < 8.0 and mean < 5e-3, (name, w, mean)
