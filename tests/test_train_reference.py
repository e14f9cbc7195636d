"""The layer's training route against the reference's own training forward (CPU).

The reference trains ``WanSelfAttentionRoLa`` through its non-fused forward
(sparkdiffusion/networks/wan_rola_attention.py:452-559): eager projections,
``WanRMSNorm``, ``rope_apply``, ``_lowrank_attn``, the gate and ``self.o``, with
the block-sparse attention from the external SLA package (``_sparse_attn``,
:293-327).  Here both layers get the same weights, and both sides' block-sparse
attention is replaced by the oracle (selection from its own q / k, then the
exact masked softmax attention), so everything else is compared: the output and
the gradients of x and of every parameter, in fp32 on the CPU.  The kernels
behind ``train.sparse_attention`` are checked on the GPU (tests/test_backward.py).

The reference is imported from ``SPARKDIFFUSION_REF``, ``baseline/_ref`` or the
read-only checkout; the tests skip where none of them exists (the GPU box).
"""

import sys

import pytest
import torch

from conftest import reference_path
from oracle import rola_oracle as orc
from sparkdiffusion_b200 import train
from sparkdiffusion_b200.layer import WanSelfAttentionRoLaB200
from sparkdiffusion_b200.rope import wan_rope_freqs


def _reference_path():
    return reference_path(allow_checkout=True)


@pytest.fixture(scope="module")
def ref_modules():
    path = _reference_path()
    if path is None:
        pytest.skip("the SparkDiffusion reference is not importable here")
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        import sparkdiffusion.networks.wan2pt1 as w
        import sparkdiffusion.networks.wan_rola_attention as r
    except Exception as e:  # pragma: no cover - a missing optional dependency of the reference
        pytest.skip(f"reference import failed: {e}")
    return w, r


def _oracle_sparse(q, k, v, ratio, blk):
    """Block-sparse attention of [B, H, L, D] with the oracle's own selection."""
    B, H, L, _ = q.shape
    NB = (L + blk - 1) // blk
    lut = orc.block_select(q.detach().float(), k.detach().float(), blk, blk, orc.topk_count(ratio, NB))[0]
    o, _ = orc.block_sparse_attention(q, k, v, lut, blk, blk, dtype=q.dtype)
    return o


@pytest.mark.parametrize("blk", [128, 64])
def test_training_route_matches_reference_training_forward(ref_modules, monkeypatch, blk):
    wan2pt1, rola = ref_modules
    # the reference's rope_apply falls back to its torch restatement without flash-attn's rotary kernel
    monkeypatch.setattr(wan2pt1, "flash_apply_rotary_emb", None)
    dim, H, L, ratio = 256, 2, 600, 0.3
    torch.manual_seed(0)
    ref = rola.WanSelfAttentionRoLa(dim, H, True, 1e-6, rola_topk_ratio=ratio, rola_rank=64, rola_blkq=blk,
                                    rola_blkk=blk).train()
    ours = WanSelfAttentionRoLaB200(dim, H, True, 1e-6, rola_topk_ratio=ratio, rola_rank=64, rola_blkq=blk,
                                    rola_blkk=blk).train()
    with torch.no_grad():
        ref.gate_proj.weight.normal_(0.0, 0.05)
        ref.norm_q.weight.uniform_(0.5, 1.5)
        ref.norm_k.weight.uniform_(0.5, 1.5)
    res = ours.load_state_dict(ref.state_dict(), strict=True)
    assert not res.missing_keys and not res.unexpected_keys

    monkeypatch.setattr(ref, "_sparse_attn", lambda q, k, v: _oracle_sparse(q, k, v, ratio, blk), raising=False)
    monkeypatch.setattr(train, "sparse_attention", lambda q, k, v, r, bq, bk: _oracle_sparse(q, k, v, r, bq))

    freqs = wan_rope_freqs(3, 10, 20)  # L = 600 (a ragged last block for both sizes)
    x = torch.randn(1, L, dim)
    x_ref = x.clone().requires_grad_(True)
    y_ref = ref(x_ref, torch.tensor([L]), freqs)
    x_our = x.clone().requires_grad_(True)
    y_our = ours.o(train.training_attention_core(ours, x_our, freqs))
    torch.testing.assert_close(y_our, y_ref, rtol=1e-5, atol=1e-5)

    w = torch.randn_like(y_ref)
    (y_ref * w).sum().backward()
    (y_our * w).sum().backward()
    torch.testing.assert_close(x_our.grad, x_ref.grad, rtol=1e-4, atol=1e-5)
    ref_params = dict(ref.named_parameters())
    for name, prm in ours.named_parameters():
        assert prm.grad is not None, name
        torch.testing.assert_close(prm.grad, ref_params[name].grad, rtol=1e-4, atol=1e-5, msg=lambda m: f"{name}: {m}")
