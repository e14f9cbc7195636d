"""GPU parity of the training path: the block-sparse attention's forward (with
the row log-sum-exp) and its backward kernels against the oracle's exact
gradient, and the layers' training forward/backward.

Tolerances (fp64 oracle on the same bf16 inputs).  Gradients of random
attention are heavy-tailed (the largest elements sit ~20x above the RMS), so
the per-element bound is the larger of a fraction of the RMS and a number of
bf16 steps of the element's own magnitude:

* against the oracle with the kernels' materialisation points (delta from the
  forward's bf16 output, whose P was rounded before P.V; P and dS rounded to
  bf16 before their MMAs): max(2e-2 of the RMS, 4 steps), mean-abs <= 1.5e-3
  of the RMS (measured on a B200: mean 1.05-1.16e-3, worst element 3.3
  steps or 2.1e-2 of the RMS; what remains are rounding flips of individual
  P / dS terms);
* against the exact gradient: max(2e-2 of the RMS, 4 steps), mean-abs <=
  3e-3 of the RMS (delta from the rounded forward output moves dS where
  dP - delta cancels: ~0.5 % at the worst element).  Where the algorithm
  itself sits further from the exact gradient -- rows whose softmax runs over
  two keys (a 2-row key block selected alone), where dS = P1 P2 (dP1 - dP2)
  cancels and the bf16 output's delta moves it by up to ~4 bounds -- the
  kernel may sit at most 1.25x as far from it as the staged oracle does;
* lse within 1e-3 absolute (log2 units);
* a whole layer's training step (fp32 parameters, the attention in bf16)
  against the same layer with the oracle's fp64 attention: max-abs <= 5e-2
  and mean-abs <= 5e-3 of the RMS of each gradient.
"""

import pytest
import torch

from conftest import assert_bf16_close, bf16_bound_ratio
from oracle import rola_oracle as orc
from sparkdiffusion_b200 import _lib, ops, train

pytestmark = pytest.mark.gpu

GRAD_MAX, GRAD_STEPS, GRAD_MEAN = 2e-2, 4.0, 3e-3
STAGED_MAX, STAGED_STEPS, STAGED_MEAN = 2e-2, 4.0, 1.5e-3
LAYER_MAX, LAYER_MEAN = 5e-2, 5e-3


def _lut(BH, NB, k, seed, skip=None):
    g = torch.Generator().manual_seed(seed)
    rows = []
    for _ in range(BH * NB):
        cand = torch.randperm(NB, generator=g)
        if skip is not None:
            cand = cand[cand != skip]
        rows.append(cand[:k].sort().values)
    return torch.stack(rows).reshape(BH, NB, k).int()


def _inputs(B, H, L, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, L, 128, generator=g).to(torch.bfloat16) for _ in range(4)]


def _paired(lut, blk, k):
    if blk == 128:
        return None
    BH, NB, _ = lut.shape
    out = torch.empty(BH, (NB + 1) // 2, 2 * k + 1, device="cuda", dtype=torch.int32)
    _lib.call("rola_b200_pair_blocks", ops._ptr(lut), BH, NB, k, ops._ptr(out), ops._stream())
    return out


def _run(q, k, v, do, lut, blk, topk):
    qg, kg, vg, dog = (t.cuda() for t in (q, k, v, do))
    lg = lut.cuda()
    paired = _paired(lg, blk, topk)
    o, lse = ops.sparse_attention_fwd_lse(qg, kg, vg, lg if blk == 128 else paired, blk, topk)
    dq, dk, dv = ops.sparse_attention_bwd(qg, kg, vg, o, dog, lg, paired, lse, blk, topk)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return o, lse, dq, dk, dv


CASES = {
    # block 128, ragged tail (1000 = 7*128 + 104), 2 heads
    "b128_tail": (1, 2, 1000, 128, 3),
    # block 64, ragged tail (1000 = 15*64 + 40), odd block count, 2 heads
    "b64_tail": (1, 2, 1000, 64, 5),
    # batch 2, no tail, block 128
    "b128_batch2": (2, 1, 768, 128, 2),
    # block 64, even block count
    "b64_even": (1, 1, 768, 64, 4),
    # short sequences: one full and one 36-row block of 64 (a single 128-row tile), top-1
    "b64_short": (1, 1, 100, 64, 1),
    # a 2-row last block of 128, top-1
    "b128_short": (1, 1, 130, 128, 1),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_sparse_attention_backward_matches_oracle(case):
    B, H, L, blk, topk = CASES[case]
    q, k, v, do = _inputs(B, H, L, seed=sorted(CASES).index(case))
    NB = (L + blk - 1) // blk
    lut = _lut(B * H, NB, topk, seed=7)
    o, lse, dq, dk, dv = _run(q, k, v, do, lut, blk, topk)
    ref_o, ref_lse = orc.block_sparse_attention(q, k, v, lut, blk, blk)
    exact = orc.block_sparse_attention_backward(q, k, v, lut, do, blk, blk)
    o_fwd = orc.sparse_attn_lut(q, k, v, lut, blk, blk)  # the forward's bf16 output, restated
    staged = orc.block_sparse_attention_backward(q, k, v, lut, do, blk, blk, round_dtype=torch.bfloat16,
                                                 o_fwd=o_fwd)
    assert_bf16_close(o, ref_o, f"{case} o", ulp_floor=True)
    lse_err = (lse[:, :L].cpu().double() - ref_lse.reshape(B * H, L)).abs().max().item()
    assert lse_err < 1e-3, f"{case} lse: max abs err {lse_err:.2e}"
    assert torch.isinf(lse[:, L:]).all() and (lse[:, L:] > 0).all()
    for name, got, ref, rs in zip(("dq", "dk", "dv"), (dq, dk, dv), exact, staged):
        assert_bf16_close(got, rs, f"{case} {name} (staged)", max_tol=STAGED_MAX, mean_tol=STAGED_MEAN,
                          ulp_floor=True, steps=STAGED_STEPS)
        algo_worst, _, algo_mean = bf16_bound_ratio(rs, ref, GRAD_MAX, GRAD_STEPS)
        worst, mx, mn = bf16_bound_ratio(got, ref, GRAD_MAX, GRAD_STEPS)
        assert worst <= max(1.0, 1.25 * algo_worst) and mn <= max(GRAD_MEAN, 1.25 * algo_mean), (
            f"{case} {name} (exact): max-abs/rms={mx:.3e} ({worst:.2f} of the per-element bound, the staged "
            f"oracle {algo_worst:.2f}), mean-abs/rms={mn:.3e} (staged oracle {algo_mean:.3e})")


def test_backward_deterministic_and_unselected_key_block_zero():
    B, H, L, blk, topk = 1, 2, 1000, 128, 3
    q, k, v, do = _inputs(B, H, L, seed=11)
    NB = (L + blk - 1) // blk
    lut = _lut(B * H, NB, topk, seed=5, skip=2)  # no query block selects key block 2
    _, _, dq1, dk1, dv1 = _run(q, k, v, do, lut, blk, topk)
    _, _, dq2, dk2, dv2 = _run(q, k, v, do, lut, blk, topk)
    assert torch.equal(dq1, dq2) and torch.equal(dk1, dk2) and torch.equal(dv1, dv2)
    assert (dk1[:, :, 256:384] == 0).all() and (dv1[:, :, 256:384] == 0).all()
    assert dk1[:, :, :256].abs().sum() > 0


def test_dense_attention_autograd_matches_sdpa():
    """train.dense_attention (every key block selected) against fp32 SDPA autograd."""
    B, H, L = 1, 2, 900
    q, k, v, do = (t.cuda() for t in _inputs(B, H, L, seed=3))
    qs, ks, vs = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    o = train.dense_attention(qs, ks, vs)
    o.backward(do)
    qr, kr, vr = (t.detach().float().clone().requires_grad_(True) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr)
    ref.backward(do.float())
    assert_bf16_close(o, ref, "dense o", ulp_floor=True)
    for name, got, r in (("dq", qs.grad, qr.grad), ("dk", ks.grad, kr.grad), ("dv", vs.grad, vr.grad)):
        assert_bf16_close(got, r, f"dense {name}", max_tol=GRAD_MAX, mean_tol=GRAD_MEAN, ulp_floor=True,
                          steps=GRAD_STEPS)


@pytest.mark.parametrize("blk", [128, 64])
def test_rola_layer_training_step(blk, monkeypatch):
    """One training step of the drop-in layer: loss.backward() through the
    B200 attention gives the same gradients as the same eager layer whose
    block-sparse attention is the oracle's fp64 autograd (same LUT)."""
    from sparkdiffusion_b200.layer import WanSelfAttentionRoLaB200
    from sparkdiffusion_b200.rope import wan_rope_freqs

    torch.manual_seed(0)
    dim, H, L = 256, 2, 1000
    layer = WanSelfAttentionRoLaB200(dim, H, rola_topk_ratio=0.3, rola_blkq=blk, rola_blkk=blk).cuda().train()
    with torch.no_grad():
        layer.gate_proj.weight.normal_(0, 0.05)
    freqs = wan_rope_freqs(4, 10, 25).cuda()
    x = torch.randn(1, L, dim, device="cuda")
    seen = {}
    real_select = train.select_blocks

    def recording_select(q, k, ratio, b):
        lut, topk, paired = real_select(q, k, ratio, b)
        seen["lut"] = lut.clone()
        return lut, topk, paired

    monkeypatch.setattr(train, "select_blocks", recording_select)
    x1 = x.clone().requires_grad_(True)
    y = layer(x1, None, freqs)
    y.float().pow(2).mean().backward()
    grads = {n: p.grad.clone() for n, p in layer.named_parameters() if p.grad is not None}
    gx = x1.grad.clone()
    assert _lib.device_status() == 0
    layer.zero_grad(set_to_none=True)

    # same layer, the attention on the oracle (on the GPU tensors, fp64 autograd)
    def oracle_sparse_dev(q, k, v, ratio, bq, bk):
        lut = seen["lut"].cpu()
        Lq = q.shape[2]
        mask = orc.block_mask(lut, Lq, bq, bk).reshape(q.shape[0], q.shape[1], Lq, Lq).to(q.device)
        s = (q.double() @ k.double().transpose(-1, -2)) * q.shape[-1] ** -0.5
        p = torch.softmax(s.masked_fill(~mask, float("-inf")), -1)
        return (p @ v.double()).to(torch.bfloat16).to(q.dtype)

    monkeypatch.setattr(train, "sparse_attention", oracle_sparse_dev)
    x2 = x.clone().requires_grad_(True)
    y_ref = layer(x2, None, freqs)
    y_ref.float().pow(2).mean().backward()
    assert_bf16_close(y, y_ref, f"blk{blk} layer output", max_tol=LAYER_MAX, mean_tol=LAYER_MEAN)
    assert_bf16_close(gx, x2.grad, f"blk{blk} dx", max_tol=LAYER_MAX, mean_tol=LAYER_MEAN)
    for n, g in grads.items():
        assert_bf16_close(g, dict(layer.named_parameters())[n].grad, f"blk{blk} d{n}", max_tol=LAYER_MAX,
                          mean_tol=LAYER_MEAN)


def test_backward_identities_at_full_c4_size():
    """Size-independent identities of the exact gradient at C4's full shape
    (L = 75600, 40 heads, top-18 of 591 blocks of 128), where the oracle is too
    slow: every query row's softmax weights sum to 1, so the sum of dV over all
    key rows equals the sum of dO over all query rows (per head and dimension);
    and sum_i q_i . dQ_i = sum_j k_j . dK_j = D^-1/2 sum_ij dS_ij (q_i . k_j), one
    side from each backward kernel.  Bounds: 1e-2 of the natural scale
    (sqrt of the sum of squares of the summed terms); bf16 rounding of the
    outputs and of P / dS stays orders of magnitude below it."""
    B, H, L, blk = 1, 40, 75600, 128
    g = torch.Generator(device="cuda").manual_seed(21)

    def mk():
        return torch.randn(B, L, H, 128, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)

    q, k, v, do = mk(), mk(), mk(), mk()
    lut, topk, _ = train.select_blocks(q, k, 18.5 / 591, blk)
    assert topk == 18
    o, lse = ops.sparse_attention_fwd_lse(q, k, v, lut, blk, topk)
    dq, dk, dv = ops.sparse_attention_bwd(q, k, v, o, do, lut, None, lse, blk, topk)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    for t in (dq, dk, dv):
        assert torch.isfinite(t).all()
    # (1) sum over key rows of dV == sum over query rows of dO, per (head, d)
    s_dv = dv.float().sum(dim=2)
    s_do = do.float().sum(dim=2)
    scale_v = dv.float().pow(2).sum(dim=2).sqrt()
    worst_v = ((s_dv - s_do).abs() / scale_v).max().item()
    assert worst_v <= 1e-2, f"sum dV vs sum dO: {worst_v:.3e} of the scale"
    # (2) sum_i q_i . dQ_i == sum_j k_j . dK_j, per head (the dq and dkdv kernels against each other)
    qdq = (q.float() * dq.float()).sum(-1)  # [B, H, L]
    kdk = (k.float() * dk.float()).sum(-1)
    lhs, rhs = qdq.sum(-1), kdk.sum(-1)
    scale_s = torch.maximum(qdq.pow(2).sum(-1).sqrt(), kdk.pow(2).sum(-1).sqrt())
    worst_s = ((lhs - rhs).abs() / scale_s).max().item()
    assert worst_s <= 1e-2, f"sum q.dQ vs sum k.dK: {worst_s:.3e} of the scale"
