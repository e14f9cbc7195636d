"""FP8 (e4m3) QKV projection, the reference's FP8 inference mode
(sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:270-285 with the row-wise
recipe of sparkdiffusion/ops/quantization/fp8_linear.py:45-61).

* The row quantization is bit-exact against the oracle's restatement (which a
  CPU test pins to the reference's own functions where they import).
* The tcgen05 e4m3 GEMM matches the oracle's torch._scaled_mm restatement to the
  bf16 rounding; the rest of the layer, from the GPU's projections, meets the
  stated bound.
* The drop-in layer takes q/k/v and o converted to the reference's FP8Linear
  buffers (weight_fp8, w_scale_t, bias) and runs them through these kernels.
"""

import os
import sys

import pytest
import torch

from conftest import assert_bf16_close, assert_ulp_close
from oracle import rola_oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rows(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g) * torch.exp(torch.randn(M, 1, generator=g) * 2)  # row scales over decades
    x[0, :5] = torch.tensor([1e-3, -3e-6, 0.0, 7.0, -7.5])
    return x.to(torch.bfloat16)


def test_oracle_fp8_recipe_pinned_to_reference():
    ref = None
    for p in (os.environ.get("SPARKDIFFUSION_REF", ""), os.path.join(ROOT, "baseline", "_ref"), "/root/reference"):
        if p and os.path.isdir(os.path.join(p, "sparkdiffusion", "ops", "quantization")):
            ref = p
            break
    if ref is None:
        pytest.skip("the SparkDiffusion reference is not importable here")
    sys.path.insert(0, ref)
    try:
        from sparkdiffusion.ops.quantization import fp8_linear as f8
    except Exception as e:  # pragma: no cover
        pytest.skip(f"reference import failed: {e}")
    x = _rows(64, 256, 1)
    q_ref, s_ref = f8.quantize_activation_rowwise(x)
    q, s = orc.quantize_rows_e4m3(x)
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8)) and torch.equal(s, s_ref.reshape(-1))
    w_ref, ws_ref = f8.quantize_weight_rowwise(x)
    assert torch.equal(w_ref.view(torch.uint8), q.view(torch.uint8)) and torch.equal(ws_ref.reshape(-1), s)


@pytest.mark.gpu
def test_quantize_rows_bit_exact():
    from sparkdiffusion_b200 import _lib, ops

    x = _rows(300, 640, 2)
    q, s = ops.quantize_rows_e4m3(x.cuda())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    q_ref, s_ref = orc.quantize_rows_e4m3(x)
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))


@pytest.mark.gpu
def test_fp8_gemm():
    from sparkdiffusion_b200 import _lib, ops

    M, K, N = 300, 512, 768
    x, w = _rows(M, K, 3), (_rows(N, K, 4).float() * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(5)) * 0.1).to(torch.bfloat16)
    xq, xs = ops.quantize_rows_e4m3(x.cuda())
    wq, ws = ops.prequantize_qkv_weight(w.cuda())
    ssq = torch.empty(M, N // 256, device="cuda", dtype=torch.float32)
    got = ops.qkv_gemm_fp8(xq, xs, wq, ws, b.cuda(), ssq)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = orc.scaled_mm_rowwise(xq.cpu(), xs.cpu(), wq.cpu(), ws.cpu(), b, out_dtype=torch.float32)
    # the rows span decades (max/rms ~260), so the bound is per element: one
    # bf16 rounding of the fp32 result (the accumulation order differs only in
    # fp32), and at most one element in 10^4 one step further
    assert_bf16_close(got.cpu(), ref, "fp8 gemm", ulp_floor=True)
    assert_ulp_close(got.cpu(), ref.to(torch.bfloat16), "fp8 gemm", ulps=1, max_frac=1e-4)
    r = got.cpu().float().view(M, N // 256, 256)
    torch.testing.assert_close(ssq.cpu(), r.pow(2).sum(-1), rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
def test_fp8_layer_forward():
    """The FP8 prologue inside the full forward; then everything after the GEMM
    against the oracle fed with the GPU's own projections."""
    from sparkdiffusion_b200 import _lib, ops
    from sparkdiffusion_b200.rope import prepare_cos_sin, prepare_lowrank_cos_sin, wan_rope_freqs
    from sparkdiffusion_b200.workloads import C3, make_inputs

    wl = C3.scaled(H=4, grid=(5, 12, 20))
    wl = wl.__class__(**{**wl.__dict__, "topk": 3})
    inp = make_inputs(wl, device="cpu")
    freqs = wan_rope_freqs(*wl.grid)
    cos_sin = prepare_cos_sin(freqs, wl.L, 128)
    lr_cos, lr_sin, rope_dim = prepare_lowrank_cos_sin(freqs, wl.L, wl.rank, torch.bfloat16)
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    wq, ws = ops.prequantize_qkv_weight(g["w_qkv"])
    out, ex = ops.rola_attention_core(g["x"], wq, None, cos_sin.cuda(), lr_cos.cuda(), lr_sin.cuda(), rope_dim,
                                      g["norm_wq"], g["norm_wk"], g["proj_q"], g["proj_k"], g["gate_w"],
                                      g["gate_b"], wl.H, wl.blk, wl.topk, keep=True, w_scale=ws)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    dim, B, L = wl.dim, wl.B, wl.L
    xq, xs = orc.quantize_rows_e4m3(inp["x"].reshape(B * L, dim))
    raw = orc.scaled_mm_rowwise(xq, xs, wq.cpu(), ws.cpu()).view(B, L, 3 * dim)
    qkv = ex["qkv"].cpu()
    assert_ulp_close(qkv, raw, "fp8 qkv")
    ref = orc.rola_attention_core(qkv[..., :dim], qkv[..., dim:2 * dim], qkv[..., 2 * dim:], inp["x"], cos_sin,
                                  lr_cos, lr_sin, rope_dim, inp["norm_wq"], inp["norm_wk"], inp["proj_q"],
                                  inp["proj_k"], inp["gate_w"], inp["gate_b"], wl.H, wl.blk, wl.blk, wl.topk,
                                  out_dtype=torch.float32)
    assert torch.equal(ex["lut"].cpu(), ref["lut"].reshape_as(ex["lut"].cpu()))
    assert_bf16_close(out.cpu(), ref["out"], "fp8 layer out (from the GPU's projections)")


class _FP8LinearLike(torch.nn.Module):
    """The buffers the reference's FP8Linear holds (fp8_linear.py:120-138)."""

    def __init__(self, lin: torch.nn.Linear):
        super().__init__()
        q, s = orc.quantize_rows_e4m3(lin.weight.detach().to(torch.bfloat16).cpu())
        self.register_buffer("weight_fp8", q.to(lin.weight.device))
        self.register_buffer("w_scale_t", s.reshape(1, -1).to(lin.weight.device))
        self.register_buffer("bias", lin.bias.detach().clone())
        self.out_features = lin.out_features


@pytest.mark.gpu
def test_layer_takes_reference_fp8_linears():
    from sparkdiffusion_b200 import _lib, ops
    from sparkdiffusion_b200.layer import WanSelfAttentionRoLaB200
    from sparkdiffusion_b200.rope import wan_rope_freqs

    torch.manual_seed(0)
    grid = (3, 10, 20)
    L = grid[0] * grid[1] * grid[2]
    layer = WanSelfAttentionRoLaB200(512, 4, True, 1e-6, rola_topk_ratio=2.5 / 5, rola_rank=64)
    layer = layer.to(torch.bfloat16).cuda().eval()
    x = torch.randn(1, L, 512, device="cuda").to(torch.bfloat16)
    freqs = wan_rope_freqs(*grid).cuda()
    with torch.no_grad():
        for n in ("q", "k", "v", "o"):
            setattr(layer, n, _FP8LinearLike(getattr(layer, n)))
        y = layer(x, torch.tensor([L]), freqs)
        core = layer.attention_core(x, freqs)
        xq, xs = ops.quantize_rows_e4m3(core.reshape(L, 512))
        ref = orc.scaled_mm_rowwise(xq.cpu(), xs.cpu(), layer.o.weight_fp8.cpu(), layer.o.w_scale_t.cpu(),
                                    layer.o.bias.cpu(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert y.shape == (1, L, 512)
    assert_bf16_close(y.float().cpu().view(L, 512), ref, "fp8 output projection")
