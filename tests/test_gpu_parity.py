"""GPU parity of every stage of the B200 RoLa forward against the CPU oracle.

Selection (pooled means, smooth-K centre, scores, LUT) is checked bit for bit
against the oracle run on the bf16 q/k the GPU produced; floating-point
outputs are checked against the bf16 tolerance (max-abs <= 2e-2 and
mean-abs <= 2e-3 of the output RMS).  Shapes are reduced (2-4 heads, a few
hundred to ~1.2k tokens, ragged tail blocks) so the oracle runs in seconds.
"""

import pytest
import torch

from conftest import assert_bf16_close, assert_ulp_close
from oracle import rola_oracle as orc
from sparkdiffusion_b200 import _lib, ops
from sparkdiffusion_b200.rope import prepare_cos_sin, prepare_lowrank_cos_sin, wan_rope_freqs
from sparkdiffusion_b200.workloads import C2, C3, make_inputs

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _setup(wl):
    inp = make_inputs(wl, device="cpu")
    freqs = wan_rope_freqs(*wl.grid)
    cos_sin = prepare_cos_sin(freqs, wl.L, 128)
    lr_cos, lr_sin, rope_dim = prepare_lowrank_cos_sin(freqs, wl.L, wl.rank, torch.bfloat16)
    return inp, cos_sin, lr_cos, lr_sin, rope_dim


def _cuda(d):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def _run_gpu_from_qkv(wl, inp, cos_sin, lr_cos, lr_sin, rope_dim, lut=None):
    g = _cuda(inp)
    out, ex = ops.rola_attention_from_qkv(
        g["q_raw"], g["k_raw"], g["v_raw"], g["x"], cos_sin.cuda(), lr_cos.cuda(), lr_sin.cuda(), rope_dim,
        g["norm_wq"], g["norm_wk"], g["proj_q"], g["proj_k"], g["gate_w"], g["gate_b"], wl.H, wl.blk, wl.topk,
        keep=True, lut=lut)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return out, ex


CASES = {
    # ragged tail (600 = 4*128 + 88), 2 heads, qkv input mode
    "qkv_tail": C2.scaled(H=2, grid=(3, 10, 20)),
    # no tail, 3 heads, batch 2
    "qkv_b2": C2.scaled(H=3, grid=(2, 16, 32), B=2),
}
for _k, _wl in list(CASES.items()):
    CASES[_k] = _wl.__class__(**{**_wl.__dict__, "topk": 2 if _k == "qkv_tail" else 3})


@pytest.fixture(scope="module", params=sorted(CASES))
def qkv_case(request):
    wl = CASES[request.param]
    inp, cos_sin, lr_cos, lr_sin, rope_dim = _setup(wl)
    out, ex = _run_gpu_from_qkv(wl, inp, cos_sin, lr_cos, lr_sin, rope_dim)
    return wl, inp, cos_sin, lr_cos, lr_sin, rope_dim, out, ex


def _heads(t, wl):
    """token-major [B, L, H*D] -> [B, H, L, D]"""
    return t.float().cpu().view(wl.B, wl.L, wl.H, 128).permute(0, 2, 1, 3).to(torch.bfloat16)


def test_prologue_epilogue(qkv_case):
    wl, inp, cos_sin, *_, out, ex = qkv_case
    q_rope, k_rope, v, q_n, k_n = orc.qkv_epilogue(inp["q_raw"], inp["k_raw"], inp["v_raw"], cos_sin,
                                                   inp["norm_wq"], inp["norm_wk"], wl.H)
    assert_ulp_close(_heads(ex["q_rope"], wl), q_rope.view(wl.B, wl.H, wl.L, 128), "q_rope")
    assert_ulp_close(_heads(ex["k_rope"], wl), k_rope.view(wl.B, wl.H, wl.L, 128), "k_rope")
    assert_ulp_close(ex["q_normed"].cpu().view(wl.B, wl.L, wl.H, 128), q_n, "q_normed")
    assert_ulp_close(ex["k_normed"].cpu().view(wl.B, wl.L, wl.H, 128), k_n, "k_normed")


def test_pooling_bit_exact(qkv_case):
    wl, *_, out, ex = qkv_case
    q4, k4 = _heads(ex["q_rope"], wl), _heads(ex["k_rope"], wl)
    assert torch.equal(ex["pooled_q"].cpu(), orc.mean_pool(q4, wl.blk))
    ks = orc.block_sums(k4, wl.blk)  # [B, H, NB, D]
    assert torch.equal(ex["ksum"].cpu(), ks.permute(0, 2, 1, 3).reshape(wl.B, wl.NB, wl.dim))
    c = orc.smooth_k_center(k4, wl.blk)
    assert torch.equal(ex["center"].cpu(), c)
    assert torch.equal(ex["pooled_k"].cpu(), orc.mean_pool(k4, wl.blk, center=c))


def test_selection_bit_exact(qkv_case):
    wl, *_, out, ex = qkv_case
    s = orc.block_scores(ex["pooled_q"].cpu(), ex["pooled_k"].cpu()).reshape(wl.B * wl.H, wl.NB, wl.NB)
    if ex["scores"] is not None:  # only materialised by the two-kernel path (NB > 768)
        assert torch.equal(ex["scores"].cpu(), s)
    assert torch.equal(ex["lut"].cpu(), orc.select_topk(s, wl.topk))
    # end to end from the GPU's roped q/k
    lut, *_ = orc.block_select(_heads(ex["q_rope"], wl), _heads(ex["k_rope"], wl), wl.blk, wl.blk, wl.topk)
    assert torch.equal(ex["lut"].cpu(), lut.reshape(wl.B * wl.H, wl.NB, wl.topk))


def test_lowrank(qkv_case):
    wl, inp, cos_sin, lr_cos, lr_sin, rope_dim, out, ex = qkv_case
    qn = ex["q_normed"].cpu().view(wl.B, wl.L, wl.H, 128)
    kn = ex["k_normed"].cpu().view(wl.B, wl.L, wl.H, 128)
    q_lr = orc.proj_silu_rope(qn, inp["proj_q"], lr_cos, lr_sin, rope_dim)  # [BH, L, R]
    got = ex["q_lr"].cpu().view(wl.B, wl.L, wl.H, wl.rank).permute(0, 2, 1, 3).reshape(wl.B * wl.H, wl.L, wl.rank)
    assert_ulp_close(got, q_lr, "q_lr")
    k_lr = orc.proj_silu_rope(kn, inp["proj_k"], lr_cos, lr_sin, rope_dim)
    v4 = inp["v_raw"].view(wl.B, wl.L, wl.H, 128).permute(0, 2, 1, 3).reshape(wl.B * wl.H, wl.L, 128)
    C = orc.lowrank_kv(k_lr, v4, wl.B, wl.H)
    assert_ulp_close(ex["C"].cpu().view_as(C), C, "C")
    assert torch.equal(ex["Ct"].cpu(), ex["C"].cpu().transpose(-1, -2))


def test_sparse_attention_lut_injected(qkv_case):
    wl, inp, *_, out, ex = qkv_case
    q4, k4 = _heads(ex["q_rope"], wl), _heads(ex["k_rope"], wl)
    v4 = inp["v_raw"].view(wl.B, wl.L, wl.H, 128).permute(0, 2, 1, 3)
    o_ref = orc.sparse_attn_lut(q4, k4, v4, ex["lut"].cpu(), wl.blk, wl.blk, out_dtype=torch.float32)
    assert_bf16_close(_heads(ex["o_sparse"], wl), o_ref, "o_sparse")


def test_gate_epilogue_stage(qkv_case):
    """The fused epilogue (o_lr = q_lr C, RMS fusion, gate) on the GPU's own
    o_sparse, q_lr and C, against the oracle with the final rounding removed."""
    wl, inp, *_, out, ex = qkv_case
    BH, R = wl.B * wl.H, wl.rank
    q_lr = ex["q_lr"].cpu().view(wl.B, wl.L, wl.H, R).permute(0, 2, 1, 3).float()
    o_lr = torch.matmul(q_lr, ex["C"].cpu().float().view(wl.B, wl.H, R, 128)).to(torch.bfloat16)
    ref = orc.fused_gate(o_lr, _heads(ex["o_sparse"], wl), inp["x"], inp["gate_w"], inp["gate_b"],
                         out_dtype=torch.float32)
    assert_bf16_close(out.cpu(), ref, "out (stage)")


def test_full_output(qkv_case):
    wl, inp, cos_sin, lr_cos, lr_sin, rope_dim, out, ex = qkv_case
    ref = orc.rola_attention_core(inp["q_raw"], inp["k_raw"], inp["v_raw"], inp["x"], cos_sin, lr_cos, lr_sin,
                                  rope_dim, inp["norm_wq"], inp["norm_wk"], inp["proj_q"], inp["proj_k"],
                                  inp["gate_w"], inp["gate_b"], wl.H, wl.blk, wl.blk, wl.topk,
                                  out_dtype=torch.float32)
    assert torch.equal(ex["lut"].cpu(), ref["lut"].reshape_as(ex["lut"].cpu()))
    assert_bf16_close(out.cpu(), ref["out"], "out")


def test_norm_pack_for_ulysses():
    """The sequence-parallel pre-exchange pass: q_normed, k_normed, v and the
    gate written into per-destination send blocks [B][p][L][Hl*D] / [B][p][L][Hl]."""
    wl = C3.scaled(H=4, grid=(2, 8, 20), B=2)  # L = 320
    B, L, H, dim, p = wl.B, wl.L, wl.H, wl.dim, 2
    Hl = H // p
    inp = make_inputs(wl, device="cpu")
    g = _cuda(inp)
    ssq = torch.empty(B * L, 3 * dim // 256, device="cuda", dtype=torch.float32)
    qkv = ops.qkv_gemm(g["x"].reshape(B * L, dim), g["w_qkv"], None, ssq)
    send = [torch.empty(B, p, L, Hl * 128, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    g_send = torch.empty(B, p, L, Hl, device="cuda", dtype=torch.bfloat16)
    gb = inp["gate_b"].reshape(-1).to(torch.bfloat16).cuda()
    _lib.call("rola_b200_qk_norm_pack", qkv.data_ptr(), qkv[:, dim:].data_ptr(), qkv[:, 2 * dim:].data_ptr(),
              3 * dim, ssq.data_ptr(), ssq.shape[1], g["x"].data_ptr(), g["norm_wq"].data_ptr(),
              g["norm_wk"].data_ptr(), g["gate_w"].reshape(-1).data_ptr(), gb.data_ptr(), B, L, H, Hl, 1e-6,
              send[0].data_ptr(), send[1].data_ptr(), send[2].data_ptr(), g_send.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    raw = qkv.cpu().view(B, L, 3 * dim)
    cos_sin = prepare_cos_sin(wan_rope_freqs(*wl.grid), L, 128)
    _, _, _, q_n, k_n = orc.qkv_epilogue(raw[..., :dim], raw[..., dim:2 * dim], raw[..., 2 * dim:], cos_sin,
                                         inp["norm_wq"], inp["norm_wk"], H)

    def unpack(t):  # [B, p, L, Hl*X] -> [B, L, H*X]
        return t.cpu().permute(0, 2, 1, 3).reshape(B, L, -1)

    assert_ulp_close(unpack(send[0]), q_n.reshape(B, L, dim), "q_normed send")
    assert_ulp_close(unpack(send[1]), k_n.reshape(B, L, dim), "k_normed send")
    assert torch.equal(unpack(send[2]), raw[..., 2 * dim:])
    gate = orc.gate_values(inp["x"], inp["gate_w"], inp["gate_b"], H)
    assert_ulp_close(unpack(g_send), gate, "gate send")


def test_gemm_parity():
    torch.manual_seed(0)
    M, K, N = 300, 512, 768
    x = torch.randn(M, K).to(torch.bfloat16)
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N) * 0.1).to(torch.bfloat16)
    got = ops.qkv_gemm(x.cuda(), w.cuda(), b.cuda())
    torch.cuda.synchronize()
    ref = orc.qkv_linear(x, w, b, out_dtype=torch.float32)
    assert_bf16_close(got.cpu(), ref, "gemm")


def test_full_layer_from_x():
    wl = C3.scaled(H=4, grid=(5, 12, 20))
    wl = wl.__class__(**{**wl.__dict__, "topk": 3})
    inp, cos_sin, lr_cos, lr_sin, rope_dim = _setup(wl)
    g = _cuda(inp)
    out, ex = ops.rola_attention_core(g["x"], g["w_qkv"], None, cos_sin.cuda(), lr_cos.cuda(), lr_sin.cuda(),
                                      rope_dim, g["norm_wq"], g["norm_wk"], g["proj_q"], g["proj_k"], g["gate_w"],
                                      g["gate_b"], wl.H, wl.blk, wl.topk, keep=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    dim = wl.dim
    wq, wk, wv = inp["w_qkv"][:dim], inp["w_qkv"][dim:2 * dim], inp["w_qkv"][2 * dim:]
    ref = orc.rola_attention_forward(inp["x"], wq, None, wk, None, wv, None, cos_sin=cos_sin, lr_cos=lr_cos,
                                     lr_sin=lr_sin, rope_dim=rope_dim, norm_wq=inp["norm_wq"],
                                     norm_wk=inp["norm_wk"], proj_q=inp["proj_q"], proj_k=inp["proj_k"],
                                     gate_w=inp["gate_w"], gate_b=inp["gate_b"], num_heads=wl.H, blkq=wl.blk,
                                     blkk=wl.blk, topk=wl.topk)
    qkv = ex["qkv"].cpu()
    # the GEMM: every q/k/v element within the bf16 rounding of the oracle's fp32-accumulated product
    assert_ulp_close(qkv[..., :dim], ref["q_raw"], "q_raw")
    assert_ulp_close(qkv[..., dim:2 * dim], ref["k_raw"], "k_raw")
    assert_ulp_close(qkv[..., 2 * dim:], ref["v_raw"], "v_raw")
    # selection from the GPU's own q/k is bit exact
    lut, *_ = orc.block_select(_heads(ex["q_rope"], wl), _heads(ex["k_rope"], wl), wl.blk, wl.blk, wl.topk)
    assert torch.equal(ex["lut"].cpu(), lut.reshape_as(ex["lut"].cpu()))
    # everything after the GEMM, from the GPU's own projections (GEMM outputs that
    # differ from the oracle's by one bf16 rounding step would otherwise propagate
    # through the norm, the attention and the gate): the stated bound
    ref2 = orc.rola_attention_core(qkv[..., :dim], qkv[..., dim:2 * dim], qkv[..., 2 * dim:], inp["x"], cos_sin,
                                   lr_cos, lr_sin, rope_dim, inp["norm_wq"], inp["norm_wk"], inp["proj_q"],
                                   inp["proj_k"], inp["gate_w"], inp["gate_b"], wl.H, wl.blk, wl.blk, wl.topk,
                                   out_dtype=torch.float32)
    assert torch.equal(ex["lut"].cpu(), ref2["lut"].reshape_as(ex["lut"].cpu()))
    assert_bf16_close(out.cpu(), ref2["out"], "out (from the GPU's projections)")


def test_topk_ties_lower_index():
    # rows with many exact ties: the kept set must prefer lower indices
    rows, nb, k = 6, 40, 7
    s = torch.zeros(rows, nb)
    s[0] = 1.0                       # all equal -> 0..6
    s[1, ::2] = 3.0                  # ties among evens -> 0,2,...,12
    s[2] = torch.arange(nb).float() % 5  # value 4 at 4,9,14,... -> those first
    s[3, 35:] = 2.0
    s[4] = -torch.arange(nb).float()
    s[5, 10] = float("inf")
    scores = s.cuda()
    got = _topk_only(scores, k)
    ref = orc.select_topk(s, k)
    assert torch.equal(got.cpu(), ref)


def test_select_two_kernel_path_large_nb():
    """More than 768 key blocks: scores go through global memory (scores_kernel +
    topk_kernel); LUT and scores bit-exact, ties included."""
    g = torch.Generator().manual_seed(5)
    B, H, NBq, NBk, k = 1, 2, 40, 900, 9
    pq = torch.randn(B, H, NBq, 128, generator=g).to(torch.bfloat16)
    pk = torch.randn(B, H, NBk, 128, generator=g).to(torch.bfloat16)
    pk[:, :, 500:520] = pk[:, :, 10:11]  # 21 identical key blocks -> exact score ties
    lut = ops.block_select(pq.cuda(), pk.cuda(), k)
    torch.cuda.synchronize()
    s = orc.block_scores(pq, pk).reshape(B * H, NBq, NBk)
    assert torch.equal(lut.cpu(), orc.select_topk(s, k))


def _topk_only(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Run block_select with pooled vectors chosen so the fp32 scores equal ``scores`` exactly.

    pooled_q[m] = e_0 (unit vector), pooled_k[j] = scores[j] * e_0 in bf16: exact when
    the scores are bf16-representable (the test values are)."""
    rows, nb = scores.shape
    pq = torch.zeros(1, rows, 1, 128, dtype=torch.bfloat16, device="cuda")
    pq[..., 0] = 1.0
    pk = torch.zeros(1, rows, nb, 128, dtype=torch.bfloat16, device="cuda")
    pk[0, :, :, 0] = scores.to(torch.bfloat16)
    return ops.block_select(pq, pk, k).view(rows, k)


def test_reference_api_sparse_attn():
    # reference-named API: q, k, v [B*H, L, D] head-major in, [B, H, L, D] out
    wl = C2.scaled(H=2, grid=(2, 12, 20))
    B, H, L = wl.B, wl.H, wl.L
    torch.manual_seed(3)
    q = torch.randn(B * H, L, 128).to(torch.bfloat16)
    k = torch.randn(B * H, L, 128).to(torch.bfloat16)
    v = torch.randn(B * H, L, 128).to(torch.bfloat16)
    nb = wl.NB
    topk = 2
    o = ops.fused_sparse_attn(q.cuda(), k.cuda(), v.cuda(), topk_ratio=(topk + 0.5) / nb, blkq=128, blkk=128,
                              num_heads=H)
    torch.cuda.synchronize()
    q4, k4, v4 = (t.view(B, H, L, 128) for t in (q, k, v))
    lut, *_ = orc.block_select(q4, k4, 128, 128, topk)
    ref = orc.sparse_attn_lut(q4, k4, v4, lut, 128, 128, out_dtype=torch.float32)
    assert_bf16_close(o.cpu(), ref, "fused_sparse_attn")
    with pytest.raises(ValueError):
        ops.fused_sparse_attn(q.cuda(), k.cuda(), v.cuda(), num_heads=3)


def test_host_pipeline_matches_device_forward():
    """rola_b200_pipeline_forward (pinned host in/out, overlapped steps) gives
    exactly the device-buffer forward's output for every step."""
    wl = C3.scaled(H=4, grid=(3, 10, 20))
    wl = wl.__class__(**{**wl.__dict__, "topk": 3})
    inp, cos_sin, lr_cos, lr_sin, rope_dim = _setup(wl)
    g = _cuda(inp)
    common = (cos_sin.cuda(), lr_cos.cuda(), lr_sin.cuda(), rope_dim, g["norm_wq"], g["norm_wk"], g["proj_q"],
              g["proj_k"], g["gate_w"], g["gate_b"])
    xs = [g["x"] * s for s in (1.0, 0.5, -1.0, 2.0)]
    refs = [ops.rola_forward_capi(x, g["w_qkv"], None, *common, wl.H, wl.topk).cpu() for x in xs]
    pipe = ops.ForwardPipeline(xs[0].numel() * 2, xs[0].numel() * 2)
    hosts = [x.cpu().pin_memory() for x in xs]
    outs = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for x in xs]
    for xh, oh in zip(hosts, outs):
        pipe.forward(xh, oh, g["w_qkv"], None, *common, wl.H, wl.topk)
    pipe.wait()
    torch.cuda.synchronize()
    pipe.close()
    assert _lib.device_status() == 0
    for i, (o, r) in enumerate(zip(outs, refs)):
        assert torch.equal(o, r), f"step {i} differs"


def test_layer_forward_with_output_projection():
    """The drop-in layer: attention core followed by self.o on the tcgen05 GEMM
    equals the core output projected in fp32 (bf16 tolerance)."""
    from sparkdiffusion_b200.layer import WanSelfAttentionRoLaB200

    torch.manual_seed(0)
    grid = (3, 10, 20)
    L = grid[0] * grid[1] * grid[2]
    layer = WanSelfAttentionRoLaB200(512, 4, True, 1e-6, rola_topk_ratio=2.5 / 5, rola_rank=64).cuda().eval()
    x = torch.randn(1, L, 512, device="cuda").to(torch.bfloat16)
    freqs = wan_rope_freqs(*grid).cuda()
    with torch.no_grad():
        y = layer(x, torch.tensor([L]), freqs)
        core = layer.attention_core(x, freqs)
        ref = torch.nn.functional.linear(core.float(), layer.o.weight.float(), layer.o.bias.float())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert y.shape == (1, L, 512) and y.dtype == layer.o.weight.dtype
    assert_bf16_close(y.float().cpu(), ref.cpu(), "layer output projection")


def test_gate_from_hidden_states_in_epilogue(qkv_case):
    """The attention epilogue's other gate source: the gate computed from the
    hidden-state tile x (rola_b200_sparse_attn with x) instead of precomputed
    gate values; same output within the bf16 tolerance (the gate's dot product
    is summed in another order)."""
    wl, inp, *_, out, ex = qkv_case
    g = _cuda(inp)
    lr_cos, lr_sin, rope_dim = qkv_case[3], qkv_case[4], qkv_case[5]
    got = ops.head_local_attention(ex["q_rope"], ex["k_rope"], ex["q_normed"], ex["k_normed"], ex["v"], None,
                                   ex["pooled_q"], ex["ksum"], lr_cos.cuda(), lr_sin.cuda(), rope_dim, g["proj_q"],
                                   g["proj_k"], wl.H, wl.blk, wl.topk, lut=ex["lut"], x=g["x"].contiguous(),
                                   gate_w=g["gate_w"], gate_b=g["gate_b"])
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert_bf16_close(got.float().cpu(), out.float().cpu(), "gate from x vs gate values")


def test_dense_attention_full_lut():
    """Dense attention (every key block kept) against the oracle's recurrence
    with the full LUT; ragged tail block."""
    B, H, L = 1, 2, 600
    torch.manual_seed(5)
    q = torch.randn(B * H, L, 128).to(torch.bfloat16)
    k = torch.randn(B * H, L, 128).to(torch.bfloat16)
    v = torch.randn(B * H, L, 128).to(torch.bfloat16)
    o = ops.dense_attention(q.cuda(), k.cuda(), v.cuda(), num_heads=H)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    NB = (L + 127) // 128
    lut = torch.arange(NB, dtype=torch.int32).expand(B * H, NB, NB).reshape(B, H, NB, NB)
    q4, k4, v4 = (t.view(B, H, L, 128) for t in (q, k, v))
    ref = orc.sparse_attn_lut(q4, k4, v4, lut, 128, 128, out_dtype=torch.float32)
    # Every query averages all 600 values, so the output's largest elements sit
    # ~4.5x above its RMS and one bf16 rounding step of them is already ~2e-2 of
    # the RMS: the bound allows one step per element (ulp_floor), and element by
    # element against the oracle rounded like the kernel's output at most 0.1 %
    # of the elements may differ by more than one step.
    assert_ulp_close(o.cpu(), ref.to(torch.bfloat16), "dense attention", ulps=1, max_frac=1e-3)
    assert_bf16_close(o.cpu(), ref, "dense attention", ulp_floor=True)

