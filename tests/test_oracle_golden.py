"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py`` from the
SparkDiffusion reference: its Triton kernels under the Triton interpreter in
fp32 (configuration C1) and its eager PyTorch pieces in bf16.  CPU only.
"""

import os

import pytest
import torch

from conftest import assert_bf16_close, assert_ulp_close, rel_err
from oracle import rola_oracle as orc
from sparkdiffusion_b200 import rope as host_rope
from sparkdiffusion_b200.workloads import C1, make_inputs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FP32_TOL = 1e-4  # fp32 on the CPU configuration within 1e-4 (relative to the RMS)


@pytest.fixture(scope="module")
def c1():
    g = torch.load(os.path.join(GOLDEN, "c1_fp32.pt"))
    wl = C1
    inp = make_inputs(wl, device="cpu")
    for k, cs in g["input_checksums"].items():
        got = inp[k].double()
        assert abs(float(got.sum()) - cs[0]) <= 1e-6 * max(1.0, abs(cs[0])), f"input {k} changed"
        assert abs(float(got.abs().sum()) - cs[1]) <= 1e-6 * cs[1], f"input {k} changed"
    freqs = orc.wan_rope_freqs(*wl.grid)
    cos_sin = orc.prepare_cos_sin(freqs, wl.L, 128)
    lr_cos, lr_sin, rope_dim = orc.prepare_lowrank_cos_sin(freqs, wl.L, wl.rank, torch.float32)
    res = orc.rola_attention_core(inp["q_raw"], inp["k_raw"], inp["v_raw"], inp["x"], cos_sin, lr_cos, lr_sin,
                                  rope_dim, inp["norm_wq"], inp["norm_wk"], inp["proj_q"], inp["proj_k"],
                                  inp["gate_w"], inp["gate_b"], wl.H, wl.blk, wl.blk, wl.topk)
    return g, res, freqs


def _sub(t4, g):
    return t4[:, g["heads"], :: g["token_stride"]].float()


def test_c1_freqs_checksum(c1):
    g, res, freqs = c1
    f = freqs.double()
    assert [float(f.sum()), float(f.abs().sum())] == pytest.approx(g["freqs_checksum"][:2], rel=1e-12)


def test_c1_lut_matches_reference(c1):
    g, res, _ = c1
    ours = res["lut"].reshape_as(g["lut_sorted"]).to(torch.int16)
    assert torch.equal(ours, g["lut_sorted"])


def test_c1_selection_margin(c1):
    # the reference's fp32 scores have no ties at the k-th boundary, so the set is well defined
    g, _, _ = c1
    s = g["scores"].sort(-1, descending=True).values
    k = C1.topk
    assert (s[..., k - 1] - s[..., k]).min() > 0


def test_c1_pool_and_scores(c1):
    g, res, _ = c1
    for name in ("pooled_q", "pooled_k"):
        mx, _ = rel_err(res[name], g[name])
        assert mx <= FP32_TOL, f"{name}: {mx:.2e}"
    mx, _ = rel_err(res["scores"].reshape_as(g["scores"]), g["scores"])
    assert mx <= FP32_TOL


@pytest.mark.parametrize("name", ["q_rope", "k_normed", "o_sparse", "o_lr", "out"])
def test_c1_outputs_fp32(c1, name):
    g, res, _ = c1
    B, H, L, D = C1.B, C1.H, C1.L, 128
    if name == "q_rope":
        ours = res["q_rope"].view(B, H, L, D)
    elif name == "k_normed":
        ours = res["k_normed"].permute(0, 2, 1, 3)
    elif name == "out":
        ours = res["out"].view(B, L, H, D).permute(0, 2, 1, 3)
    else:
        ours = res[name]
    mx, mn = rel_err(_sub(ours, g), g[name])
    assert mx <= FP32_TOL, f"{name}: max-abs/rms {mx:.2e} mean {mn:.2e}"


# ------------------------------------------------------------------ bf16 eager
@pytest.fixture(scope="module")
def eager():
    return torch.load(os.path.join(GOLDEN, "eager_bf16.pt"))


def test_rope_freqs_exact(eager):
    small = orc.wan_rope_freqs(3, 5, 7)
    assert torch.equal(small, eager["freqs_small"])
    assert torch.equal(host_rope.wan_rope_freqs(3, 5, 7), eager["freqs_small"])
    assert torch.equal(orc.wan_rope_freqs(21, 30, 52)[::997], eager["freqs_c2_rows"])
    assert torch.equal(host_rope.wan_rope_freqs(21, 45, 80)[::997], eager["freqs_c4_rows"])


def test_rmsnorm_and_rope_bf16(eager):
    x, w = eager["rms_in"], eager["rms_w"]
    B, L, dim = x.shape
    H = eager["config"]["H"]
    cos_sin = orc.prepare_cos_sin(eager["rope_freqs"], L, 128)
    q_rope, _, _, q_n, _ = orc.qkv_epilogue(x, x, x, cos_sin, w, w, H)
    assert_ulp_close(q_n.reshape(B, L, dim), eager["rms_out"], "WanRMSNorm", ulps=1)
    ref_rope = eager["rope_out"].permute(0, 2, 1, 3).reshape(B * H, L, 128)
    assert_ulp_close(q_rope, ref_rope, "rope_apply", ulps=1)


def test_lowrank_bf16(eager):
    e = eager
    R = e["config"]["R"]
    L = e["lr_q"].shape[1]
    cos, sin, rope_dim = orc.prepare_lowrank_cos_sin(e["rope_freqs"], L, R, torch.bfloat16)
    o_lr, *_ = orc.fused_lowrank(e["lr_q"], e["lr_k"], e["lr_v"], e["lr_pq"], e["lr_pk"], cos, sin, rope_dim)
    assert_ulp_close(o_lr, e["lr_out"], "fused_lowrank_ref")


def test_gate_bf16(eager):
    e = eager
    out = orc.fused_gate(e["g_olr"], e["g_os"], e["g_x"], e["g_w"], e["g_b"])
    assert_ulp_close(out, e["g_out"], "fused_gate_ref")
    assert_bf16_close(out, e["g_out"], "fused_gate_ref")


def test_select_topk_policy():
    s = torch.tensor([[1.0, 3.0, 3.0, 3.0, 0.5, 3.0]])
    # reference torch.topk may return {1,2,3,5} in any order for the tied 3s; the
    # build keeps the lowest indices among equal scores, ascending
    assert orc.select_topk(s, 3).tolist() == [[1, 2, 3]]
    assert orc.topk_count(0.1, 256) == 25 and orc.topk_count((26 + 0.5) / 256, 256) == 26
