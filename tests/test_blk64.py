"""Block size 64, the reference's inference default (rola_blkq = rola_blkk = 64,
sparkdiffusion/configs/defaults/net.py:52-59, wan2pt1_t2v_distilled_infer.py:66,72).

Selection runs on 64-token blocks; the attention kernel's 128-row query tiles
hold two 64-token query blocks and attend to the union of their kept key
blocks (rola_b200_pair_blocks), each row masked to its own block's.  Checked
against the oracle run with blk 64: LUT bit for bit, the pairing table against
a direct restatement, o_sparse and the gated output within the bf16 tolerance.
Shapes: C1's (H = 12, grid 6x16x16 -> L = 1536, top-6; rank 64, the only rank
of this build) and a ragged odd case (L = 1200: 19 blocks, the last query tile
half empty, a 48-token tail block).
"""

import dataclasses

import pytest
import torch

from conftest import assert_bf16_close, assert_ulp_close
from oracle import rola_oracle as orc
from sparkdiffusion_b200 import _lib, ops
from sparkdiffusion_b200.rope import prepare_cos_sin, prepare_lowrank_cos_sin, wan_rope_freqs
from sparkdiffusion_b200.workloads import C1, C2, make_inputs

pytestmark = pytest.mark.gpu

CASES = {
    "c1_shape": dataclasses.replace(C2, H=12, grid=C1.grid, blk=64, topk=6),
    "odd_tail": dataclasses.replace(C2, H=3, grid=(3, 16, 25), blk=64, topk=5),
}


def _heads(t, wl):
    return t.float().cpu().view(wl.B, wl.L, wl.H, 128).permute(0, 2, 1, 3).to(torch.bfloat16)


def _pair_reference(lut, NB, k):
    """Restatement of the pairing table, rows of the tile in ascending order."""
    BH = lut.shape[0]
    NT = (NB + 1) // 2
    out = torch.full((BH, NT, 2 * k + 1), -1, dtype=torch.int32)
    for bh in range(BH):
        for t in range(NT):
            sel = {}
            for half in range(2):
                m = 2 * t + half
                if m < NB:
                    for j in lut[bh, m].tolist():
                        sel[j] = sel.get(j, 0) | (1 << (28 + half))
            ent = [j | sel[j] for j in sorted(sel)]
            out[bh, t, 1:1 + len(ent)] = torch.tensor(ent, dtype=torch.int32)
            out[bh, t, 0] = (len(ent) + 1) // 2
    return out


@pytest.mark.parametrize("name", sorted(CASES))
def test_blk64_forward(name):
    wl = CASES[name]
    B, L, H, blk, k = wl.B, wl.L, wl.H, 64, wl.topk
    NB = (L + blk - 1) // blk
    inp = make_inputs(wl, device="cpu")
    freqs = wan_rope_freqs(*wl.grid)
    cos_sin = prepare_cos_sin(freqs, L, 128)
    lr_cos, lr_sin, rope_dim = prepare_lowrank_cos_sin(freqs, L, wl.rank, torch.bfloat16)
    g = {kk: (v.cuda() if isinstance(v, torch.Tensor) else v) for kk, v in inp.items()}
    out, ex = ops.rola_attention_from_qkv(g["q_raw"], g["k_raw"], g["v_raw"], g["x"], cos_sin.cuda(), lr_cos.cuda(),
                                          lr_sin.cuda(), rope_dim, g["norm_wq"], g["norm_wk"], g["proj_q"],
                                          g["proj_k"], g["gate_w"], g["gate_b"], H, blk, k, keep=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    q4, k4 = _heads(ex["q_rope"], wl), _heads(ex["k_rope"], wl)
    # selection on 64-token blocks, bit for bit
    lut, *_ = orc.block_select(q4, k4, blk, blk, k)
    assert torch.equal(ex["lut"].cpu(), lut.reshape(B * H, NB, k))
    # the pairing table
    paired = torch.empty(B * H, (NB + 1) // 2, 2 * k + 1, device="cuda", dtype=torch.int32)
    _lib.call("rola_b200_pair_blocks", ex["lut"].data_ptr(), B * H, NB, k, paired.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(paired.cpu(), _pair_reference(ex["lut"].cpu(), NB, k))
    # attention with the GPU's LUT
    v4 = inp["v_raw"].view(B, L, H, 128).permute(0, 2, 1, 3)
    o_ref = orc.sparse_attn_lut(q4, k4, v4, ex["lut"].cpu(), blk, blk, out_dtype=torch.float32)
    assert_bf16_close(_heads(ex["o_sparse"], wl), o_ref, f"o_sparse blk64 ({name})", ulp_floor=True)
    # the kernel takes one running max per 128-key tile (two 64-key blocks),
    # the oracle one per 64-key block, so P is rounded to bf16 relative to a
    # different max now and then: ~0.5 % of the elements land 1-2 steps apart
    assert_ulp_close(_heads(ex["o_sparse"], wl), o_ref.to(torch.bfloat16), f"o_sparse blk64 ({name})", ulps=2,
                     max_frac=1e-2)
    # the gated output: the fused epilogue on the GPU's own o_sparse, q_lr and C
    # against the oracle's (final rounding removed), at the strict bound
    R = wl.rank
    q_lr = ex["q_lr"].cpu().view(B, L, H, R).permute(0, 2, 1, 3).float()
    o_lr = torch.matmul(q_lr, ex["C"].cpu().float().view(B, H, R, 128)).to(torch.bfloat16)
    ref = orc.fused_gate(o_lr, _heads(ex["o_sparse"], wl), inp["x"], inp["gate_w"], inp["gate_b"],
                         out_dtype=torch.float32)
    assert_bf16_close(out.cpu(), ref, f"out blk64 ({name})")


def test_blk64_reference_named_api():
    B, H, L = 1, 2, 1000  # 16 blocks of 64, a 40-token tail
    torch.manual_seed(4)
    q, k, v = (torch.randn(B * H, L, 128).to(torch.bfloat16) for _ in range(3))
    topk = 3
    o = ops.fused_sparse_attn(q.cuda(), k.cuda(), v.cuda(), topk_ratio=(topk + 0.5) / 16, blkq=64, blkk=64,
                              num_heads=H)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    q4, k4, v4 = (t.view(B, H, L, 128) for t in (q, k, v))
    lut, *_ = orc.block_select(q4, k4, 64, 64, topk)
    ref = orc.sparse_attn_lut(q4, k4, v4, lut, 64, 64, out_dtype=torch.float32)
    assert_bf16_close(o.cpu(), ref, "fused_sparse_attn blk64", ulp_floor=True)
