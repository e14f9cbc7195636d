"""Ulysses sequence<->head exchange on 2 gloo CPU ranks.

Each rank holds a sequence shard of the hidden states; the per-rank compute is
the CPU oracle, laid out exactly like the CUDA path (norm pass writes
per-destination send blocks [B][p][Ls][Hl*D], the all-to-alls move them to head
shards, the head-local stages run over the full sequence, the output goes back
to the sequence owner).  The result must match the single-process oracle:
identical block selection, output within bf16 tolerance.
"""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import rola_oracle as orc
from sparkdiffusion_b200.workloads import C3, make_inputs

WL = C3.scaled(H=4, grid=(2, 10, 32), B=2)  # L = 640, NB = 5, two batch elements
WL = WL.__class__(**{**WL.__dict__, "topk": 2})


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tables(wl):
    freqs = orc.wan_rope_freqs(*wl.grid)
    cos_sin = orc.prepare_cos_sin(freqs, wl.L, 128)
    lr_cos, lr_sin, rope_dim = orc.prepare_lowrank_cos_sin(freqs, wl.L, wl.rank, torch.bfloat16)
    return cos_sin, lr_cos, lr_sin, rope_dim


def _rank_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from sparkdiffusion_b200.ulysses import head_to_seq, seq_to_head

    wl = WL
    p = world
    B, L, H, D, dim = wl.B, wl.L, wl.H, 128, wl.dim
    Ls, Hl = L // p, H // p
    inp = make_inputs(wl, device="cpu")
    cos_sin, lr_cos, lr_sin, rope_dim = _tables(wl)
    w = inp["w_qkv"]
    x_local = inp["x"][:, rank * Ls:(rank + 1) * Ls].contiguous()
    # sequence-parallel half: projections, qk-RMSNorm and gate on the shard
    q_raw = orc.qkv_linear(x_local, w[:dim])
    k_raw = orc.qkv_linear(x_local, w[dim:2 * dim])
    v_raw = orc.qkv_linear(x_local, w[2 * dim:])
    _, _, _, q_n, k_n = orc.qkv_epilogue(q_raw, k_raw, v_raw, cos_sin[rank * Ls:], inp["norm_wq"], inp["norm_wk"], H)
    gate = orc.gate_values(x_local, inp["gate_w"], inp["gate_b"], H)

    def pack(t):  # [B, Ls, H*X] -> send blocks [B, p, Ls, Hl*X] (what the norm pass writes)
        X = t.shape[-1] // H
        return t.reshape(B, Ls, p, Hl * X).permute(0, 2, 1, 3).contiguous()

    q_h, _ = seq_to_head(pack(q_n.reshape(B, Ls, dim)))
    k_h, _ = seq_to_head(pack(k_n.reshape(B, Ls, dim)))
    v_h, _ = seq_to_head(pack(v_raw))
    g_h, _ = seq_to_head(pack(gate))
    q_h, k_h, v_h, g_h = (t.reshape(B, L, -1) for t in (q_h, k_h, v_h, g_h))
    # head-local half over the full sequence (global RoPE positions)
    q_rope, k_rope, v4, _, _ = orc.qkv_epilogue(q_h, k_h, v_h, cos_sin, None, None, Hl)
    q4, k4, v4 = (t.reshape(B, Hl, L, D) for t in (q_rope, k_rope, v4))
    lut, *_ = orc.block_select(q4, k4, 128, 128, wl.topk)
    o_sparse = orc.sparse_attn_lut(q4, k4, v4, lut, 128, 128)
    o_lr, *_ = orc.fused_lowrank(q_h.reshape(B, L, Hl, D), k_h.reshape(B, L, Hl, D), v4.reshape(B * Hl, L, D),
                                 inp["proj_q"], inp["proj_k"], lr_cos, lr_sin, rope_dim)
    out_heads = orc.fused_gate(o_lr, o_sparse, None, None, None, gate=g_h)
    out_local = head_to_seq(out_heads, p)
    luts = [torch.empty_like(lut) for _ in range(p)]
    dist.all_gather(luts, lut.contiguous())
    outs = [torch.empty_like(out_local) for _ in range(p)]
    dist.all_gather(outs, out_local.contiguous())
    if rank == 0:
        torch.save({"lut": torch.cat(luts, dim=1), "out": torch.cat(outs, dim=1)}, out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_ulysses_two_ranks_match_single_process(tmp_path):
    out_path = str(tmp_path / "ulysses.pt")
    mp.start_processes(_rank_main, args=(2, _free_port(), out_path), nprocs=2, start_method="spawn")
    got = torch.load(out_path)
    wl = WL
    inp = make_inputs(wl, device="cpu")
    cos_sin, lr_cos, lr_sin, rope_dim = _tables(wl)
    dim = wl.dim
    w = inp["w_qkv"]
    ref = orc.rola_attention_forward(inp["x"], w[:dim], None, w[dim:2 * dim], None, w[2 * dim:], None,
                                     cos_sin=cos_sin, lr_cos=lr_cos, lr_sin=lr_sin, rope_dim=rope_dim,
                                     norm_wq=inp["norm_wq"], norm_wk=inp["norm_wk"], proj_q=inp["proj_q"],
                                     proj_k=inp["proj_k"], gate_w=inp["gate_w"], gate_b=inp["gate_b"],
                                     num_heads=wl.H, blkq=128, blkk=128, topk=wl.topk)
    assert torch.equal(got["lut"], ref["lut"])
    r = ref["out"].float()
    d = (got["out"].float() - r).abs()
    rms = r.pow(2).mean().sqrt()
    assert (d.mean() / rms) <= 2e-3 and (d.max() / rms) <= 2e-2
