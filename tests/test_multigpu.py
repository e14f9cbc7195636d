"""Ulysses sequence<->head parallel forward on 2, 4 and 8 GPUs vs the 1-GPU forward.

Skipped unless enough CUDA devices are visible.  Each rank holds a sequence
shard of the hidden states; the result gathered from all ranks must match the
single-GPU forward bit for bit: every stage computes the same values in the
same order on both paths (the low-rank C sums fixed 1024-token chunks in
order, whatever the heads per GPU and hence the number of CTA columns).  Both
transports run: the exchanges fused into the kernels over peer memory, and the
NCCL all-to-all.  With 8 ranks the shards (360 tokens) do not align with the
128-token blocks, so blocks straddle ranks in both exchanges.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _workload():
    from sparkdiffusion_b200.workloads import C3

    wl = C3.scaled(H=8, grid=(4, 16, 45), B=1)  # L = 2880 (NB = 23, ragged tail of 64)
    return wl.__class__(**{**wl.__dict__, "topk": 3})


def _inputs(wl, dev):
    from sparkdiffusion_b200.rope import prepare_cos_sin, prepare_lowrank_cos_sin, wan_rope_freqs
    from sparkdiffusion_b200.workloads import make_inputs

    inp = make_inputs(wl, device="cpu")
    inp = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    freqs = wan_rope_freqs(*wl.grid)
    cos_sin = prepare_cos_sin(freqs, wl.L, 128).to(dev)
    lr_cos, lr_sin, rope_dim = prepare_lowrank_cos_sin(freqs, wl.L, wl.rank, torch.bfloat16)
    common = (cos_sin, lr_cos.to(dev), lr_sin.to(dev), rope_dim, inp["norm_wq"], inp["norm_wk"], inp["proj_q"],
              inp["proj_k"], inp["gate_w"], inp["gate_b"])
    return inp, common


def _rank_main(rank, world, transport, chunks, port, out_path):
    import datetime

    import torch.distributed as dist

    from sparkdiffusion_b200 import _lib, peer
    from sparkdiffusion_b200.ulysses import ulysses_rola_attention_params

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    wl = _workload()
    inp, common = _inputs(wl, dev)
    Ls = wl.L // world
    x_local = inp["x"][:, rank * Ls:(rank + 1) * Ls].contiguous()
    outs = []
    for _ in range(3):  # both alternating output buffers, then the first again
        out = ulysses_rola_attention_params(x_local, inp["w_qkv"], None, *common, wl.H, wl.topk,
                                            transport=transport, chunks=chunks)
        outs.append(out.clone())
    torch.cuda.synchronize()
    status = _lib.device_status()
    parts = [torch.empty_like(outs[0]) for _ in range(world)]
    dist.all_gather(parts, outs[0])
    repeat_equal = all(torch.equal(o, outs[0]) for o in outs[1:])
    if rank == 0:
        torch.save({"out": torch.cat(parts, dim=1).cpu(), "status": status, "repeat_equal": repeat_equal},
                   out_path)
    peer.release_all()
    dist.barrier()
    dist.destroy_process_group()


# (ranks, transport, token chunks of the GEMM / scatter overlap: None = the
# automatic plan, 1 = no overlap); with 8 ranks and 2 chunks the 360-token
# shards split into 256 + 104 tokens
CASES = [(2, "peer", None), (2, "peer", 1), (2, "nccl", 1), (4, "peer", None), (8, "peer", 2)]


@pytest.mark.parametrize("world,transport,chunks", CASES, ids=[f"{w}gpu-{t}-c{c}" for w, t, c in CASES])
def test_ulysses_matches_single_gpu(tmp_path, world, transport, chunks):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from sparkdiffusion_b200 import ops

    out_path = str(tmp_path / "ulysses.pt")
    mp.start_processes(_rank_main, args=(world, transport, chunks, _free_port(), out_path), nprocs=world,
                       start_method="spawn")
    got = torch.load(out_path)
    assert got["status"] == 0
    assert got["repeat_equal"]
    wl = _workload()
    inp, common = _inputs(wl, "cuda:0")
    ref = ops.rola_attention_core(inp["x"], inp["w_qkv"], None, *common, wl.H, 128, wl.topk)
    torch.cuda.synchronize()
    assert torch.equal(got["out"], ref.cpu()), f"ulysses {world} GPUs ({transport}) differs from the single GPU"
