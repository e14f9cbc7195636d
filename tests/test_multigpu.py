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


def _layer_rank_main(rank, world, blk, port, out_path):
    """The drop-in layer under the model's context-parallel hook: each rank gets
    its sequence shard of the hidden states and of the RoPE frequencies (as
    WanModel passes them, wan2pt1.py:825-826), the layer runs the Ulysses route."""
    import datetime

    import torch.distributed as dist

    from sparkdiffusion_b200 import peer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    layer, x, freqs = _layer_case(blk, dev)
    L = x.shape[1]
    Ls = L // world
    layer.set_context_parallel_group(dist.group.WORLD, list(range(world)), torch.cuda.Stream())
    with torch.no_grad():
        y = layer(x[:, rank * Ls:(rank + 1) * Ls].contiguous(), torch.tensor([L]),
                  freqs[rank * Ls:(rank + 1) * Ls])
    torch.cuda.synchronize()
    parts = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(parts, y.contiguous())
    if rank == 0:
        torch.save({"out": torch.cat(parts, dim=1).cpu()}, out_path)
    peer.release_all()
    dist.barrier()
    dist.destroy_process_group()


def _layer_case(blk, dev):
    from sparkdiffusion_b200.layer import WanSelfAttentionRoLaB200
    from sparkdiffusion_b200.rope import wan_rope_freqs

    torch.manual_seed(11)
    grid = (4, 16, 30)  # L = 1920: 15 blocks of 128 / 30 of 64
    layer = WanSelfAttentionRoLaB200(1024, 8, True, 1e-6, rola_topk_ratio=0.25, rola_rank=64, rola_blkq=blk,
                                     rola_blkk=blk)
    with torch.no_grad():  # a gate that varies per token (the trained layer's is not constant)
        layer.gate_proj.weight.normal_(0.0, 0.05)
        layer.norm_q.weight.uniform_(0.5, 1.5)
        layer.norm_k.weight.uniform_(0.5, 1.5)
    layer = layer.to(torch.bfloat16).to(dev).eval()
    g = torch.Generator().manual_seed(12)
    x = torch.randn(1, grid[0] * grid[1] * grid[2], 1024, generator=g).to(torch.bfloat16).to(dev)
    return layer, x, wan_rope_freqs(*grid).to(dev)


@pytest.mark.parametrize("blk", [128, 64])
def test_layer_context_parallel_matches_single_gpu(tmp_path, blk):
    """WanSelfAttentionRoLaB200 after set_context_parallel_group on 2 ranks equals
    the same layer on one GPU, bit for bit (output projection included)."""
    world = 2
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out_path = str(tmp_path / "layer_cp.pt")
    mp.start_processes(_layer_rank_main, args=(world, blk, _free_port(), out_path), nprocs=world,
                       start_method="spawn")
    got = torch.load(out_path)["out"]
    layer, x, freqs = _layer_case(blk, torch.device("cuda", 0))
    with torch.no_grad():
        ref = layer(x, torch.tensor([x.shape[1]]), freqs)
    torch.cuda.synchronize()
    assert torch.equal(got, ref.cpu()), f"context-parallel layer (blk {blk}) differs from the single GPU"


# ---------------------------------------------------------------------------
# the whole model: the reference's WanModel with this package's layer, its own
# context-parallel split / gather (wan2pt1.py:767-866, enable_context_parallel
# :953-960) on 2 ranks against the same model on one GPU
# ---------------------------------------------------------------------------
MODEL_TINY = dict(model_type="t2v", patch_size=(1, 2, 2), text_len=8, in_dim=4, dim=1024, ffn_dim=2048, freq_dim=32,
                  text_dim=32, out_dim=4, num_heads=8, num_layers=2)
MODEL_ROLA = dict(rola_topk_ratio=0.25, rola_rank=64, rola_blkq=128, rola_blkk=128)


def _reference_package_path():
    """The installed reference (``baseline/_ref`` or ``SPARKDIFFUSION_REF``); the
    read-only source checkout is not used here."""
    from conftest import reference_path

    return reference_path(allow_checkout=False)


def _model_case(ref_path, dev):
    import sys

    if ref_path not in sys.path:
        sys.path.insert(0, ref_path)
    import sparkdiffusion.networks.wan2pt1 as wan2pt1

    from sparkdiffusion_b200 import registry

    registry.register_into_reference()
    torch.manual_seed(0)
    model = wan2pt1.WanModel(**MODEL_TINY, attn_variant="rola_b200", attn_variant_kwargs=dict(MODEL_ROLA))
    with torch.no_grad():
        for blk in model.blocks:  # a gate that varies per token (a trained layer's is not constant)
            blk.self_attn.gate_proj.weight.normal_(0.0, 0.05)
        for prm in model.head.parameters():  # the reference zero-initialises the output head
            prm.normal_(0.0, 0.02)
    model = model.to(dev).eval()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, 4, 4, 32, 60, generator=g).to(dev)  # L = 4 * 16 * 30 = 1920 tokens after patchify
    t = torch.full((1, 1), 500.0).to(dev)
    ctx = torch.randn(1, 8, 32, generator=g).to(dev)
    return model, (x, t, ctx)


def _model_rank_main(rank, world, port, ref_path, out_path):
    import datetime

    import torch.distributed as dist

    from sparkdiffusion_b200 import _lib, peer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    model, args = _model_case(ref_path, dev)
    model.enable_context_parallel(dist.group.WORLD)
    with torch.no_grad():
        y = model(*args)
    torch.cuda.synchronize()
    if rank == 0:
        torch.save({"out": y.cpu(), "status": _lib.device_status()}, out_path)
    peer.release_all()
    dist.barrier()
    dist.destroy_process_group()


def test_wanmodel_context_parallel_matches_single_gpu(tmp_path):
    """The reference's WanModel built with attn_variant="rola_b200", run with its
    own context parallelism on 2 ranks (inputs broadcast, sequence split before
    the blocks, outputs gathered after the head), equals the same model on one
    GPU: this layer attends over the whole sequence under the model's hook
    (where the reference's context-parallel RoLa attends within each rank's
    shard).  Tolerance: max-abs <= 2e-2 and mean-abs <= 2e-3 of the output RMS
    (the other layers run fp32 GEMMs on shards of a different length, whose
    library kernels may sum in another order)."""
    world = 2
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ref_path = _reference_package_path()
    if ref_path is None:
        pytest.skip("the reference package (baseline/_ref) is not installed")
    out_path = str(tmp_path / "model_cp.pt")
    mp.start_processes(_model_rank_main, args=(world, _free_port(), ref_path, out_path), nprocs=world,
                       start_method="spawn")
    got = torch.load(out_path)
    assert got["status"] == 0
    model, args = _model_case(ref_path, torch.device("cuda", 0))
    with torch.no_grad():
        ref = model(*args)
    torch.cuda.synchronize()
    g, r = got["out"].float(), ref.float().cpu()
    rms = r.pow(2).mean().sqrt()
    assert rms > 0 and torch.isfinite(r).all() and torch.isfinite(g).all()
    mx, mn = ((g - r).abs().max() / rms).item(), ((g - r).abs().mean() / rms).item()
    assert mx <= 2e-2 and mn <= 2e-3, f"context-parallel WanModel: max-abs/rms={mx:.3e} mean-abs/rms={mn:.3e}"
