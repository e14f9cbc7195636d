"""Training path of the block-sparse attention: forward with the row
log-sum-exp and the backward, timed on the B200.

The reference trains RoLa through the external SLA kernel
(sparkdiffusion/networks/wan_rola_attention.py:293-327), which is not part of
the reference tree nor of this image, so there is no reference arm here: the
numbers are reported against the roofline (the measured burst bf16 peak in
MEASURED_PEAKS.json).  Inputs: seeded bf16 q/k/v/dO of the given shape in the
token-major layout the layer produces, the selection from the B200 selection
kernels.  FLOPs are algorithmic, from the LUT: forward 4*D per selected
(query row, key) pair (two GEMMs), backward 10*D (five GEMMs: S, dP, dV, dK,
dQ).  The kernels recompute S and dP in both backward kernels (seven GEMMs
executed, ``tflops_executed``), which the algorithmic figure does not credit.

    python -m sparkdiffusion_b200.bench_backward --seq 75600 --heads 40 --blk 128

``--dense``: dense attention (every key block selected) forward + backward
against PyTorch SDPA with the cuDNN backend, which the reference's dense layers
train through (sparkdiffusion/utils/attention.py:122-186), on the same inputs;
FLOPs 4*L^2*D*H*B forward, 2.5x that backward.

    python -m sparkdiffusion_b200.bench_backward --dense --seq 32760 --heads 40
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from . import _lib, ops, train
from .workloads import attn_flops_lut


def _peak() -> tuple[float, str]:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured burst bf16"
    except (OSError, KeyError, ValueError, TypeError):
        return 1590.0, "fallback bf16"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=75600)
    ap.add_argument("--heads", type=int, default=40)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--blk", type=int, default=128, choices=(64, 128))
    ap.add_argument("--topk-ratio", type=float, default=18.5 / 591)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--dense", action="store_true")
    args = ap.parse_args(argv)
    if args.dense:
        return dense(args)
    B, H, L, blk = args.batch, args.heads, args.seq, args.blk
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)

    def mk():
        return torch.randn(B, L, H, 128, device=dev, generator=g).to(torch.bfloat16).transpose(1, 2)

    q, k, v, do = mk(), mk(), mk(), mk()
    lut, topk, paired = train.select_blocks(q, k, args.topk_ratio, blk)
    flut = lut if blk == 128 else paired
    flops_fwd = attn_flops_lut(lut, L, blk)
    flops_bwd = 2.5 * flops_fwd
    for _ in range(args.warmup):
        o, lse = ops.sparse_attention_fwd_lse(q, k, v, flut, blk, topk)
        ops.sparse_attention_bwd(q, k, v, o, do, lut, paired, lse, blk, topk)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    for e in ev:
        e[0].record()
        o, lse = ops.sparse_attention_fwd_lse(q, k, v, flut, blk, topk)
        e[1].record()
        ops.sparse_attention_bwd(q, k, v, o, do, lut, paired, lse, blk, topk)
        e[2].record()
    torch.cuda.synchronize()
    if _lib.device_status() != 0:
        raise RuntimeError(f"device error {_lib.device_status()}")
    tf = sorted(e[0].elapsed_time(e[1]) for e in ev)[len(ev) // 2]
    tb = sorted(e[1].elapsed_time(e[2]) for e in ev)[len(ev) // 2]
    peak, kind = _peak()
    res = {"what": "block-sparse attention training path (forward with lse, backward), bf16",
           "B": B, "H": H, "L": L, "blk": blk, "topk": topk, "fwd_tflop": flops_fwd / 1e12,
           "fwd": {"ms": tf, "tflops": flops_fwd / tf / 1e9, "frac": flops_fwd / tf / 1e9 / peak},
           "bwd": {"ms": tb, "tflops_algorithmic": flops_bwd / tb / 1e9, "frac": flops_bwd / tb / 1e9 / peak,
                   "tflops_executed": 3.5 * flops_fwd / tb / 1e9},
           "peak_tflops": peak, "peak_kind": kind}
    print(json.dumps(res))


def dense(args) -> None:
    B, H, L = args.batch, args.heads, args.seq
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)

    def mk():
        return torch.randn(B, H, L, 128, device=dev, generator=g).to(torch.bfloat16)

    q0, k0, v0, do = mk(), mk(), mk(), mk()
    flops = 4.0 * B * H * L * L * 128
    peak, kind = _peak()

    def run(fn):
        q, k, v = (t.detach().clone().requires_grad_(True) for t in (q0, k0, v0))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        o = fn(q, k, v)
        ev[1].record()
        o.backward(do)
        ev[2].record()
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), (o.detach(), q.grad, k.grad, v.grad)

    from torch.nn.attention import SDPBackend, sdpa_kernel

    def sdpa(q, k, v):
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            return torch.nn.functional.scaled_dot_product_attention(q, k, v)

    res = {"what": "dense attention forward + backward, bf16, [B, H, L, 128], no mask", "B": B, "H": H, "L": L,
           "fwd_tflop": flops / 1e12, "peak_tflops": peak, "peak_kind": kind}
    outs = {}
    for name, fn in (("ours", train.dense_attention), ("sdpa_cudnn", sdpa)):
        try:
            for _ in range(args.warmup):
                run(fn)
            ts = [run(fn) for _ in range(args.steps)]
        except RuntimeError as exc:  # backend not available for this shape / build
            res[name] = {"unavailable": str(exc).splitlines()[0][:200]}
            continue
        tf = sorted(t[0] for t in ts)[len(ts) // 2]
        tb = sorted(t[1] for t in ts)[len(ts) // 2]
        outs[name] = ts[-1][2]
        res[name] = {"fwd_ms": tf, "bwd_ms": tb, "fwd_tflops": flops / tf / 1e9, "bwd_tflops": 2.5 * flops / tb / 1e9}
    if len(outs) == 2:
        rows = torch.randint(0, L, (512,), generator=torch.Generator().manual_seed(1)).to(dev)
        cmp = {}
        for i, n in enumerate(("o", "dq", "dk", "dv")):
            a, r = outs["ours"][i][:, :, rows].float(), outs["sdpa_cudnn"][i][:, :, rows].float()
            rms = r.pow(2).mean().sqrt()
            cmp[n] = {"max_rel": ((a - r).abs().max() / rms).item(), "mean_rel": ((a - r).abs().mean() / rms).item()}
        res["ours_vs_sdpa"] = cmp
    if _lib.device_status() != 0:
        raise RuntimeError(f"device error {_lib.device_status()}")
    print(json.dumps(res))


if __name__ == "__main__":
    main()
