"""Dense attention on the B200 kernels against the reference's dense attention
backend on the same GPU.

The reference's dense layers (``WanSelfAttention``, sparkdiffusion/networks/wan2pt1.py:282-324)
run scaled-dot-product attention through ``sparkdiffusion/utils/attention.py:122-186``,
which on sm_100 prefers PyTorch SDPA with the cuDNN backend.  This module times
``ops.dense_attention_strided`` (the block-sparse tcgen05 kernel with every key
block kept) and SDPA (cuDNN, and flash where PyTorch offers it) on the same
seeded ``[B, H, L, 128]`` bf16 q/k/v, with CUDA events on the launching stream,
and prints one JSON line: ms per call, TFLOP/s (4 * L^2 * D * H * B), and the
difference between the two outputs on sampled rows.

    python -m sparkdiffusion_b200.bench_dense --seq 75600 --heads 40
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.nn.functional as F

from . import ops


def _time(fn, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=75600)
    ap.add_argument("--heads", type=int, default=40)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    B, H, L, D = args.batch, args.heads, args.seq, 128
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    q, k, v = (torch.randn(B, H, L, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    out = torch.empty_like(q)
    s = q.stride()
    strides = (s[0], s[1], s[2])

    def ours():
        ops.dense_attention_strided(q, k, v, B, L, H, strides, strides, out, strides)

    flops = 4.0 * B * H * L * L * D
    res = {"what": "dense attention, bf16, [B, H, L, 128] q/k/v, no mask", "B": B, "H": H, "L": L,
           "tflop_per_call": flops / 1e12}
    t = _time(ours, args.steps, args.warmup)
    res["ours"] = {"kernel": "sparse_attn_tcgen05 (every key block kept)", "ms": t, "tflops": flops / t / 1e9}
    rows = torch.randint(0, L, (256,), generator=torch.Generator().manual_seed(1)).to(dev)
    from torch.nn.attention import SDPBackend, sdpa_kernel

    for name, backend in (("sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("sdpa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel(backend):
                ref = F.scaled_dot_product_attention(q, k, v)
                t = _time(lambda: F.scaled_dot_product_attention(q, k, v), args.steps, args.warmup)
        except RuntimeError as exc:  # backend not available for this shape / build
            res[name] = {"unavailable": str(exc).splitlines()[0][:200]}
            continue
        a, r = out[:, :, rows].float(), ref[:, :, rows].float()
        rms = r.pow(2).mean().sqrt()
        res[name] = {"ms": t, "tflops": flops / t / 1e9, "ours_vs_this_max_rel": ((a - r).abs().max() / rms).item(),
                     "ours_vs_this_mean_rel": ((a - r).abs().mean() / rms).item()}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
