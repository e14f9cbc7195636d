"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs ONLY in a container where the SparkDiffusion reference checkout is
importable (its path is taken from ``SPARKDIFFUSION_REF`` or the first
argument); the GPU box never runs this script.  Two fixture files are written
next to this script:

* ``c1_fp32.pt``: configuration C1 (B=1, H=12, grid 6x16x16 -> L=1536, block 64,
  top-6, rank 16, fp32) run through the reference's own fused inference path
  -- the prologue's ``_epilogue_kernel`` (C1 starts from projected q/k/v),
  ``fused_sparse_attn``, ``fused_lowrank`` and ``fused_gate`` -- with their
  Triton kernels executed by the Triton interpreter in fp32 (autotuners pinned
  to one configuration, since autotuning needs a GPU).
  Stored: the reference's LUT (as kept sets), pooled q/k, scores, and heads 0
  and 11 (every 4th token) of q_rope, o_sparse, o_lr and the gated output.
* ``eager_bf16.pt``: the reference's eager PyTorch pieces in bf16 on small
  shapes (WanRMSNorm, the fp32 rope_apply fallback, ``fused_lowrank_ref``,
  ``fused_gate_ref``) and the Wan 3D RoPE angles of two grids.

Inputs are not stored: the tests regenerate them from
``sparkdiffusion_b200.workloads.make_inputs`` and compare checksums recorded here.
"""

from __future__ import annotations

import importlib
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from sparkdiffusion_b200.workloads import C1, make_inputs  # noqa: E402

HEADS = [0, 11]
TOKEN_STRIDE = 4


class _Pinned:
    """Stand-in for a triton Autotuner: launches its kernel with one fixed config."""

    def __init__(self, autotuner, meta):
        self.fn = autotuner.fn
        self.meta = dict(meta)

    def __getitem__(self, grid):
        def launch(*args, **kw):
            meta = dict(kw)
            meta.update(self.meta)
            g = grid(meta) if callable(grid) else grid
            return self.fn[g](*args, **meta)

        return launch


class _PaddedEmpty:
    """The Triton interpreter touches the addresses of masked-out lanes; with
    H=12 padded to 16 those lie past the end of the reference's own output
    buffers.  While active, torch.empty over-allocates and returns a view, so
    the masked addresses land in padding."""

    PAD = 1 << 22

    def __enter__(self):
        self.orig = torch.empty

        def empty(*size, **kw):
            shape = tuple(size[0]) if len(size) == 1 and isinstance(size[0], (tuple, list, torch.Size)) else size
            n = 1
            for s in shape:
                n *= int(s)
            flat = self.orig(n + self.PAD, **kw)
            return flat[:n].view(*shape)

        torch.empty = empty
        return self

    def __exit__(self, *exc):
        torch.empty = self.orig


def _import_reference(path: str):
    sys.path.insert(0, path)
    w21 = importlib.import_module("sparkdiffusion.networks.wan2pt1")
    fq = importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_qkv_rope")
    fs = importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_sparse_attn")
    fl = importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_lowrank")
    fg = importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_gate")
    fu = importlib.import_module("sparkdiffusion.ops.fused_kernel.utils")
    # the eager RoPE falls back to its own fp32 formula when flash_attn is absent
    w21.flash_apply_rotary_emb = None
    # pin the autotuned kernels (autotuning needs a CUDA driver)
    fq._epilogue_kernel = _Pinned(fq._epilogue_kernel, {})
    fs._rola_fwd_kernel = _Pinned(fs._rola_fwd_kernel, {})
    fl._proj_silu_rope_kernel = _Pinned(fl._proj_silu_rope_kernel, {"BLOCK_L": 64})
    fg._gate_fusion_kernel = _Pinned(fg._gate_fusion_kernel, {"BLOCK_L": 64})
    return w21, fq, fs, fl, fg, fu


def _rope_freqs(w21, T, H, W, head_dim=128):
    emb = w21.VideoRopePosition3DEmb(head_dim=head_dim, len_h=128, len_w=128, len_t=32)
    orig = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self  # cache_parameters() moves tables to CUDA
    try:
        return emb.generate_embeddings(torch.Size([1, T, H, W, head_dim])).contiguous()
    finally:
        torch.Tensor.cuda = orig


def _checksum(t: torch.Tensor) -> list:
    f = t.double()
    return [float(f.sum()), float(f.abs().sum()), float(f.reshape(-1)[:: max(1, f.numel() // 97)].sum())]


def _heads_tokens(t4: torch.Tensor) -> torch.Tensor:
    """[B, H, L, X] -> heads HEADS, every TOKEN_STRIDE-th token."""
    return t4[:, HEADS, ::TOKEN_STRIDE].float().clone()  # compact copy (no padded storage)


def make_c1(mods) -> dict:
    w21, fq, fs, fl, fg, fu = mods
    wl = C1
    B, L, H, D, dim = wl.B, wl.L, wl.H, wl.head_dim, wl.dim
    inp = make_inputs(wl, device="cpu")
    freqs = _rope_freqs(w21, *wl.grid)
    cos_sin = fq.prepare_cos_sin(freqs, L, D)
    # The reference's prologue epilogue kernel run directly on the projected
    # q/k/v (C1 starts from q/k/v, not from hidden states); arguments as
    # fused_qkv_gemm_rope passes them (fused_qkv_rope.py:297-329).
    M = B * L
    q_raw, k_raw, v_raw = (inp[n].reshape(M, dim).contiguous() for n in ("q_raw", "k_raw", "v_raw"))
    with torch.no_grad(), _PaddedEmpty():
        q_rope = torch.empty(B * H, L, D)
        k_rope = torch.empty(B * H, L, D)
        v_out = torch.empty(B * H, L, D)
        q_n = torch.empty(B, L, H, D)
        k_n = torch.empty(B, L, H, D)
        fq._epilogue_kernel[(M,)](
            q_raw, k_raw, v_raw, cos_sin, inp["norm_wq"], inp["norm_wk"], q_rope, k_rope, v_out, q_n, k_n,
            L, H, dim, L * D, D, HEAD_DIM=D, NUM_HEADS=H, DIM=dim, PAD_H=16, PAD_D=128, EPS=1e-6,
            HAS_NORM=True, RETURN_NORMED=True)
        # the selection, recorded from inside fused_sparse_attn
        rec = {}
        orig_topk = torch.topk

        def topk_rec(x, k, *a, **kw):
            r = orig_topk(x, k, *a, **kw)
            rec["scores"], rec["lut"] = x.clone(), r.indices.clone()
            return r

        torch.topk = topk_rec
        try:
            ratio = (wl.topk + 0.5) / wl.NB
            o_sparse = fs.fused_sparse_attn(q_rope, k_rope, v_out, topk_ratio=ratio, blkq=wl.blk, blkk=wl.blk,
                                            num_heads=H)
        finally:
            torch.topk = orig_topk
        q4, k4 = q_rope.view(B, H, L, D), k_rope.view(B, H, L, D)
        pooled_q = fu.mean_pool(q4, wl.blk)
        pooled_k = fu.mean_pool(k4, wl.blk, center=k4.mean(dim=-2))
        rope_tables = fl.prepare_lowrank_cos_sin(freqs, L, wl.rank, torch.float32)
        o_lr = fl.fused_lowrank(q_n, k_n, v_out, freqs, proj_q_weight=inp["proj_q"], proj_k_weight=inp["proj_k"],
                                rola_rank=wl.rank, eps=1e-6, rope_tables=rope_tables)
        out = fg.fused_gate(o_lr, o_sparse, inp["x"], gate_proj_weight=inp["gate_w"],
                            gate_bias=inp["gate_b"].view(H))
    kept = torch.sort(rec["lut"].reshape(B * H, wl.NB, -1), dim=-1).values.to(torch.int16)
    return {
        "config": dict(B=B, H=H, grid=wl.grid, blk=wl.blk, topk=wl.topk, rank=wl.rank, L=L),
        "heads": HEADS,
        "token_stride": TOKEN_STRIDE,
        "input_checksums": {k: _checksum(v) for k, v in inp.items() if isinstance(v, torch.Tensor)},
        "freqs_checksum": _checksum(freqs),
        "lut_sorted": kept.clone(),
        "scores": rec["scores"].reshape(B * H, wl.NB, wl.NB).float().clone(),
        "pooled_q": pooled_q.float().clone(),
        "pooled_k": pooled_k.float().clone(),
        "q_rope": _heads_tokens(q_rope.view(B, H, L, D)).float(),
        "k_normed": _heads_tokens(k_n.permute(0, 2, 1, 3)).float(),
        "o_sparse": _heads_tokens(o_sparse).float(),
        "o_lr": _heads_tokens(o_lr).float(),
        "out": _heads_tokens(out.view(B, L, H, D).permute(0, 2, 1, 3)).float(),
    }


def make_eager_bf16(mods) -> dict:
    w21, fq, fs, fl, fg, fu = mods
    g = torch.Generator().manual_seed(7)
    bf = torch.bfloat16
    B, L, H, D, R = 1, 192, 2, 128, 64
    dim = H * D
    res = {"config": dict(B=B, L=L, H=H, R=R, seed=7)}
    x = (torch.randn(B, L, dim, generator=g) * 1.5).to(bf)
    w = (1.0 + 0.1 * torch.randn(dim, generator=g)).to(bf)
    norm = w21.WanRMSNorm(dim, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(w)
        normed = norm.to(bf)(x)
    freqs = _rope_freqs(w21, 2, 8, 12)
    roped = w21.rope_apply(normed.view(B, L, H, D), freqs)
    res.update(rms_in=x, rms_w=w, rms_out=normed, rope_freqs=freqs, rope_out=roped)
    # low-rank eager reference
    q = (torch.randn(B, L, H, D, generator=g) * 0.7).to(bf)
    k = (torch.randn(B, L, H, D, generator=g) * 0.7).to(bf)
    v = torch.randn(B * H, L, D, generator=g).to(bf)
    pq = (torch.randn(R, D, generator=g) / D ** 0.5).to(bf)
    pk = (torch.randn(R, D, generator=g) / D ** 0.5).to(bf)
    o_lr = fl.fused_lowrank_ref(q, k, v, freqs=freqs, proj_q_weight=pq, proj_k_weight=pk, rola_rank=R)
    res.update(lr_q=q, lr_k=k, lr_v=v, lr_pq=pq, lr_pk=pk, lr_out=o_lr)
    # gate eager reference
    o_sp = (torch.randn(B, H, L, D, generator=g) * 0.3).to(bf)
    xg = torch.randn(B, L, dim, generator=g).to(bf)
    gw = (torch.randn(1, D, generator=g) * 0.02).to(bf)
    gb = torch.full((H,), -1.946).to(bf)
    gout = fg.fused_gate_ref(o_lr, o_sp, xg, gate_proj_weight=gw, gate_bias=gb)
    res.update(g_olr=o_lr, g_os=o_sp, g_x=xg, g_w=gw, g_b=gb, g_out=gout)
    # Wan 3D RoPE angles: a full small grid and sampled rows of the C2/C4 grids
    res["freqs_small"] = _rope_freqs(w21, 3, 5, 7)
    for name, grid in (("freqs_c2_rows", (21, 30, 52)), ("freqs_c4_rows", (21, 45, 80))):
        f = _rope_freqs(w21, *grid)
        res[name] = f[::997].contiguous()
    return res


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPARKDIFFUSION_REF", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_golden.py <path to the SparkDiffusion reference checkout>")
    mods = _import_reference(ref)
    torch.save(make_eager_bf16(mods), os.path.join(HERE, "eager_bf16.pt"))
    torch.save(make_c1(mods), os.path.join(HERE, "c1_fp32.pt"))


if __name__ == "__main__":
    main()
