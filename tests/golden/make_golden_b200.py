"""Generate the B200 golden fixtures: the reference's own bf16 fused path run on a B200.

Test infrastructure only.  The reference's Triton interpreter cannot do bf16
arithmetic on the CPU, so its bf16 kernels only run on a GPU.  This script runs
the unmodified SparkDiffusion fused inference path -- ``_epilogue_kernel`` /
``fused_qkv_gemm_rope``, ``fused_sparse_attn``, ``fused_lowrank`` and
``fused_gate``, called as ``WanSelfAttentionRoLa.fused_forward`` calls them
(sparkdiffusion/networks/wan_rola_attention.py:414-446), with
``topk_ratio=(k+0.5)/NB`` so that ``int(ratio*NB)`` is the configuration's k --
on seeded inputs and stores what the GPU tests need to compare against it:

* ``ref_b200_c2.pt``: configuration C2 (B=1, H=12, L=32760, block 128, top-26,
  rank 64; from projected q/k/v through the reference's prologue epilogue
  kernel), all heads.
* ``ref_b200_c4.pt``: configuration C4 (B=1, H=40, L=75600, block 128, top-18,
  rank 64; from hidden states through the reference's cuBLAS projections and
  epilogue), the first ``C4_HEADS`` heads for selection, attention, low rank
  and gate (heads are independent after the prologue).
* ``ref_b200_c5.pt``: configuration C5 (B=2: cond and uncond batched, H=40,
  L=32760, top-13; from hidden states like C4), the first ``C4_HEADS`` heads of
  both batch elements.

Per configuration: the reference's LUT in its own (``torch.topk(sorted=False)``)
order, its bf16 pooled scores of the top ``k + EXTRA`` key blocks of every row
(values and indices, for classifying selection mismatches), and ``o_sparse``,
the gated output and ``q_rope`` on a seeded sample of token rows.  Also recorded:
the spread of the reference's own ``o_sparse`` against the CPU oracle's
recurrence on the reference's own q/k/v and LUT (``ref_vs_oracle``), which
tells how far a correct bf16 implementation sits from the fp32-accumulated
restatement.

The reference comes from a ``pip install --target`` of the checkout (default
``<repo>/baseline/_ref``; override with ``SPARKDIFFUSION_REF`` or the first
argument).  Fixtures are written to ``gpurun_out/`` (or the second argument)
and committed under ``tests/golden/`` by hand; the tests never import the
reference.
"""

from __future__ import annotations

import importlib
import os
import sys
import time
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import rola_oracle as orc  # noqa: E402
from sparkdiffusion_b200.rope import prepare_cos_sin, prepare_lowrank_cos_sin, wan_rope_freqs  # noqa: E402
from sparkdiffusion_b200.workloads import C2, C4, C5, make_inputs  # noqa: E402

EXTRA = 38          # stored scores per row: top k + EXTRA
C2_TOKENS = 192     # sampled token rows
C4_TOKENS = 256
C5_TOKENS = 192
C4_HEADS = 4
ORACLE_HEADS = 2    # heads of C2 on which the reference is compared with the oracle


def sample_tokens(L: int, n: int, seed: int) -> torch.Tensor:
    """Sorted seeded sample of ``n`` token rows, always including the last (tail) token."""
    g = torch.Generator().manual_seed(seed)
    idx = torch.randperm(L - 1, generator=g)[: n - 1]
    return torch.cat([idx, torch.tensor([L - 1])]).sort().values


def checksum(t: torch.Tensor) -> list:
    f = t.double().cpu()
    return [float(f.sum()), float(f.abs().sum())]


def import_reference(path: str):
    sys.path.insert(0, path)
    mods = types.SimpleNamespace(
        fq=importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_qkv_rope"),
        fs=importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_sparse_attn"),
        fl=importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_lowrank"),
        fg=importlib.import_module("sparkdiffusion.ops.fused_kernel.fused_gate"),
    )
    return mods


class TopkRecorder:
    """Records the scores and indices of the reference's ``torch.topk`` call
    inside ``fused_sparse_attn`` (fused_sparse_attn.py:197-198)."""

    def __enter__(self):
        self.orig = torch.topk
        self.rec = {}

        def topk(x, k, *a, **kw):
            r = self.orig(x, k, *a, **kw)
            self.rec["scores"], self.rec["lut"] = x.detach().clone(), r.indices.detach().clone()
            return r

        torch.topk = topk
        return self.rec

    def __exit__(self, *exc):
        torch.topk = self.orig


def top_scores(scores: torch.Tensor, n: int):
    """Top ``n`` bf16 scores per row (value desc, index asc among equal values)."""
    # a stable descending sort keeps ascending index order among equal values
    order = torch.sort(scores.float(), dim=-1, descending=True, stable=True).indices
    top = order[..., :n]
    return torch.gather(scores, -1, top).to(torch.bfloat16).cpu(), top.to(torch.int16).cpu()


def run_reference_tail(m, q_rope, k_rope, v, q_n, k_n, x, inp, wl, H, lr_tables, heads=None):
    """fused_sparse_attn -> fused_lowrank -> fused_gate as fused_forward chains them."""
    B, L = wl.B, wl.L
    if heads is not None:
        q_rope, k_rope, v = (t.view(B, -1, L, 128)[:, heads].reshape(-1, L, 128).contiguous()
                             for t in (q_rope, k_rope, v))
        q_n, k_n = (t[:, :, heads].contiguous() for t in (q_n, k_n))
        x = x[:, :, heads.start * 128: heads.stop * 128]
        H = heads.stop - heads.start
    gate_b = inp["gate_b"].reshape(-1)[: H].cuda()
    with TopkRecorder() as rec:
        o_sparse = m.fs.fused_sparse_attn(q_rope, k_rope, v, topk_ratio=wl.reference_topk_ratio, blkq=wl.blk,
                                          blkk=wl.blk, num_heads=H)
    o_lr = m.fl.fused_lowrank(q_n, k_n, v, None, norm_q_weight=None, norm_k_weight=None,
                              proj_q_weight=inp["proj_q"].cuda(), proj_k_weight=inp["proj_k"].cuda(),
                              rola_rank=wl.rank, eps=1e-6, rope_tables=lr_tables)
    out = m.fg.fused_gate(o_lr, o_sparse, x, gate_proj_weight=inp["gate_w"].cuda(), gate_bias=gate_b.view(H))
    torch.cuda.synchronize()
    return dict(q_rope=q_rope, k_rope=k_rope, v=v, o_sparse=o_sparse, o_lr=o_lr, out=out, scores=rec["scores"],
                lut=rec["lut"], H=H)


def pack_result(wl, r, tokens, inp_checksums, extra_info):
    B, L, H = wl.B, wl.L, r["H"]
    k = r["lut"].shape[-1]
    vals, idx = top_scores(r["scores"].reshape(B * H, wl.NB, wl.NB), k + EXTRA)
    tok = tokens.cuda()
    heads4 = lambda t: t.view(B, H, L, 128)[:, :, tok].to(torch.bfloat16).cpu().clone()  # noqa: E731
    return {
        "config": dict(name=wl.name, B=B, H=H, L=L, grid=wl.grid, blk=wl.blk, topk=k, rank=wl.rank),
        "input_checksums": inp_checksums,
        "tokens": tokens.to(torch.int32),
        "lut": r["lut"].reshape(B * H, wl.NB, k).to(torch.int16).cpu(),
        "score_vals": vals,
        "score_idx": idx,
        "o_sparse": heads4(r["o_sparse"]),
        "q_rope": heads4(r["q_rope"]),
        "out": r["out"].view(B, L, H * 128)[:, tok].to(torch.bfloat16).cpu().clone(),
        **extra_info,
    }


def ref_vs_oracle(r, wl, heads: int) -> dict:
    """The reference's own o_sparse against the oracle's recurrence on the
    reference's own q/k/v and LUT (CPU), over the first ``heads`` heads."""
    B, L = wl.B, wl.L
    sl = lambda t: t.view(B, -1, L, 128)[:, :heads].cpu()  # noqa: E731
    q4, k4, v4 = sl(r["q_rope"]), sl(r["k_rope"]), sl(r["v"])
    lut = r["lut"].view(B, -1, wl.NB, r["lut"].shape[-1])[:, :heads].cpu()
    ref = orc.sparse_attn_lut(q4, k4, v4, lut, wl.blk, wl.blk, out_dtype=torch.float32)
    got = sl(r["o_sparse"]).float()
    rms = ref.pow(2).mean().sqrt()
    d = (got - ref).abs()
    return {"heads": heads, "max_rel": float(d.max() / rms), "mean_rel": float(d.mean() / rms)}


def make_c2(m) -> dict:
    wl = C2
    B, L, H, dim = wl.B, wl.L, wl.H, wl.dim
    inp = make_inputs(wl, device="cpu")
    sums = {k: checksum(v) for k, v in inp.items() if isinstance(v, torch.Tensor)}
    freqs = wan_rope_freqs(*wl.grid)
    cos_sin = prepare_cos_sin(freqs, L, 128).cuda()
    lr_tables = tuple(t.cuda() if isinstance(t, torch.Tensor) else t
                      for t in m.fl.prepare_lowrank_cos_sin(freqs, L, wl.rank, torch.bfloat16))
    M = B * L
    q_raw, k_raw, v_raw = (inp[n].reshape(M, dim).cuda() for n in ("q_raw", "k_raw", "v_raw"))
    e = lambda *s: torch.empty(*s, device="cuda", dtype=torch.bfloat16)  # noqa: E731
    q_rope, k_rope, v_out = e(B * H, L, 128), e(B * H, L, 128), e(B * H, L, 128)
    q_n, k_n = e(B, L, H, 128), e(B, L, H, 128)
    # the prologue's epilogue kernel on the projected q/k/v, arguments as
    # fused_qkv_gemm_rope passes them (fused_qkv_rope.py:297-329)
    m.fq._epilogue_kernel[(M,)](
        q_raw, k_raw, v_raw, cos_sin, inp["norm_wq"].cuda(), inp["norm_wk"].cuda(), q_rope, k_rope, v_out, q_n, k_n,
        L, H, dim, L * 128, 128, HEAD_DIM=128, NUM_HEADS=H, DIM=dim, PAD_H=16, PAD_D=128, EPS=1e-6,
        HAS_NORM=True, RETURN_NORMED=True)
    r = run_reference_tail(m, q_rope, k_rope, v_out, q_n, k_n, inp["x"].cuda(), inp, wl, H, lr_tables)
    t0 = time.time()
    rvo = ref_vs_oracle(r, wl, ORACLE_HEADS)
    print(f"C2 reference vs oracle ({ORACLE_HEADS} heads, {time.time() - t0:.1f} s): {rvo}", flush=True)
    return pack_result(wl, r, sample_tokens(L, C2_TOKENS, 11), sums, {"ref_vs_oracle": rvo})


def make_c4(m, wl=C4, tokens=C4_TOKENS, seed=12) -> dict:
    B, L, H, dim = wl.B, wl.L, wl.H, wl.dim
    inp = make_inputs(wl, device="cpu")
    sums = {k: checksum(v) for k, v in inp.items() if isinstance(v, torch.Tensor)}
    freqs = wan_rope_freqs(*wl.grid)
    cos_sin = prepare_cos_sin(freqs, L, 128).cuda()
    lr_tables = tuple(t.cuda() if isinstance(t, torch.Tensor) else t
                      for t in m.fl.prepare_lowrank_cos_sin(freqs, L, wl.rank, torch.bfloat16))
    x = inp["x"].cuda()
    w = inp["w_qkv"].cuda()
    lin = lambda wt: types.SimpleNamespace(weight=wt, bias=None)  # noqa: E731
    q_rope, k_rope, v_out, q_n, k_n = m.fq.fused_qkv_gemm_rope(
        x, lin(w[:dim]), lin(w[dim:2 * dim]), lin(w[2 * dim:]), freqs.cuda(), inp["norm_wq"].cuda(),
        inp["norm_wk"].cuda(), H, 128, eps=1e-6, return_normed=True, fp8_weights=None, cos_sin=cos_sin)
    r = run_reference_tail(m, q_rope, k_rope, v_out, q_n, k_n, x, inp, wl, H, lr_tables,
                           heads=slice(0, C4_HEADS))
    return pack_result(wl, r, sample_tokens(L, tokens, seed), sums, {})


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPARKDIFFUSION_REF",
                                                              os.path.join(ROOT, "baseline", "_ref"))
    out_dir = sys.argv[2] if len(sys.argv) > 2 else os.path.join(ROOT, "gpurun_out")
    which = (sys.argv[3] if len(sys.argv) > 3 else "c2,c4,c5").split(",")
    if not os.path.isdir(os.path.join(ref, "sparkdiffusion")):
        raise SystemExit(f"reference package not found under {ref}")
    if not torch.cuda.is_available():
        raise SystemExit("needs a CUDA device (the reference's bf16 kernels are Triton GPU kernels)")
    os.makedirs(out_dir, exist_ok=True)
    torch.cuda.set_device(0)
    m = import_reference(ref)
    makers = {"c2": lambda: make_c2(m), "c4": lambda: make_c4(m),
              "c5": lambda: make_c4(m, C5, C5_TOKENS, 13)}
    with torch.no_grad():
        for name in which:
            t0 = time.time()
            fx = makers[name]()
            torch.save(fx, os.path.join(out_dir, f"ref_b200_{name}.pt"))
            print(f"{name} done in {time.time() - t0:.1f} s", flush=True)
            del fx
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
