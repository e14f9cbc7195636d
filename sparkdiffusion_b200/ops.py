"""Host-side ops of the B200 RoLa attention forward.

Two layers of API:

* ``rola_attention_core`` / ``rola_attention_from_qkv``: the fused B200 path
  used by the drop-in layer.  Activations stay token-major ``[B, L, H*D]``
  from the QKV GEMM to the gated output; the kernels gather per-head tiles
  with TMA, so no layout transform is ever materialised.
* reference-named functions mirroring ``sparkdiffusion.ops.fused_kernel``
  (``fused_qkv_gemm_rope``, ``mean_pool``, ``fused_sparse_attn``) with the
  reference's argument meaning, layouts and ``ValueError``s, so callers and
  tests written against the reference read the same.

Every function launches librola_b200 kernels on the current CUDA stream and
raises if the library is missing or the tensors are not on a CUDA device:
there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .rope import prepare_cos_sin

BF16 = torch.bfloat16
HEAD_DIM = 128
FUSED_SELECT_MAX_NB = 768  # up to this many key blocks the scores stay on chip (no scores buffer)


_SIDE: dict = {}


def _side_streams(dev) -> tuple:
    """Three side streams per device for the concurrent head-local branches: the
    low-rank C^T and q_lr at the lowest priority, the selection chain at the
    device's greatest priority (the hardware then dispatches its few,
    latency-bound CTAs ahead of the low-rank kernels' many queued ones)."""
    key = torch.device(dev).index if torch.device(dev).index is not None else torch.cuda.current_device()
    s = _SIDE.get(key)
    if s is None:
        least, greatest = torch.cuda.Stream.priority_range()
        s = _SIDE[key] = (torch.cuda.Stream(device=key, priority=least), torch.cuda.Stream(device=key, priority=least),
                          torch.cuda.Stream(device=key, priority=greatest))
    return s


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("sparkdiffusion_b200 ops run on CUDA tensors only (no CPU fallback)")
        if t.dtype not in (torch.bfloat16, torch.float32, torch.int32, torch.float8_e4m3fn):
            raise ValueError(f"unsupported dtype {t.dtype}")


def _bf16_vec(t: torch.Tensor, n: int, name: str) -> torch.Tensor:
    t = t.reshape(-1).to(BF16).contiguous()
    if t.numel() != n:
        raise ValueError(f"{name} must have {n} elements, got {t.numel()}")
    return t


def topk_count(topk_ratio: float, nb: int) -> int:
    """k = max(1, min(NB, int(ratio*NB))) (fused_sparse_attn.py:197)."""
    return max(1, min(nb, int(topk_ratio * nb)))


LOWRANK_CHUNK_TILES = 16  # 64-token tiles per fp32 partial of C (kKvChunk in csrc/kernels.h)


def lowrank_chunks(L: int) -> int:
    """Fp32 partials of the low-rank C reduction: one per 1024 tokens."""
    return ((L + 63) // 64 + LOWRANK_CHUNK_TILES - 1) // LOWRANK_CHUNK_TILES


def default_splits(B: int, H: int, L: int) -> int:
    """The C ABI's ``splits`` argument of the low-rank reduction (kept for ABI
    compatibility; the kernel is persistent and C follows fixed token chunks)."""
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return max(1, min(lowrank_chunks(L), (2 * sms) // (B * H)))


# ---------------------------------------------------------------------------
# fused B200 path
# ---------------------------------------------------------------------------
def qkv_gemm(x2d: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
             ssq: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = x[M, K] w[N, K]^T (+ bias) on tcgen05 (bf16 in/out, fp32 accumulate).
    ``ssq`` (fp32 ``[M, N/256]``) receives each row's sum of squares of its bf16
    outputs per 256-column tile.  ``out`` (contiguous bf16 ``[M, N]``) is
    written in place when given."""
    _require_cuda(x2d, w, bias)
    if x2d.dtype != BF16 or w.dtype != BF16:
        raise ValueError("qkv_gemm: bf16 operands required")
    x2d = x2d.contiguous()
    w = w.contiguous()
    M, K = x2d.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"qkv_gemm: weight {tuple(w.shape)} does not match x {tuple(x2d.shape)}")
    if out is None:
        out = torch.empty(M, N, device=x2d.device, dtype=BF16)
    elif out.shape != (M, N) or out.dtype != BF16 or not out.is_contiguous():
        raise ValueError("qkv_gemm: out must be a contiguous bf16 [M, N] tensor")
    b = None if bias is None else bias.to(BF16).contiguous()
    if ssq is not None and (ssq.dtype != torch.float32 or ssq.shape != (M, N // 256) or not ssq.is_contiguous()):
        raise ValueError("qkv_gemm: ssq must be a contiguous fp32 [M, N/256] tensor")
    _lib.call("rola_b200_qkv_gemm", _ptr(x2d), _ptr(w), _ptr(b), _ptr(out), _ptr(ssq), M, N, K, _stream())
    return out


def quantize_rows_e4m3(x2d: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Row-wise FP8 quantization of bf16 ``[M, K]`` (the reference's
    quantize_activation_rowwise / quantize_weight_rowwise,
    sparkdiffusion/ops/quantization/fp8_linear.py:45-61) -> ``(xq float8_e4m3fn
    [M, K], scale fp32 [M])`` with ``x ~= xq * scale[:, None]``."""
    _require_cuda(x2d)
    if x2d.dtype != BF16 or x2d.dim() != 2 or x2d.stride(1) != 1:
        raise ValueError("quantize_rows_e4m3: bf16 [M, K] rows with unit column stride required")
    M, K = x2d.shape
    xq = torch.empty(M, K, device=x2d.device, dtype=torch.float8_e4m3fn)
    scale = torch.empty(M, device=x2d.device, dtype=torch.float32)
    _lib.call("rola_b200_quantize_rows_e4m3", _ptr(x2d), x2d.stride(0), M, K, _ptr(xq), _ptr(scale), _stream())
    return xq, scale


def qkv_gemm_fp8(xq: torch.Tensor, x_scale: torch.Tensor, wq: torch.Tensor, w_scale: torch.Tensor,
                 bias: torch.Tensor | None = None, ssq: torch.Tensor | None = None) -> torch.Tensor:
    """``out[M, N] = bf16((xq . wq^T) * x_scale[:, None] * w_scale[None, :] + bias)`` on
    tcgen05 with e4m3 operands (the reference's FP8 prologue, torch._scaled_mm with
    row-wise scales, fused_qkv_rope.py:270-285).  ``ssq`` as in ``qkv_gemm``."""
    _require_cuda(xq, wq, x_scale, w_scale, bias)
    if xq.dtype != torch.float8_e4m3fn or wq.dtype != torch.float8_e4m3fn:
        raise ValueError("qkv_gemm_fp8: float8_e4m3fn operands required")
    M, K = xq.shape
    N = wq.shape[0]
    if wq.shape[1] != K:
        raise ValueError(f"qkv_gemm_fp8: weight {tuple(wq.shape)} does not match x {tuple(xq.shape)}")
    xs = x_scale.reshape(-1).to(torch.float32).contiguous()
    ws = w_scale.reshape(-1).to(torch.float32).contiguous()
    if xs.numel() != M or ws.numel() != N:
        raise ValueError("qkv_gemm_fp8: one scale per row of x and per output channel required")
    out = torch.empty(M, N, device=xq.device, dtype=BF16)
    b = None if bias is None else bias.to(BF16).contiguous()
    if ssq is not None and (ssq.dtype != torch.float32 or ssq.shape != (M, N // 256) or not ssq.is_contiguous()):
        raise ValueError("qkv_gemm_fp8: ssq must be a contiguous fp32 [M, N/256] tensor")
    _lib.call("rola_b200_qkv_gemm_fp8", _ptr(xq.contiguous()), _ptr(xs), _ptr(wq.contiguous()), _ptr(ws), _ptr(b),
              _ptr(out), _ptr(ssq), M, N, K, _stream())
    return out


def prequantize_qkv_weight(w_qkv: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """FP8 copy of the concatenated ``[Wq; Wk; Wv]`` with per-output-channel scales
    (quantize_weight_rowwise, fp8_linear.py:45-53) -> ``(w_fp8, w_scale [3*dim])``."""
    return quantize_rows_e4m3(w_qkv.to(BF16).contiguous())


def head_local_attention(q_rope, k_rope, q_normed, k_normed, v, gate, pooled_q, ksum, lr_cos, lr_sin, rope_dim,
                         proj_q, proj_k, num_heads: int, blk: int, topk: int, splits: int | None = None,
                         keep: bool = False, lut=None, events: dict | None = None, x=None, gate_w=None,
                         gate_b=None, scatter: dict | None = None):
    """Selection, low-rank branch and fused attention for ``num_heads`` heads
    over the full sequence.  q_rope/k_rope/q_normed/k_normed/v are token-major
    ``[B, L, H*D]`` (unit column stride; q/k tensors contiguous), pooled_q
    ``[B, H, NB, D]`` and ksum ``[B, NB, H*D]`` come from the prologue pass.  The
    gate is either given (``gate [B, L, H]``) or computed inside the attention
    epilogue from the hidden states ``x [B, L, H*D]`` with ``gate_w``/``gate_b``.
    Returns the gated output ``[B, L, H*D]``, or None with ``scatter``
    (``dst``: per-rank output pointers, ``world``, ``head_offset``, ``H_total``),
    which stores each output row straight into the rank owning its token
    (``rola_b200_sparse_attn_scatter``)."""
    B, L, dim = q_rope.shape
    H = num_heads
    dev = q_rope.device
    NB = (L + blk - 1) // blk
    R = proj_q.shape[0]
    splits = splits or default_splits(B, H, L)
    st = _stream()
    e = lambda *s, dt=BF16: torch.empty(*s, device=dev, dtype=dt)  # noqa: E731
    center = e(B, H, HEAD_DIM)
    pooled_k = e(B, H, NB, HEAD_DIM)
    q_lr = e(B, L, H * R)
    c_part = e(lowrank_chunks(L), B * H, R, HEAD_DIM, dt=torch.float32)
    C = e(B * H, R, HEAD_DIM) if keep else None
    Ct = e(B * H, HEAD_DIM, R)
    out = e(B, L, dim) if scatter is None else None
    o_sparse = e(B, L, dim) if keep else None
    scores = None
    # three independent branches run concurrently on side streams (each
    # under-fills the GPU on its own): the selection chain (queued first, high
    # priority), the low-rank C^T and q_lr; the attention waits for all three
    main = torch.cuda.current_stream(dev)
    s_kv, s_q, s_sel = _side_streams(dev)
    pq_, pk_ = proj_q.to(BF16).contiguous(), proj_k.to(BF16).contiguous()
    lc = None if lr_cos is None else lr_cos.to(BF16).contiguous()
    ls = None if lr_sin is None else lr_sin.to(BF16).contiguous()
    vs = v.stride()
    ks = k_normed.stride()
    qs = q_normed.stride()
    # fork once every input of the side branches (the conversions just queued
    # included) is on this stream
    s_kv.wait_stream(main)
    s_q.wait_stream(main)
    s_sel.wait_stream(main)
    for t in (center, pooled_k):
        t.record_stream(s_sel)
    lut_in = lut
    if lut is None:
        scores = e(B * H, NB, NB, dt=torch.float32) if NB > FUSED_SELECT_MAX_NB else None
        lut = e(B * H, NB, topk, dt=torch.int32)
        for t in (scores, lut):
            if t is not None:
                t.record_stream(s_sel)
    else:
        lut = lut.to(device=dev, dtype=torch.int32).reshape(B * H, NB, -1).contiguous()
        topk = lut.shape[-1]
    _lib.call("rola_b200_center_from_sums", _ptr(ksum), B, NB, dim, L, _ptr(center), s_sel.cuda_stream)
    _lib.call("rola_b200_mean_pool", _ptr(k_rope), L * dim, HEAD_DIM, dim, B, H, L, blk, _ptr(center),
              _ptr(pooled_k), s_sel.cuda_stream)
    if lut_in is None:
        _lib.call("rola_b200_block_select", _ptr(pooled_q), _ptr(pooled_k), B * H, NB, NB, topk, _ptr(scores),
                  _ptr(lut), s_sel.cuda_stream)
    for t in (pq_, pk_, lc, ls):
        if t is not None:
            t.record_stream(s_kv)
            t.record_stream(s_q)
    for t in (c_part, C, Ct):
        if t is not None:
            t.record_stream(s_kv)
    q_lr.record_stream(s_q)
    _lib.call("rola_b200_lowrank_kv", _ptr(k_normed), ks[0], HEAD_DIM, ks[1], _ptr(v), vs[0], HEAD_DIM, vs[1],
              _ptr(pk_), _ptr(lc), _ptr(ls), rope_dim, B, L, H, R, splits, _ptr(c_part), _ptr(C), _ptr(Ct),
              s_kv.cuda_stream)
    _lib.call("rola_b200_lowrank_q", _ptr(q_normed), qs[0], HEAD_DIM, qs[1], _ptr(pq_), _ptr(lc), _ptr(ls),
              rope_dim, B, L, H, R, _ptr(q_lr), s_q.cuda_stream)
    main.wait_stream(s_sel)
    main.wait_stream(s_kv)
    main.wait_stream(s_q)
    attn_lut = lut
    if blk == 64:
        # 128-row query tiles of two 64-token blocks: the union of their kept key
        # blocks with selection masks (rola_b200_pair_blocks)
        attn_lut = e(B * H, (NB + 1) // 2, 2 * topk + 1, dt=torch.int32)
        _lib.call("rola_b200_pair_blocks", _ptr(lut), B * H, NB, topk, _ptr(attn_lut), st)
    eps_lr = float(torch.finfo(BF16).eps)
    if events is not None:
        events["attn"][0].record()
    if x is not None:
        xs = x.stride()
        gw = _bf16_vec(gate_w, HEAD_DIM, "gate_w")
        gb = _bf16_vec(gate_b, H, "gate_b")
        gate = None
    else:
        xs, gw, gb = (0, 0, 0), None, None
    if scatter is not None:
        _lib.call("rola_b200_sparse_attn_scatter", _ptr(q_rope), _ptr(k_rope), L * dim, HEAD_DIM, dim, _ptr(v),
                  vs[0], HEAD_DIM, vs[1], _ptr(attn_lut), B, L, H, blk, topk, _ptr(q_lr), _ptr(Ct), _ptr(gate), eps_lr,
                  scatter["dst"], scatter["world"], scatter["head_offset"], scatter["H_total"], st)
    else:
        _lib.call("rola_b200_sparse_attn", _ptr(q_rope), _ptr(k_rope), L * dim, HEAD_DIM, dim, _ptr(v), vs[0],
                  HEAD_DIM, vs[1], _ptr(attn_lut), B, L, H, blk, topk, _ptr(q_lr), _ptr(Ct), _ptr(gate), _ptr(x),
                  xs[0], HEAD_DIM, xs[1], _ptr(gw), _ptr(gb), eps_lr, _ptr(out), _ptr(o_sparse), L * dim, HEAD_DIM,
                  dim, st)
    if events is not None:
        events["attn"][1].record()
    if not keep:
        return out
    return out, dict(pooled_k=pooled_k, center=center, scores=scores, lut=lut, q_lr=q_lr, C=C, Ct=Ct,
                     o_sparse=o_sparse)


def rola_attention_from_qkv(q_raw, k_raw, v_raw, x, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq, norm_wk,
                            proj_q, proj_k, gate_w, gate_b, num_heads: int, blk: int = 128, topk: int = 1,
                            eps: float = 1e-6, splits: int | None = None, keep: bool = False, lut=None,
                            events: dict | None = None, ssq: torch.Tensor | None = None):
    """RoLa forward from projected q/k/v (token-major ``[B, L, H*D]`` views
    with unit column stride; q and k share a row stride) to the gated output
    ``[B, L, H*D]``.  ``keep`` returns the intermediates too.  ``lut`` (int32
    ``[B*H, NB, k]``) replaces the kernel's own selection.  ``ssq`` are the QKV
    GEMM's per-tile sums of squares (``qkv_gemm``), which make the norm pass a
    pure stream.
    """
    _require_cuda(q_raw, k_raw, v_raw, x)
    B, L, dim = q_raw.shape
    H = num_heads
    if dim != H * HEAD_DIM:
        raise ValueError(f"hidden size {dim} != num_heads*128")
    if blk not in (64, 128):
        raise ValueError("the B200 attention kernel supports block sizes 64 and 128")
    for t in (q_raw, k_raw, v_raw):
        if t.stride(2) != 1:
            raise ValueError("q/k/v must have unit column stride")
    if q_raw.stride() != k_raw.stride():
        raise ValueError("q_raw and k_raw must share strides")
    dev = q_raw.device
    NB = (L + blk - 1) // blk
    if not 1 <= topk <= NB:
        raise ValueError(f"topk must be in [1, {NB}]")
    st = _stream()
    e = lambda *s, dt=BF16: torch.empty(*s, device=dev, dtype=dt)  # noqa: E731
    q_rope, k_rope = e(B, L, dim), e(B, L, dim)
    q_normed, k_normed = e(B, L, dim), e(B, L, dim)
    pooled_q = e(B, H, NB, HEAD_DIM)
    ksum = e(B, NB, dim, dt=torch.float32)
    nwq = None if norm_wq is None else _bf16_vec(norm_wq, dim, "norm_wq")
    nwk = None if norm_wk is None else _bf16_vec(norm_wk, dim, "norm_wk")
    cos_sin = cos_sin.to(torch.float32).contiguous()
    xc = x.contiguous()
    ssq_ld = 0 if ssq is None else ssq.shape[-1]
    # the gate values come out of the same streaming pass (it reads x beside q and k)
    gate = e(B, L, H)
    _lib.call("rola_b200_qk_norm_rope", _ptr(q_raw), _ptr(k_raw), q_raw.stride(1), _ptr(ssq), ssq_ld, _ptr(xc),
              _ptr(nwq), _ptr(nwk), _ptr(cos_sin), _ptr(_bf16_vec(gate_w, HEAD_DIM, "gate_w")),
              _ptr(_bf16_vec(gate_b, H, "gate_b")), B, L, H, blk, eps, _ptr(q_rope), _ptr(k_rope), _ptr(q_normed),
              _ptr(k_normed), _ptr(gate), _ptr(pooled_q), _ptr(ksum), st)
    res = head_local_attention(q_rope, k_rope, q_normed, k_normed, v_raw, gate, pooled_q, ksum, lr_cos, lr_sin,
                               rope_dim, proj_q, proj_k, H, blk, topk, splits, keep, lut, events)
    if not keep:
        return res
    out, extra = res
    extra.update(q_rope=q_rope, k_rope=k_rope, q_normed=q_normed, k_normed=k_normed, pooled_q=pooled_q, ksum=ksum,
                 v=v_raw, gate=gate)
    return out, extra


def rola_attention_core(x, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq, norm_wk, proj_q, proj_k,
                        gate_w, gate_b, num_heads: int, blk: int = 128, topk: int = 1, eps: float = 1e-6,
                        splits: int | None = None, keep: bool = False, events: dict | None = None,
                        w_scale: torch.Tensor | None = None):
    """RoLa forward from hidden states ``x [B, L, H*D]`` up to (excluding) the
    output projection: ``WanSelfAttentionRoLa.fused_forward`` minus ``self.o``
    (sparkdiffusion/networks/wan_rola_attention.py:414-446).  ``w_qkv`` is the
    concatenated ``[Wq; Wk; Wv]`` of shape ``[3*dim, dim]``: bf16, or float8_e4m3fn
    with per-output-channel scales ``w_scale [3*dim]`` (the reference's FP8 mode:
    the hidden states are quantized per token once for all three projections,
    fused_qkv_rope.py:270-285)."""
    B, L, dim = x.shape
    ssq = torch.empty(B * L, 3 * dim // 256, device=x.device, dtype=torch.float32)
    if events is not None:
        events["gemm"][0].record()
    if w_scale is not None:
        xq, xs = quantize_rows_e4m3(x.reshape(B * L, dim))
        qkv = qkv_gemm_fp8(xq, xs, w_qkv, w_scale, b_qkv, ssq).view(B, L, 3 * dim)
    else:
        qkv = qkv_gemm(x.reshape(B * L, dim), w_qkv, b_qkv, ssq).view(B, L, 3 * dim)
    if events is not None:
        events["gemm"][1].record()
    res = rola_attention_from_qkv(qkv[..., :dim], qkv[..., dim:2 * dim], qkv[..., 2 * dim:], x, cos_sin, lr_cos,
                                  lr_sin, rope_dim, norm_wq, norm_wk, proj_q, proj_k, gate_w, gate_b, num_heads,
                                  blk, topk, eps, splits, keep, events=events, ssq=ssq)
    if keep:
        out, extra = res
        extra["qkv"] = qkv
        return out, extra
    return res


def rola_forward_capi(x, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq, norm_wk, proj_q, proj_k,
                      gate_w, gate_b, num_heads: int, topk: int, eps: float = 1e-6, splits: int | None = None,
                      workspace: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """Same forward through the single C entry point ``rola_b200_rola_forward``."""
    B, L, dim = x.shape
    H = num_heads
    R = proj_q.shape[0]
    splits = splits or default_splits(B, H, L)
    need = _lib.lib().rola_b200_forward_workspace_bytes(B, L, H, 128, R, splits)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=x.device, dtype=torch.uint8)
    if out is None:
        out = torch.empty(B, L, dim, device=x.device, dtype=BF16)
    _lib.call("rola_b200_rola_forward", _ptr(x), _ptr(w_qkv), _ptr(b_qkv), _ptr(_bf16_vec(norm_wq, dim, "norm_wq")),
              _ptr(_bf16_vec(norm_wk, dim, "norm_wk")), _ptr(cos_sin), _ptr(lr_cos), _ptr(lr_sin), rope_dim,
              _ptr(proj_q), _ptr(proj_k), _ptr(_bf16_vec(gate_w, HEAD_DIM, "gate_w")),
              _ptr(_bf16_vec(gate_b, H, "gate_b")), B, L, H, 128, topk, R, splits, eps, _ptr(workspace), need,
              _ptr(out), None, _stream())
    return out


class ForwardPipeline:
    """Host-buffer forward through ``rola_b200_pipeline_forward``: every call
    uploads pinned ``x_host [B, L, dim]``, runs the forward and downloads into
    pinned ``out_host``; consecutive calls overlap uploads and downloads with
    the previous / next step's kernels.  ``wait()`` orders the current stream
    after every submitted step."""

    def __init__(self, x_bytes: int, out_bytes: int):
        self._lib = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(self._lib.rola_b200_pipeline_create(x_bytes, out_bytes, ctypes.byref(h)),
                   "rola_b200_pipeline_create")
        self._h = h
        self._ws = None

    def forward(self, x_host, out_host, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq, norm_wk, proj_q,
                proj_k, gate_w, gate_b, num_heads: int, topk: int, eps: float = 1e-6, splits: int | None = None):
        if not (x_host.is_pinned() and out_host.is_pinned()):
            raise ValueError("ForwardPipeline: x_host and out_host must be pinned host tensors")
        B, L, dim = x_host.shape
        H = num_heads
        R = proj_q.shape[0]
        splits = splits or default_splits(B, H, L)
        need = self._lib.rola_b200_forward_workspace_bytes(B, L, H, 128, R, splits)
        dev = w_qkv.device
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, device=dev, dtype=torch.uint8)
        _lib.call("rola_b200_pipeline_forward", self._h, _ptr(x_host), _ptr(w_qkv), _ptr(b_qkv),
                  _ptr(_bf16_vec(norm_wq, dim, "norm_wq")), _ptr(_bf16_vec(norm_wk, dim, "norm_wk")), _ptr(cos_sin),
                  _ptr(lr_cos), _ptr(lr_sin), rope_dim, _ptr(proj_q), _ptr(proj_k),
                  _ptr(_bf16_vec(gate_w, HEAD_DIM, "gate_w")), _ptr(_bf16_vec(gate_b, H, "gate_b")), B, L, H, 128,
                  topk, R, splits, eps, _ptr(self._ws), need, _ptr(out_host), _stream())

    def wait(self) -> None:
        _lib.call("rola_b200_pipeline_wait", self._h, _stream())

    def close(self) -> None:
        if self._h is not None:
            _lib.call("rola_b200_pipeline_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# reference-named API (sparkdiffusion.ops.fused_kernel)
# ---------------------------------------------------------------------------
def mean_pool(x: torch.Tensor, BLK: int, *, center: torch.Tensor | None = None) -> torch.Tensor:
    """Block mean pooling of ``x [B, H, L, D]`` -> ``[B, H, NB, D]``
    (sparkdiffusion/ops/fused_kernel/utils.py:57-82)."""
    _require_cuda(x, center)
    B, H, L, D = x.shape
    if D != HEAD_DIM:
        raise ValueError("head dim must be 128")
    if center is not None:
        if center.shape != (B, H, D):
            raise ValueError(f"center must have shape {(B, H, D)}, got {tuple(center.shape)}")
        if center.device != x.device or center.dtype != x.dtype:
            raise ValueError("center must have the same device and dtype as x")
        center = center.contiguous()
    if x.dtype != BF16:
        raise ValueError("mean_pool: bf16 input required")
    if x.stride(3) != 1:
        x = x.contiguous()
    NB = (L + BLK - 1) // BLK
    out = torch.empty(B, H, NB, D, device=x.device, dtype=x.dtype)
    sB, sH, sT, _ = x.stride()
    _lib.call("rola_b200_mean_pool", _ptr(x), sB, sH, sT, B, H, L, BLK, _ptr(center), _ptr(out), _stream())
    return out


def smooth_k_center(k4: torch.Tensor, blk: int) -> torch.Tensor:
    """Smooth-K centre ``k.mean(dim=-2)`` of ``k [B, H, L, D]`` -> ``[B, H, D]``."""
    _require_cuda(k4)
    B, H, L, D = k4.shape
    NB = (L + blk - 1) // blk
    ws = torch.empty(B, NB, H * D, device=k4.device, dtype=torch.float32)
    c = torch.empty(B, H, D, device=k4.device, dtype=BF16)
    sB, sH, sT, _ = k4.stride()
    _lib.call("rola_b200_smooth_k_center", _ptr(k4), sB, sH, sT, B, H, L, blk, _ptr(ws), _ptr(c), _stream())
    return c


def block_select(pooled_q: torch.Tensor, pooled_k: torch.Tensor, topk: int) -> torch.Tensor:
    """fp32 pooled scores + top-k (ties toward the lower index), int32 ascending
    ``[B*H, NBq, topk]``."""
    _require_cuda(pooled_q, pooled_k)
    B, H, NBq, D = pooled_q.shape
    NBk = pooled_k.shape[2]
    pq, pk = pooled_q.contiguous(), pooled_k.contiguous()
    scores = (torch.empty(B * H, NBq, NBk, device=pq.device, dtype=torch.float32)
              if NBk > FUSED_SELECT_MAX_NB else None)
    lut = torch.empty(B * H, NBq, topk, device=pq.device, dtype=torch.int32)
    _lib.call("rola_b200_block_select", _ptr(pq), _ptr(pk), B * H, NBq, NBk, topk, _ptr(scores), _ptr(lut),
              _stream())
    return lut


def fused_sparse_attn(q, k, v, topk_ratio: float = 0.1, blkq: int = 64, blkk: int = 64, num_heads=None,
                      force_local_sink: bool = False):
    """Block-sparse attention over ``q, k, v [B*H, L, D]`` (already normed and
    roped) -> ``[B, H, L, D]`` (sparkdiffusion/ops/fused_kernel/fused_sparse_attn.py:151-215).

    Selection uses the build's contract (fp32 scores, lower-index ties, LUT
    ascending).  ``force_local_sink`` is not supported (off in the reference)."""
    BH, L, D = q.shape
    if num_heads is None or BH % num_heads != 0:
        raise ValueError(f"invalid num_heads={num_heads} for leading dimension {BH}")
    if force_local_sink:
        raise ValueError("force_local_sink is not supported by the B200 path")
    if blkq != blkk or blkq not in (64, 128):
        raise ValueError("the B200 attention kernel supports blkq == blkk in (64, 128)")
    _require_cuda(q, k, v)
    H = num_heads
    B = BH // H
    q4, k4, v4 = (t.view(B, H, L, D).contiguous() for t in (q, k, v))
    NB = (L + blkq - 1) // blkq
    topk = topk_count(topk_ratio, NB)
    pq = mean_pool(q4, blkq)
    pk = mean_pool(k4, blkk, center=smooth_k_center(k4, blkk))
    lut = block_select(pq, pk, topk)
    if blkq == 64:
        paired = torch.empty(B * H, (NB + 1) // 2, 2 * topk + 1, device=q.device, dtype=torch.int32)
        _lib.call("rola_b200_pair_blocks", _ptr(lut), B * H, NB, topk, _ptr(paired), _stream())
        lut = paired
    o = torch.empty_like(v4)
    s = q4.stride()
    vs = v4.stride()
    _lib.call("rola_b200_sparse_attn", _ptr(q4), _ptr(k4), s[0], s[1], s[2], _ptr(v4), vs[0], vs[1], vs[2],
              _ptr(lut), B, L, H, blkq, topk, None, None, None, None, 0, 0, 0, None, None, 0.0, None, _ptr(o), s[0],
              s[1], s[2], _stream())
    return o


_FULL_LUT: dict = {}


def _full_lut(BH: int, NB: int, dev) -> torch.Tensor:
    """LUT that keeps every key block of every query block, ascending (dense attention)."""
    key = (BH, NB, str(dev))
    lut = _FULL_LUT.get(key)
    if lut is None:
        lut = torch.arange(NB, device=dev, dtype=torch.int32).expand(BH, NB, NB).contiguous()
        _FULL_LUT[key] = lut
    return lut


def dense_attention_strided(q, k, v, B: int, L: int, H: int, qk_strides, v_strides, out, o_strides) -> None:
    """Dense softmax attention through the block-sparse kernel with every key
    block selected (the reference's dense path runs SDPA / flash attention after
    the same prologue, sparkdiffusion/networks/wan2pt1.py:282-320).  Element
    (b, h, t, d) of each tensor at ``base + sB*b + sH*h + sT*t + d``."""
    NB = (L + 127) // 128
    lut = _full_lut(B * H, NB, q.device)
    _lib.call("rola_b200_sparse_attn", _ptr(q), _ptr(k), *qk_strides, _ptr(v), *v_strides, _ptr(lut), B, L, H, 128,
              NB, None, None, None, None, 0, 0, 0, None, None, 0.0, None, _ptr(out), *o_strides, _stream())


def dense_attention(q, k, v, num_heads: int):
    """Dense attention over ``q, k, v [B*H, L, D]`` (normed and roped, the
    layouts ``fused_qkv_gemm_rope`` returns) -> ``[B, H, L, D]``; the reference
    computes it with its attention op after the fused prologue
    (sparkdiffusion/networks/wan2pt1.py:282-320)."""
    BH, L, D = q.shape
    if num_heads <= 0 or BH % num_heads != 0:
        raise ValueError(f"invalid num_heads={num_heads} for leading dimension {BH}")
    if D != HEAD_DIM:
        raise ValueError("head dim must be 128")
    _require_cuda(q, k, v)
    H = num_heads
    B = BH // H
    q4, k4, v4 = (t.view(B, H, L, D).contiguous() for t in (q, k, v))
    o = torch.empty_like(v4)
    s, vs = q4.stride(), v4.stride()
    dense_attention_strided(q4, k4, v4, B, L, H, (s[0], s[1], s[2]), (vs[0], vs[1], vs[2]), o, (s[0], s[1], s[2]))
    return o


def fused_qkv_gemm_rope(x, q_proj, k_proj, v_proj, freqs, norm_q_weight, norm_k_weight, num_heads, head_dim,
                        eps: float = 1e-6, return_normed: bool = False, fp8_weights=None, cos_sin=None):
    """QKV projection + full-width qk-RMSNorm + interleaved RoPE
    (sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:228-333).  Returns q, k,
    v as ``[B*H, L, D]`` (and q/k normed ``[B, L, H, D]``), the reference's layouts."""
    if head_dim != HEAD_DIM:
        raise ValueError("head_dim must be 128")
    B, L, dim = x.shape
    H = num_heads
    bias = None
    if q_proj.bias is not None:
        bias = torch.cat([q_proj.bias, k_proj.bias, v_proj.bias], 0).to(BF16)
    ssq = torch.empty(B * L, 3 * dim // 256, device=x.device, dtype=torch.float32) if H % 2 == 0 else None
    if fp8_weights is not None:
        # {'q'|'k'|'v': (w_fp8 [dim, dim], w_scale_t [1, dim])} from the reference's prequantize_qkv:
        # one activation quantization shared by the three projections (fused_qkv_rope.py:270-285)
        w8 = torch.cat([fp8_weights[n][0].view(torch.uint8) for n in ("q", "k", "v")], 0).view(torch.float8_e4m3fn)
        ws = torch.cat([fp8_weights[n][1].reshape(-1) for n in ("q", "k", "v")], 0)
        xq, xs = quantize_rows_e4m3(x.reshape(B * L, dim).to(BF16).contiguous())
        qkv = qkv_gemm_fp8(xq, xs, w8, ws, bias, ssq).view(B, L, 3 * dim)
    else:
        w = torch.cat([q_proj.weight, k_proj.weight, v_proj.weight], 0).to(BF16)
        qkv = qkv_gemm(x.reshape(B * L, dim), w, bias, ssq).view(B, L, 3 * dim)
    if cos_sin is None:
        cos_sin = prepare_cos_sin(freqs, L, head_dim)
    e = lambda: torch.empty(B, L, dim, device=x.device, dtype=BF16)  # noqa: E731
    q_rope, k_rope, q_n, k_n = e(), e(), e(), e()
    has_norm = norm_q_weight is not None and norm_k_weight is not None
    nwq = _bf16_vec(norm_q_weight, dim, "norm_q_weight") if has_norm else None
    nwk = _bf16_vec(norm_k_weight, dim, "norm_k_weight") if has_norm else None
    _lib.call("rola_b200_qk_norm_rope", _ptr(qkv), _ptr(qkv[..., dim:]), 3 * dim, _ptr(ssq if has_norm else None),
              0 if ssq is None else ssq.shape[-1], None, _ptr(nwq), _ptr(nwk),
              _ptr(cos_sin.to(torch.float32).contiguous()), None, None, B, L, H, 128, eps, _ptr(q_rope),
              _ptr(k_rope), _ptr(q_n), _ptr(k_n), None, None, None, _stream())

    def bhld(t):
        return t.view(B, L, H, head_dim).permute(0, 2, 1, 3).reshape(B * H, L, head_dim)

    outs = (bhld(q_rope), bhld(k_rope), bhld(qkv[..., 2 * dim:]))
    if return_normed:
        return (*outs, q_n.view(B, L, H, head_dim), k_n.view(B, L, H, head_dim))
    return outs


# ---------------------------------------------------------------------------
# training: block-sparse attention forward with the row log-sum-exp, backward
# ---------------------------------------------------------------------------
def _head_view_ok(t: torch.Tensor) -> bool:
    """``[B, H, L, 128]`` view the kernels can map: unit d stride, 16-byte rows."""
    return (t.dim() == 4 and t.shape[-1] == HEAD_DIM and t.stride(3) == 1 and t.data_ptr() % 16 == 0
            and all(s % 8 == 0 for s in t.stride()[:3]))


def _token_major(t: torch.Tensor) -> torch.Tensor:
    """``[B, H, L, D]`` view of a contiguous ``[B, L, H, D]`` copy of ``t``."""
    return t.transpose(1, 2).contiguous().transpose(1, 2)


def lse_rows(L: int) -> int:
    """Row stride of the ``lse`` table: L rounded up to whole 128-row tiles."""
    return 128 * ((L + 127) // 128)


def sparse_attention_fwd_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lut: torch.Tensor, blk: int,
                             topk: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Block-sparse attention over ``q, k, v [B, H, L, 128]`` (bf16) with the
    selection ``lut`` (block 128: ``[B*H, NB, topk]``; block 64: the paired
    table of ``rola_b200_pair_blocks``).  Returns ``(o [B, H, L, 128]`` (a view
    of a token-major ``[B, L, H, 128]`` tensor), ``lse [B*H, Lpad]`` fp32)``."""
    _require_cuda(q, k, v, lut)
    if not (q.dtype == k.dtype == v.dtype == BF16):
        raise ValueError("sparse_attention_fwd_lse: bf16 q, k, v required")
    B, H, L, D = q.shape
    if k.shape != q.shape or v.shape != q.shape or D != HEAD_DIM:
        raise ValueError("sparse_attention_fwd_lse: q, k, v must all be [B, H, L, 128]")
    if not (_head_view_ok(q) and _head_view_ok(k) and q.stride() == k.stride()):
        q, k = _token_major(q), _token_major(k)
    if not _head_view_ok(v):
        v = _token_major(v)
    o = torch.empty(B, L, H, D, device=q.device, dtype=BF16).transpose(1, 2)
    lse = torch.empty(B * H, lse_rows(L), device=q.device, dtype=torch.float32)
    lut = lut.contiguous()
    _lib.call("rola_b200_sparse_attn_fwd_lse", _ptr(q), _ptr(k), *q.stride()[:3], _ptr(v), *v.stride()[:3],
              _ptr(lut), B, L, H, blk, topk, _ptr(o), *o.stride()[:3], _ptr(lse), _stream())
    return o, lse


def sparse_attention_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, do: torch.Tensor,
                         lut: torch.Tensor, paired: torch.Tensor | None, lse: torch.Tensor, blk: int,
                         topk: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients ``(dq, dk, dv)`` ``[B, H, L, 128]`` bf16 of
    ``sparse_attention_fwd_lse`` given ``do = dL/do``; ``lut`` is the selection
    ``[B*H, NB, topk]`` and ``paired`` its block-64 pairing (the forward's lut;
    None for block 128)."""
    _require_cuda(q, k, v, o, do, lut, paired, lse)
    B, H, L, D = q.shape
    if not (_head_view_ok(q) and _head_view_ok(k) and q.stride() == k.stride()):
        q, k = _token_major(q), _token_major(k)
    if not _head_view_ok(v):
        v = _token_major(v)
    if not _head_view_ok(o):
        raise ValueError("sparse_attention_bwd: o must be the forward's output")
    do = do.to(BF16)
    if do.stride() != o.stride() or do.data_ptr() % 16:
        d2 = torch.empty_like(o)
        d2.copy_(do)
        do = d2
    g = torch.empty(3, B, L, H, D, device=q.device, dtype=BF16)
    dq, dk, dv = (g[i].transpose(1, 2) for i in range(3))
    ws_bytes = _lib.lib().rola_b200_sparse_attn_bwd_workspace(B, L, H, blk)
    if ws_bytes == 0:
        raise ValueError("sparse_attention_bwd: bad sizes")
    ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
    _lib.call("rola_b200_sparse_attn_bwd", _ptr(q), _ptr(k), *q.stride()[:3], _ptr(v), *v.stride()[:3], _ptr(o),
              _ptr(do), *o.stride()[:3], _ptr(lut.contiguous()), _ptr(None if paired is None else paired.contiguous()),
              _ptr(lse), B, L, H, blk, topk, _ptr(dq), _ptr(dk), _ptr(dv), *dq.stride()[:3], _ptr(ws), ws_bytes,
              _stream())
    return dq, dk, dv
