"""Ulysses sequence<->head parallel RoLa attention across GPUs (NCCL).

The layer's input arrives sequence-sharded: rank r holds tokens
[r*Ls, (r+1)*Ls) of every head (Ls = L / p).  The qk-RMSNorm couples all heads
of a token (sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:146-149), so

1. the QKV GEMM, the qk-RMSNorm and the gate run on the sequence shard, the
   norm pass writing q_normed, k_normed, v and the gate straight into
   per-destination send blocks ``[B][p][Ls][Hl*D]`` (Hl = H / p);
2. one all-to-all per tensor (per batch element) moves them to head shards:
   rank r now holds heads [r*Hl, (r+1)*Hl) of the whole sequence;
3. RoPE (global positions), pooling, selection, the low-rank branch and the
   fused block-sparse attention run head-local over the full sequence;
4. an all-to-all sends each rank's output rows back to their sequence owner,
   which interleaves the head groups into ``[B, Ls, H*D]``.

This follows the reference's DistributedAttention pattern
(sparkdiffusion/utils/a2a_cp.py:146-186) but applies it to RoLa, so the
multi-GPU result equals the single-GPU one (the reference's own context
parallel RoLa attends only within each rank's shard).

Two transports carry steps 2 and 4:

* ``"peer"`` (default): the exchanges are fused into the kernels.  The norm
  pass stores each head group's rows straight into the owning rank's buffers
  (``rola_b200_qk_norm_scatter``) and the attention epilogue stores each output
  row into the buffer of the rank that owns its token
  (``rola_b200_sparse_attn_scatter``); the buffers are CUDA-IPC peer mappings
  (``peer.PeerBuffer``) and a stream-ordered barrier follows each scatter.  No
  all-to-all, send buffer or output permutation is left.
* ``"nccl"``: send buffers plus NCCL ``all_to_all_single`` (the reference's
  pattern), kept as the comparison point.

``seq_to_head`` / ``head_to_seq`` are device-agnostic (they also run on gloo
CPU ranks in the tests); ``ulysses_rola_attention`` runs the CUDA kernels.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops, peer
from .ops import BF16, HEAD_DIM, _bf16_vec, _ptr, _stream


def seq_to_head(send: torch.Tensor, group=None, async_op: bool = False):
    """``send [B, p, Ls, X]`` (block j goes to rank j) -> ``recv [B, p, Ls, X]``
    whose block i came from rank i, i.e. ``[B, L, X]`` in global token order."""
    recv = torch.empty_like(send)
    works = [dist.all_to_all_single(recv[b], send[b], group=group, async_op=async_op) for b in range(send.shape[0])]
    return recv, works


def head_to_seq(out_heads: torch.Tensor, p: int, group=None) -> torch.Tensor:
    """``out_heads [B, L, X]`` (this rank's head group, all tokens) ->
    ``[B, Ls, p*X]``: this rank's tokens with the p head groups side by side."""
    B, L, X = out_heads.shape
    Ls = L // p
    send = out_heads.contiguous().view(B, p, Ls, X)
    recv = torch.empty_like(send)
    for b in range(B):
        dist.all_to_all_single(recv[b], send[b], group=group)
    return recv.permute(0, 2, 1, 3).reshape(B, Ls, p * X)


def _peer_layout(B: int, Ls: int, H: int, p: int) -> dict:
    L, Hl = Ls * p, H // p
    return {"q": ((B, L, Hl * HEAD_DIM), BF16), "k": ((B, L, Hl * HEAD_DIM), BF16),
            "v": ((B, L, Hl * HEAD_DIM), BF16), "gate": ((B, L, Hl), BF16),
            "out0": ((B, Ls, H * HEAD_DIM), BF16), "out1": ((B, Ls, H * HEAD_DIM), BF16)}


_out_slot: dict = {}


def _scatter_args(qkv, ssq, xc, nwq, nwk, gw, gb, H, p, L, eps, buf, b, r0, t0, t1):
    """rola_scatter_args of tokens [t0, t1) of batch b (rows r0.. of qkv) into
    rows rank*Ls + t0.. of every rank's head buffers (buf)."""
    dim = H * HEAD_DIM
    Hl = H // p
    a = _lib.ScatterArgs()
    a.q_raw, a.k_raw, a.v_raw = _ptr(qkv[r0]), _ptr(qkv[r0, dim:]), _ptr(qkv[r0, 2 * dim:])
    a.ld_raw = 3 * dim
    a.ssq, a.ssq_ld = _ptr(ssq[r0]), ssq.shape[-1]
    a.B, a.L, a.H, a.world, a.eps = 1, t1 - t0, H, p, eps
    a.dst_rows, a.dst_row0 = L, t0
    a.x = _ptr(xc[r0])
    a.norm_wq, a.norm_wk, a.gate_w, a.gate_b = _ptr(nwq), _ptr(nwk), _ptr(gw), _ptr(gb)
    boff = b * L * Hl * HEAD_DIM * 2
    goff = b * L * Hl * 2
    for name, field, off in (("q", "q_dst", boff), ("k", "k_dst", boff), ("v", "v_dst", boff),
                             ("gate", "g_dst", goff)):
        tab = getattr(a, field)
        for r, ptr in enumerate(buf.region(name).table):
            tab[r] = ptr + off
    return a


def chunk_plan(rows: int, n_tiles: int, sms: int, chunks: int | None = None) -> list[int]:
    """Token-chunk sizes of the GEMM / scatter overlap.  ``chunks`` given: equal
    chunks of whole 128-row tiles.  Otherwise a halving sequence (each chunk's
    GEMM hides the previous chunk's scatter; the last, exposed one is small) of
    sizes whose ``m_tiles * n_tiles`` output tiles fill the ``sms`` persistent
    CTAs in whole waves where possible."""
    m_tiles = -(-rows // 128)
    if chunks is not None:
        step = -(-m_tiles // max(1, chunks))
        sizes = [step] * (m_tiles // step) + ([m_tiles % step] if m_tiles % step else [])
    else:
        def eff(s):
            t = s * n_tiles
            return t / (-(-t // sms) * sms)

        sizes, left = [], m_tiles
        while left > 8:
            target = left // 2
            s = max(range(max(1, (3 * target) // 4), target + 1), key=lambda c: (round(eff(c), 2), c))
            sizes.append(s)
            left -= s
        if left:
            sizes.append(left)
    out, start = [], 0
    for s in sizes:
        n = min(rows - start, s * 128)
        if n > 0:
            out.append(n)
            start += n
    return out


def _gemm_scatter_overlapped(x_local, w_qkv, b_qkv, nwq, nwk, gw, gb, xc, H, p, rank, eps, buf, chunks, events):
    """QKV GEMM and the scattering norm pass in token chunks: the persistent
    GEMM of chunk c carries the scatter of chunk c-1 on spare warps
    (rola_b200_qkv_gemm_scatter), so the NVLink traffic hides under the
    tensor-core work; the last chunk's scatter runs on its own."""
    B, Ls, dim = x_local.shape
    dev = x_local.device
    st = _stream()
    L = Ls * p
    x2d = x_local.reshape(B * Ls, dim)
    xc2 = xc.view(B * Ls, dim)
    qkv = torch.empty(B * Ls, 3 * dim, device=dev, dtype=BF16)
    ssq = torch.empty(B * Ls, 3 * dim // 256, device=dev, dtype=torch.float32)
    bias = None if b_qkv is None else b_qkv.to(BF16).contiguous()
    w = w_qkv.contiguous()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    plan = chunk_plan(Ls, 3 * dim // 256, sms, chunks)
    if events is not None:
        events["gemm"][0].record()
    prev = None
    for b in range(B):
        t1 = 0
        for n in plan:
            t0, t1 = t1, t1 + n
            r0, r1 = b * Ls + t0, b * Ls + t1
            if prev is None:
                # the first chunk on the single-SM kernel too (side job NULL): every chunk of
                # the overlapped exchange runs on one GEMM kernel
                _lib.call("rola_b200_qkv_gemm_scatter", _ptr(x2d[r0]), _ptr(w), _ptr(bias), _ptr(qkv[r0]),
                          _ptr(ssq[r0]), r1 - r0, 3 * dim, dim, None, st)
            else:
                _lib.call("rola_b200_qkv_gemm_scatter", _ptr(x2d[r0]), _ptr(w), _ptr(bias), _ptr(qkv[r0]),
                          _ptr(ssq[r0]), r1 - r0, 3 * dim, dim, ctypes.byref(prev), st)
            prev = _scatter_args(qkv, ssq, xc2, nwq, nwk, gw, gb, H, p, L, eps, buf, b, r0, rank * Ls + t0,
                                 rank * Ls + t1)
    _lib.call("rola_b200_qk_norm_scatter", ctypes.byref(prev), 0, st)
    if events is not None:
        events["gemm"][1].record()


def ulysses_rola_attention_params(x_local, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, norm_wq, norm_wk,
                                  proj_q, proj_k, gate_w, gate_b, num_heads: int, topk: int, group=None,
                                  eps: float = 1e-6, splits: int | None = None, events: dict | None = None,
                                  transport: str = "peer", chunks: int | None = None, record: dict | None = None,
                                  blk: int = 128):
    """Sequence-sharded RoLa forward: ``x_local [B, Ls, H*D]`` on this rank ->
    ``[B, Ls, H*D]`` (excluding the output projection).  ``cos_sin`` and the
    low-rank tables cover the whole sequence (global positions).

    With ``transport="peer"`` the result is a view of one of two alternating
    peer-mapped output buffers: it stays valid until the second-next call with
    the same shapes and group, and consumers must run on the current stream.
    The peer transport overlaps the QKV GEMM with the scattering norm pass in
    token chunks (``chunk_plan``; ``chunks`` forces that many equal chunks,
    1 turns the overlap off).  ``record`` (a dict) receives this rank's LUT
    (``lut``, int32 ``[B*Hl, NB, k]`` of heads ``rank*Hl ...``).  ``blk``: the
    selection block size (128 or 64)."""
    if transport not in ("peer", "nccl"):
        raise ValueError(f"unknown transport {transport!r}")
    p = dist.get_world_size(group)
    B, Ls, dim = x_local.shape
    H = num_heads
    if H % p != 0:
        raise ValueError(f"num_heads={H} must be divisible by the sequence-parallel size {p}")
    Hl = H // p
    L = Ls * p
    if cos_sin.shape[0] < L:
        raise ValueError("cos_sin must cover the full (global) sequence")
    dev = x_local.device
    st = _stream()
    gw = _bf16_vec(gate_w, HEAD_DIM, "gate_w")
    gb = _bf16_vec(gate_b, H, "gate_b")
    nwq = _bf16_vec(norm_wq, dim, "norm_wq")
    nwk = _bf16_vec(norm_wk, dim, "norm_wk")
    xc = x_local.contiguous()
    rank = dist.get_rank(group)
    if transport == "peer":
        key = ("ulysses", B, Ls, H, str(dev))
        buf = peer.cached_buffer(key, _peer_layout(B, Ls, H, p), group)
        rq, rk, rv, rg = (buf.region(n) for n in ("q", "k", "v", "gate"))
        if chunks is None or chunks > 1:
            _gemm_scatter_overlapped(x_local, w_qkv, b_qkv, nwq, nwk, gw, gb, xc, H, p, rank, eps, buf, chunks,
                                     events)
        else:
            ssq = torch.empty(B * Ls, 3 * dim // 256, device=dev, dtype=torch.float32)
            if events is not None:
                events["gemm"][0].record()
            qkv = ops.qkv_gemm(x_local.reshape(B * Ls, dim), w_qkv, b_qkv, ssq)
            if events is not None:
                events["gemm"][1].record()
            a = _scatter_args(qkv, ssq, xc.view(B * Ls, dim), nwq, nwk, gw, gb, H, p, L, eps, buf, 0, 0,
                              rank * Ls, rank * Ls + Ls)
            a.B = B
            _lib.call("rola_b200_qk_norm_scatter", ctypes.byref(a), 0, st)
        peer.stream_barrier(group)
        q_n, k_n, v, gate = rq.tensor, rk.tensor, rv.tensor, rg.tensor
    else:
        ssq = torch.empty(B * Ls, 3 * dim // 256, device=dev, dtype=torch.float32)
        if events is not None:
            events["gemm"][0].record()
        qkv = ops.qkv_gemm(x_local.reshape(B * Ls, dim), w_qkv, b_qkv, ssq)
        if events is not None:
            events["gemm"][1].record()
        q_send = torch.empty(B, p, Ls, Hl * HEAD_DIM, device=dev, dtype=BF16)
        k_send = torch.empty_like(q_send)
        v_send = torch.empty_like(q_send)
        g_send = torch.empty(B, p, Ls, Hl, device=dev, dtype=BF16)
        _lib.call("rola_b200_qk_norm_pack", _ptr(qkv), _ptr(qkv[:, dim:]), _ptr(qkv[:, 2 * dim:]), 3 * dim,
                  _ptr(ssq), ssq.shape[-1], _ptr(xc), _ptr(nwq), _ptr(nwk), _ptr(gw), _ptr(gb), B, Ls, H, Hl, eps,
                  _ptr(q_send), _ptr(k_send), _ptr(v_send), _ptr(g_send), st)
        q_n, w1 = seq_to_head(q_send, group, async_op=True)
        k_n, w2 = seq_to_head(k_send, group, async_op=True)
        v, w3 = seq_to_head(v_send, group, async_op=True)
        gate, w4 = seq_to_head(g_send, group, async_op=True)
        for w in (*w1, *w2, *w3, *w4):
            w.wait()
        q_n = q_n.view(B, L, Hl * HEAD_DIM)
        k_n = k_n.view(B, L, Hl * HEAD_DIM)
        v = v.view(B, L, Hl * HEAD_DIM)
        gate = gate.view(B, L, Hl)
    if blk not in (64, 128):
        raise ValueError("block size must be 64 or 128")
    NB = (L + blk - 1) // blk
    q_rope = torch.empty_like(q_n)
    k_rope = torch.empty_like(k_n)
    pooled_q = torch.empty(B, Hl, NB, HEAD_DIM, device=dev, dtype=BF16)
    ksum = torch.empty(B, NB, Hl * HEAD_DIM, device=dev, dtype=torch.float32)
    cs = cos_sin.to(torch.float32).contiguous()
    _lib.call("rola_b200_rope_pool", _ptr(q_n), _ptr(k_n), Hl * HEAD_DIM, _ptr(cs), B, L, Hl, blk, _ptr(q_rope),
              _ptr(k_rope), _ptr(pooled_q), _ptr(ksum), st)
    if transport == "peer":
        slot = _out_slot.get(key, 0)
        _out_slot[key] = slot ^ 1
        rout = buf.region(f"out{slot}")
        res = ops.head_local_attention(q_rope, k_rope, q_n, k_n, v, gate, pooled_q, ksum, lr_cos, lr_sin, rope_dim,
                                       proj_q, proj_k, Hl, blk, topk, splits, keep=record is not None,
                                       events=events,
                                       scatter=dict(dst=rout.table, world=p, head_offset=rank * Hl, H_total=H))
        if record is not None:
            record["lut"] = res[1]["lut"]
        peer.stream_barrier(group)
        return rout.tensor
    res = ops.head_local_attention(q_rope, k_rope, q_n, k_n, v, gate, pooled_q, ksum, lr_cos, lr_sin,
                                   rope_dim, proj_q, proj_k, Hl, blk, topk, splits, keep=record is not None,
                                   events=events)
    if record is not None:
        res, extra = res
        record["lut"] = extra["lut"]
    return head_to_seq(res, p, group)


def ulysses_rola_attention(layer, x_local, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, nwq, nwk):
    """Entry used by WanSelfAttentionRoLaB200 when a sequence-parallel group is set.

    The model passes RoPE tables of the local shard (wan2pt1.py:825-826); the
    head-local stages need the whole sequence, so the tables are all-gathered."""
    group = layer._pg
    p = dist.get_world_size(group)
    B, Ls, dim = x_local.shape
    L = Ls * p
    if cos_sin.shape[0] == Ls and p > 1:
        cos_sin = _all_gather_rows(cos_sin, group)
        lr_cos = _all_gather_rows(lr_cos, group)
        lr_sin = _all_gather_rows(lr_sin, group)
    blk = layer.rola_blkq
    NB = (L + blk - 1) // blk
    topk = ops.topk_count(layer.rola_topk_ratio, NB)
    return ulysses_rola_attention_params(x_local, w_qkv, b_qkv, cos_sin, lr_cos, lr_sin, rope_dim, nwq, nwk,
                                         layer.proj_q.weight, layer.proj_k.weight, layer.gate_proj.weight,
                                         layer.gate_bias, layer.num_heads, topk, group, layer.eps, blk=blk)


def _all_gather_rows(t: torch.Tensor, group) -> torch.Tensor:
    p = dist.get_world_size(group)
    parts = [torch.empty_like(t) for _ in range(p)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.cat(parts, 0)
