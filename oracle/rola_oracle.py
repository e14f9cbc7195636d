"""CPU oracle for the RoLa attention forward.  TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the algorithm of
SparkDiffusion's fused RoLa inference path so that the CUDA path in
``sparkdiffusion_b200`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import it, and only as the checker or as the
timed CPU baseline.  The product path never calls it.

Parity pin: the functions below were checked against the reference itself run
in the build container (its Triton kernels under the Triton interpreter in
fp32 and its eager PyTorch pieces in bf16); the resulting golden vectors live
in ``tests/golden`` together with the script that made them
(``tests/golden/make_golden.py``).

The training section (f4) restates the gradient of the block-sparse attention
that the reference takes from the external SLA package; the package is absent,
so that section is pinned against torch.autograd of its own forward
restatement (parity of the backward against the SLA kernel itself: unpinned).

Every function cites the reference file:line it restates (paths relative to
the SparkDiffusion project root).

Rounding convention: ``_r(t, dt)`` rounds an fp32 tensor through ``dt`` and
back, i.e. it marks a point where the reference materialises a value in the
data dtype (bf16 in production, a no-op in the fp32 CPU configuration).

Build-defined orders (where the reference's order is implementation defined and
the build needs bit-exact block selection):

* block sums (``mean_pool``) add the rows of a block sequentially in fp32,
  row 0 first;
* the smooth-K centre adds the per-block sums sequentially over blocks;
* a pooled score is a sequential fp32 sum over the head dimension of exact
  bf16 x bf16 products (equivalently a chain of fused multiply-adds);
* top-k keeps the k largest scores, ties broken toward the lower block index,
  and the selected indices are returned sorted ascending as int32.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

F32 = torch.float32
LOG2E = 1.4426950408889634


def _r(t: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    """Round through ``dt`` (a materialisation point) and return fp32."""
    return t.to(dt).to(F32)


# ---------------------------------------------------------------------------
# (a2) Wan 3D RoPE angles            sparkdiffusion/networks/wan2pt1.py:45-137
# ---------------------------------------------------------------------------
def wan_rope_freqs(T: int, H: int, W: int, head_dim: int = 128, theta: float = 10000.0) -> torch.Tensor:
    """Raw RoPE angles ``[T*H*W, head_dim//2]`` fp32, token order (t h w).

    ``VideoRopePosition3DEmb``: the head dim splits into t/h/w parts with
    dim_h = dim_w = head_dim//6*2 and dim_t = head_dim - 2*dim_h (44/42/42 at
    128) (wan2pt1.py:61-63); per-axis frequencies theta^(-2i/dim_axis)
    (:82-83,111-117, NTK factor 1); angles = position x frequency (:121-126),
    concatenated [t, h, w] (:128-137).
    """
    dim_h = head_dim // 6 * 2
    dim_t = head_dim - 2 * dim_h
    seq = torch.arange(max(H, W, T)).float()
    spatial = torch.arange(0, dim_h, 2)[: dim_h // 2].float() / dim_h
    temporal = torch.arange(0, dim_t, 2)[: dim_t // 2].float() / dim_t
    h_freqs = 1.0 / (theta ** spatial)
    w_freqs = 1.0 / (theta ** spatial)
    t_freqs = 1.0 / (theta ** temporal)
    ft = torch.outer(seq[:T], t_freqs)
    fh = torch.outer(seq[:H], h_freqs)
    fw = torch.outer(seq[:W], w_freqs)
    out = torch.cat(
        [
            ft[:, None, None, :].expand(T, H, W, -1),
            fh[None, :, None, :].expand(T, H, W, -1),
            fw[None, None, :, :].expand(T, H, W, -1),
        ],
        dim=-1,
    )
    return out.reshape(T * H * W, -1).float().contiguous()


# ---------------------------------------------------------------------------
# (a3) cos/sin tables
# ---------------------------------------------------------------------------
def prepare_cos_sin(freqs: torch.Tensor, L: int, D: int) -> torch.Tensor:
    """Interleaved fp32 ``[L, D]`` table [cos0, sin0, cos1, sin1, ...].

    sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:37-50 (trig in the
    angle dtype, fp32 tables).
    """
    f = freqs[:L, : D // 2]
    cos = torch.cos(f).to(F32)
    sin = torch.sin(f).to(F32)
    return torch.stack([cos, sin], dim=-1).reshape(L, D).contiguous()


def prepare_lowrank_cos_sin(freqs: torch.Tensor, L: int, rank: int, dtype: torch.dtype):
    """Low-rank RoPE tables: angles cast to the data dtype before cos/sin.

    sparkdiffusion/ops/fused_kernel/fused_lowrank.py:254-267.  Returns
    (cos [L, rope_dim] dtype, sin, rope_dim); no power-of-two padding (the
    padding in the reference only serves Triton's arange).
    """
    rope_dim = min(rank // 2, freqs.shape[-1])
    f = freqs[:L, :rope_dim].to(dtype)
    return torch.cos(f).contiguous(), torch.sin(f).contiguous(), rope_dim


# ---------------------------------------------------------------------------
# (a4) QKV projection + full-width qk-RMSNorm + interleaved RoPE
# ---------------------------------------------------------------------------
def qkv_epilogue(q_raw, k_raw, v_raw, cos_sin, norm_wq, norm_wk, num_heads: int, eps: float = 1e-6):
    """Epilogue of the fused prologue.

    Restates ``_epilogue_kernel`` (fused_qkv_rope.py:53-225):
    RMSNorm over the full hidden width H*D in fp32 (:144-149), unit value
    materialised in the data dtype, times the weight, materialised again
    (:150-159); interleaved RoPE in fp32 on the normed value (:170-176).

    Inputs ``[B, L, H*D]`` (data dtype), ``cos_sin [L, D]`` fp32, norm weights
    ``[H*D]`` or None.  Returns q_rope, k_rope, v as ``[B*H, L, D]`` and
    q_normed, k_normed as ``[B, L, H, D]`` (all data dtype).
    """
    dt = q_raw.dtype
    B, L, dim = q_raw.shape
    H = num_heads
    D = dim // H
    cs = cos_sin[:L].reshape(L, D // 2, 2).to(F32)
    cos = cs[..., 0][None, :, None, :]
    sin = cs[..., 1][None, :, None, :]

    def one(raw, w):
        x = raw.to(F32)
        if w is not None:
            ss = (x * x).sum(-1, keepdim=True)
            rstd = torch.rsqrt(ss / dim + eps)
            unit = _r(x * rstd, dt)
            normed = _r(unit * w.to(F32)[None, None, :], dt)
        else:
            normed = x
        n4 = normed.reshape(B, L, H, D)
        e, o = n4[..., 0::2], n4[..., 1::2]
        rot = torch.stack([e * cos - o * sin, e * sin + o * cos], dim=-1).reshape(B, L, H, D)
        rope = rot.to(dt).permute(0, 2, 1, 3).reshape(B * H, L, D).contiguous()
        return rope, n4.to(dt).contiguous()

    q_rope, q_normed = one(q_raw, norm_wq)
    k_rope, k_normed = one(k_raw, norm_wk)
    v = v_raw.reshape(B, L, H, D).permute(0, 2, 1, 3).reshape(B * H, L, D).contiguous()
    return q_rope, k_rope, v, q_normed, k_normed


def qkv_linear(x, w, b=None, out_dtype=None):
    """bf16(x W^T + b) with fp32 accumulation (fused_qkv_rope.py:287-289).
    ``out_dtype=torch.float32`` returns the value before the final rounding."""
    y = x.to(F32) @ w.to(F32).t()
    if b is not None:
        y = y + b.to(F32)
    return y.to(out_dtype or x.dtype)


def quantize_rows_e4m3(x2: torch.Tensor):
    """Row-wise FP8 quantization, the reference's quantize_activation_rowwise /
    quantize_weight_rowwise (sparkdiffusion/ops/quantization/fp8_linear.py:45-61):
    scale = amax|row| (of the bf16 values) / 448 + 1e-12 in fp32; q =
    e4m3(bf16(x / bf16(scale))).  Returns (q float8_e4m3fn, scale fp32 [M])."""
    scale = x2.abs().amax(dim=1, keepdim=True).float() / 448.0 + 1e-12
    q = (x2 / scale.to(x2.dtype)).to(torch.float8_e4m3fn)
    return q, scale.reshape(-1)


def scaled_mm_rowwise(xq, x_scale, wq, w_scale, bias=None, out_dtype=torch.bfloat16):
    """torch._scaled_mm(xq, wq.t(), scale_a=x_scale[:, None], scale_b=w_scale[None, :],
    bias, out_dtype) as the reference's FP8 prologue calls it (fused_qkv_rope.py:274-285):
    fp32 products of the e4m3 values, times both scales, plus the bias."""
    y = (xq.to(F32) @ wq.to(F32).t()) * x_scale.reshape(-1, 1).to(F32) * w_scale.reshape(1, -1).to(F32)
    if bias is not None:
        y = y + bias.to(F32)
    return y.to(out_dtype)


def fused_qkv_gemm_rope(x, wq, bq, wk, bk, wv, bv, cos_sin, norm_wq, norm_wk, num_heads, eps=1e-6):
    """fused_qkv_rope.py:228-333 (bf16 branch): three linears, then the epilogue."""
    q_raw = qkv_linear(x, wq, bq)
    k_raw = qkv_linear(x, wk, bk)
    v_raw = qkv_linear(x, wv, bv)
    return qkv_epilogue(q_raw, k_raw, v_raw, cos_sin, norm_wq, norm_wk, num_heads, eps)


# ---------------------------------------------------------------------------
# (a5, a6) block mean-pool and smooth-K centre
# ---------------------------------------------------------------------------
def block_sums(x4: torch.Tensor, blk: int) -> torch.Tensor:
    """fp32 per-block column sums ``[B, H, NB, D]``, rows added sequentially.

    Tail rows beyond L contribute nothing (utils.py:46-50 masks them to 0 after the subtraction).
    """
    B, H, L, D = x4.shape
    NB = (L + blk - 1) // blk
    pad = NB * blk - L
    xf = x4.to(F32)
    if pad:
        xf = torch.cat([xf, xf.new_zeros(B, H, pad, D)], dim=2)
    xb = xf.reshape(B, H, NB, blk, D)
    acc = torch.zeros(B, H, NB, D, dtype=F32)
    for r in range(blk):
        acc = acc + xb[:, :, :, r, :]
    return acc


def block_counts(L: int, blk: int) -> torch.Tensor:
    """Valid rows per block ``nx = min(blk, L - m*blk)`` (utils.py:52)."""
    NB = (L + blk - 1) // blk
    return torch.tensor([min(blk, L - m * blk) for m in range(NB)], dtype=F32)


def mean_pool(x4: torch.Tensor, blk: int, center: torch.Tensor | None = None) -> torch.Tensor:
    """Block mean in the data dtype (utils.py:19-82, ``compress_kernel``).

    Without a centre: bf16(sum_fp32(x) / nx) (:52-54).  With a centre:
    each row is first materialised as bf16(x - c) and tail rows are zeroed
    after the subtraction (:40-50).
    """
    dt = x4.dtype
    B, H, L, D = x4.shape
    if center is not None:
        xc = _r(x4.to(F32) - center.to(F32)[:, :, None, :], dt)
        src = xc
    else:
        src = x4.to(F32)
    sums = block_sums(src, blk)
    nx = block_counts(L, blk)
    return (sums / nx[None, None, :, None]).to(dt)


def smooth_k_center(k4: torch.Tensor, blk: int) -> torch.Tensor:
    """Smooth-K centre c = dtype(mean over L of k) (fused_sparse_attn.py:180).

    Build-defined order: the sequential per-block sums of ``block_sums`` added
    sequentially over blocks, then divided by L.
    """
    B, H, L, D = k4.shape
    sums = block_sums(k4, blk)
    acc = torch.zeros(B, H, D, dtype=F32)
    for m in range(sums.shape[2]):
        acc = acc + sums[:, :, m, :]
    return (acc / float(L)).to(k4.dtype)


# ---------------------------------------------------------------------------
# (a7) pooled scores and top-k selection
# ---------------------------------------------------------------------------
def block_scores(pq: torch.Tensor, pk: torch.Tensor) -> torch.Tensor:
    """fp32 scores ``[B, H, NBq, NBk]`` = pooled_q . pooled_k.

    The reference multiplies the bf16 pooled tensors with cuBLAS and gets bf16
    scores (fused_sparse_attn.py:181).  The build scores in fp32 with a fixed
    order: a sequential sum over d of exact products.
    """
    a = pq.to(F32)
    b = pk.to(F32)
    D = a.shape[-1]
    acc = torch.zeros(a.shape[:-1] + (b.shape[-2],), dtype=F32)
    for d in range(D):
        acc = acc + a[..., :, d, None] * b[..., None, :, d]
    return acc


def topk_count(topk_ratio: float, nb: int) -> int:
    """k = max(1, min(NB, int(ratio*NB))) (fused_sparse_attn.py:197)."""
    return max(1, min(nb, int(topk_ratio * nb)))


def select_topk(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k block indices, ties toward the lower index, sorted ascending.

    Replaces ``torch.topk(sorted=False)`` (fused_sparse_attn.py:198) whose
    order and tie handling are implementation defined.  Returns int32
    ``[..., k]``.
    """
    nb = scores.shape[-1]
    idx = torch.arange(nb).expand_as(scores)
    # stable sort of -score keeps the lower index first among equal scores
    order = torch.sort(-scores, dim=-1, stable=True).indices
    sel = torch.gather(idx, -1, order[..., :k])
    return torch.sort(sel, dim=-1).values.to(torch.int32)


def block_select(q4: torch.Tensor, k4: torch.Tensor, blkq: int, blkk: int, topk: int):
    """Pool, smooth-K, score, select.  Returns (lut, pooled_q, pooled_k, scores, center)."""
    pq = mean_pool(q4, blkq)
    c = smooth_k_center(k4, blkk)
    pk = mean_pool(k4, blkk, center=c)
    s = block_scores(pq, pk)
    return select_topk(s, topk), pq, pk, s, c


# ---------------------------------------------------------------------------
# (a8) block-sparse online-softmax attention over the LUT
# ---------------------------------------------------------------------------
def sparse_attn_lut(q4, k4, v4, lut, blkq: int, blkk: int, out_dtype=None) -> torch.Tensor:
    """Restates ``_rola_fwd_kernel`` (fused_sparse_attn.py:55-144).

    For each query block, iterate the LUT in its stored order: s = (q.k) *
    D^-1/2 * log2(e) in fp32 (:107,200); columns past L are -inf for a
    partial key block (:100-109); online base-2 softmax (:118-124); the
    accumulator is rescaled by alpha and P is materialised in the data dtype
    before P.V (:136-138); o = acc / l (:143).  ``lut`` is ``[B*H, NBq, k]``
    or ``[B, H, NBq, k]``.  Returns ``[B, H, L, D]`` in the data dtype
    (``out_dtype=torch.float32``: before the final rounding).
    """
    dt = q4.dtype
    B, H, L, D = q4.shape
    NBq = (L + blkq - 1) // blkq
    NBk = (L + blkk - 1) // blkk
    lut = lut.reshape(B * H, NBq, -1).long()
    topk = lut.shape[-1]
    scale = D ** -0.5 * LOG2E

    def pad_blocks(t, blk, nb):
        p = nb * blk - L
        tf = t.to(F32).reshape(B * H, L, D)
        if p:
            tf = torch.cat([tf, tf.new_zeros(B * H, p, D)], dim=1)
        return tf.reshape(B * H, nb, blk, D)

    qb = pad_blocks(q4, blkq, NBq)
    kb = pad_blocks(k4, blkk, NBk)
    vb = pad_blocks(v4, blkk, NBk)
    bh = torch.arange(B * H)[:, None].expand(B * H, NBq)
    m_i = torch.full((B * H, NBq, blkq), -math.inf)
    l_i = torch.zeros(B * H, NBq, blkq)
    acc = torch.zeros(B * H, NBq, blkq, D)
    col = torch.arange(blkk)
    for t in range(topk):
        j = lut[:, :, t]
        kj = kb[bh, j]
        vj = vb[bh, j]
        s = torch.matmul(qb, kj.transpose(-1, -2)) * scale
        valid = col[None, None, :] < (L - j * blkk)[:, :, None]
        s = torch.where(valid[:, :, None, :], s, torch.tensor(-math.inf))
        new_m = torch.maximum(m_i, s.amax(-1))
        p = torch.exp2(s - new_m[..., None])
        alpha = torch.exp2(m_i - new_m)
        acc = acc * alpha[..., None] + torch.matmul(_r(p, dt), vj)
        l_i = l_i * alpha + p.sum(-1)
        m_i = new_m
    o = (acc / l_i[..., None]).to(out_dtype or dt)
    return o.reshape(B, H, NBq * blkq, D)[:, :, :L].contiguous()


# ---------------------------------------------------------------------------
# (f4) training: the block-sparse attention and its exact gradient
# ---------------------------------------------------------------------------
# The reference trains through the external SLA package
# (`_attention.apply(q, k, v, sparse_map, lut, real_topk, BLKQ, BLKK)`,
# wan_rola_attention.py:293-327; the package is loaded from `SLA_SRC`,
# :97-109, and is not part of the reference tree nor of this container, so no
# version is pinned).  Its published algorithm is block-sparse softmax
# attention, each query block attending to the key blocks of its LUT row, and
# its backward is the exact gradient of that function.  Parity of the backward
# is therefore pinned against torch.autograd of ``block_sparse_attention``
# below (tests/test_oracle_backward.py), not against outputs of the SLA kernel.
def block_mask(lut: torch.Tensor, L: int, blkq: int, blkk: int) -> torch.Tensor:
    """``[B*H, L, L]`` bool: row t may attend to column u when the key block of
    u is in the LUT row of the query block of t (small cases only)."""
    lut = lut.long()
    BH, NBq, _ = lut.shape
    NBk = (L + blkk - 1) // blkk
    sel = torch.zeros(BH, NBq, NBk, dtype=torch.bool)
    sel.scatter_(-1, lut, True)
    rows = torch.arange(L) // blkq
    cols = torch.arange(L) // blkk
    return sel[:, rows][:, :, cols]


def block_sparse_attention(q4, k4, v4, lut, blkq: int, blkk: int, dtype=torch.float64):
    """o = softmax_masked(q k^T D^-1/2) v over ``[B, H, L, D]`` in ``dtype``,
    with the base-2 log-sum-exp per row (units of D^-1/2 log2 e, the forward
    kernel's ``lse``).  Differentiable (plain torch ops)."""
    B, H, L, D = q4.shape
    mask = block_mask(lut.reshape(B * H, -1, lut.shape[-1]), L, blkq, blkk).reshape(B, H, L, L)
    s = torch.matmul(q4.to(dtype), k4.to(dtype).transpose(-1, -2)) * D ** -0.5
    s = s.masked_fill(~mask, -math.inf)
    o = torch.matmul(torch.softmax(s, dim=-1), v4.to(dtype))
    lse2 = torch.logsumexp(s, dim=-1) * LOG2E
    return o, lse2


def block_sparse_attention_backward(q4, k4, v4, lut, do4, blkq: int, blkk: int, dtype=torch.float64,
                                    round_dtype=None, o_fwd=None):
    """Exact gradient (dq, dk, dv) of ``block_sparse_attention``, written out:
    P = softmax_masked(S), dV = P^T dO, dP = dO V^T, delta = rowsum(dO * O),
    dS = P (dP - delta), dQ = D^-1/2 dS K, dK = D^-1/2 dS^T Q.

    ``round_dtype`` (e.g. bf16) models the materialisation points of a
    flash-style backward: P and dS are rounded before the products that take
    them (dV, dQ, dK), and delta uses ``o_fwd``, the forward's materialised
    output (``sparse_attn_lut``, whose P was rounded before P.V), when given."""
    B, H, L, D = q4.shape
    mask = block_mask(lut.reshape(B * H, -1, lut.shape[-1]), L, blkq, blkk).reshape(B, H, L, L)
    q, k, v, do = (t.to(dtype) for t in (q4, k4, v4, do4))

    def rnd(t):
        return t if round_dtype is None else t.to(round_dtype).to(dtype)

    s = (torch.matmul(q, k.transpose(-1, -2)) * D ** -0.5).masked_fill(~mask, -math.inf)
    p = torch.softmax(s, dim=-1)
    o = rnd(torch.matmul(p, v)) if o_fwd is None else o_fwd.to(dtype)
    dv = torch.matmul(rnd(p).transpose(-1, -2), do)
    dp = torch.matmul(do, v.transpose(-1, -2))
    delta = (do * o).sum(-1, keepdim=True)
    ds = rnd(p * (dp - delta))
    dq = torch.matmul(ds, k) * D ** -0.5
    dk = torch.matmul(ds.transpose(-1, -2), q) * D ** -0.5
    return dq, dk, dv


# ---------------------------------------------------------------------------
# (a9) low-rank branch
# ---------------------------------------------------------------------------
def proj_silu_rope(x_blhd, proj_w, cos, sin, rope_dim: int) -> torch.Tensor:
    """Restates ``_proj_silu_rope_kernel`` (fused_lowrank.py:31-152) without norm.

    lin = dtype(x . P^T) (:97), silu in fp32 then dtype (:99-102); interleaved
    RoPE on the first 2*rope_dim columns with every product and sum rounded
    to the data dtype (:123-135); remaining columns pass through.
    Input ``[B, L, H, D]``; returns ``[B*H, L, R]``.
    """
    dt = x_blhd.dtype
    B, L, H, D = x_blhd.shape
    R = proj_w.shape[0]
    x = x_blhd.permute(0, 2, 1, 3).to(F32)
    lin = _r(torch.matmul(x, proj_w.to(F32).t()), dt)
    o = _r(lin * torch.sigmoid(lin), dt)
    if rope_dim > 0:
        c = cos[:L, :rope_dim].to(F32)[None, None]
        s = sin[:L, :rope_dim].to(F32)[None, None]
        rot = o[..., : 2 * rope_dim]
        e, od = rot[..., 0::2], rot[..., 1::2]
        ec, os_ = _r(e * c, dt), _r(od * s, dt)
        es, oc = _r(e * s, dt), _r(od * c, dt)
        re = _r(ec - os_, dt)
        ro = _r(es + oc, dt)
        rot_out = torch.stack([re, ro], dim=-1).reshape(B, H, L, 2 * rope_dim)
        o = torch.cat([rot_out, o[..., 2 * rope_dim:]], dim=-1)
    return o.to(dt).reshape(B * H, L, R).contiguous()


def lowrank_kv(k_lr, v, B: int, H: int) -> torch.Tensor:
    """C = dtype(k_lr^T v) ``[B, H, R, D]`` (fused_lowrank.py:355-358)."""
    L, R = k_lr.shape[1], k_lr.shape[2]
    D = v.shape[-1]
    kl = k_lr.reshape(B, H, L, R).to(F32)
    vv = v.reshape(B, H, L, D).to(F32)
    return torch.matmul(kl.transpose(-1, -2), vv).to(v.dtype)


def fused_lowrank(q_normed, k_normed, v, proj_q, proj_k, cos, sin, rope_dim: int):
    """fused_lowrank.py:270-364 with no re-norm (as called from
    wan_rola_attention.py:432-439).  Returns (o_lr [B,H,L,D], q_lr, k_lr, C)."""
    B, L, H, D = q_normed.shape
    q_lr = proj_silu_rope(q_normed, proj_q, cos, sin, rope_dim)
    k_lr = proj_silu_rope(k_normed, proj_k, cos, sin, rope_dim)
    C = lowrank_kv(k_lr, v, B, H)
    R = q_lr.shape[-1]
    o_lr = torch.matmul(q_lr.reshape(B, H, L, R).to(F32), C.to(F32)).to(v.dtype)
    return o_lr, q_lr, k_lr, C


# ---------------------------------------------------------------------------
# (a10) gated fusion
# ---------------------------------------------------------------------------
def gate_values(x, gate_w, gate_b, num_heads: int) -> torch.Tensor:
    """gate = dtype(sigmoid(dtype(dtype(x_h . w_g) + b_h))) ``[B, L, H]``.

    fused_gate.py:97-114 (the bias is cast to the data dtype at :199).
    """
    dt = x.dtype
    B, L, dim = x.shape
    D = dim // num_heads
    xh = x.reshape(B, L, num_heads, D).to(F32)
    lin = _r((xh * gate_w.reshape(-1).to(F32)).sum(-1), dt)
    logit = _r(lin + gate_b.reshape(-1).to(dt).to(F32)[None, None, :], dt)
    return _r(1.0 / (1.0 + torch.exp(-logit)), dt)


def fused_gate(o_lr, o_sparse, x, gate_w, gate_b, out_dtype=None, gate=None) -> torch.Tensor:
    """Restates ``_gate_fusion_kernel`` (fused_gate.py:27-127).

    o_lr_n = dtype(o_lr * rsqrt(mean(o_lr^2) + eps_lr)), eps_lr =
    finfo(dtype).eps (:72-77,220); os_rms through the dtype chain
    pow -> mean -> +1e-5 -> sqrt (:84-95); out = (os/os_rms + gate*o_lr_n) *
    os_rms in fp32 (:120-121), stored ``[B, L, H*D]`` (:123-127).  ``gate``
    (``[B, L, H]`` from ``gate_values``) may replace x, gate_w and gate_b.
    """
    dt = o_lr.dtype
    B, H, L, D = o_lr.shape
    eps_lr = torch.finfo(dt).eps
    olr = o_lr.to(F32)
    rms_sq = (olr * olr).sum(-1, keepdim=True) / D + eps_lr
    olr_n = _r(olr * torch.rsqrt(rms_sq), dt)
    os_ = o_sparse.to(F32)
    os_sq = _r(os_ * os_, dt)
    os_mean = _r(os_sq.sum(-1, keepdim=True) / D, dt)
    os_mean_eps = _r(os_mean + 1e-5, dt)
    os_rms = _r(torch.sqrt(os_mean_eps), dt)
    if gate is None:
        gate = gate_values(x, gate_w, gate_b, H)
    gate = gate.to(F32).permute(0, 2, 1)[..., None]
    out = (os_ / os_rms + gate * olr_n) * os_rms
    return out.to(out_dtype or dt).permute(0, 2, 1, 3).reshape(B, L, H * D).contiguous()


# ---------------------------------------------------------------------------
# (a1) whole layer (without the output projection)
# ---------------------------------------------------------------------------
def rola_attention_core(q_raw, k_raw, v_raw, x, cos_sin, lr_cos, lr_sin, rope_dim,
                        norm_wq, norm_wk, proj_q, proj_k, gate_w, gate_b,
                        num_heads: int, blkq: int, blkk: int, topk: int, eps: float = 1e-6,
                        lut: torch.Tensor | None = None, out_dtype=None):
    """RoLa forward from the projected q/k/v to the gated output ``[B, L, H*D]``.

    wan_rola_attention.py:414-446 (``fused_forward`` minus ``self.o``).
    If ``lut`` is given it replaces the oracle's own selection (used to check
    attention output parity independently of selection).  Returns a dict of
    every intermediate; ``out_dtype=torch.float32`` leaves the final output
    unrounded.
    """
    B, L, dim = q_raw.shape
    H = num_heads
    D = dim // H
    q_rope, k_rope, v, q_normed, k_normed = qkv_epilogue(q_raw, k_raw, v_raw, cos_sin, norm_wq, norm_wk, H, eps)
    q4, k4, v4 = (t.reshape(B, H, L, D) for t in (q_rope, k_rope, v))
    sel_lut, pq, pk, scores, center = block_select(q4, k4, blkq, blkk, topk)
    use_lut = sel_lut if lut is None else lut
    o_sparse = sparse_attn_lut(q4, k4, v4, use_lut, blkq, blkk)
    o_lr, q_lr, k_lr, C = fused_lowrank(q_normed, k_normed, v, proj_q, proj_k, lr_cos, lr_sin, rope_dim)
    out = fused_gate(o_lr, o_sparse, x, gate_w, gate_b, out_dtype=out_dtype)
    return dict(q_rope=q_rope, k_rope=k_rope, v=v, q_normed=q_normed, k_normed=k_normed,
                lut=sel_lut, pooled_q=pq, pooled_k=pk, scores=scores, center=center,
                o_sparse=o_sparse, o_lr=o_lr, q_lr=q_lr, k_lr=k_lr, C=C, out=out)


def rola_attention_forward(x, wq, bq, wk, bk, wv, bv, **kw):
    """Full prologue from hidden states: linears, then ``rola_attention_core``."""
    q_raw = qkv_linear(x, wq, bq)
    k_raw = qkv_linear(x, wk, bk)
    v_raw = qkv_linear(x, wv, bv)
    res = rola_attention_core(q_raw, k_raw, v_raw, x, **kw)
    res.update(q_raw=q_raw, k_raw=k_raw, v_raw=v_raw)
    return res
