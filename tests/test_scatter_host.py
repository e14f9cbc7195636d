"""Host side of the fused sequence->head exchange (CPU): the ctypes mirror of
``rola_scatter_args`` matches the C header's layout, and the scatter
description of a token chunk points where the kernels must write."""

import ctypes
import os
import shutil
import subprocess

import pytest
import torch

from sparkdiffusion_b200 import _lib
from sparkdiffusion_b200.ulysses import _peer_layout, _scatter_args

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIELDS = [f[0] for f in _lib.ScatterArgs._fields_]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_ctypes_struct_matches_c_header(tmp_path):
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "rola_b200.h"', "int main(void) {",
             '  printf("size %zu\\n", sizeof(rola_scatter_args));']
    lines += [f'  printf("{f} %zu\\n", offsetof(rola_scatter_args, {f}));' for f in FIELDS]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(_lib.ScatterArgs)
    for f in FIELDS:
        assert int(out[f]) == getattr(_lib.ScatterArgs, f).offset, f


SPAN = 1 << 36  # fake address space of one rank's region (larger than any region here)


class _Region:
    def __init__(self, base, world):
        self.table = (ctypes.c_void_p * world)(*[base + SPAN * r for r in range(world)])


class _Buf:
    def __init__(self, world):
        self.regions = {n: _Region(16 * SPAN * (i + 1), world) for i, n in enumerate(("q", "k", "v", "gate"))}

    def region(self, name):
        return self.regions[name]


def test_scatter_args_of_a_chunk():
    H, p, Ls, B = 8, 4, 300, 2
    dim, L = H * 128, Ls * p
    qkv = torch.zeros(B * Ls, 3 * dim, dtype=torch.bfloat16)
    ssq = torch.zeros(B * Ls, 3 * dim // 256)
    xc = torch.zeros(B * Ls, dim, dtype=torch.bfloat16)
    w = torch.ones(dim, dtype=torch.bfloat16)
    buf = _Buf(p)
    rank, b, t0, t1 = 2, 1, 128, 300
    r0 = b * Ls + t0
    a = _scatter_args(qkv, ssq, xc, w, w, w, w, H, p, L, 1e-6, buf, b, r0, rank * Ls + t0, rank * Ls + t1)
    row = qkv.data_ptr() + r0 * 3 * dim * 2
    assert (a.q_raw, a.k_raw, a.v_raw) == (row, row + dim * 2, row + 2 * dim * 2)
    assert a.ld_raw == 3 * dim and a.ssq == ssq.data_ptr() + r0 * ssq.shape[1] * 4
    assert a.x == xc.data_ptr() + r0 * dim * 2
    assert (a.B, a.L, a.H, a.world) == (1, t1 - t0, H, p)
    assert (a.dst_rows, a.dst_row0) == (L, rank * Ls + t0)
    Hl = H // p
    for name, field, per_row in (("q", "q_dst", Hl * 128 * 2), ("gate", "g_dst", Hl * 2)):
        tab = getattr(a, field)
        for r in range(p):
            # batch b of every destination buffer [B, L, Hl*D] (gate [B, L, Hl])
            assert tab[r] == buf.region(name).table[r] + b * L * per_row


def test_peer_layout_sizes():
    lay = _peer_layout(2, 300, 8, 4)
    assert lay["q"][0] == (2, 1200, 2 * 128) and lay["gate"][0] == (2, 1200, 2)
    assert lay["out0"][0] == lay["out1"][0] == (2, 300, 8 * 128)


def _replay_exchange(monkeypatch, B, Ls, H, p, chunks):
    """Run every rank's host side of the overlapped QKV GEMM / scatter
    (``_gemm_scatter_overlapped``) on CPU with the library calls recorded, and
    replay what the kernels would do with the recorded arguments: the GEMM
    writes rows [out, out + M) of qkv and their sums of squares; a scatter
    (the GEMM's side job or the standalone pass) reads row ``b * L + t`` from
    its q_raw / ssq / x pointers and writes token t of batch b to
    ``dst[chunk] + b * dst_sB + (dst_row0 + t) * chunk_cols + col - chunk * chunk_cols``
    (prologue.cu ``chunk_dst``; the gate ``gate_dst``), over work items of 32
    tokens x 8 heads (capi.cu ``scatter_params``).  Returns, per region, the
    written destination elements with the source row and the issuing rank."""
    import types

    from sparkdiffusion_b200 import ulysses

    dim, L, hpc = H * 128, Ls * p, H // p
    monkeypatch.setattr(ulysses, "_stream", lambda: 0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda dev: types.SimpleNamespace(
        multi_processor_count=148))
    buf = _Buf(p)
    bases = {n: [buf.region(n).table[r] for r in range(p)] for n in ("q", "gate")}
    written = {"q": {}, "gate": {}}
    plans = []  # per rank: (GEMM rows, with a side job) of each GEMM call
    for rank in range(p):
        calls = []
        monkeypatch.setattr(_lib, "call", lambda name, *args: calls.append((name, args)))
        x = torch.zeros(B, Ls, dim, dtype=torch.bfloat16)
        w = torch.zeros(3 * dim, dim, dtype=torch.bfloat16)
        v = torch.ones(dim, dtype=torch.bfloat16)
        # qkv / ssq are allocated inside: take their base pointers from the first GEMM call
        ulysses._gemm_scatter_overlapped(x, w, None, v, v, v, v, x, H, p, rank, 1e-6, buf, chunks, None)
        gemm = [a for n, a in calls if n == "rola_b200_qkv_gemm_scatter"]
        plans.append([(a[5], a[8] is not None) for a in gemm])
        qkv0, ssq0 = gemm[0][3], gemm[0][4]
        row_of = lambda ptr: (ptr - qkv0) // (3 * dim * 2)  # noqa: E731
        done = set()  # qkv rows the GEMM calls so far have written
        for name, args in calls:
            if name == "rola_b200_qkv_gemm_scatter":
                out, ssq, M, side = args[3], args[4], args[5], args[8]
                r0 = row_of(out)
                assert (ssq - ssq0) // (3 * dim // 256 * 4) == r0
                rows = set(range(r0, r0 + M))
                assert not rows & done, "a GEMM chunk overlaps an earlier one"
                scatters = [side._obj] if side is not None else []
            else:
                assert name == "rola_b200_qk_norm_scatter"
                rows, scatters = set(), [args[0]._obj]
            for a in scatters:
                assert a.world == p and a.H == H and a.dst_rows == L and a.ld_raw == 3 * dim
                src0 = row_of(a.q_raw)
                assert (a.ssq - ssq0) // (a.ssq_ld * 4) == src0 and (a.x - x.data_ptr()) // (dim * 2) == src0
                dst_sB = a.dst_rows * hpc * 128
                for b in range(a.B):
                    for m in range((a.L + 31) // 32):  # work items of 32 tokens (all head groups)
                        for t in range(32 * m, min(a.L, 32 * m + 32)):
                            src = src0 + b * a.L + t
                            # the side job reads only rows written by earlier GEMM calls
                            assert src in done, f"rank {rank}: row {src} read before it is written"
                            for h in range(H):
                                c = h // hpc
                                q = a.q_dst[c] + 2 * (b * dst_sB + (a.dst_row0 + t) * hpc * 128 + (h - c * hpc) * 128)
                                g = a.g_dst[c] + 2 * (b * (dst_sB // 128) + (a.dst_row0 + t) * hpc + (h - c * hpc))
                                for region, ptr in (("q", q), ("gate", g)):
                                    assert ptr not in written[region], f"{region} element written twice"
                                    written[region][ptr] = (rank, src, c, h)
            done |= rows
    return written, bases, dim, L, hpc, plans


@pytest.mark.parametrize("B,Ls,H,p,chunks", [(1, 1440, 8, 2, None), (1, 1440, 8, 2, 1), (2, 1440, 8, 2, None),
                                             (1, 360, 8, 8, 2), (1, 720, 8, 4, None),
                                             (1, 37800, 40, 2, None)])  # C4 on 2 GPUs, the automatic plan
def test_overlapped_exchange_writes_every_element_once(monkeypatch, B, Ls, H, p, chunks):
    """Every element of every rank's q / gate buffer is written exactly once,
    by the rank that owns its token, from the qkv row of that token, after
    the GEMM chunk that produced the row (the plan of the 2-GPU case with
    chunks of 768 + 672 rows per rank, the same routine with one chunk, batch
    2, the 8- and 4-rank plans, and C4 on 2 ranks)."""
    written, bases, dim, L, hpc, plans = _replay_exchange(monkeypatch, B, Ls, H, p, chunks)
    if (B, Ls, p, chunks) == (1, 1440, 2, None):  # the case that differed on 2 GPUs
        assert plans == [[(768, False), (672, True)]] * 2
    for region, per_tok in (("q", hpc * 128 * 2), ("gate", hpc * 2)):
        for d in range(p):
            base = bases[region][d]
            got = {ptr: v for ptr, v in written[region].items() if 0 <= ptr - base < SPAN}
            head_stride = 128 * 2 if region == "q" else 2
            expect = {base + b * L * per_tok + row * per_tok + j * head_stride
                      for b in range(B) for row in range(L) for j in range(hpc)}
            assert set(got) == expect, f"{region} buffer of rank {d}: {len(expect - set(got))} missing"
            for ptr, (rank, src, c, h) in got.items():
                off = ptr - base
                b, row = off // (L * per_tok), off % (L * per_tok) // per_tok
                assert c == d and h // hpc == d  # heads of rank d
                assert rank == row // Ls  # written by the rank that owns the token
                assert src == b * Ls + row % Ls  # from that token's qkv row
