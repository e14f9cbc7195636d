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


class _Region:
    def __init__(self, base, world):
        self.table = (ctypes.c_void_p * world)(*[base + 0x1000000 * r for r in range(world)])


class _Buf:
    def __init__(self, world):
        self.regions = {n: _Region(0x10000000 * (i + 1), world) for i, n in enumerate(("q", "k", "v", "gate"))}

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
