"""The allocation-free low-rank reduction entry point (rola_b200_lowrank_kv_noalloc).

It exists for callers that cannot give the library device memory for its
scratch (a host framework owning a fixed memory pool, a latency-critical loop
that must not call cudaMalloc, a binding without a CUDA allocator).  Checked
through the C ABI against the allocating entry point rola_b200_lowrank_kv on
two calls in a row with different inputs, so stale scratch contents from the
first call cannot leak into the second.  This file is named to be collected
last; it also passes when run alone in a fresh process.
"""

import math

import pytest
import torch

from sparkdiffusion_b200 import _lib
from sparkdiffusion_b200.rope import prepare_lowrank_cos_sin, wan_rope_freqs

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 4 << 20  # the fixed 16 MiB scratch of the entry point


def _case(B, H, grid, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    L = grid[0] * grid[1] * grid[2]
    dim = H * 128
    k = torch.randn(B, L, dim, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, L, dim, generator=g).to(torch.bfloat16).cuda()
    pk = (torch.randn(64, 128, generator=g) / math.sqrt(128)).to(torch.bfloat16).cuda()
    cos, sin, rope_dim = prepare_lowrank_cos_sin(wan_rope_freqs(*grid), L, 64, torch.bfloat16)
    return k, v, pk, cos.cuda(), sin.cuda(), rope_dim, B, L, H


def _strides(t):
    return t.stride(0), 128, t.stride(1)


def _run(name, case, splits, scratch=None):
    k, v, pk, cos, sin, rope_dim, B, L, H = case
    C = torch.empty(B * H, 64, 128, dtype=torch.bfloat16, device="cuda")
    Ct = torch.empty(B * H, 128, 64, dtype=torch.bfloat16, device="cuda")
    args = [k.data_ptr(), *_strides(k), v.data_ptr(), *_strides(v), pk.data_ptr(), cos.data_ptr(), sin.data_ptr(),
            rope_dim, B, L, H, 64, splits]
    if scratch is not None:
        args.append(scratch.data_ptr())
    args += [C.data_ptr(), Ct.data_ptr(), torch.cuda.current_stream().cuda_stream]
    _lib.call(name, *args)
    return C, Ct


def test_noalloc_matches_allocating_entry_point_twice():
    lib = _lib.load_library()
    first = _case(1, 4, (3, 12, 30), seed=1)   # 1080 tokens, ragged tail tile
    second = _case(2, 2, (2, 10, 20), seed=2)  # different shape and batch
    for case, splits in ((first, 6), (second, 3)):
        k, v, pk, cos, sin, rope_dim, B, L, H = case
        chunks = ((L + 63) // 64 + 15) // 16  # one fp32 partial of C per 1024 tokens
        scratch = torch.empty(chunks * B * H * 64 * 128, dtype=torch.float32, device="cuda")
        C_ref, Ct_ref = _run("rola_b200_lowrank_kv", case, splits, scratch)
        C, Ct = _run("rola_b200_lowrank_kv_noalloc", case, splits)
        torch.cuda.synchronize()
        # same kernels, same split order and the same fixed-order reduction:
        # the results are identical bit for bit
        assert torch.equal(C.cpu(), C_ref.cpu()), "C (noalloc) differs from the allocating entry point"
        assert torch.equal(Ct.cpu(), Ct_ref.cpu()), "Ct (noalloc) differs from the allocating entry point"
    assert lib.rola_b200_device_status(1) == 0


def test_noalloc_rejects_requests_beyond_the_scratch():
    case = _case(1, 4, (2, 8, 16), seed=3)
    k, v, pk, cos, sin, rope_dim, B, L, H = case
    # a sequence with more 1024-token chunks than the scratch holds partials
    # for: refused by the size check before any memory is touched
    max_chunks = SCRATCH_FLOATS // (B * H * 64 * 128)
    too_long = (k, v, pk, cos, sin, rope_dim, B, (max_chunks + 1) * 1024, H)
    with pytest.raises(ValueError, match="exceed the fixed"):
        _run("rola_b200_lowrank_kv_noalloc", too_long, 4)
