"""The C ABI library loads and exports every symbol declared in include/*.h (CPU)."""

import ctypes
import glob
import os
import re

import pytest

from sparkdiffusion_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(rola_b200_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "rola_b200_sparse_attn" in names and "rola_b200_rola_forward" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_python_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_abi_version_and_validation_without_gpu():
    lib = _lib.load_library()
    assert lib.rola_b200_abi_version() == _lib.ABI_VERSION
    # argument validation runs on the host before any launch: a bad size is
    # rejected with ROLA_ERR_INVALID and a message, no GPU needed
    rc = lib.rola_b200_qkv_gemm(None, None, None, None, None, 0, 0, 0, None)
    assert rc == _lib.ROLA_ERR_INVALID
    assert b"null pointer" in lib.rola_b200_last_error()
    rc = lib.rola_b200_block_select(ctypes.c_void_p(16), ctypes.c_void_p(16), 1, 4, 4, 9, ctypes.c_void_p(16),
                                    ctypes.c_void_p(16), None)
    assert rc == _lib.ROLA_ERR_INVALID and b"topk" in lib.rola_b200_last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "block_select")


def test_workspace_size_monotone():
    lib = _lib.load_library()
    a = lib.rola_b200_forward_workspace_bytes(1, 1024, 4, 128, 64, 2)
    b = lib.rola_b200_forward_workspace_bytes(1, 2048, 4, 128, 64, 2)
    assert 0 < a < b
    assert lib.rola_b200_forward_workspace_bytes(0, 1024, 4, 128, 64, 2) == 0


def test_training_entry_points_validate_without_gpu():
    """The training forward / backward entries reject bad arguments on the host
    (ROLA_ERR_INVALID with a message) before any launch; the backward's workspace
    size is 0 for bad sizes and grows with the sequence."""
    lib = _lib.load_library()
    p = ctypes.c_void_p(256)  # a 16-byte aligned stand-in; validation fails before any use
    ws = lib.rola_b200_sparse_attn_bwd_workspace
    assert ws(1, 1024, 2, 96) == 0 and ws(0, 1024, 2, 128) == 0
    assert 0 < ws(1, 1024, 2, 128) < ws(1, 2048, 2, 128)
    assert ws(1, 1024, 2, 64) > ws(1, 1024, 2, 128)  # the byte map grows with the 64-token block count
    # forward with lse: no lse pointer
    rc = lib.rola_b200_sparse_attn_fwd_lse(p, p, 1024 * 256, 128, 256, p, 1024 * 256, 128, 256, p, 1, 1024, 2, 128, 2,
                                           p, 1024 * 256, 128, 256, None, None)
    assert rc == _lib.ROLA_ERR_INVALID and b"null pointer" in lib.rola_b200_last_error()
    # backward: block size 96, block 64 without the paired table, topk beyond NB, workspace too small
    args = dict(B=1, L=1024, H=2, topk=2)
    base = (p, p, 1024 * 256, 128, 256, p, 1024 * 256, 128, 256, p, p, 1024 * 256, 128, 256)

    def bwd(blk, paired, topk, ws_bytes):
        return lib.rola_b200_sparse_attn_bwd(*base, p, paired, p, args["B"], args["L"], args["H"], blk, topk, p, p, p,
                                             1024 * 256, 128, 256, p, ws_bytes, None)

    big = ws(1, 1024, 2, 64)
    assert bwd(96, p, 2, big) == _lib.ROLA_ERR_INVALID and b"block size" in lib.rola_b200_last_error()
    assert bwd(64, None, 2, big) == _lib.ROLA_ERR_INVALID and b"paired" in lib.rola_b200_last_error()
    assert bwd(128, None, 9, big) == _lib.ROLA_ERR_INVALID and b"topk" in lib.rola_b200_last_error()
    assert bwd(128, None, 2, 16) == _lib.ROLA_ERR_INVALID and b"workspace" in lib.rola_b200_last_error()
