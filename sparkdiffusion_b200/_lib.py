"""ctypes binding of ``librola_b200.so`` (the C ABI declared in include/rola_b200.h).

The library is built in-tree (``sparkdiffusion_b200/librola_b200.so``) by
``sparkdiffusion_b200.build.build_library``.  There is no fallback: if the
shared library is missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librola_b200.so")
ABI_VERSION = 2
PEER_HANDLE_BYTES = 64

ROLA_OK = 0
ROLA_ERR_INVALID = 1
ROLA_ERR_CUDA = 2
ROLA_ERR_DEVICE = 3

DEVICE_ERRORS = {
    0: "ok",
    1: "timeout waiting for a TMA load",
    2: "timeout waiting for an MMA completion",
    3: "timeout waiting for the softmax hand-off",
    4: "LUT entry outside [0, NB)",
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_Z = ctypes.c_size_t

# name -> argument types (return type is int unless listed in _RESTYPES)
SIGNATURES = {
    "rola_b200_abi_version": [],
    "rola_b200_last_error": [],
    "rola_b200_device_status": [_I],
    "rola_b200_check_wait_timeout": [ctypes.c_uint, _P],
    "rola_b200_qkv_gemm": [_P, _P, _P, _P, _P, _L, _L, _L, _P],
    "rola_b200_quantize_rows_e4m3": [_P, _L, _L, _L, _P, _P, _P],
    "rola_b200_qkv_gemm_fp8": [_P, _P, _P, _P, _P, _P, _P, _L, _L, _L, _P],
    "rola_b200_qk_norm_rope": [_P, _P, _L, _P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F,
                               _P, _P, _P, _P, _P, _P, _P, _P],
    "rola_b200_qk_norm_pack": [_P, _P, _P, _L, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F,
                               _P, _P, _P, _P, _P],
    "rola_b200_qk_norm_scatter": [_P, _I, _P],
    "rola_b200_qkv_gemm_scatter": [_P, _P, _P, _P, _P, _L, _L, _L, _P, _P],
    "rola_b200_rope_pool": [_P, _P, _L, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P],
    "rola_b200_mean_pool": [_P, _L, _L, _L, _I, _I, _I, _I, _P, _P, _P],
    "rola_b200_smooth_k_center": [_P, _L, _L, _L, _I, _I, _I, _I, _P, _P, _P],
    "rola_b200_center_from_sums": [_P, _I, _I, _I, _I, _P, _P],
    "rola_b200_block_select": [_P, _P, _I, _I, _I, _I, _P, _P, _P],
    "rola_b200_pair_blocks": [_P, _I, _I, _I, _P, _P],
    "rola_b200_lowrank_q": [_P, _L, _L, _L, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P],
    "rola_b200_lowrank_kv": [_P, _L, _L, _L, _P, _L, _L, _L, _P, _P, _P, _I, _I, _I, _I, _I, _I,
                             _P, _P, _P, _P],
    "rola_b200_sparse_attn": [_P, _P, _L, _L, _L, _P, _L, _L, _L, _P, _I, _I, _I, _I, _I, _P, _P, _P,
                              _P, _L, _L, _L, _P, _P, _F, _P, _P, _L, _L, _L, _P],
    "rola_b200_sparse_attn_scatter": [_P, _P, _L, _L, _L, _P, _L, _L, _L, _P, _I, _I, _I, _I, _I, _P, _P,
                                      _P, _F, _P, _I, _I, _I, _P],
    "rola_b200_sparse_attn_fwd_lse": [_P, _P, _L, _L, _L, _P, _L, _L, _L, _P, _I, _I, _I, _I, _I, _P, _L, _L, _L,
                                      _P, _P],
    "rola_b200_sparse_attn_bwd_workspace": [_I, _I, _I, _I],
    "rola_b200_sparse_attn_bwd": [_P, _P, _L, _L, _L, _P, _L, _L, _L, _P, _P, _L, _L, _L, _P, _P, _P, _I, _I, _I,
                                  _I, _I, _P, _P, _P, _L, _L, _L, _P, _Z, _P],
    "rola_b200_peer_alloc": [_Z, ctypes.POINTER(_P), _P],
    "rola_b200_peer_open": [_P, ctypes.POINTER(_P)],
    "rola_b200_peer_close": [_P],
    "rola_b200_peer_free": [_P],
    "rola_b200_lowrank_kv_noalloc": [_P, _L, _L, _L, _P, _L, _L, _L, _P, _P, _P, _I, _I, _I, _I, _I, _I,
                                     _P, _P, _P],
    "rola_b200_forward_workspace_bytes": [_I, _I, _I, _I, _I, _I],
    "rola_b200_pipeline_create": [_Z, _Z, ctypes.POINTER(_P)],
    "rola_b200_pipeline_forward": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I,
                                   _I, _F, _P, _Z, _P, _P],
    "rola_b200_pipeline_wait": [_P, _P],
    "rola_b200_pipeline_destroy": [_P],
    "rola_b200_rola_forward": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I,
                               _I, _I, _F, _P, _Z, _P, _P, _P],
}
_RESTYPES = {
    "rola_b200_last_error": ctypes.c_char_p,
    "rola_b200_forward_workspace_bytes": _Z,
    "rola_b200_sparse_attn_bwd_workspace": _Z,
}

MAX_RANKS = 8


class ScatterArgs(ctypes.Structure):
    """``rola_scatter_args`` of include/rola_b200.h."""

    _fields_ = [("q_raw", _P), ("k_raw", _P), ("v_raw", _P), ("ld_raw", _L), ("ssq", _P), ("ssq_ld", ctypes.c_int32),
                ("B", ctypes.c_int32), ("L", ctypes.c_int32), ("H", ctypes.c_int32), ("world", ctypes.c_int32),
                ("eps", _F), ("dst_rows", _L), ("dst_row0", _L), ("x", _P), ("norm_wq", _P), ("norm_wk", _P),
                ("gate_w", _P), ("gate_b", _P), ("q_dst", _P * MAX_RANKS), ("k_dst", _P * MAX_RANKS),
                ("v_dst", _P * MAX_RANKS), ("g_dst", _P * MAX_RANKS)]


_lock = threading.Lock()
_lib = None


class RolaError(RuntimeError):
    """A librola_b200 entry point returned an error code."""


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the shared library; raise if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RolaError(
                f"librola_b200.so not found at {path}; build it with "
                "`python -c 'import sparkdiffusion_b200.build as b; b.build_library()'`"
            )
        lib = ctypes.CDLL(path)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, _I)
        got = lib.rola_b200_abi_version()
        if got != ABI_VERSION:
            raise RolaError(f"librola_b200.so ABI version {got}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load_library()


def check(rc: int, what: str) -> None:
    """Map a non-zero return code to an exception carrying the library's message."""
    if rc == ROLA_OK:
        return
    msg = lib().rola_b200_last_error().decode(errors="replace")
    if rc == ROLA_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RolaError(f"{what}: {msg} (code {rc})")


def device_status(clear: bool = True) -> int:
    """Synchronise and return the device-side error flag (0 = ok)."""
    v = lib().rola_b200_device_status(1 if clear else 0)
    if v < 0:
        raise RolaError("rola_b200_device_status: CUDA error while reading the device flag")
    return v


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
