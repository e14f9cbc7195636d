"""Sparse-attention plugin registry (same contract as the reference's).

Mirrors ``sparkdiffusion/networks/sparse_attn_registry.py``: a name -> class
map, the trainable parameter names each variant adds, a decorator that refuses
to bind an existing name to a different class (ValueError, :46-48) and a
lookup that raises KeyError with the registered names (:54-62).

``register_into_reference()`` binds this package's variant into the
reference's own registry when ``sparkdiffusion`` is importable, which is the
drop-in route: ``WanModel(attn_variant="rola_b200", ...)`` then builds it with
no change to the reference's files.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Type

SPARSE_ATTN_REGISTRY: Dict[str, Type] = {}
SPARSE_ATTN_PARAM_NAMES: Dict[str, List[str]] = {}


def register_sparse_attn(name: str, sparse_param_names: Optional[List[str]] = None):
    def _decorator(cls):
        if name in SPARSE_ATTN_REGISTRY and SPARSE_ATTN_REGISTRY[name] is not cls:
            raise ValueError(f"sparse attention variant '{name}' is already registered as {SPARSE_ATTN_REGISTRY[name]}")
        SPARSE_ATTN_REGISTRY[name] = cls
        SPARSE_ATTN_PARAM_NAMES[name] = list(sparse_param_names or [])
        return cls

    return _decorator


def get_sparse_attn_class(name: str) -> Type:
    if name not in SPARSE_ATTN_REGISTRY:
        raise KeyError(
            f"unknown attn_variant='{name}'. Registered: {sorted(SPARSE_ATTN_REGISTRY)}. "
            f"Register your sparse-attention class with @register_sparse_attn('{name}') and import its module."
        )
    return SPARSE_ATTN_REGISTRY[name]


def get_sparse_param_names(name: str) -> List[str]:
    return list(SPARSE_ATTN_PARAM_NAMES.get(name, []))


def register_into_reference() -> bool:
    """Register every variant of this registry into the reference's registry.

    Returns False when ``sparkdiffusion`` is not importable."""
    try:
        from sparkdiffusion.networks import sparse_attn_registry as ref  # type: ignore
    except Exception:
        return False
    for name, cls in SPARSE_ATTN_REGISTRY.items():
        ref.register_sparse_attn(name, sparse_param_names=SPARSE_ATTN_PARAM_NAMES[name])(cls)
    return True
