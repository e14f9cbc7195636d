"""B200-native (sm_100a) RoLa attention forward for SparkDiffusion's Wan models.

The package holds the host mirror of the reference's plugin/operator interface
(``registry``, ``layer``, ``ops``), the Ulysses multi-GPU exchange
(``ulysses``), and the CUDA sources of ``librola_b200.so`` (``csrc``), whose C
ABI is declared in ``include/rola_b200.h``.
"""

from .registry import get_sparse_attn_class, get_sparse_param_names, register_sparse_attn, register_into_reference
from .layer import WanSelfAttentionRoLaB200

__all__ = [
    "WanSelfAttentionRoLaB200",
    "register_sparse_attn",
    "get_sparse_attn_class",
    "get_sparse_param_names",
    "register_into_reference",
]
