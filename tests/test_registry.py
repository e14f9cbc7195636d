"""Plugin boundary on CPU: registry contract, constructor, parameter names."""

import pytest
import torch

from sparkdiffusion_b200 import registry
from sparkdiffusion_b200.layer import WanSelfAttentionRoLaB200

# parameter names/shapes of the reference's WanSelfAttentionRoLa
# (sparkdiffusion/networks/wan_rola_attention.py:241-264) for dim=256, 2 heads, rank 64
REFERENCE_PARAMS = {
    "q.weight": (256, 256), "q.bias": (256,), "k.weight": (256, 256), "k.bias": (256,),
    "v.weight": (256, 256), "v.bias": (256,), "o.weight": (256, 256), "o.bias": (256,),
    "norm_q.weight": (256,), "norm_k.weight": (256,),
    "proj_q.weight": (64, 128), "proj_k.weight": (64, 128), "gate_proj.weight": (1, 128),
    "gate_bias": (1, 2, 1, 1),
}


def test_registered_variant():
    cls = registry.get_sparse_attn_class("rola_b200")
    assert cls is WanSelfAttentionRoLaB200
    assert registry.get_sparse_param_names("rola_b200") == ["proj_q", "proj_k", "gate_proj", "gate_bias"]


def test_registry_errors():
    with pytest.raises(KeyError):
        registry.get_sparse_attn_class("no_such_variant")

    @registry.register_sparse_attn("_tmp_variant")
    class A:  # noqa: N801
        pass

    registry.register_sparse_attn("_tmp_variant")(A)  # same class: allowed
    with pytest.raises(ValueError):
        @registry.register_sparse_attn("_tmp_variant")
        class B:  # noqa: N801
            pass
    registry.SPARSE_ATTN_REGISTRY.pop("_tmp_variant")
    registry.SPARSE_ATTN_PARAM_NAMES.pop("_tmp_variant")


def test_state_dict_matches_reference_layer():
    m = WanSelfAttentionRoLaB200(256, 2, True, 1e-6, rola_rank=64)
    got = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert got == REFERENCE_PARAMS
    assert torch.all(m.gate_bias == -1.946)
    assert torch.all(m.gate_proj.weight == 0)


def test_forward_refuses_cpu_and_grad():
    m = WanSelfAttentionRoLaB200(256, 2)
    x = torch.randn(1, 256, 256)
    freqs = torch.zeros(256, 64)
    with torch.no_grad():
        with pytest.raises(RuntimeError):
            m.eval()(x, None, freqs)
    m.train()
    with pytest.raises(RuntimeError):
        m(x, None, freqs)


def test_constructor_validation():
    with pytest.raises(ValueError):
        WanSelfAttentionRoLaB200(256, 2, attn_precision="fp4")


def test_dense_layer_params_match_reference_dense_layer():
    """WanSelfAttentionB200 carries WanSelfAttention's parameters (wan2pt1.py:221-239)."""
    from sparkdiffusion_b200.layer import WanSelfAttentionB200

    m = WanSelfAttentionB200(256, 2, True, 1e-6)
    got = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    dense = {k: v for k, v in REFERENCE_PARAMS.items() if k.split(".")[0] in ("q", "k", "v", "o", "norm_q", "norm_k")}
    assert got == dense
    assert torch.all(m.q.bias == 0) and torch.all(m.norm_q.weight == 1)


def test_dense_path_validates_on_the_host():
    from sparkdiffusion_b200 import ops
    from sparkdiffusion_b200.layer import WanSelfAttentionB200

    q = torch.zeros(4, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.dense_attention(q, q, q, num_heads=3)  # 4 is not a multiple of 3
    with pytest.raises(ValueError):
        ops.dense_attention(q[..., :64], q[..., :64], q[..., :64], num_heads=2)  # head dim 64
    with pytest.raises((RuntimeError, ValueError)):
        ops.dense_attention(q, q, q, num_heads=2)  # CPU tensors: no fallback
    m = WanSelfAttentionB200(256, 2).eval()
    with torch.no_grad(), pytest.raises(RuntimeError):
        m(torch.zeros(1, 256, 256), torch.tensor([256]), torch.zeros(256, 64))
