"""The drop-in boundary against the reference itself (CPU).

* ``register_into_reference()`` binds ``"rola_b200"`` into the reference's own
  sparse-attention registry, after which the reference's ``WanModel`` builds
  this package's layer from ``attn_variant="rola_b200"``
  (sparkdiffusion/networks/wan2pt1.py:663-667) and loads a RoLa model's state
  dict key for key, as ``load_checkpoint_auto`` does (model_utils.py:175).
* The layer traces under ``torch.compile`` (the Wan inference entry points
  compile the whole model, inference_optimization.py:122) as custom operators
  with no graph break: run on meta tensors, only the operators' shape
  functions execute.

The reference is imported from ``SPARKDIFFUSION_REF``, ``baseline/_ref`` or the
read-only checkout; the tests skip where none of them exists (the GPU box).
"""

import sys

import pytest
import torch

from conftest import reference_path
from sparkdiffusion_b200 import registry
from sparkdiffusion_b200.layer import WanSelfAttentionRoLaB200


def _reference_path():
    return reference_path(allow_checkout=True)


@pytest.fixture(scope="module")
def wan2pt1():
    path = _reference_path()
    if path is None:
        pytest.skip("the SparkDiffusion reference is not importable here")
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        import sparkdiffusion.networks.wan2pt1 as w
    except Exception as e:  # pragma: no cover - a missing optional dependency of the reference
        pytest.skip(f"reference import failed: {e}")
    return w


TINY = dict(model_type="t2v", patch_size=(1, 2, 2), text_len=8, in_dim=4, dim=256, ffn_dim=512, freq_dim=32,
            text_dim=32, out_dim=4, num_heads=2, num_layers=2)
ROLA = dict(rola_topk_ratio=0.25, rola_rank=64, rola_blkq=128, rola_blkk=128)


def test_wanmodel_builds_and_loads_reference_rola_checkpoint(wan2pt1):
    assert registry.register_into_reference()
    from sparkdiffusion.networks import sparse_attn_registry as ref_reg

    assert ref_reg.get_sparse_attn_class("rola_b200") is WanSelfAttentionRoLaB200
    torch.manual_seed(0)
    ref_model = wan2pt1.WanModel(**TINY, use_rola_attn=True, **ROLA)
    ours = wan2pt1.WanModel(**TINY, attn_variant="rola_b200", attn_variant_kwargs=dict(ROLA))
    for blk_ref, blk in zip(ref_model.blocks, ours.blocks):
        assert type(blk_ref.self_attn).__name__ == "WanSelfAttentionRoLa"
        assert isinstance(blk.self_attn, WanSelfAttentionRoLaB200)
    sd = ref_model.state_dict()
    res = ours.load_state_dict(sd, strict=True)
    assert not res.missing_keys and not res.unexpected_keys
    for name, t in ours.state_dict().items():
        assert torch.equal(t, sd[name]), name
    # the RoLa-specific parameters are the registry's trainable sparse parameters
    names = registry.get_sparse_param_names("rola_b200")
    own = {n.split(".")[-2] if n.endswith(".weight") else n.split(".")[-1]
           for n, _ in ours.blocks[0].self_attn.named_parameters() if any(k in n for k in names)}
    assert own == set(names)


def test_layer_compiles_to_custom_ops_without_graph_break():
    graphs = []

    def backend(gm, example_inputs):
        graphs.append(gm)
        return gm.forward

    torch.manual_seed(0)
    layer = WanSelfAttentionRoLaB200(256, 2, True, 1e-6, **ROLA).to("meta").eval()
    L = 384
    x = torch.empty(1, L, 256, device="meta", dtype=torch.bfloat16)
    freqs = torch.empty(L, 64, device="meta", dtype=torch.float32)
    with torch.no_grad():
        y = torch.compile(layer, backend=backend, fullgraph=True)(x, torch.tensor([L]), freqs)
    assert y.shape == (1, L, 256) and y.device.type == "meta" and y.dtype == layer.o.weight.dtype
    code = "".join(g.code for g in graphs)
    assert "rola_b200.attention_core" in code and "rola_b200.qkv_gemm" in code


def test_custom_op_shape_functions():
    m = "meta"
    bf = torch.bfloat16
    assert torch.ops.rola_b200.qkv_gemm(torch.empty(300, 512, device=m, dtype=bf),
                                        torch.empty(768, 512, device=m, dtype=bf), None).shape == (300, 768)
    lut = torch.ops.rola_b200.block_select(torch.empty(1, 3, 5, 128, device=m, dtype=bf),
                                           torch.empty(1, 3, 7, 128, device=m, dtype=bf), 2)
    assert lut.shape == (3, 5, 2) and lut.dtype == torch.int32
    q = torch.empty(6, 600, 128, device=m, dtype=bf)
    assert torch.ops.rola_b200.fused_sparse_attn(q, q, q, 0.5, 128, 128, 3).shape == (2, 3, 600, 128)
    assert torch.ops.rola_b200.dense_attention(q, q, q, 3).shape == (2, 3, 600, 128)


def test_custom_ops_refuse_cpu_tensors():
    bf = torch.bfloat16
    with pytest.raises((ValueError, RuntimeError)):
        torch.ops.rola_b200.qkv_gemm(torch.zeros(4, 256, dtype=bf), torch.zeros(256, 256, dtype=bf), None)
