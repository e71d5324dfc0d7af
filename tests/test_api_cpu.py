"""Host-side API checks (no GPU): reference names/shapes, errors instead of
a CPU fallback, checkpoint interchange."""
import pytest
import torch

import mhc_ascend_b200 as mhc
from mhc_ascend_b200 import ops


def test_public_api_matches_reference():
    assert set(mhc.__all__) == {"MHCLayer", "MHCResidualWrapper", "create_mhc_layer",
                                "replace_residual_with_mhc", "sinkhorn_knopp", "rmsnorm",
                                "stream_aggregate", "stream_distribute_mix_add"}
    assert mhc.__version__ == "0.1.0"


def test_dynamic_parameters_match_reference_names_and_shapes():
    layer = mhc.MHCLayer(hidden_dim=64, expansion_rate=4)
    shapes = {k: tuple(v.shape) for k, v in layer.state_dict().items()}
    assert shapes == {"rmsnorm_weight": (64,), "phi_pre": (4, 256), "phi_post": (4, 256),
                      "phi_res": (16, 256), "b_pre": (4,), "b_post": (4,), "b_res": (4, 4),
                      "alpha_pre": (), "alpha_post": (), "alpha_res": ()}
    assert float(layer.alpha_pre) == pytest.approx(0.01)


def test_static_parameters_match_reference():
    layer = mhc.create_mhc_layer(hidden_dim=32, expansion_rate=2, use_dynamic_h=False)
    assert {k: tuple(v.shape) for k, v in layer.state_dict().items()} == {
        "rmsnorm_weight": (32,), "H_pre": (2,), "H_post": (2,), "H_res": (2, 2)}


def test_reference_checkpoint_with_bf16_weight_loads():
    layer = mhc.MHCLayer(hidden_dim=16, expansion_rate=4)
    sd = {k: v.clone() for k, v in layer.state_dict().items()}
    sd["rmsnorm_weight"] = torch.full((16,), 1.5, dtype=torch.bfloat16)
    layer.load_state_dict(sd)
    assert layer.rmsnorm_weight.dtype == torch.float32
    assert torch.all(layer.rmsnorm_weight == 1.5)


@pytest.mark.parametrize("fn,args", [
    (mhc.sinkhorn_knopp, (torch.rand(2, 4, 4),)),
    (mhc.rmsnorm, (torch.rand(2, 8), torch.ones(8))),
    (mhc.stream_aggregate, (torch.rand(2, 4, 8), torch.rand(2, 4))),
    (mhc.stream_distribute_mix_add, (torch.rand(2, 8), torch.rand(2, 4), torch.rand(2, 4, 4),
                                     torch.rand(2, 4, 8))),
])
def test_cpu_tensors_raise_no_fallback(fn, args):
    with pytest.raises(RuntimeError, match="CUDA"):
        fn(*args)


def test_layer_on_cpu_raises():
    layer = mhc.MHCLayer(hidden_dim=8, expansion_rate=4)
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.randn(2, 4, 8))


def test_wrapper_modes():
    w = mhc.replace_residual_with_mhc(hidden_dim=8, expansion_rate=4, residual_mode="bogus")
    with pytest.raises(ValueError):
        w(torch.randn(2, 8), torch.randn(2, 8))
    assert w.use_post_norm is False
