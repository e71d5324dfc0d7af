"""The CPU oracle (oracle/mhc_oracle.py) against the golden fixtures that
tests/golden/make_golden.py froze from the reference's own formulation."""
import pytest
import torch

from oracle import mhc_oracle as O
from tests.helpers import golden

DYN_CASES = ["dynamic_cfg1_B32_n4_C256", "dynamic_strong_B8_n4_C64",
             "dynamic_strong_B4_n8_C32", "dynamic_strong_B6_n2_C100"]

PARAM_KEYS = {"rmsnorm_weight": "w", "phi_pre": "phi_pre", "phi_post": "phi_post",
              "phi_res": "phi_res", "alpha_pre": "alpha_pre", "alpha_post": "alpha_post",
              "alpha_res": "alpha_res", "b_pre": "b_pre", "b_post": "b_post", "b_res": "b_res"}


@pytest.fixture(autouse=True)
def _single_thread():
    # The fixtures were generated with one intra-op thread; with the same
    # summation order the restatement reproduces them bit for bit.
    prev = torch.get_num_threads()
    torch.set_num_threads(1)
    yield
    torch.set_num_threads(prev)


def _tight(a, e, what):
    torch.testing.assert_close(a, e, rtol=0, atol=0, msg=what)


@pytest.mark.parametrize("case", DYN_CASES)
def test_dynamic_layer_matches_reference(case):
    z = golden(case)
    params = {k: z[v] for k, v in PARAM_KEYS.items()}
    out, grads = O.dynamic_fwd_bwd(z["x"], params, z.get("grad_out"))
    _tight(out, z["out"], f"{case}: out")
    _tight(grads["x"], z["grad_x"], f"{case}: grad_x")
    for k, v in PARAM_KEYS.items():
        _tight(grads[k], z["grad_" + v], f"{case}: grad_{k}")


def test_static_layer_matches_reference():
    z = golden("static_B16_n4_C128")
    out, grads = O.static_fwd_bwd(z["x"], z["w"], z["H_pre"], z["H_post"], z["H_res"])
    _tight(out, z["out"], "out")
    _tight(grads["x"], z["grad_x"], "grad_x")
    _tight(grads["rmsnorm_weight"], z["grad_w"], "grad_w")
    for k in ("H_pre", "H_post", "H_res"):
        _tight(grads[k], z["grad_" + k], k)


@pytest.mark.parametrize("case", ["sinkhorn_B256_N4", "sinkhorn_B32_N8", "sinkhorn_B64_N2",
                                  "sinkhorn_B8_N16"])
def test_sinkhorn_matches_reference(case):
    z = golden(case)
    inp = z["inp"].clone().requires_grad_(True)
    out = O.sinkhorn_knopp(inp, 20, 1e-8)
    out.backward(z["grad"])
    _tight(out, z["out"], "out")
    _tight(inp.grad, z["grad_inp"], "grad")


def test_sinkhorn_doubly_stochastic():
    z = golden("sinkhorn_B256_N4")
    out = O.sinkhorn_knopp(z["inp"].double(), 20, 1e-8)
    torch.testing.assert_close(out.sum(-1), torch.ones(256, 4, dtype=torch.float64), rtol=0,
                               atol=1e-3)
    torch.testing.assert_close(out.sum(-2), torch.ones(256, 4, dtype=torch.float64), rtol=0,
                               atol=1e-6)


def test_ops_match_reference():
    z = golden("rmsnorm_B16_C4096")
    x = z["x"].clone().requires_grad_(True)
    w = z["w"].clone().requires_grad_(True)
    out = O.rmsnorm(x, w, 1e-5)
    out.backward(z["grad"])
    _tight(out, z["out"], "rmsnorm out")
    _tight(x.grad, z["grad_x"], "rmsnorm grad_x")
    _tight(w.grad, z["grad_w"], "rmsnorm grad_w")

    z = golden("aggregate_B32_n4_C256")
    x = z["x"].clone().requires_grad_(True)
    h = z["H_pre"].clone().requires_grad_(True)
    out = O.stream_aggregate(x, h)
    out.backward(z["grad"])
    _tight(out, z["out"], "aggregate out")
    _tight(x.grad, z["grad_x"], "aggregate grad_x")
    _tight(h.grad, z["grad_H_pre"], "aggregate grad_H")

    z = golden("distribute_B8_n4_C96")
    t = {k: z[k].clone().requires_grad_(True) for k in ("y", "H_post", "M", "x")}
    out = O.stream_distribute_mix_add(t["y"], t["H_post"], t["M"], t["x"])
    out.backward(z["grad"])
    _tight(out, z["out"], "distribute out")
    for k in ("y", "H_post", "M", "x"):
        _tight(t[k].grad, z["grad_" + k], "distribute grad_" + k)


def test_residual_pack_decay():
    r = torch.randn(2, 3, 8)
    b = torch.randn(2, 3, 8)
    s, shape = O.residual_wrapper_pack(r, b, 4)
    assert shape == (2, 3, 8)
    torch.testing.assert_close(s[:, 0], r.reshape(6, 8))
    torch.testing.assert_close(s[:, 1], b.reshape(6, 8))
    torch.testing.assert_close(s[:, 3], r.reshape(6, 8) * 0.01)
