"""The drop-in ``mhc_ascend`` module (mhc_ascend_b200.mhc_ascend_shim).

CPU: every call the reference's ops.py makes into its native module
(recorded from the source by tests/golden/make_callsites.py) binds to the
shim's signature.  GPU: the shim driven the way ops.py drives the native
module -- the four operator autograd classes (ops.py:32-265) and the fused
layer's forward -> saved tensors -> backward round trip (ops.py:394-564) --
against the fp64 oracle.  The reference file itself cannot be loaded on the
GPU box, so the test restates those call sequences (same call order,
argument order and dtype casts, with the line of each).
"""
import inspect
import json
import os

import pytest
import torch

from mhc_ascend_b200 import mhc_ascend_shim as shim
from oracle import mhc_oracle as O
from tests.helpers import GOLDEN, close, close_param


def _callsites():
    with open(os.path.join(GOLDEN, "mhc_ascend_callsites.json")) as f:
        return json.load(f)["calls"]


def test_shim_binds_every_reference_call_site():
    sites = _callsites()
    assert len(sites) >= 13
    for c in sites:
        fn = getattr(shim, c["function"], None)
        assert fn is not None, f"ops.py:{c['line']} calls mhc_ascend.{c['function']}"
        args = [object()] * c["positional"]
        kwargs = {k: object() for k in c["keywords"]}
        inspect.signature(fn).bind(*args, **kwargs)  # raises TypeError on mismatch


def test_shim_parameter_names_follow_the_pybind_module():
    # py::arg names of bindings.cpp:1024-1098
    expect = {
        "sinkhorn_knopp_fwd": ["inp", "num_iters", "eps"],
        "sinkhorn_knopp_bwd": ["grad_out", "inp", "out", "num_iters", "eps"],
        "rmsnorm_fwd": ["inp", "weight", "eps"],
        "rmsnorm_bwd": ["grad_out", "inp", "weight", "rms"],
        "stream_aggregate_fwd": ["inp", "H_pre_raw"],
        "stream_aggregate_bwd": ["grad_out", "inp", "H_pre_activated"],
        "stream_distribute_mix_add_fwd": ["y_norm", "H_post_raw", "M", "x_inp"],
        "stream_distribute_mix_add_bwd": ["grad_out", "x_inp", "y_norm", "M", "H_post_activated"],
        "fused_rmsnorm_matmul_fwd": ["inp", "weight"],
        "fused_rmsnorm_matmul_bwd": ["grad_out", "x_flat", "phi_concat"],
        "compute_rms_fwd": ["inp", "eps"],
    }
    for name, params in expect.items():
        assert list(inspect.signature(getattr(shim, name)).parameters) == params, name
    assert set(shim.__all__) >= set(expect) | {"mhc_layer_fwd_dynamic", "mhc_layer_bwd_dynamic"}


@pytest.mark.gpu
def test_shim_operator_calls_as_ops_py_makes_them(cuda):
    gen = torch.Generator().manual_seed(31)
    B, n, C = 16, 4, 256
    # SinkhornKnoppFunction (ops.py:48, 58)
    inp = torch.rand(64, n, n, generator=gen)
    g = torch.randn(64, n, n, generator=gen)
    out = shim.sinkhorn_knopp_fwd(inp.to(cuda), 20, 1e-8)
    gi = shim.sinkhorn_knopp_bwd(g.to(cuda), inp.to(cuda), out, 20, 1e-8)
    r = inp.double().requires_grad_(True)
    ro = O.sinkhorn_knopp(r, 20, 1e-8)
    ro.backward(g.double())
    close(out, ro, what="shim sinkhorn out")
    close(gi, r.grad, what="shim sinkhorn grad")
    # StreamAggregateFunction (ops.py:160, 169): the caller applies sigma'
    x = torch.randn(B, n, C, generator=gen)
    hraw = torch.randn(B, n, generator=gen)
    ga = torch.randn(B, C, generator=gen)
    out, h_act = shim.stream_aggregate_fwd(x.to(cuda), hraw.to(cuda))
    gx, gh_act = shim.stream_aggregate_bwd(ga.to(cuda), x.to(cuda), h_act)
    gh = gh_act * h_act * (1.0 - h_act)
    rx, rh = x.double().requires_grad_(True), hraw.double().requires_grad_(True)
    ro = O.stream_aggregate(rx, rh)
    ro.backward(ga.double())
    close(out, ro, what="shim aggregate out")
    close(gx, rx.grad, what="shim aggregate grad_x")
    close(gh, rh.grad, what="shim aggregate grad_H_pre")
    # StreamDistributeMixAddFunction (ops.py:223, 236)
    y = torch.randn(B, C, generator=gen)
    hq = torch.randn(B, n, generator=gen)
    M = torch.rand(B, n, n, generator=gen)
    gd = torch.randn(B, n, C, generator=gen)
    out, hq_act = shim.stream_distribute_mix_add_fwd(y.to(cuda), hq.to(cuda), M.to(cuda), x.to(cuda))
    gxd, gy, gM, ghq_act = shim.stream_distribute_mix_add_bwd(gd.to(cuda), x.to(cuda), y.to(cuda),
                                                              M.to(cuda), hq_act)
    ghq = ghq_act * hq_act * (1.0 - hq_act / 2.0)
    ts = [t.double().requires_grad_(True) for t in (y, hq, M, x)]
    ro = O.stream_distribute_mix_add(*ts)
    ro.backward(gd.double())
    close(out, ro, what="shim distribute out")
    for a, t, k in zip((gy, ghq, gM, gxd), ts, ("y", "H_post", "M", "x")):
        close(a, t.grad, what="shim distribute grad_" + k)
    # FusedProjectionFunction (ops.py:279, 290) and compute_rms (ops.py:330)
    xf = torch.randn(B, n * C, generator=gen)
    phi = torch.randn(24, n * C, generator=gen) * 0.02
    gp = torch.randn(B, 24, generator=gen)
    p = shim.fused_rmsnorm_matmul_fwd(xf.to(cuda), phi.to(cuda))
    gxf, gphi = shim.fused_rmsnorm_matmul_bwd(gp.to(cuda), xf.to(cuda), phi.to(cuda))
    close(p, xf.double() @ phi.double().t(), what="shim projection")
    close(gxf, gp.double() @ phi.double(), what="shim projection grad_x")
    close_param(gphi, gp.double().t() @ xf.double(), what="shim projection grad_phi")
    close(shim.compute_rms_fwd(xf.to(cuda), 1e-5), O.compute_rms(xf.double(), 1e-5),
          what="shim compute_rms")


@pytest.mark.gpu
def test_shim_fused_layer_round_trip(cuda):
    """ops.py:424-446 (forward: cat of phi, alphas as host floats, 9 outputs,
    all saved) then ops.py:518-541 (backward: the saved tensors handed back in
    order, 11 gradients)."""
    B, n, C = 48, 4, 512
    gen = torch.Generator().manual_seed(32)
    x = torch.randn(B, n, C, generator=gen)
    params = O.make_dynamic_params(n, C, gen, alpha=0.5, bias_std=0.5, weight="rand")
    grad = torch.randn(B, n, C, generator=gen)
    d = {k: v.to(cuda) for k, v in params.items()}
    phi_concat = torch.cat([d["phi_pre"], d["phi_post"], d["phi_res"].view(n * n, -1)], 0).contiguous()
    res = shim.mhc_layer_fwd_dynamic(
        x.to(cuda).contiguous(), d["rmsnorm_weight"], phi_concat, float(d["alpha_pre"].item()),
        float(d["alpha_post"].item()), float(d["alpha_res"].item()), d["b_pre"], d["b_post"],
        d["b_res"], 20, 1e-8, 1e-5)
    assert len(res) == 9
    output, rms, x_agg_bf16, h_pre, h_post, M, y_norm_bf16, x_flat_bf16, rms_h = res
    grads = shim.mhc_layer_bwd_dynamic(
        grad.to(cuda), x.to(cuda), d["rmsnorm_weight"], rms.contiguous(), x_agg_bf16.contiguous(),
        h_pre.contiguous(), h_post.contiguous(), M.contiguous(), y_norm_bf16.contiguous(),
        x_flat_bf16.contiguous(), rms_h.contiguous(), d["phi_pre"], d["phi_post"], d["phi_res"],
        float(d["alpha_pre"].item()), float(d["alpha_post"].item()), float(d["alpha_res"].item()),
        d["b_pre"], d["b_post"], d["b_res"], 20, 1e-8, 1e-5)
    assert len(grads) == 11
    ro, rg = O.dynamic_fwd_bwd(x.double(), {k: v.double() for k, v in params.items()},
                               grad.double())
    close(output, ro, what="shim layer out")
    close(grads[0], rg["x"], what="shim layer grad_x")
    names = ("rmsnorm_weight", "phi_pre", "phi_post", "phi_res", "alpha_pre", "alpha_post",
             "alpha_res", "b_pre", "b_post", "b_res")
    for gv, k in zip(grads[1:], names):
        close_param(gv.reshape(rg[k].shape), rg[k], what="shim layer grad_" + k)
    # the record's views carry the reference's per-token quantities
    xo = x.double()
    rmsh = torch.sqrt((xo.reshape(B, -1) ** 2).mean(-1) + 1e-5)
    close(rms_h, rmsh, what="shim layer rms_h")
    with pytest.raises(RuntimeError, match="record"):
        shim.mhc_layer_bwd_dynamic(grad.to(cuda), x.to(cuda), d["rmsnorm_weight"], rms,
                                   torch.empty(0, device=cuda), h_pre, h_post, M, y_norm_bf16,
                                   x_flat_bf16, rms_h, d["phi_pre"], d["phi_post"], d["phi_res"],
                                   0.5, 0.5, 0.5, d["b_pre"], d["b_post"], d["b_res"])
