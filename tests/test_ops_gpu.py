"""Per-operator parity of the CUDA kernels with the reference formulation
(golden fixtures from the reference, plus the CPU oracle on random inputs)."""
import pytest
import torch

import mhc_ascend_b200 as mhc
from mhc_ascend_b200 import ops
from oracle import mhc_oracle as O
from tests.helpers import close, close_param, close_ref, golden

pytestmark = pytest.mark.gpu


def _grad_of(fn, inputs, grad, dev):
    ts = [t.to(dev).clone().requires_grad_(True) for t in inputs]
    out = fn(*ts)
    out.backward(grad.to(dev))
    return out, [t.grad for t in ts]


@pytest.mark.parametrize("case", ["sinkhorn_B256_N4", "sinkhorn_B32_N8", "sinkhorn_B64_N2",
                                  "sinkhorn_B8_N16"])
def test_sinkhorn_golden(cuda, case):
    z = golden(case)
    out, (g,) = _grad_of(lambda a: mhc.sinkhorn_knopp(a, 20, 1e-8), [z["inp"]], z["grad"], cuda)
    ref = z["inp"].double().requires_grad_(True)
    ro = O.sinkhorn_knopp(ref, 20, 1e-8)
    ro.backward(z["grad"].double())
    close_ref(out, z["out"], ro, what="sinkhorn out")
    close_ref(g, z["grad_inp"], ref.grad, what="sinkhorn grad")


@pytest.mark.parametrize("B,N,iters", [(65536, 4, 20), (1, 4, 20), (7, 3, 50), (5, 32, 20),
                                       (9, 5, 0), (3, 8, 1),
                                       # warp-per-matrix sizes with idle lanes, several blocks,
                                       # and more iterations than one saved segment
                                       (6, 12, 20), (4, 17, 33), (3, 31, 20), (2, 9, 5),
                                       (41, 16, 20)])
def test_sinkhorn_oracle(cuda, B, N, iters):
    gen = torch.Generator().manual_seed(B * 31 + N)
    inp = torch.rand(B, N, N, generator=gen)
    grad = torch.randn(B, N, N, generator=gen)
    ref = inp.double().requires_grad_(True)
    ro = O.sinkhorn_knopp(ref, iters, 1e-8)
    ro.backward(grad.double())
    out, (g,) = _grad_of(lambda a: mhc.sinkhorn_knopp(a, iters, 1e-8), [inp], grad, cuda)
    close(out, ro, what="sinkhorn out")
    close(g, ref.grad, what="sinkhorn grad")


def test_sinkhorn_doubly_stochastic_full_size(cuda):
    inp = torch.rand(65536, 4, 4, device=cuda)
    out = mhc.sinkhorn_knopp(inp, 20, 1e-8)
    assert torch.allclose(out.sum(-2), torch.ones_like(out.sum(-2)), atol=1e-5)
    assert torch.allclose(out.sum(-1), torch.ones_like(out.sum(-1)), atol=2e-2)


def test_rmsnorm_golden(cuda):
    z = golden("rmsnorm_B16_C4096")
    out, (gx, gw) = _grad_of(lambda a, w: mhc.rmsnorm(a, w, 1e-5), [z["x"], z["w"]], z["grad"], cuda)
    rx, rw = z["x"].double().requires_grad_(True), z["w"].double().requires_grad_(True)
    ro = O.rmsnorm(rx, rw, 1e-5)
    ro.backward(z["grad"].double())
    close_ref(out, z["out"], ro, what="rmsnorm out")
    close_ref(gx, z["grad_x"], rx.grad, what="rmsnorm grad_x")
    close_ref(gw, z["grad_w"], rw.grad, what="rmsnorm grad_w", scaled=True)


@pytest.mark.parametrize("B,C", [(1024, 4096), (3, 100), (1, 4097)])
def test_rmsnorm_oracle(cuda, B, C):
    gen = torch.Generator().manual_seed(B + C)
    x = torch.randn(B, C, generator=gen)
    w = torch.rand(C, generator=gen) + 0.5
    grad = torch.randn(B, C, generator=gen)
    rx, rw = x.double().requires_grad_(True), w.double().requires_grad_(True)
    ro = O.rmsnorm(rx, rw, 1e-5)
    ro.backward(grad.double())
    out, (gx, gw) = _grad_of(lambda a, b: mhc.rmsnorm(a, b, 1e-5), [x, w], grad, cuda)
    close(out, ro, what="out")
    close(gx, rx.grad, what="grad_x")
    close_param(gw, rw.grad, what="grad_w")


def test_aggregate_golden(cuda):
    z = golden("aggregate_B32_n4_C256")
    out, (gx, gh) = _grad_of(mhc.stream_aggregate, [z["x"], z["H_pre"]], z["grad"], cuda)
    close(out, z["out"], what="aggregate out")
    close(gx, z["grad_x"], what="aggregate grad_x")
    close(gh, z["grad_H_pre"], what="aggregate grad_H_pre")


def test_distribute_golden(cuda):
    z = golden("distribute_B8_n4_C96")
    out, grads = _grad_of(mhc.stream_distribute_mix_add, [z["y"], z["H_post"], z["M"], z["x"]],
                          z["grad"], cuda)
    close(out, z["out"], what="distribute out")
    for g, k in zip(grads, ("y", "H_post", "M", "x")):
        close(g, z["grad_" + k], what="distribute grad_" + k)


@pytest.mark.parametrize("B,n,C", [(4, 8, 333), (2, 1, 5), (70000, 2, 4)])
def test_stream_ops_oracle(cuda, B, n, C):
    gen = torch.Generator().manual_seed(B + n + C)
    x = torch.randn(B, n, C, generator=gen)
    h = torch.randn(B, n, generator=gen)
    y = torch.randn(B, C, generator=gen)
    M = torch.rand(B, n, n, generator=gen)
    ga = torch.randn(B, C, generator=gen)
    gd = torch.randn(B, n, C, generator=gen)
    r = [t.double().requires_grad_(True) for t in (x, h)]
    ro = O.stream_aggregate(*r)
    ro.backward(ga.double())
    out, grads = _grad_of(mhc.stream_aggregate, [x, h], ga, cuda)
    close(out, ro, what="aggregate")
    close(grads[0], r[0].grad, what="aggregate gx")
    close(grads[1], r[1].grad, what="aggregate gh")
    r = [t.double().requires_grad_(True) for t in (y, h, M, x)]
    ro = O.stream_distribute_mix_add(*r)
    ro.backward(gd.double())
    out, grads = _grad_of(mhc.stream_distribute_mix_add, [y, h, M, x], gd, cuda)
    close(out, ro, what="distribute")
    for g, rr, k in zip(grads, r, "y h M x".split()):
        close(g, rr.grad, what="distribute grad " + k)


@pytest.mark.parametrize("B,K,O_", [(64, 16384, 24), (5, 1000, 7)])
def test_projection_and_rms(cuda, B, K, O_):
    gen = torch.Generator().manual_seed(K)
    x = torch.randn(B, K, generator=gen)
    w = torch.randn(O_, K, generator=gen) * 0.02
    g = torch.randn(B, O_, generator=gen)
    rx, rw = x.double().requires_grad_(True), w.double().requires_grad_(True)
    ro = rx @ rw.t()
    ro.backward(g.double())
    xs, ws = x.to(cuda).requires_grad_(True), w.to(cuda).requires_grad_(True)
    out = ops.fused_rmsnorm_matmul(xs, ws)
    out.backward(g.to(cuda))
    close(out, ro, what="proj")
    close(xs.grad, rx.grad, what="proj grad_x")
    close_param(ws.grad, rw.grad, what="proj grad_w")
    rms = ops.compute_rms(x.to(cuda), 1e-5)
    close(rms, O.compute_rms(x.double(), 1e-5), what="compute_rms")
