"""Fused mHC layer parity (dynamic and static H, forward and backward) with the
reference formulation: golden fixtures, the CPU oracle at random shapes, and
size-independent properties at the BASELINE full sizes."""
import pytest
import torch

import mhc_ascend_b200 as mhc
from oracle import mhc_oracle as O
from tests.helpers import close, close_param, close_ref, golden, rel_err

pytestmark = pytest.mark.gpu

KEYS = {"rmsnorm_weight": "w", "phi_pre": "phi_pre", "phi_post": "phi_post", "phi_res": "phi_res",
        "alpha_pre": "alpha_pre", "alpha_post": "alpha_post", "alpha_res": "alpha_res",
        "b_pre": "b_pre", "b_post": "b_post", "b_res": "b_res"}


def make_layer(params, n, C, dev, iters=20, s_eps=1e-8, r_eps=1e-5):
    layer = mhc.MHCLayer(hidden_dim=C, expansion_rate=n, num_sinkhorn_iters=iters,
                         sinkhorn_eps=s_eps, rmsnorm_eps=r_eps).to(dev)
    with torch.no_grad():
        for k, v in params.items():
            getattr(layer, k).copy_(v.reshape(getattr(layer, k).shape))
    return layer


def run_layer(layer, x, grad_out=None):
    x = x.clone().requires_grad_(True)
    out = layer(x)
    if grad_out is None:
        (out ** 2).sum().backward()
    else:
        out.backward(grad_out)
    grads = {"x": x.grad}
    grads.update({k: p.grad for k, p in layer.named_parameters()})
    return out.detach(), grads


@pytest.mark.parametrize("case", ["dynamic_cfg1_B32_n4_C256", "dynamic_strong_B8_n4_C64",
                                  "dynamic_strong_B4_n8_C32", "dynamic_strong_B6_n2_C100"])
def test_dynamic_golden(cuda, case):
    z = golden(case)
    B, n, C = z["x"].shape
    layer = make_layer({k: z[v] for k, v in KEYS.items()}, n, C, cuda)
    g = z["grad_out"].to(cuda) if "grad_out" in z else None
    out, grads = run_layer(layer, z["x"].to(cuda), g)
    ro, rg = O.dynamic_fwd_bwd(z["x"].double(), {k: z[v].double() for k, v in KEYS.items()},
                               z["grad_out"].double() if "grad_out" in z else None)
    close_ref(out, z["out"], ro, what="out")
    close_ref(grads["x"], z["grad_x"], rg["x"], what="grad_x")
    for k, v in KEYS.items():
        close_ref(grads[k], z["grad_" + v], rg[k], what="grad_" + k, scaled=True)


def oracle_case(B, n, C, seed, alpha=0.01, bias_std=0.0, weight=None):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, n, C, generator=gen)
    params = O.make_dynamic_params(n, C, gen, alpha=alpha, bias_std=bias_std, weight=weight)
    grad = torch.randn(B, n, C, generator=gen)
    return x, params, grad


@pytest.mark.parametrize("B,n,C,alpha,bias", [
    (64, 4, 4096, 0.01, 0.0),     # BASELINE shape family (cfg3 channels)
    (37, 4, 4096, 1.0, 1.0),      # strong gating, token count not a tile multiple
    (5, 4, 4097, 0.5, 0.5),       # C not a multiple of 4: scalar paths
    (3, 8, 256, 0.5, 0.5),
    (11, 2, 100, 1.0, 1.0),
    (6, 3, 96, 1.0, 1.0),
    (4, 1, 64, 1.0, 1.0),
    (2, 6, 72, 0.5, 0.5),
    (1, 4, 32, 1.0, 1.0),         # single token
    # wide expansion rates (GEMM projection, warp Sinkhorn, n x n mixes)
    (9, 16, 64, 0.5, 0.5),
    (5, 32, 96, 1.0, 1.0),
    (130, 12, 40, 0.5, 0.5),      # tokens span two GEMM row tiles
    (3, 9, 33, 1.0, 1.0),         # odd n, odd C
    (32, 32, 1280, 0.01, 0.0),    # the reference's paper shape (benchmark.py:302-312)
    (1024, 6, 64, 0.5, 0.5),      # n = 6, 7 switch to the wide-rate kernels from 1024 tokens
    (1100, 7, 40, 1.0, 1.0),
    (1023, 7, 40, 1.0, 1.0),      # ... and stay on the fused kernels below
])
def test_dynamic_vs_oracle(cuda, B, n, C, alpha, bias):
    x, params, grad = oracle_case(B, n, C, seed=B * 7 + n * 13 + C, alpha=alpha, bias_std=bias,
                                  weight="rand")
    ro, rg = O.dynamic_fwd_bwd(x.double(), {k: v.double() for k, v in params.items()},
                               grad.double())
    layer = make_layer(params, n, C, cuda)
    out, grads = run_layer(layer, x.to(cuda), grad.to(cuda))
    close(out, ro, what="out")
    close(grads["x"], rg["x"], what="grad_x")
    for k in KEYS:
        close_param(grads[k], rg[k], what="grad_" + k)


def test_dynamic_inference_matches_training_forward(cuda):
    x, params, _ = oracle_case(16, 4, 512, seed=5, alpha=1.0, bias_std=1.0)
    layer = make_layer(params, 4, 512, cuda)
    xd = x.to(cuda)
    out_train = layer(xd)
    layer.eval()
    with torch.no_grad():
        out_inf = layer(xd)
    assert torch.equal(out_train.detach(), out_inf)


@pytest.mark.parametrize("B,n,C", [(512, 4, 1024), (64, 32, 256)])
def test_dynamic_backward_is_deterministic(cuda, B, n, C):
    x, params, grad = oracle_case(B, n, C, seed=9)
    layer = make_layer(params, n, C, cuda)
    _, g1 = run_layer(layer, x.to(cuda), grad.to(cuda))
    layer.zero_grad()
    _, g2 = run_layer(layer, x.to(cuda), grad.to(cuda))
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


def test_dynamic_cfg3_full_size(cuda):
    """BASELINE cfg3: B=8192, n=4, C=4096.  The CPU oracle runs the whole batch
    (a few seconds); additionally the parameter gradients are linear in the
    batch: grads(full) == grads(first half) + grads(second half)."""
    B, n, C = 8192, 4, 4096
    x, params, grad = oracle_case(B, n, C, seed=0)
    layer = make_layer(params, n, C, cuda)
    xd, gd = x.to(cuda), grad.to(cuda)
    out, grads = run_layer(layer, xd, gd)
    ro, rg = O.dynamic_fwd_bwd(x, params, grad)
    close(out, ro, what="out")
    close(grads["x"], rg["x"], what="grad_x")
    for k in KEYS:
        close_param(grads[k], rg[k], what="grad_" + k)
    halves = []
    for sl in (slice(0, B // 2), slice(B // 2, B)):
        layer.zero_grad()
        _, gh = run_layer(layer, xd[sl], gd[sl])
        halves.append(gh)
    for k in KEYS:
        close_param(halves[0][k] + halves[1][k], grads[k], what="linearity " + k)


def test_static_golden(cuda):
    z = golden("static_B16_n4_C128")
    layer = mhc.MHCLayer(hidden_dim=128, expansion_rate=4, use_dynamic_h=False).to(cuda)
    with torch.no_grad():
        layer.rmsnorm_weight.copy_(z["w"])
        layer.H_pre.copy_(z["H_pre"])
        layer.H_post.copy_(z["H_post"])
        layer.H_res.copy_(z["H_res"])
    out, grads = run_layer(layer, z["x"].to(cuda))
    ro, rg = O.static_fwd_bwd(z["x"].double(), z["w"].double(), z["H_pre"].double(),
                              z["H_post"].double(), z["H_res"].double())
    close_ref(out, z["out"], ro, what="out")
    close_ref(grads["x"], z["grad_x"], rg["x"], what="grad_x")
    close_ref(grads["rmsnorm_weight"], z["grad_w"], rg["rmsnorm_weight"], what="grad_w", scaled=True)
    for k in ("H_pre", "H_post", "H_res"):
        close_ref(grads[k], z["grad_" + k], rg[k], what=k, scaled=True)


@pytest.mark.parametrize("B,n,C", [(64, 4, 4096), (7, 4, 7168), (3, 8, 100), (5, 2, 4097),
                                   (2, 4, 20000), (6, 16, 96), (4, 32, 64), (3, 9, 33)])
def test_static_vs_oracle(cuda, B, n, C):
    gen = torch.Generator().manual_seed(B + C)
    x = torch.randn(B, n, C, generator=gen)
    Hp, Hq, Hr = (torch.randn(n, generator=gen), torch.randn(n, generator=gen),
                  torch.randn(n, n, generator=gen))
    w = torch.rand(C, generator=gen) + 0.5
    grad = torch.randn(B, n, C, generator=gen)
    ro, rg = O.static_fwd_bwd(x.double(), w.double(), Hp.double(), Hq.double(), Hr.double(),
                              grad.double())
    layer = mhc.MHCLayer(hidden_dim=C, expansion_rate=n, use_dynamic_h=False).to(cuda)
    with torch.no_grad():
        layer.rmsnorm_weight.copy_(w); layer.H_pre.copy_(Hp)
        layer.H_post.copy_(Hq); layer.H_res.copy_(Hr)
    out, grads = run_layer(layer, x.to(cuda), grad.to(cuda))
    close(out, ro, what="out")
    close(grads["x"], rg["x"], what="grad_x")
    for k in ("rmsnorm_weight", "H_pre", "H_post", "H_res"):
        close_param(grads[k], rg[k], what=k)
    layer.eval()
    with torch.no_grad():
        close(layer(x.to(cuda)), ro, what="inference out")


def test_static_bf16_io(cuda):
    """bf16 storage, fp32 arithmetic: compare with the oracle on the same
    bf16-rounded input; the only extra error is the bf16 rounding of the output
    (relative 2^-9), so the stated tolerance is rtol 8e-3 / atol 1e-2."""
    B, n, C = 256, 4, 4096
    gen = torch.Generator().manual_seed(4)
    x = torch.randn(B, n, C, generator=gen).bfloat16()
    Hp, Hq, Hr = torch.randn(n, generator=gen), torch.randn(n, generator=gen), torch.randn(n, n, generator=gen)
    layer = mhc.MHCLayer(hidden_dim=C, expansion_rate=n, use_dynamic_h=False, bf16_io=True).to(cuda)
    with torch.no_grad():
        layer.H_pre.copy_(Hp); layer.H_post.copy_(Hq); layer.H_res.copy_(Hr)
    layer.eval()
    with torch.no_grad():
        out = layer(x.to(cuda))
    assert out.dtype == torch.bfloat16
    ro = O.mhc_layer_static(x.double(), torch.ones(C, dtype=torch.float64), Hp.double(),
                            Hq.double(), Hr.double())
    close(out.float(), ro, rtol=8e-3, atol=1e-2, what="bf16 out")


@pytest.mark.parametrize("B,C", [(256, 4096), (37, 1024)])
def test_dynamic_bf16_io(cuda, B, C):
    """bf16 streams (x, out, grad_out, grad_x) with fp32 arithmetic, against the
    oracle in fp64 on the same bf16-rounded x and grad_out.  out and grad_x
    carry one bf16 rounding of the result (relative 2^-9): rtol 8e-3 / atol
    1e-2 at the tensor's scale.  The parameter gradients are fp32 and keep the
    fp32 tolerances."""
    n = 4
    x, params, grad = oracle_case(B, n, C, seed=B + C, alpha=0.5, bias_std=0.5, weight="rand")
    xb, gb = x.bfloat16(), grad.bfloat16()
    ro, rg = O.dynamic_fwd_bwd(xb.double(), {k: v.double() for k, v in params.items()},
                               gb.double())
    layer = make_layer(params, n, C, cuda)
    layer.bf16_io = True
    xd = xb.to(cuda).requires_grad_(True)
    out = layer(xd)
    assert out.dtype == torch.bfloat16
    out.backward(gb.to(cuda))
    assert xd.grad.dtype == torch.bfloat16
    close(out.float(), ro, rtol=8e-3, atol=1e-2, what="bf16 out")
    close(xd.grad.float(), rg["x"], rtol=8e-3, atol=1e-2, what="bf16 grad_x")
    for k in KEYS:
        close_param(getattr(layer, k).grad, rg[k], what="grad_" + k)
    layer.eval()
    with torch.no_grad():
        assert torch.equal(layer(xb.to(cuda)), out.detach())


def test_dynamic_bf16_io_rejects_unsupported_shapes(cuda):
    """bf16 streams need the tensor-core kernels: other shapes fail loudly
    (no silent fp32 or CPU fallback)."""
    for n, C, train in ((4, 96, False), (2, 128, True)):
        x, params, grad = oracle_case(8, n, C, seed=3, alpha=0.5, bias_std=0.5)
        layer = make_layer(params, n, C, cuda)
        layer.bf16_io = True
        xd = x.bfloat16().to(cuda).requires_grad_(train)
        with pytest.raises(RuntimeError, match="bf16"):
            if train:
                layer(xd).backward(grad.bfloat16().to(cuda))
            else:
                with torch.no_grad():
                    layer.eval()
                    layer(xd)
        torch.cuda.synchronize()


@pytest.mark.parametrize("n,mode,shape", [(4, "decay", (2, 5, 64)), (4, "zero", (3, 64)),
                                          (8, "decay", (2, 3, 33)), (2, "decay", (7, 96)),
                                          (1, "decay", (4, 64)), (32, "decay", (1, 3, 64))])
def test_residual_wrapper(cuda, n, mode, shape):
    """Wrapper forward and input / parameter gradients against the oracle's
    packing + layer + mean, in fp64 autograd."""
    gen = torch.Generator().manual_seed(3 + n)
    r, b = torch.randn(*shape, generator=gen), torch.randn(*shape, generator=gen)
    C = shape[-1]
    w = mhc.replace_residual_with_mhc(hidden_dim=C, expansion_rate=n, residual_mode=mode).to(cuda)
    rd, bd = r.to(cuda).requires_grad_(True), b.to(cuda).requires_grad_(True)
    out = w(rd, bd)
    gout = torch.randn(*shape, generator=gen)
    out.backward(gout.to(cuda))
    rr, br_ = r.double().requires_grad_(True), b.double().requires_grad_(True)
    streams, _ = O.residual_wrapper_pack(rr, br_, n, mode)
    params = {k: p.detach().cpu().double().requires_grad_(True) for k, p in w.mhc.named_parameters()}
    ref = O.mhc_layer_dynamic(streams, *[params[k] for k in O.DYNAMIC_PARAM_ORDER]).mean(dim=1)
    ref = ref.reshape(shape)
    ref.backward(gout.double())
    close(out, ref, what="wrapper out")
    close(rd.grad, rr.grad, what="wrapper grad residual")
    if n >= 2:
        close(bd.grad, br_.grad, what="wrapper grad branch")
    else:
        assert bd.grad is None and br_.grad is None
    for k, p in w.mhc.named_parameters():
        close_param(p.grad, params[k].grad, what="wrapper grad " + k)


@pytest.mark.parametrize("mode,shape,alpha", [("decay", (3, 345, 4096), 0.01),
                                              ("zero", (700, 1024), 0.5),
                                              ("decay", (2, 64, 7168), 0.5)])
def test_residual_wrapper_fused(cuda, mode, shape, alpha):
    """n = 4, dynamic H: MHCResidualWrapper builds the streams inside the layer
    kernels and writes the stream mean directly (mhc_wrapper_fwd/bwd_dynamic).
    Checked against the unfused composition (pack -> layer -> mean, the
    reference's layer.py:287-316 over this library's kernels) and against the
    fp64 oracle on a token sample."""
    from mhc_ascend_b200 import ops
    n, C = 4, shape[-1]
    gen = torch.Generator().manual_seed(17 + C)
    r, b = torch.randn(*shape, generator=gen), torch.randn(*shape, generator=gen)
    gout = torch.randn(*shape, generator=gen)
    params = O.make_dynamic_params(n, C, gen, alpha=alpha, bias_std=0.5, weight="rand")
    w = mhc.replace_residual_with_mhc(hidden_dim=C, expansion_rate=n, residual_mode=mode).to(cuda)
    with torch.no_grad():
        for k, v in params.items():
            getattr(w.mhc, k).copy_(v.reshape(getattr(w.mhc, k).shape))
    T = r.numel() // C
    assert ops.wrapper_fused_supported(r.reshape(T, C).to(cuda), b.reshape(T, C).to(cuda), n, C)
    rd, bd = r.to(cuda).requires_grad_(True), b.to(cuda).requires_grad_(True)
    out = w(rd, bd)
    out.backward(gout.to(cuda))
    fused = {"out": out.detach(), "res": rd.grad, "br": bd.grad}
    fused.update({k: p.grad.clone() for k, p in w.mhc.named_parameters()})
    # unfused: pack -> layer -> mean
    w.mhc.zero_grad(set_to_none=True)
    ru, bu = r.to(cuda).requires_grad_(True), b.to(cuda).requires_grad_(True)
    x = ops.wrapper_pack(ru.reshape(T, C), bu.reshape(T, C), n, mode)
    ref = ops.stream_mean(w.mhc(x)).reshape(shape)
    ref.backward(gout.to(cuda))
    close(fused["out"], ref.detach(), rtol=1e-6, atol=1e-6, what="fused vs unfused out")
    close(fused["res"], ru.grad, rtol=1e-6, atol=1e-6, what="fused vs unfused grad residual")
    close(fused["br"], bu.grad, rtol=1e-6, atol=1e-6, what="fused vs unfused grad branch")
    for k, p in w.mhc.named_parameters():
        close_param(fused[k], p.grad, rtol=1e-5, atol=1e-6, what="fused vs unfused grad " + k)
    # fp64 oracle on a token sample (per-token rows depend on their token only)
    idx = torch.randperm(T, generator=gen)[:64]
    rs, bs = r.reshape(T, C)[idx].double(), b.reshape(T, C)[idx].double()
    streams, _ = O.residual_wrapper_pack(rs, bs, n, mode)
    p64 = {k: v.double() for k, v in params.items()}
    o64 = O.mhc_layer_dynamic(streams, *[p64[k] for k in O.DYNAMIC_PARAM_ORDER]).mean(dim=1)
    close(fused["out"].reshape(T, C)[idx.to(cuda)], o64, what="fused wrapper out vs fp64")


@pytest.mark.parametrize("mode,shape,alpha", [("decay", (3, 345, 4096), 0.5),
                                              ("zero", (700, 1024), 0.01),
                                              ("decay", (2, 64, 7168), 0.5),
                                              ("decay", (5, 96), 0.5)])
def test_residual_wrapper_prenorm(cuda, mode, shape, alpha):
    """MHCResidualWrapper.forward_prenorm: the hidden state and the next
    branch's input RMSNorm of it from one output pass (n = 4 dynamic H; C = 96
    takes the unfused path).  Forward and every gradient, with upstream
    gradients on both outputs, against the unfused composition (wrapper ->
    rmsnorm over this library's kernels) and, on a token sample, the fp64
    oracle (reference layer.py:287-316 then ops_pytorch_backward rmsnorm)."""
    from mhc_ascend_b200 import ops
    n, C = 4, shape[-1]
    gen = torch.Generator().manual_seed(23 + C)
    r, b = torch.randn(*shape, generator=gen), torch.randn(*shape, generator=gen)
    gh, gn = torch.randn(*shape, generator=gen), torch.randn(*shape, generator=gen)
    w2 = torch.rand(C, generator=gen) + 0.5
    params = O.make_dynamic_params(n, C, gen, alpha=alpha, bias_std=0.5, weight="rand")
    w = mhc.replace_residual_with_mhc(hidden_dim=C, expansion_rate=n, residual_mode=mode).to(cuda)
    with torch.no_grad():
        for k, v in params.items():
            getattr(w.mhc, k).copy_(v.reshape(getattr(w.mhc, k).shape))
    rd, bd = r.to(cuda).requires_grad_(True), b.to(cuda).requires_grad_(True)
    w2d = w2.to(cuda).requires_grad_(True)
    hid, nrm = w.forward_prenorm(rd, bd, w2d, 1e-5)
    torch.autograd.backward([hid, nrm], [gh.to(cuda), gn.to(cuda)])
    fused = {"hid": hid.detach(), "nrm": nrm.detach(), "res": rd.grad, "br": bd.grad,
             "w2": w2d.grad.clone()}
    fused.update({k: p.grad.clone() for k, p in w.mhc.named_parameters()})
    w.mhc.zero_grad(set_to_none=True)
    ru, bu = r.to(cuda).requires_grad_(True), b.to(cuda).requires_grad_(True)
    w2u = w2.to(cuda).requires_grad_(True)
    hu = w(ru, bu)
    nu = ops.rmsnorm(hu.reshape(-1, C), w2u, 1e-5).reshape(shape)
    torch.autograd.backward([hu, nu], [gh.to(cuda), gn.to(cuda)])
    close(fused["hid"], hu.detach(), rtol=1e-6, atol=1e-6, what="prenorm hidden vs unfused")
    close(fused["nrm"], nu.detach(), rtol=1e-5, atol=1e-6, what="prenorm normed vs unfused")
    close(fused["res"], ru.grad, rtol=1e-5, atol=1e-6, what="prenorm grad residual vs unfused")
    close(fused["br"], bu.grad, rtol=1e-5, atol=1e-6, what="prenorm grad branch vs unfused")
    close_param(fused["w2"], w2u.grad, rtol=1e-5, atol=1e-6, what="prenorm grad norm weight")
    for k, p in w.mhc.named_parameters():
        close_param(fused[k], p.grad, rtol=1e-5, atol=1e-6, what="prenorm grad " + k)
    # fp64 oracle on a token sample
    T = r.numel() // C
    idx = torch.randperm(T, generator=gen)[:64]
    rs, bs = r.reshape(T, C)[idx].double(), b.reshape(T, C)[idx].double()
    streams, _ = O.residual_wrapper_pack(rs, bs, n, mode)
    p64 = {k: v.double() for k, v in params.items()}
    h64 = O.mhc_layer_dynamic(streams, *[p64[k] for k in O.DYNAMIC_PARAM_ORDER]).mean(dim=1)
    n64 = O.rmsnorm(h64, w2.double(), 1e-5)
    di = idx.to(cuda)
    close(fused["hid"].reshape(T, C)[di], h64, what="prenorm hidden vs fp64")
    close(fused["nrm"].reshape(T, C)[di], n64, what="prenorm normed vs fp64")


@pytest.mark.parametrize("n,mode,shape", [(4, "decay", (2, 9, 4096)), (6, "decay", (5, 33)),
                                          (3, "zero", (4, 64))])
def test_residual_wrapper_bf16_inputs(cuda, n, mode, shape):
    """bf16 residual / branch: the reference packs the streams in bf16
    (layer.py:299-308: zeros in residual.dtype, decayed copies rounded to bf16),
    then runs the layer in fp32 and returns fp32.  Packing is bit-exact with the
    oracle's bf16 packing; the output meets the fp32 tolerance against the fp64
    layer on those packed streams; input gradients come back bf16 (one bf16
    rounding: rtol 8e-3 / atol 1e-2)."""
    from mhc_ascend_b200 import ops
    gen = torch.Generator().manual_seed(11 + n)
    r = torch.randn(*shape, generator=gen).bfloat16()
    b = torch.randn(*shape, generator=gen).bfloat16()
    C = shape[-1]
    streams_bf16, _ = O.residual_wrapper_pack(r, b, n, mode)
    assert streams_bf16.dtype == torch.bfloat16
    packed = ops.wrapper_pack(r.reshape(-1, C).to(cuda), b.reshape(-1, C).to(cuda), n, mode)
    assert packed.dtype == torch.float32
    assert torch.equal(packed.cpu(), streams_bf16.float())
    w = mhc.replace_residual_with_mhc(hidden_dim=C, expansion_rate=n, residual_mode=mode).to(cuda)
    with torch.no_grad():
        for k, p in w.mhc.named_parameters():
            if k.startswith("alpha"):
                p.fill_(0.5)
            elif k.startswith("b_"):
                p.copy_(torch.randn(p.shape, generator=gen) * 0.5)
    rd, bd = r.to(cuda).requires_grad_(True), b.to(cuda).requires_grad_(True)
    out = w(rd, bd)
    assert out.dtype == torch.float32 and out.shape == shape
    gout = torch.randn(*shape, generator=gen)
    out.backward(gout.to(cuda))
    assert rd.grad.dtype == torch.bfloat16 and bd.grad.dtype == torch.bfloat16
    params = {k: p.detach().cpu().double() for k, p in w.mhc.named_parameters()}
    x64 = streams_bf16.double().requires_grad_(True)
    ref = O.mhc_layer_dynamic(x64, *[params[k] for k in O.DYNAMIC_PARAM_ORDER]).mean(dim=1)
    close(out.reshape(-1, C), ref, what="bf16 wrapper out")
    ref.backward(gout.reshape(-1, C).double())
    gx = x64.grad  # [T, n, C]; the pack's reverse in fp64
    sc = [1.0, 0.0] + [(0.1 ** (i - 1) if mode == "decay" else 0.0) for i in range(2, n)]
    g_res = sum(sc[i] * gx[:, i] for i in range(n) if i != 1)
    close(rd.grad.float().reshape(-1, C), g_res, rtol=8e-3, atol=1e-2, what="bf16 wrapper grad residual")
    close(bd.grad.float().reshape(-1, C), gx[:, 1], rtol=8e-3, atol=1e-2, what="bf16 wrapper grad branch")


@pytest.mark.parametrize("n,mode,C", [(4, "decay", 4096), (6, "decay", 33), (5, "zero", 64),
                                      (1, "zero", 8), (32, "decay", 100)])
def test_wrapper_pack_and_mean_ops(cuda, n, mode, C):
    """Packing is bit-exact with the reference's fp32 ops (same fp32 scale
    products); the mean and both reverses match torch's fp32 formulas."""
    from mhc_ascend_b200 import ops
    gen = torch.Generator().manual_seed(n * 100 + C)
    T = 37
    r, b = torch.randn(T, C, generator=gen), torch.randn(T, C, generator=gen)
    packed = ops.wrapper_pack(r.to(cuda), b.to(cuda), n, mode)
    ref, _ = O.residual_wrapper_pack(r, b, n, mode)
    assert torch.equal(packed.cpu(), ref)
    x = torch.randn(T, n, C, generator=gen)
    m = ops.stream_mean(x.to(cuda))
    close(m, x.mean(dim=1), rtol=1e-6, atol=1e-6, what="stream mean")
    # reverses
    g = torch.randn(T, n, C, generator=gen)
    rd, bd = r.to(cuda).requires_grad_(True), b.to(cuda).requires_grad_(True)
    ops.wrapper_pack(rd, bd, n, mode).backward(g.to(cuda))
    rr, bb = r.clone().requires_grad_(True), b.clone().requires_grad_(True)
    O.residual_wrapper_pack(rr, bb, n, mode)[0].backward(g)
    close(rd.grad, rr.grad, rtol=1e-6, atol=1e-6, what="pack grad residual")
    if n >= 2:
        close(bd.grad, bb.grad, rtol=0, atol=0, what="pack grad branch")
    else:
        assert bd.grad is None and bb.grad is None
    xd = x.to(cuda).requires_grad_(True)
    gm = torch.randn(T, C, generator=gen)
    ops.stream_mean(xd).backward(gm.to(cuda))
    assert torch.equal(xd.grad.cpu(), (gm / n).unsqueeze(1).expand(T, n, C))


def test_no_device_wait_timed_out(cuda):
    """The TMA-pipelined kernels bound every mbarrier wait; none may have run out."""
    from mhc_ascend_b200 import _C
    x, params, grad = oracle_case(333, 4, 4096, seed=21)
    layer = make_layer(params, 4, 4096, cuda)
    run_layer(layer, x.to(cuda), grad.to(cuda))
    torch.cuda.synchronize()
    assert _C.device_error_word(reset=True) == 0
