"""Generate the golden fixtures in this directory from the reference itself.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/mHC_Ascend

It imports the reference's fp32 PyTorch formulation
(``src/python/mhc/ops_pytorch_backward.py``) by file path -- the package's
``__init__`` cannot be imported without the Ascend extension -- composes the
dynamic layer in the order of ``src/python/bindings.cpp:880-952`` and the
static layer in the order of ``src/python/mhc/layer.py:142-170``, runs autograd
backward, and freezes inputs, outputs and gradients into ``*.npz``.

Nothing at test time reads the reference: the tests only read the fixtures.
"""

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(ref_root):
    path = os.path.join(ref_root, "src", "python", "mhc", "ops_pytorch_backward.py")
    spec = importlib.util.spec_from_file_location("ref_ops_pytorch_backward", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def save(name, **arrays):
    out = {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v))
           for k, v in arrays.items()}
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    print("wrote", name, {k: v.shape for k, v in out.items()})


def dynamic_case(R, name, B, n, C, seed, alpha, bias_std, rand_weight, loss_sq,
                 iters=20, s_eps=1e-8, r_eps=1e-5):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, n, C, generator=g)
    nh = n * n + 2 * n
    phi = torch.randn(nh, n * C, generator=g) * 0.02
    b = (torch.randn(nh, generator=g) * bias_std) if bias_std > 0 else torch.zeros(nh)
    w = (torch.rand(C, generator=g) + 0.5) if rand_weight else torch.ones(C)
    grad_out = None if loss_sq else torch.randn(B, n, C, generator=g)

    leaves = dict(
        x=x.clone(), w=w.clone(), phi_pre=phi[:n].clone(), phi_post=phi[n:2 * n].clone(),
        phi_res=phi[2 * n:].clone(), alpha_pre=torch.tensor(alpha),
        alpha_post=torch.tensor(alpha), alpha_res=torch.tensor(alpha),
        b_pre=b[:n].clone(), b_post=b[n:2 * n].clone(), b_res=b[2 * n:].reshape(n, n).clone())
    for t in leaves.values():
        t.requires_grad_(True)
    L = leaves
    x_flat = L["x"].reshape(B, n * C)
    rms_h = R.compute_rms_pytorch(x_flat, r_eps)
    hp = R.dynamic_h_projection_pytorch(x_flat, L["phi_pre"], L["alpha_pre"], L["b_pre"], rms_h)
    hq = R.dynamic_h_projection_pytorch(x_flat, L["phi_post"], L["alpha_post"], L["b_post"], rms_h)
    hr = R.dynamic_h_projection_pytorch(x_flat, L["phi_res"], L["alpha_res"], L["b_res"], rms_h,
                                        is_res=True)
    M = R.sinkhorn_knopp_pytorch(torch.exp(hr), iters, s_eps)
    x_agg = R.stream_aggregate_pytorch(L["x"], hp)
    y = R.rmsnorm_pytorch(x_agg, L["w"], r_eps)
    out = R.stream_distribute_mix_add_pytorch(y, hq, M, L["x"])
    if grad_out is None:
        (out ** 2).sum().backward()
    else:
        out.backward(grad_out)
    arrays = {k: v.detach() for k, v in leaves.items()}
    arrays.update({"grad_" + k: v.grad for k, v in leaves.items()})
    arrays["out"] = out.detach()
    arrays["M"] = M.detach()
    arrays["rms_h"] = rms_h.detach()
    if grad_out is not None:
        arrays["grad_out"] = grad_out
    arrays["meta"] = np.array([iters, s_eps, r_eps], dtype=np.float64)
    save(name, **arrays)


def static_case(R, name, B, n, C, seed, loss_sq=True, iters=20, s_eps=1e-8, r_eps=1e-5):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, n, C, generator=g)
    H_pre = torch.randn(n, generator=g)
    H_post = torch.randn(n, generator=g)
    H_res = torch.randn(n, n, generator=g)
    w = torch.rand(C, generator=g) + 0.5
    leaves = dict(x=x, w=w, H_pre=H_pre, H_post=H_post, H_res=H_res)
    for t in leaves.values():
        t.requires_grad_(True)
    L = leaves
    hp = L["H_pre"].unsqueeze(0).expand(B, -1)
    hq = L["H_post"].unsqueeze(0).expand(B, -1)
    hr = L["H_res"].unsqueeze(0).expand(B, -1, -1)
    x_agg = R.stream_aggregate_pytorch(L["x"], hp)
    y = R.rmsnorm_pytorch(x_agg, L["w"], r_eps)
    M = R.sinkhorn_knopp_pytorch(torch.exp(hr), iters, s_eps)
    out = R.stream_distribute_mix_add_pytorch(y, hq, M, L["x"])
    (out ** 2).sum().backward()
    arrays = {k: v.detach() for k, v in leaves.items()}
    arrays.update({"grad_" + k: v.grad for k, v in leaves.items()})
    arrays["out"] = out.detach()
    arrays["meta"] = np.array([iters, s_eps, r_eps], dtype=np.float64)
    save(name, **arrays)


def op_cases(R):
    # sinkhorn_knopp: U[0,1) inputs, N(0,1) upstream gradient (BASELINE cfg2 distribution)
    for (B, N, seed) in ((256, 4, 11), (32, 8, 12), (64, 2, 13), (8, 16, 14)):
        g = torch.Generator().manual_seed(seed)
        inp = torch.rand(B, N, N, generator=g).requires_grad_(True)
        grad = torch.randn(B, N, N, generator=g)
        out = R.sinkhorn_knopp_pytorch(inp, 20, 1e-8)
        out.backward(grad)
        save(f"sinkhorn_B{B}_N{N}", inp=inp.detach(), grad=grad, out=out.detach(),
             grad_inp=inp.grad)
    # rmsnorm: x ~ N(0,1), weight ~ U[0.5,1.5)
    g = torch.Generator().manual_seed(21)
    x = torch.randn(16, 4096, generator=g).requires_grad_(True)
    w = (torch.rand(4096, generator=g) + 0.5).requires_grad_(True)
    grad = torch.randn(16, 4096, generator=g)
    out = R.rmsnorm_pytorch(x, w, 1e-5)
    out.backward(grad)
    save("rmsnorm_B16_C4096", x=x.detach(), w=w.detach(), grad=grad, out=out.detach(),
         grad_x=x.grad, grad_w=w.grad)
    # stream_aggregate: BASELINE cfg2 shape [32,4,256]
    g = torch.Generator().manual_seed(31)
    x = torch.randn(32, 4, 256, generator=g).requires_grad_(True)
    h = torch.randn(32, 4, generator=g).requires_grad_(True)
    grad = torch.randn(32, 256, generator=g)
    out = R.stream_aggregate_pytorch(x, h)
    out.backward(grad)
    save("aggregate_B32_n4_C256", x=x.detach(), H_pre=h.detach(), grad=grad, out=out.detach(),
         grad_x=x.grad, grad_H_pre=h.grad)
    # stream_distribute_mix_add
    g = torch.Generator().manual_seed(41)
    B, n, C = 8, 4, 96
    y = torch.randn(B, C, generator=g).requires_grad_(True)
    hq = torch.randn(B, n, generator=g).requires_grad_(True)
    M = torch.rand(B, n, n, generator=g).requires_grad_(True)
    x = torch.randn(B, n, C, generator=g).requires_grad_(True)
    grad = torch.randn(B, n, C, generator=g)
    out = R.stream_distribute_mix_add_pytorch(y, hq, M, x)
    out.backward(grad)
    save("distribute_B8_n4_C96", y=y.detach(), H_post=hq.detach(), M=M.detach(), x=x.detach(),
         grad=grad, out=out.detach(), grad_y=y.grad, grad_H_post=hq.grad, grad_M=M.grad,
         grad_x=x.grad)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MHC_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    torch.set_num_threads(1)
    R = load_reference(ref_root)
    # BASELINE cfg1: B=32, n=4, C=256, alpha 0.01, zero bias, unit weight, loss sum(out^2)
    dynamic_case(R, "dynamic_cfg1_B32_n4_C256", 32, 4, 256, seed=0, alpha=0.01,
                 bias_std=0.0, rand_weight=False, loss_sq=True)
    # Strong gating: alpha 1, random biases and weight, random upstream gradient
    dynamic_case(R, "dynamic_strong_B8_n4_C64", 8, 4, 64, seed=1, alpha=1.0,
                 bias_std=1.0, rand_weight=True, loss_sq=False)
    dynamic_case(R, "dynamic_strong_B4_n8_C32", 4, 8, 32, seed=2, alpha=1.0,
                 bias_std=1.0, rand_weight=True, loss_sq=False)
    dynamic_case(R, "dynamic_strong_B6_n2_C100", 6, 2, 100, seed=3, alpha=1.0,
                 bias_std=1.0, rand_weight=True, loss_sq=False)
    static_case(R, "static_B16_n4_C128", 16, 4, 128, seed=4)
    op_cases(R)


if __name__ == "__main__":
    main()
