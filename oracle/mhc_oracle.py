"""CPU oracle for the mHC layer hot path.  TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the reference's own fp32
formulation of the mHC operators (ParadoxZW/mHC_Ascend
``src/python/mhc/ops_pytorch_backward.py``) and composes them in the order the
reference's fused host orchestration uses (``src/python/bindings.cpp:880-952``).
Backward passes come from autograd, exactly as the reference's PyTorch
formulation obtains them.

Only the test-suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline arm may import this file, and only as a checker / CPU baseline.  The
product package (``mhc_ascend_b200``) never imports it: the CUDA path fails
loudly when its extension is missing.

Parity pin: ``tests/golden/make_golden.py`` imported the reference's
``ops_pytorch_backward.py`` by file path (in the build container) and froze its
outputs and gradients into ``tests/golden/*.npz``; ``tests/test_oracle.py``
checks this restatement against those fixtures.

All functions take a ``dtype``-agnostic tensor: call them with float64 inputs
for a high-precision reference, float32 for the reference's own precision.
"""

from __future__ import annotations

import torch


# --------------------------------------------------------------------------
# Operators (ops_pytorch_backward.py)
# --------------------------------------------------------------------------

def sinkhorn_knopp(inp: torch.Tensor, num_iters: int = 20, eps: float = 1e-8) -> torch.Tensor:
    """Alternating row / column normalisation of a batch [B, M, N].

    Follows ops_pytorch_backward.py:9-33: each iteration divides every row by
    (row sum + eps), then every column by (column sum + eps).
    """
    a = inp.clone()
    for _ in range(num_iters):
        a = a / (a.sum(dim=2, keepdim=True) + eps)
        a = a / (a.sum(dim=1, keepdim=True) + eps)
    return a


def stream_distribute_mix_add(y_norm, H_post_raw, M, x_inp):
    """out[b,i,c] = 2*sigmoid(H_post_raw[b,i]) * y_norm[b,c] + sum_j M[b,i,j] x[b,j,c].

    Follows ops_pytorch_backward.py:36-62.
    """
    h_post = 2.0 * torch.sigmoid(H_post_raw)
    return h_post.unsqueeze(-1) * y_norm.unsqueeze(1) + torch.bmm(M, x_inp)


def compute_rms(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """sqrt(mean(x^2, -1) + eps).  ops_pytorch_backward.py:65-75."""
    return torch.sqrt((x ** 2).mean(dim=-1) + eps)


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """(x / rms(x)) * weight.  ops_pytorch_backward.py:78-91."""
    rms = compute_rms(x, eps)
    return (x / rms.unsqueeze(-1)) * weight.unsqueeze(0)


def stream_aggregate(x: torch.Tensor, H_pre_raw: torch.Tensor) -> torch.Tensor:
    """sum_i sigmoid(H_pre_raw[b,i]) * x[b,i,:].  ops_pytorch_backward.py:94-111."""
    return (torch.sigmoid(H_pre_raw).unsqueeze(-1) * x).sum(dim=1)


def dynamic_h_projection(x_flat, phi, alpha, b, rms, is_res=False):
    """alpha * (x_flat @ phi^T) / rms + b.  ops_pytorch_backward.py:114-150."""
    p = torch.matmul(x_flat, phi.t())
    rms_inv = 1.0 / rms
    if is_res:
        tilde = alpha * p * rms_inv.unsqueeze(-1) + b.reshape(-1)
        return tilde.reshape(-1, b.size(0), b.size(1))
    return alpha * p * rms_inv.unsqueeze(-1) + b


# --------------------------------------------------------------------------
# Layer compositions
# --------------------------------------------------------------------------

def mhc_layer_dynamic(x, rmsnorm_weight, phi_pre, phi_post, phi_res,
                      alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                      sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5):
    """Dynamic-H mHC layer forward (autograd-capable).

    Composition order of bindings.cpp:880-952 (mhc_layer_fwd_dynamic):
    compute_rms(eps=rmsnorm_eps) on x_flat -> three projections -> exp ->
    Sinkhorn -> aggregate -> RMSNorm -> distribute-mix-add.  No bf16 casts:
    this is the fp32 formulation the B200 build is checked against.
    """
    B, n, C = x.shape
    x_flat = x.reshape(B, n * C)
    rms_h = compute_rms(x_flat, rmsnorm_eps)
    h_pre_raw = dynamic_h_projection(x_flat, phi_pre, alpha_pre, b_pre, rms_h)
    h_post_raw = dynamic_h_projection(x_flat, phi_post, alpha_post, b_post, rms_h)
    h_res_raw = dynamic_h_projection(x_flat, phi_res.reshape(n * n, n * C), alpha_res,
                                     b_res, rms_h, is_res=True)
    M = sinkhorn_knopp(torch.exp(h_res_raw), sinkhorn_iters, sinkhorn_eps)
    x_agg = stream_aggregate(x, h_pre_raw)
    y = rmsnorm(x_agg, rmsnorm_weight, rmsnorm_eps)
    return stream_distribute_mix_add(y, h_post_raw, M, x)


def mhc_layer_static(x, rmsnorm_weight, H_pre, H_post, H_res,
                     sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5):
    """Static-H mHC layer forward (layer.py:142-170): shared logits broadcast over B."""
    B = x.shape[0]
    h_pre_raw = H_pre.unsqueeze(0).expand(B, -1)
    h_post_raw = H_post.unsqueeze(0).expand(B, -1)
    h_res_raw = H_res.unsqueeze(0).expand(B, -1, -1)
    x_agg = stream_aggregate(x, h_pre_raw)
    y = rmsnorm(x_agg, rmsnorm_weight, rmsnorm_eps)
    M = sinkhorn_knopp(torch.exp(h_res_raw), sinkhorn_iters, sinkhorn_eps)
    return stream_distribute_mix_add(y, h_post_raw, M, x)


def residual_wrapper_pack(residual, branch_output, n, residual_mode="decay"):
    """Stream packing of MHCResidualWrapper.forward (layer.py:287-310)."""
    shape = residual.shape
    if residual.dim() == 3:
        B, T, C = shape
        residual = residual.reshape(B * T, C)
        branch_output = branch_output.reshape(B * T, C)
    else:
        B, C = shape
        T = 1
    streams = torch.zeros(B * T, n, C, dtype=residual.dtype)
    streams[:, 0] = residual
    if n >= 2:  # n == 1 packs the residual alone (layer.py:310)
        streams[:, 1] = branch_output
    if residual_mode == "decay":
        for i in range(2, n):
            streams[:, i] = residual * (0.1 ** (i - 1))
    elif residual_mode != "zero":
        raise ValueError(f"Unknown residual_mode: {residual_mode}")
    return streams, (B, T, C)


def make_dynamic_params(n, C, gen, dtype=torch.float32, alpha=0.01, phi_std=0.02,
                        bias_std=0.0, weight=None):
    """Seeded parameter set for a dynamic-H layer in the reference's shapes.

    Draw order: phi_concat [n^2+2n, nC] ~ N(0, phi_std^2) (rows pre|post|res),
    then (if bias_std > 0) the biases, then (if weight == 'rand') the RMSNorm
    weight ~ U[0.5, 1.5).
    """
    nh = n * n + 2 * n
    phi = torch.randn(nh, n * C, generator=gen, dtype=torch.float32) * phi_std
    if bias_std > 0:
        b = torch.randn(nh, generator=gen, dtype=torch.float32) * bias_std
    else:
        b = torch.zeros(nh, dtype=torch.float32)
    if weight == "rand":
        w = torch.rand(C, generator=gen, dtype=torch.float32) + 0.5
    else:
        w = torch.ones(C, dtype=torch.float32)
    p = {
        "rmsnorm_weight": w,
        "phi_pre": phi[:n].clone(),
        "phi_post": phi[n:2 * n].clone(),
        "phi_res": phi[2 * n:].clone(),
        "alpha_pre": torch.tensor(alpha),
        "alpha_post": torch.tensor(alpha),
        "alpha_res": torch.tensor(alpha),
        "b_pre": b[:n].clone(),
        "b_post": b[n:2 * n].clone(),
        "b_res": b[2 * n:].reshape(n, n).clone(),
    }
    return {k: v.to(dtype) for k, v in p.items()}


DYNAMIC_PARAM_ORDER = ("rmsnorm_weight", "phi_pre", "phi_post", "phi_res",
                       "alpha_pre", "alpha_post", "alpha_res", "b_pre", "b_post", "b_res")


def dynamic_fwd_bwd(x, params, grad_out=None, iters=20, s_eps=1e-8, r_eps=1e-5):
    """Run the dynamic layer forward + autograd backward on CPU.

    Returns (out, grads) where grads maps 'x' and every parameter name to its
    gradient.  With grad_out None the loss is sum(out^2) (BASELINE cfg1).
    """
    x = x.detach().clone().requires_grad_(True)
    ps = {k: v.detach().clone().requires_grad_(True) for k, v in params.items()}
    out = mhc_layer_dynamic(x, *[ps[k] for k in DYNAMIC_PARAM_ORDER],
                            sinkhorn_iters=iters, sinkhorn_eps=s_eps, rmsnorm_eps=r_eps)
    if grad_out is None:
        (out ** 2).sum().backward()
    else:
        out.backward(grad_out)
    grads = {"x": x.grad}
    grads.update({k: v.grad for k, v in ps.items()})
    return out.detach(), grads


def static_fwd_bwd(x, w, H_pre, H_post, H_res, grad_out=None, iters=20, s_eps=1e-8,
                   r_eps=1e-5):
    """Static-H layer forward + autograd backward on CPU."""
    x = x.detach().clone().requires_grad_(True)
    ts = [t.detach().clone().requires_grad_(True) for t in (w, H_pre, H_post, H_res)]
    out = mhc_layer_static(x, *ts, sinkhorn_iters=iters, sinkhorn_eps=s_eps,
                           rmsnorm_eps=r_eps)
    if grad_out is None:
        (out ** 2).sum().backward()
    else:
        out.backward(grad_out)
    names = ("rmsnorm_weight", "H_pre", "H_post", "H_res")
    grads = {"x": x.grad}
    grads.update({k: t.grad for k, t in zip(names, ts)})
    return out.detach(), grads
