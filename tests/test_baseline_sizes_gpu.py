"""Parity at the BASELINE configurations' own sizes.

* cfg5 shape (n=4, C=7168, dynamic H, fwd+bwd): 2048 tokens against the fp64
  oracle in full; 32768 tokens (one GPU's shard) with out / grad_x checked on a
  seeded sample of tokens (each token's rows depend only on that token) and the
  parameter gradients against the fp64 oracle summed over token chunks.
* cfg4 (static H, forward, B=65536, n=4, C=4096): fp32 and bf16 I/O with a
  non-unit RMSNorm weight, every output row against the oracle in chunks.

out and grad_x are held to the unscaled rtol 1e-4 / atol 1e-5; only the
batch-reduced parameter gradients use the tensor-scale atol (close_param).
"""
import pytest
import torch

import mhc_ascend_b200 as mhc
from oracle import mhc_oracle as O
from tests.helpers import close, close_param

pytestmark = pytest.mark.gpu

PARAMS = O.DYNAMIC_PARAM_ORDER


def _layer(params, n, C, dev):
    layer = mhc.MHCLayer(hidden_dim=C, expansion_rate=n).to(dev)
    with torch.no_grad():
        for k, v in params.items():
            getattr(layer, k).copy_(v.reshape(getattr(layer, k).shape))
    return layer


def _fwd_bwd(layer, xd, gd):
    xd = xd.clone().requires_grad_(True)
    layer.zero_grad(set_to_none=True)
    out = layer(xd)
    out.backward(gd)
    return out.detach(), xd.grad, {k: p.grad.detach().clone() for k, p in layer.named_parameters()}


def _case(B, n, C, seed, alpha, bias):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, n, C, generator=gen)
    params = O.make_dynamic_params(n, C, gen, alpha=alpha, bias_std=bias, weight="rand")
    grad = torch.randn(B, n, C, generator=gen)
    return x, params, grad


@pytest.mark.parametrize("alpha,bias", [(0.01, 0.0), (0.5, 0.5)])
def test_cfg5_shape_dynamic_vs_oracle(cuda, alpha, bias):
    B, n, C = 2048, 4, 7168
    x, params, grad = _case(B, n, C, 50 + int(alpha * 10), alpha, bias)
    layer = _layer(params, n, C, cuda)
    out, gx, pg = _fwd_bwd(layer, x.to(cuda), grad.to(cuda))
    ro, rg = O.dynamic_fwd_bwd(x.double(), {k: v.double() for k, v in params.items()},
                               grad.double())
    close(out, ro, what="cfg5 out")
    close(gx, rg["x"], what="cfg5 grad_x")
    for k in PARAMS:
        close_param(pg[k], rg[k], what="cfg5 grad_" + k)


def test_cfg5_full_shard(cuda):
    """32768 tokens x n=4 x C=7168 (3.5 GiB per stream tensor)."""
    B, n, C = 32768, 4, 7168
    x, params, grad = _case(B, n, C, 1000, 0.01, 0.0)
    layer = _layer(params, n, C, cuda)
    xd, gd = x.to(cuda), grad.to(cuda)
    out, gx, pg = _fwd_bwd(layer, xd, gd)
    # per-token rows on a seeded sample of tokens
    idx = torch.randperm(B, generator=torch.Generator().manual_seed(7))[:384].sort().values
    ro, rg = O.dynamic_fwd_bwd(x[idx].double(), {k: v.double() for k, v in params.items()},
                               grad[idx].double())
    close(out[idx.to(cuda)], ro, what="cfg5 shard out (sample)")
    close(gx[idx.to(cuda)], rg["x"], what="cfg5 shard grad_x (sample)")
    del out, gx
    # parameter gradients: fp64 oracle summed over token chunks
    ps64 = {k: v.double() for k, v in params.items()}
    tot = {k: torch.zeros_like(v) for k, v in ps64.items()}
    for c0 in range(0, B, 4096):
        _, r = O.dynamic_fwd_bwd(x[c0:c0 + 4096].double(), ps64, grad[c0:c0 + 4096].double())
        for k in PARAMS:
            tot[k] += r[k]
    for k in PARAMS:
        close_param(pg[k], tot[k], what="cfg5 shard grad_" + k)


def _static_layer(n, C, dev, bf16, seed):
    gen = torch.Generator().manual_seed(seed)
    Hp, Hq, Hr = torch.randn(n, generator=gen), torch.randn(n, generator=gen), torch.randn(n, n, generator=gen)
    w = torch.rand(C, generator=gen) + 0.5
    layer = mhc.MHCLayer(hidden_dim=C, expansion_rate=n, use_dynamic_h=False, bf16_io=bf16).to(dev)
    with torch.no_grad():
        layer.rmsnorm_weight.copy_(w); layer.H_pre.copy_(Hp)
        layer.H_post.copy_(Hq); layer.H_res.copy_(Hr)
    layer.eval()
    return layer, (w, Hp, Hq, Hr), gen


@pytest.mark.parametrize("bf16", [False, True])
def test_cfg4_static_forward_full_size(cuda, bf16):
    """B=65536, n=4, C=4096 static-H inference.  bf16 I/O: the oracle runs on the
    same bf16-rounded input; the output carries one bf16 rounding (relative
    2^-9), so rtol 8e-3 / atol 1e-2 (the stated bf16 tolerance)."""
    B, n, C = 65536, 4, 4096
    layer, (w, Hp, Hq, Hr), gen = _static_layer(n, C, cuda, bf16, 44)
    x = torch.randn(B, n, C, generator=gen)
    if bf16:
        x = x.bfloat16()
    with torch.no_grad():
        out = layer(x.to(cuda))
    assert out.dtype == (torch.bfloat16 if bf16 else torch.float32)
    rtol, atol = (8e-3, 1e-2) if bf16 else (1e-4, 1e-5)
    for c0 in range(0, B, 8192):
        sl = slice(c0, c0 + 8192)
        ro = O.mhc_layer_static(x[sl].double(), w.double(), Hp.double(), Hq.double(), Hr.double())
        close(out[sl].float(), ro, rtol=rtol, atol=atol, what=f"cfg4 out tokens {c0}+")
