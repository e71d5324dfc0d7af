"""Drop-in stand-in for the reference's native module ``mhc_ascend``.

The reference's Python package reaches its kernels through the pybind11
module ``mhc_ascend`` (src/python/bindings.cpp:1020-1117).  This module
exposes the same 13 hot-path functions, with the same argument names, order
and defaults, implemented over this library's C-ABI (``libmhc_b200.so``).  A
maintainer switches the reference package to the B200 kernels by making this
module importable under that name before ``mhc/ops.py`` runs its
``import mhc_ascend`` (ops.py:19-25)::

    import sys
    from mhc_ascend_b200 import mhc_ascend_shim
    sys.modules["mhc_ascend"] = mhc_ascend_shim
    import mhc            # the reference package, unchanged

Differences a caller can observe:

* Outputs are fp32 where the Ascend kernels return bf16 (rmsnorm_fwd out,
  stream_aggregate_fwd out); bf16 inputs are widened first.
* ``mhc_layer_fwd_dynamic`` returns the reference's 9 tensors (bindings.cpp:
  944-952), but the B200 layer keeps one fp32 per-token record instead of the
  three ``[B, nC]``/``[B, C]`` bf16 copies: the record travels in the
  ``x_agg_bf16`` slot; ``y_norm_bf16`` and ``x_flat_bf16`` are empty
  placeholders; ``rms``, ``H_pre_activated``, ``H_post_activated``, ``M`` and
  ``rms_h`` are views of the record.  ``mhc_layer_bwd_dynamic`` reads the
  record from the same slot, so ``ops.py:394-564`` runs unchanged as long as
  it hands the forward's tensors back in order (it does).
* The alphas arrive as host floats (the reference's ``.item()`` calls); they
  are copied to the device per call.
"""

from __future__ import annotations

import torch

from . import ops as _ops

__all__ = [
    "sinkhorn_knopp_fwd", "sinkhorn_knopp_bwd", "rmsnorm_fwd", "rmsnorm_bwd",
    "stream_aggregate_fwd", "stream_aggregate_bwd", "stream_distribute_mix_add_fwd",
    "stream_distribute_mix_add_bwd", "fused_rmsnorm_matmul_fwd", "fused_rmsnorm_matmul_bwd",
    "compute_rms_fwd", "mhc_layer_fwd_dynamic", "mhc_layer_bwd_dynamic",
]


def sinkhorn_knopp_fwd(inp, num_iters=20, eps=1e-8):
    """bindings.cpp:155-187 -> out [B, N, N]."""
    return _ops.sinkhorn_knopp_fwd(inp, num_iters, eps)


def sinkhorn_knopp_bwd(grad_out, inp, out, num_iters=20, eps=1e-8):
    """bindings.cpp:189-231 -> grad_inp (``out`` is accepted and unused: the
    exact reverse recomputes the iterations from ``inp``)."""
    return _ops.sinkhorn_knopp_bwd(grad_out, inp, out, num_iters, eps)


def rmsnorm_fwd(inp, weight, eps=1e-5):
    """bindings.cpp:237-265 -> (out, rms)."""
    return _ops.rmsnorm_fwd(inp, weight, eps)


def rmsnorm_bwd(grad_out, inp, weight, rms):
    """bindings.cpp:267-301 -> (grad_inp, grad_weight)."""
    return _ops.rmsnorm_bwd(grad_out, inp, weight, rms)


def stream_aggregate_fwd(inp, H_pre_raw):
    """bindings.cpp:307-335 -> (out, H_pre_activated)."""
    return _ops.stream_aggregate_fwd(inp, H_pre_raw)


def stream_aggregate_bwd(grad_out, inp, H_pre_activated):
    """bindings.cpp:337-374 -> (grad_inp, grad_H_pre_activated)."""
    return _ops.stream_aggregate_bwd(grad_out, inp, H_pre_activated)


def stream_distribute_mix_add_fwd(y_norm, H_post_raw, M, x_inp):
    """bindings.cpp:380-414 -> (out, H_post_activated)."""
    return _ops.stream_distribute_mix_add_fwd(y_norm, H_post_raw, M, x_inp)


def stream_distribute_mix_add_bwd(grad_out, x_inp, y_norm, M, H_post_activated):
    """bindings.cpp:416-460 -> (grad_x, grad_y_norm, grad_M, grad_H_post_activated)."""
    return _ops.stream_distribute_mix_add_bwd(grad_out, x_inp, y_norm, M, H_post_activated)


def fused_rmsnorm_matmul_fwd(inp, weight):
    """bindings.cpp:480-510 -> inp @ weight^T, fp32 (bf16 inputs are widened)."""
    return _ops.fused_rmsnorm_matmul_fwd(inp, weight)


def fused_rmsnorm_matmul_bwd(grad_out, x_flat, phi_concat):
    """bindings.cpp:512-541 -> (grad_x, grad_phi)."""
    return _ops.fused_rmsnorm_matmul_bwd(grad_out, x_flat, phi_concat)


def compute_rms_fwd(inp, eps=1e-8):
    """bindings.cpp:543-566 -> rms [B]."""
    return _ops.compute_rms(inp, eps)


def _split_phi(phi_concat, n, C):
    # rows pre | post | res of the concatenation (ops.py:416-418): contiguous
    # row blocks, so these are views, not copies
    phi = phi_concat.float().contiguous()
    return phi[:n], phi[n:2 * n], phi[2 * n:].reshape(n * n, n * C)


def mhc_layer_fwd_dynamic(x_expanded, rmsnorm_weight, phi_concat, alpha_pre, alpha_post,
                          alpha_res, b_pre, b_post, b_res, sinkhorn_iters=20,
                          sinkhorn_eps=1e-8, rmsnorm_eps=1e-5):
    """bindings.cpp:880-952 -> (output, rms, x_agg_bf16, H_pre_activated,
    H_post_activated, M, y_norm_bf16, x_flat_bf16, rms_h); the per-token
    record rides in the x_agg_bf16 slot (module docstring)."""
    B, n, C = x_expanded.shape
    pp, pq, pr = _split_phi(phi_concat, n, C)
    out, rec = _ops.mhc_layer_fwd_dynamic(
        x_expanded, rmsnorm_weight, pp, pq, pr, float(alpha_pre), float(alpha_post),
        float(alpha_res), b_pre, b_post, b_res, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps,
        save_state=True)
    # record fields: rms_h, r, H_pre act [n], H_post act [n], M [n, n], ...
    rms_h, rms = rec[:, 0], rec[:, 1]
    h_pre = rec[:, 2:2 + n]
    h_post = rec[:, 2 + n:2 + 2 * n]
    M = rec[:, 2 + 2 * n:2 + 2 * n + n * n].unflatten(1, (n, n))
    empty = x_expanded.new_empty(0)
    return out, rms, rec, h_pre, h_post, M, empty, empty, rms_h


def mhc_layer_bwd_dynamic(grad_output, x_expanded, rmsnorm_weight, rms, x_agg_bf16,
                          H_pre_activated, H_post_activated, M, y_norm_bf16, x_flat_bf16, rms_h,
                          phi_pre, phi_post, phi_res, alpha_pre, alpha_post, alpha_res, b_pre,
                          b_post, b_res, sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5):
    """bindings.cpp:600-874 -> (grad_x, grad_rmsnorm_weight, d_phi_pre,
    d_phi_post, d_phi_res, d_alpha_pre, d_alpha_post, d_alpha_res, d_b_pre,
    d_b_post, d_b_res).  ``x_agg_bf16`` must be the record the forward
    returned in that slot."""
    B, n, C = x_expanded.shape
    rec = x_agg_bf16
    if rec.dim() != 2 or rec.size(0) != B or rec.size(1) != _ops.token_state_stride(n) \
            or rec.dtype != torch.float32:
        raise RuntimeError("mhc_layer_bwd_dynamic: the x_agg_bf16 slot must hold the per-token "
                           "record returned by this module's mhc_layer_fwd_dynamic")
    return _ops.mhc_layer_bwd_dynamic(
        grad_output, x_expanded, rmsnorm_weight, phi_pre, phi_post, phi_res, float(alpha_pre),
        float(alpha_post), float(alpha_res), b_pre, b_post, b_res, rec.contiguous(),
        sinkhorn_iters, sinkhorn_eps, rmsnorm_eps)
