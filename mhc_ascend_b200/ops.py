"""PyTorch autograd functions over the B200 C-ABI kernels.

Mirrors the reference's ``src/python/mhc/ops.py`` (same class and function
names, same argument meaning) with the pybind module ``mhc_ascend`` replaced by
the ctypes binding of ``libmhc_b200.so``.  Differences that follow from the
B200 design, each deliberate:

* All arithmetic and all stored intermediates are fp32 (the reference casts
  to bf16 at ops.py:105-107, 218, 280-281 and bindings.cpp:906); results match
  the reference's fp32 PyTorch formulation (ops_pytorch_backward.py).
* Scalars alpha are passed to the kernels as device pointers: no ``.item()``
  host synchronisation (reference ops.py:420-422, 533-535).
* No host synchronisation anywhere (the reference syncs before every kernel
  launch, bindings.cpp:77).
* Parameter gradients are fixed-order reductions: bitwise reproducible.

Every op raises RuntimeError for inputs that are not CUDA tensors or have the
wrong rank, like the reference's TORCH_CHECKs raise for non-NPU inputs.
"""

from __future__ import annotations

from typing import Tuple

import ctypes

import torch

from . import _C

class _LazyLib:
    """Loads libmhc_b200.so on first use (so the build step can import the
    package before the library exists); a missing library raises then."""

    def __getattr__(self, name):
        return getattr(_C.load(), name)


_lib = _LazyLib()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(what, *tensors):
    for t in tensors:
        if not (torch.is_tensor(t) and t.is_cuda):
            raise RuntimeError(f"{what}: input must be a CUDA tensor")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"{what}: all tensors must be on the same device")


def _f32(t):
    return t.detach().float().contiguous() if t.dtype != torch.float32 or not t.is_contiguous() \
        else t.detach()


def _workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


class _DevGuard:
    def __init__(self, t):
        self.g = torch.cuda.device(t.device)

    def __enter__(self):
        self.g.__enter__()

    def __exit__(self, *a):
        self.g.__exit__(*a)


# =============================================================================
# Sinkhorn-Knopp
# =============================================================================

def sinkhorn_knopp_fwd(inp: torch.Tensor, num_iters: int = 20, eps: float = 1e-8) -> torch.Tensor:
    """Forward kernel call (reference: mhc_ascend.sinkhorn_knopp_fwd, bindings.cpp:155)."""
    _require_cuda("sinkhorn_knopp_fwd", inp)
    if inp.dim() != 3:
        raise RuntimeError("Input must be 3D tensor [B, M, N]")
    if inp.size(1) != inp.size(2):
        raise RuntimeError(
            f"Sinkhorn-Knopp requires square matrices (M == N), got M={inp.size(1)}, N={inp.size(2)}")
    x = _f32(inp)
    out = torch.empty_like(x)
    with _DevGuard(x):
        rc = _lib.mhc_sinkhorn_knopp_fwd(x.data_ptr(), out.data_ptr(), x.size(0), x.size(1),
                                         int(num_iters), float(eps), _stream(x.device))
    _C.check(rc, "sinkhorn_knopp_fwd")
    return out


def sinkhorn_knopp_bwd(grad_out, inp, out, num_iters: int = 20, eps: float = 1e-8):
    """Backward kernel call (reference: mhc_ascend.sinkhorn_knopp_bwd, bindings.cpp:189)."""
    _require_cuda("sinkhorn_knopp_bwd", grad_out, inp)
    if grad_out.shape != inp.shape:
        raise RuntimeError("grad_out shape must match inp")
    g = _f32(grad_out)
    x = _f32(inp)
    gi = torch.empty_like(x)
    with _DevGuard(x):
        rc = _lib.mhc_sinkhorn_knopp_bwd(g.data_ptr(), x.data_ptr(), None, gi.data_ptr(),
                                         x.size(0), x.size(1), int(num_iters), float(eps),
                                         _stream(x.device))
    _C.check(rc, "sinkhorn_knopp_bwd")
    return gi


class SinkhornKnoppFunction(torch.autograd.Function):
    """Sinkhorn-Knopp doubly stochastic matrix normalization (reference ops.py:32-61)."""

    @staticmethod
    def forward(ctx, inp, num_iters=20, eps=1e-8):
        out = sinkhorn_knopp_fwd(inp, num_iters, eps)
        ctx.save_for_backward(inp)
        ctx.num_iters = num_iters
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (inp,) = ctx.saved_tensors
        return sinkhorn_knopp_bwd(grad_out, inp, None, ctx.num_iters, ctx.eps), None, None


def sinkhorn_knopp(inp: torch.Tensor, num_iters: int = 20, eps: float = 1e-8) -> torch.Tensor:
    """Apply Sinkhorn-Knopp normalization to a batch of matrices [B, M, M] (ops.py:64-80)."""
    return SinkhornKnoppFunction.apply(inp.float(), num_iters, eps)


# =============================================================================
# RMSNorm
# =============================================================================

def rmsnorm_fwd(inp, weight, eps=1e-5):
    _require_cuda("rmsnorm_fwd", inp, weight)
    if inp.dim() != 2:
        raise RuntimeError("Input must be 2D tensor [B, C]")
    if weight.dim() != 1 or weight.size(0) != inp.size(1):
        raise RuntimeError("Weight must be 1D with size equal to hidden_dim")
    x, w = _f32(inp), _f32(weight)
    out = torch.empty_like(x)
    rms = torch.empty(x.size(0), dtype=torch.float32, device=x.device)
    with _DevGuard(x):
        rc = _lib.mhc_rmsnorm_fwd(x.data_ptr(), w.data_ptr(), out.data_ptr(), rms.data_ptr(),
                                  x.size(0), x.size(1), float(eps), _stream(x.device))
    _C.check(rc, "rmsnorm_fwd")
    return out, rms


def rmsnorm_bwd(grad_out, inp, weight, rms):
    _require_cuda("rmsnorm_bwd", grad_out, inp, weight, rms)
    g, x, w, r = _f32(grad_out), _f32(inp), _f32(weight), _f32(rms)
    B, C = x.shape
    gi = torch.empty_like(x)
    gw = torch.empty(C, dtype=torch.float32, device=x.device)
    ws = _workspace(_lib.mhc_rmsnorm_bwd_workspace_bytes(B, C), x.device)
    with _DevGuard(x):
        rc = _lib.mhc_rmsnorm_bwd(g.data_ptr(), x.data_ptr(), w.data_ptr(), r.data_ptr(),
                                  gi.data_ptr(), gw.data_ptr(), B, C, ws.data_ptr(), ws.numel(),
                                  _stream(x.device))
    _C.check(rc, "rmsnorm_bwd")
    return gi, gw


class RMSNormFunction(torch.autograd.Function):
    """Root Mean Square Normalization (reference ops.py:87-120)."""

    @staticmethod
    def forward(ctx, inp, weight, eps=1e-5):
        out, rms = rmsnorm_fwd(inp, weight, eps)
        ctx.save_for_backward(inp, weight, rms)
        ctx.eps = eps
        ctx.w_dtype = weight.dtype
        ctx.x_dtype = inp.dtype
        return out

    @staticmethod
    def backward(ctx, grad_out):
        inp, weight, rms = ctx.saved_tensors
        gi, gw = rmsnorm_bwd(grad_out, inp, weight, rms)
        return gi.to(ctx.x_dtype), gw.to(ctx.w_dtype), None


def rmsnorm(inp: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Apply RMS normalization over the last dim of [B, C] (reference ops.py:123-136)."""
    return RMSNormFunction.apply(inp, weight, eps)


# =============================================================================
# Stream aggregate
# =============================================================================

def stream_aggregate_fwd(inp, H_pre_raw):
    _require_cuda("stream_aggregate_fwd", inp, H_pre_raw)
    if inp.dim() != 3:
        raise RuntimeError("Input must be 3D tensor [B, n, C]")
    B, n, C = inp.shape
    if H_pre_raw.shape != (B, n):
        raise RuntimeError("H_pre_raw must be [B, n]")
    x, h = _f32(inp), _f32(H_pre_raw)
    out = torch.empty(B, C, dtype=torch.float32, device=x.device)
    h_act = torch.empty_like(h)
    with _DevGuard(x):
        rc = _lib.mhc_stream_aggregate_fwd(x.data_ptr(), h.data_ptr(), out.data_ptr(),
                                           h_act.data_ptr(), B, n, C, _stream(x.device))
    _C.check(rc, "stream_aggregate_fwd")
    return out, h_act


def stream_aggregate_bwd(grad_out, inp, H_pre_activated):
    _require_cuda("stream_aggregate_bwd", grad_out, inp, H_pre_activated)
    g, x, h = _f32(grad_out), _f32(inp), _f32(H_pre_activated)
    B, n, C = x.shape
    gi = torch.empty_like(x)
    gh = torch.empty_like(h)
    with _DevGuard(x):
        rc = _lib.mhc_stream_aggregate_bwd(g.data_ptr(), x.data_ptr(), h.data_ptr(),
                                           gi.data_ptr(), gh.data_ptr(), B, n, C,
                                           _stream(x.device))
    _C.check(rc, "stream_aggregate_bwd")
    return gi, gh


class StreamAggregateFunction(torch.autograd.Function):
    """Stream aggregation with sigmoid-activated weights (reference ops.py:143-173)."""

    @staticmethod
    def forward(ctx, inp, H_pre_raw):
        out, h_act = stream_aggregate_fwd(inp, H_pre_raw)
        ctx.save_for_backward(inp, h_act)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        inp, h_act = ctx.saved_tensors
        gi, gh_act = stream_aggregate_bwd(grad_out, inp, h_act)
        return gi, gh_act * h_act * (1.0 - h_act)


def stream_aggregate(inp: torch.Tensor, H_pre_raw: torch.Tensor) -> torch.Tensor:
    """sum_i sigmoid(H_pre_raw[:, i]) * inp[:, i, :] -> [B, C] (reference ops.py:176-188)."""
    return StreamAggregateFunction.apply(inp, H_pre_raw)


# =============================================================================
# Stream distribute-mix-add
# =============================================================================

def stream_distribute_mix_add_fwd(y_norm, H_post_raw, M, x_inp):
    _require_cuda("stream_distribute_mix_add_fwd", y_norm, H_post_raw, M, x_inp)
    if x_inp.dim() != 3:
        raise RuntimeError("x_inp must be 3D tensor [B, n, C]")
    B, n, C = x_inp.shape
    if y_norm.shape != (B, C) or H_post_raw.shape != (B, n) or M.shape != (B, n, n):
        raise RuntimeError("shape mismatch: y_norm [B,C], H_post_raw [B,n], M [B,n,n] expected")
    y, hq, m, x = _f32(y_norm), _f32(H_post_raw), _f32(M), _f32(x_inp)
    out = torch.empty_like(x)
    hq_act = torch.empty_like(hq)
    with _DevGuard(x):
        rc = _lib.mhc_stream_distribute_mix_add_fwd(y.data_ptr(), hq.data_ptr(), m.data_ptr(),
                                                    x.data_ptr(), out.data_ptr(),
                                                    hq_act.data_ptr(), B, n, C,
                                                    _stream(x.device))
    _C.check(rc, "stream_distribute_mix_add_fwd")
    return out, hq_act


def stream_distribute_mix_add_bwd(grad_out, x_inp, y_norm, M, H_post_activated):
    _require_cuda("stream_distribute_mix_add_bwd", grad_out, x_inp, y_norm, M, H_post_activated)
    g, x, y, m, hq = (_f32(t) for t in (grad_out, x_inp, y_norm, M, H_post_activated))
    B, n, C = x.shape
    gx = torch.empty_like(x)
    gy = torch.empty_like(y)
    gm = torch.empty_like(m)
    ghq = torch.empty_like(hq)
    with _DevGuard(x):
        rc = _lib.mhc_stream_distribute_mix_add_bwd(g.data_ptr(), x.data_ptr(), y.data_ptr(),
                                                    m.data_ptr(), hq.data_ptr(), gx.data_ptr(),
                                                    gy.data_ptr(), gm.data_ptr(), ghq.data_ptr(),
                                                    B, n, C, _stream(x.device))
    _C.check(rc, "stream_distribute_mix_add_bwd")
    return gx, gy, gm, ghq


class StreamDistributeMixAddFunction(torch.autograd.Function):
    """Stream distribution, mixing, and residual addition (reference ops.py:195-243)."""

    @staticmethod
    def forward(ctx, y_norm, H_post_raw, M, x_inp):
        out, hq_act = stream_distribute_mix_add_fwd(y_norm, H_post_raw, M, x_inp)
        ctx.save_for_backward(x_inp, y_norm, M, hq_act)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x_inp, y_norm, M, hq_act = ctx.saved_tensors
        gx, gy, gm, ghq = stream_distribute_mix_add_bwd(grad_out, x_inp, y_norm, M, hq_act)
        g_hpost = ghq * hq_act * (1.0 - hq_act / 2.0)
        return gy, g_hpost, gm, gx


def stream_distribute_mix_add(y_norm, H_post_raw, M, x_inp) -> torch.Tensor:
    """2 sigmoid(H_post_raw)_i y_norm + sum_j M_ij x_j -> [B, n, C] (reference ops.py:246-265)."""
    return StreamDistributeMixAddFunction.apply(y_norm, H_post_raw, M, x_inp)


# =============================================================================
# Dynamic-H projection and row RMS
# =============================================================================

def fused_rmsnorm_matmul_fwd(x_flat, phi_concat):
    _require_cuda("fused_rmsnorm_matmul_fwd", x_flat, phi_concat)
    if x_flat.dim() != 2 or phi_concat.dim() != 2 or phi_concat.size(1) != x_flat.size(1):
        raise RuntimeError("Weight K dimension must match input")
    x, w = _f32(x_flat), _f32(phi_concat)
    out = torch.empty(x.size(0), w.size(0), dtype=torch.float32, device=x.device)
    with _DevGuard(x):
        rc = _lib.mhc_fused_rmsnorm_matmul_fwd(x.data_ptr(), w.data_ptr(), out.data_ptr(),
                                               x.size(0), x.size(1), w.size(0),
                                               _stream(x.device))
    _C.check(rc, "fused_rmsnorm_matmul_fwd")
    return out


def fused_rmsnorm_matmul_bwd(grad_out, x_flat, phi_concat):
    _require_cuda("fused_rmsnorm_matmul_bwd", grad_out, x_flat, phi_concat)
    g, x, w = _f32(grad_out), _f32(x_flat), _f32(phi_concat)
    B, K = x.shape
    O = w.size(0)
    gx = torch.empty_like(x)
    gw = torch.empty_like(w)
    ws = _workspace(_lib.mhc_fused_rmsnorm_matmul_bwd_workspace_bytes(B, K, O), x.device)
    with _DevGuard(x):
        rc = _lib.mhc_fused_rmsnorm_matmul_bwd(g.data_ptr(), x.data_ptr(), w.data_ptr(),
                                               gx.data_ptr(), gw.data_ptr(), B, K, O,
                                               ws.data_ptr(), ws.numel(), _stream(x.device))
    _C.check(rc, "fused_rmsnorm_matmul_bwd")
    return gx, gw


class FusedProjectionFunction(torch.autograd.Function):
    """fp32 projection x_flat @ phi_concat^T (reference ops.py:272-295)."""

    @staticmethod
    def forward(ctx, x_flat, phi_concat):
        ctx.save_for_backward(x_flat, phi_concat)
        return fused_rmsnorm_matmul_fwd(x_flat, phi_concat)

    @staticmethod
    def backward(ctx, grad_out):
        x_flat, phi_concat = ctx.saved_tensors
        return fused_rmsnorm_matmul_bwd(grad_out, x_flat, phi_concat)


def fused_rmsnorm_matmul(x_flat: torch.Tensor, phi_concat: torch.Tensor) -> torch.Tensor:
    """Project x_flat [B, K] with phi_concat [out_dim, K] -> [B, out_dim] (ops.py:298-315)."""
    return FusedProjectionFunction.apply(x_flat, phi_concat)


def compute_rms(x_flat: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    """sqrt(mean(x_flat^2, -1) + eps) per row (reference ops.py:318-330)."""
    _require_cuda("compute_rms", x_flat)
    if x_flat.dim() != 2:
        raise RuntimeError("Input must be 2D tensor [B, K]")
    x = _f32(x_flat)
    rms = torch.empty(x.size(0), dtype=torch.float32, device=x.device)
    with _DevGuard(x):
        rc = _lib.mhc_compute_rms_fwd(x.data_ptr(), rms.data_ptr(), x.size(0), x.size(1),
                                      float(eps), _stream(x.device))
    _C.check(rc, "compute_rms")
    return rms


# =============================================================================
# MHCResidualWrapper stream packing and stream mean (reference layer.py:287-316)
# =============================================================================

def wrapper_stream_scales(n: int, residual_mode: str = "decay"):
    """Per-stream residual scales of MHCResidualWrapper: stream 0 is the
    residual, stream 1 the branch output, streams i >= 2 are
    residual * 0.1 ** (i - 1) ("decay", the reference's Python-float factor
    applied in fp32) or zeros ("zero")."""
    if residual_mode == "decay":
        vals = [1.0, 0.0] + [0.1 ** (i - 1) for i in range(2, n)]
    elif residual_mode == "zero":
        vals = [1.0, 0.0] + [0.0] * max(n - 2, 0)
    else:
        raise ValueError(f"Unknown residual_mode: {residual_mode}")
    return (ctypes.c_float * max(n, 1))(*vals[:max(n, 1)])


class WrapperPackFunction(torch.autograd.Function):
    """[T, C] residual and branch -> [T, n, C] mHC input in one pass."""

    @staticmethod
    def forward(ctx, residual, branch, n, residual_mode):
        sc = wrapper_stream_scales(n, residual_mode)  # unknown modes: ValueError first
        _require_cuda("wrapper_pack", residual, branch)
        if residual.dtype == torch.bfloat16 and branch.dtype == torch.bfloat16:
            # packed in bf16 like the reference (decayed copies rounded to bf16)
            r, b = residual.contiguous(), branch.contiguous()
            T, C = r.shape
            out = torch.empty(T, n, C, dtype=torch.float32, device=r.device)
            with _DevGuard(r):
                rc = _lib.mhc_wrapper_pack_fwd_bf16(r.data_ptr(), b.data_ptr(), out.data_ptr(),
                                                    sc, T, n, C, _stream(r.device))
            _C.check(rc, "mhc_wrapper_pack_fwd_bf16")
        else:
            r, b = _f32(residual), _f32(branch)
            T, C = r.shape
            out = torch.empty(T, n, C, dtype=torch.float32, device=r.device)
            with _DevGuard(r):
                rc = _lib.mhc_wrapper_pack_fwd(r.data_ptr(), b.data_ptr(), out.data_ptr(), sc,
                                               T, n, C, _stream(r.device))
            _C.check(rc, "mhc_wrapper_pack_fwd")
        ctx.n, ctx.sc, ctx.dtypes = n, sc, (residual.dtype, branch.dtype)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        g = _f32(grad_out)
        T, n, C = g.shape
        gr = torch.empty(T, C, dtype=torch.float32, device=g.device)
        gb = torch.empty(T, C, dtype=torch.float32, device=g.device) if n >= 2 else None
        with _DevGuard(g):
            rc = _lib.mhc_wrapper_pack_bwd(g.data_ptr(), gr.data_ptr(),
                                           gb.data_ptr() if n >= 2 else None, ctx.sc, T, n, C,
                                           _stream(g.device))
        _C.check(rc, "mhc_wrapper_pack_bwd")
        # at n == 1 the branch output is not an input of the layer: no gradient
        return gr.to(ctx.dtypes[0]), (gb.to(ctx.dtypes[1]) if gb is not None else None), None, None


def wrapper_pack(residual: torch.Tensor, branch: torch.Tensor, n: int,
                 residual_mode: str = "decay") -> torch.Tensor:
    """Stream packing of MHCResidualWrapper.forward (reference layer.py:300-310)."""
    return WrapperPackFunction.apply(residual, branch, n, residual_mode)


class StreamMeanFunction(torch.autograd.Function):
    """[T, n, C] -> [T, C] mean over the streams (reference layer.py:312)."""

    @staticmethod
    def forward(ctx, x):
        _require_cuda("stream_mean", x)
        xf = _f32(x)
        T, n, C = xf.shape
        out = torch.empty(T, C, dtype=torch.float32, device=xf.device)
        with _DevGuard(xf):
            rc = _lib.mhc_stream_mean_fwd(xf.data_ptr(), out.data_ptr(), T, n, C,
                                          _stream(xf.device))
        _C.check(rc, "mhc_stream_mean_fwd")
        ctx.shape, ctx.dtype = (T, n, C), x.dtype
        return out

    @staticmethod
    def backward(ctx, grad_out):
        g = _f32(grad_out)
        T, n, C = ctx.shape
        gx = torch.empty(T, n, C, dtype=torch.float32, device=g.device)
        with _DevGuard(g):
            rc = _lib.mhc_stream_mean_bwd(g.data_ptr(), gx.data_ptr(), T, n, C,
                                          _stream(g.device))
        _C.check(rc, "mhc_stream_mean_bwd")
        return gx.to(ctx.dtype)


def stream_mean(x: torch.Tensor) -> torch.Tensor:
    return StreamMeanFunction.apply(x)


# =============================================================================
# Fused dynamic-H layer
# =============================================================================

def token_state_stride(n: int) -> int:
    return int(_lib.mhc_token_state_stride(int(n)))


def _as_scalar_tensor(a, like):
    if torch.is_tensor(a):
        return a.detach().reshape(1).float().contiguous()
    return torch.tensor([float(a)], dtype=torch.float32, device=like.device)


def mhc_layer_fwd_dynamic(x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre, alpha_post,
                          alpha_res, b_pre, b_post, b_res, sinkhorn_iters=20, sinkhorn_eps=1e-8,
                          rmsnorm_eps=1e-5, save_state=True, bf16_io=False):
    """One fused dynamic-H forward (reference mhc_ascend.mhc_layer_fwd_dynamic,
    bindings.cpp:880-952).  Returns (out, token_state or None).  With bf16_io
    x must be bf16 and out is bf16 (fp32 arithmetic inside; n <= 4 and
    hidden % 64 == 0)."""
    _require_cuda("mhc_layer_fwd_dynamic", x, rmsnorm_weight, phi_pre, phi_post, phi_res)
    if x.dim() != 3:
        raise RuntimeError("x_expanded must be [B, n, C]")
    B, n, C = x.shape
    if bf16_io and x.dtype != torch.bfloat16:
        raise RuntimeError("bf16_io needs a bf16 input")
    xf = x.contiguous() if bf16_io else _f32(x)
    w = _f32(rmsnorm_weight)
    pp, pq, pr = _f32(phi_pre), _f32(phi_post), _f32(phi_res).reshape(n * n, n * C)
    if pp.shape != (n, n * C) or pq.shape != (n, n * C) or w.shape != (C,):
        raise RuntimeError("parameter shapes do not match x [B, n, C]")
    ap, aq, ar = (_as_scalar_tensor(a, xf) for a in (alpha_pre, alpha_post, alpha_res))
    bp, bq, br = _f32(b_pre), _f32(b_post), _f32(b_res)
    out = torch.empty_like(xf)
    state = torch.empty(B, token_state_stride(n), dtype=torch.float32, device=xf.device) \
        if save_state else None
    ws = _workspace(_lib.mhc_layer_fwd_dynamic_workspace_bytes(B, n, C), xf.device)
    fn = _lib.mhc_layer_fwd_dynamic_bf16 if bf16_io else _lib.mhc_layer_fwd_dynamic
    with _DevGuard(xf):
        rc = fn(
            xf.data_ptr(), w.data_ptr(), pp.data_ptr(), pq.data_ptr(), pr.data_ptr(),
            ap.data_ptr(), aq.data_ptr(), ar.data_ptr(), bp.data_ptr(), bq.data_ptr(),
            br.data_ptr(), out.data_ptr(), _ptr(state), B, n, C, int(sinkhorn_iters),
            float(sinkhorn_eps), float(rmsnorm_eps), ws.data_ptr(), ws.numel(),
            _stream(xf.device))
    _C.check(rc, "mhc_layer_fwd_dynamic_bf16" if bf16_io else "mhc_layer_fwd_dynamic")
    return out, state


def mhc_layer_bwd_dynamic(grad_output, x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                          alpha_post, alpha_res, b_pre, b_post, b_res, token_state,
                          sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5, bf16_io=False):
    """Fused dynamic-H backward (reference mhc_ascend.mhc_layer_bwd_dynamic,
    bindings.cpp:600-874).  Returns the 11 gradients in the reference's order.
    With bf16_io, grad_output / x are read and grad_x written in bf16 (n == 4,
    hidden % 32 == 0); the parameter gradients stay fp32."""
    B, n, C = x.shape
    if bf16_io:
        g = grad_output.to(torch.bfloat16).contiguous()
        xf = x.contiguous()
    else:
        g = _f32(grad_output)
        xf = _f32(x)
    w = _f32(rmsnorm_weight)
    pp, pq, pr = _f32(phi_pre), _f32(phi_post), _f32(phi_res).reshape(n * n, n * C)
    ap, aq, ar = (_as_scalar_tensor(a, xf) for a in (alpha_pre, alpha_post, alpha_res))
    bp, bq, br = _f32(b_pre), _f32(b_post), _f32(b_res)
    dev = xf.device
    gx = torch.empty_like(xf)
    # all parameter gradients live in one flat fp32 buffer, in the order of
    # MHCLayer.parameters() (weight, phi_pre/post/res, b_pre/post/res,
    # alpha_pre/post/res): data-parallel training all-reduces it as it is
    nC = n * C
    sizes = [C, n * nC, n * nC, n * n * nC, n, n, n * n, 3]
    flat = torch.empty(sum(sizes), dtype=torch.float32, device=dev)
    parts = list(torch.split(flat, sizes))
    gw = parts[0]
    gpp, gpq, gpr = parts[1].view(n, nC), parts[2].view(n, nC), parts[3].view(n * n, nC)
    gbp, gbq, gbr = parts[4], parts[5], parts[6].view(n, n)
    galpha = parts[7]
    ws = _workspace(_lib.mhc_layer_bwd_dynamic_workspace_bytes(B, n, C), dev)
    a0 = galpha.data_ptr()
    fn = _lib.mhc_layer_bwd_dynamic_bf16 if bf16_io else _lib.mhc_layer_bwd_dynamic
    with _DevGuard(xf):
        rc = fn(
            g.data_ptr(), xf.data_ptr(), w.data_ptr(), pp.data_ptr(), pq.data_ptr(),
            pr.data_ptr(), ap.data_ptr(), aq.data_ptr(), ar.data_ptr(), bp.data_ptr(),
            bq.data_ptr(), br.data_ptr(), token_state.data_ptr(), gx.data_ptr(), gw.data_ptr(),
            gpp.data_ptr(), gpq.data_ptr(), gpr.data_ptr(), a0, a0 + 4, a0 + 8, gbp.data_ptr(),
            gbq.data_ptr(), gbr.data_ptr(), B, n, C, int(sinkhorn_iters), float(sinkhorn_eps),
            float(rmsnorm_eps), ws.data_ptr(), ws.numel(), _stream(dev))
    _C.check(rc, "mhc_layer_bwd_dynamic_bf16" if bf16_io else "mhc_layer_bwd_dynamic")
    return (gx, gw, gpp, gpq, gpr.reshape(phi_res.shape), galpha[0], galpha[1], galpha[2],
            gbp, gbq, gbr)


def mhc_layer_fused_dynamic_inference(x_expanded, rmsnorm_weight, phi_pre, phi_post, phi_res,
                                      alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                                      sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5,
                                      bf16_io=False):
    """Fused dynamic-H forward without autograd (reference ops.py:337-380)."""
    out, _ = mhc_layer_fwd_dynamic(x_expanded, rmsnorm_weight, phi_pre, phi_post, phi_res,
                                   alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                                   sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, save_state=False,
                                   bf16_io=bf16_io)
    return out


class MHCLayerDynamicFunction(torch.autograd.Function):
    """MHC layer with dynamic H for training (reference ops.py:387-564).

    Saves x, the parameters and one fp32 per-token record (rms_h, rms,
    H_pre/H_post activations, M and the raw projections) instead of the
    reference's 19 tensors.
    """

    @staticmethod
    def forward(ctx, x_expanded, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                alpha_post, alpha_res, b_pre, b_post, b_res, sinkhorn_iters, sinkhorn_eps,
                rmsnorm_eps, bf16_io=False):
        out, state = mhc_layer_fwd_dynamic(x_expanded, rmsnorm_weight, phi_pre, phi_post,
                                           phi_res, alpha_pre, alpha_post, alpha_res, b_pre,
                                           b_post, b_res, sinkhorn_iters, sinkhorn_eps,
                                           rmsnorm_eps, save_state=True, bf16_io=bf16_io)
        ctx.save_for_backward(x_expanded, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                              alpha_post, alpha_res, b_pre, b_post, b_res, state)
        ctx.hp = (sinkhorn_iters, sinkhorn_eps, rmsnorm_eps)
        ctx.bf16_io = bf16_io
        return out

    @staticmethod
    def backward(ctx, grad_output):
        (x, w, pp, pq, pr, ap, aq, ar, bp, bq, br, state) = ctx.saved_tensors
        grads = mhc_layer_bwd_dynamic(grad_output, x, w, pp, pq, pr, ap, aq, ar, bp, bq, br,
                                      state, *ctx.hp, bf16_io=ctx.bf16_io)
        (gx, gw, gpp, gpq, gpr, gap, gaq, gar, gbp, gbq, gbr) = grads
        gx = gx.to(x.dtype)
        gw = gw.to(w.dtype)
        gap = gap.to(ap.dtype).view_as(ap)
        gaq = gaq.to(aq.dtype).view_as(aq)
        gar = gar.to(ar.dtype).view_as(ar)
        return (gx, gw, gpp.to(pp.dtype), gpq.to(pq.dtype), gpr.to(pr.dtype), gap, gaq, gar,
                gbp.to(bp.dtype), gbq.to(bq.dtype), gbr.to(br.dtype), None, None, None, None)


def mhc_layer_fused_dynamic_training(x_expanded, rmsnorm_weight, phi_pre, phi_post, phi_res,
                                     alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                                     sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5,
                                     bf16_io=False):
    """Dynamic-H layer forward with autograd support (reference ops.py:567-628)."""
    dev = phi_pre.device
    if not torch.is_tensor(alpha_pre):
        alpha_pre = torch.tensor(alpha_pre, device=dev, dtype=torch.float32)
    if not torch.is_tensor(alpha_post):
        alpha_post = torch.tensor(alpha_post, device=dev, dtype=torch.float32)
    if not torch.is_tensor(alpha_res):
        alpha_res = torch.tensor(alpha_res, device=dev, dtype=torch.float32)
    return MHCLayerDynamicFunction.apply(x_expanded, rmsnorm_weight, phi_pre, phi_post, phi_res,
                                         alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                                         sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, bf16_io)


# =============================================================================
# MHCResidualWrapper in one piece (n = 4, fp32): streams built in the kernels
# =============================================================================

def wrapper_fused_supported(residual, branch, n, hidden, dynamic=True):
    """Whether the fused wrapper entry points take this call: n = 4, dynamic
    H, fp32 CUDA [tokens, hidden] inputs, hidden % 32 == 0, 16-byte aligned."""
    if not (dynamic and n == 4 and hidden % 32 == 0):
        return False
    for t in (residual, branch):
        if (t is None or not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous()
                or t.data_ptr() % 16):
            return False
    return True


def _flat_param_grads(n, C, dev):
    nC = n * C
    sizes = [C, n * nC, n * nC, n * n * nC, n, n, n * n, 3]
    flat = torch.empty(sum(sizes), dtype=torch.float32, device=dev)
    parts = list(torch.split(flat, sizes))
    return (parts[0], parts[1].view(n, nC), parts[2].view(n, nC), parts[3].view(n * n, nC),
            parts[4], parts[5], parts[6].view(n, n), parts[7])


class WrapperDynamicFunction(torch.autograd.Function):
    """MHCResidualWrapper.forward for a dynamic-H layer at n = 4 (reference
    layer.py:287-316 around ops.py:387-564): the packed streams, the layer
    output and their gradients stay inside the kernels."""

    @staticmethod
    def forward(ctx, residual, branch, residual_mode, rmsnorm_weight, phi_pre, phi_post,
                phi_res, alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res, sinkhorn_iters,
                sinkhorn_eps, rmsnorm_eps):
        n = 4
        T, C = residual.shape
        sc = wrapper_stream_scales(n, residual_mode)
        w = _f32(rmsnorm_weight)
        pp, pq, pr = _f32(phi_pre), _f32(phi_post), _f32(phi_res).reshape(n * n, n * C)
        ap, aq, ar = (_as_scalar_tensor(a, residual) for a in (alpha_pre, alpha_post, alpha_res))
        bp, bq, br = _f32(b_pre), _f32(b_post), _f32(b_res)
        mean = torch.empty(T, C, dtype=torch.float32, device=residual.device)
        state = torch.empty(T, token_state_stride(n), dtype=torch.float32, device=residual.device)
        ws = _workspace(_lib.mhc_layer_fwd_dynamic_workspace_bytes(T, n, C), residual.device)
        with _DevGuard(residual):
            rc = _lib.mhc_wrapper_fwd_dynamic(
                residual.data_ptr(), branch.data_ptr(), sc, w.data_ptr(), pp.data_ptr(),
                pq.data_ptr(), pr.data_ptr(), ap.data_ptr(), aq.data_ptr(), ar.data_ptr(),
                bp.data_ptr(), bq.data_ptr(), br.data_ptr(), mean.data_ptr(), state.data_ptr(),
                T, n, C, int(sinkhorn_iters), float(sinkhorn_eps), float(rmsnorm_eps),
                ws.data_ptr(), ws.numel(), _stream(residual.device))
        _C.check(rc, "mhc_wrapper_fwd_dynamic")
        ctx.save_for_backward(residual, branch, rmsnorm_weight, phi_pre, phi_post, phi_res,
                              alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res, state)
        ctx.sc = sc
        ctx.hp = (sinkhorn_iters, sinkhorn_eps, rmsnorm_eps)
        return mean

    @staticmethod
    def backward(ctx, grad_mean):
        grads = _wrapper_dynamic_bwd(ctx.saved_tensors, ctx.sc, ctx.hp, _f32(grad_mean))
        return (grads[0], grads[1], None, *grads[2:], None, None, None)


def _wrapper_dynamic_bwd(saved, sc, hp, g):
    """Backward of the fused n = 4 wrapper forward for the stream-mean gradient
    g: (grad residual, grad branch, then the gradients of rmsnorm_weight,
    phi_pre, phi_post, phi_res, alpha_pre, alpha_post, alpha_res, b_pre, b_post,
    b_res in their parameters' dtypes)."""
    (res, brn, w0, pp0, pq0, pr0, ap0, aq0, ar0, bp0, bq0, br0, state) = saved
    n = 4
    T, C = res.shape
    w = _f32(w0)
    pp, pq, pr = _f32(pp0), _f32(pq0), _f32(pr0).reshape(n * n, n * C)
    ap, aq, ar = (_as_scalar_tensor(a, res) for a in (ap0, aq0, ar0))
    bp, bq, br = _f32(bp0), _f32(bq0), _f32(br0)
    gres = torch.empty_like(res)
    gbrn = torch.empty_like(brn)
    gw, gpp, gpq, gpr, gbp, gbq, gbr, galpha = _flat_param_grads(n, C, res.device)
    ws = _workspace(_lib.mhc_layer_bwd_dynamic_workspace_bytes(T, n, C), res.device)
    a0 = galpha.data_ptr()
    with _DevGuard(res):
        rc = _lib.mhc_wrapper_bwd_dynamic(
            g.data_ptr(), res.data_ptr(), brn.data_ptr(), sc, w.data_ptr(),
            pp.data_ptr(), pq.data_ptr(), pr.data_ptr(), ap.data_ptr(), aq.data_ptr(),
            ar.data_ptr(), bp.data_ptr(), bq.data_ptr(), br.data_ptr(), state.data_ptr(),
            gres.data_ptr(), gbrn.data_ptr(), gw.data_ptr(), gpp.data_ptr(), gpq.data_ptr(),
            gpr.data_ptr(), a0, a0 + 4, a0 + 8, gbp.data_ptr(), gbq.data_ptr(),
            gbr.data_ptr(), T, n, C, int(hp[0]), float(hp[1]), float(hp[2]),
            ws.data_ptr(), ws.numel(), _stream(res.device))
    _C.check(rc, "mhc_wrapper_bwd_dynamic")
    return (gres, gbrn, gw.to(w0.dtype), gpp.to(pp0.dtype), gpq.to(pq0.dtype),
            gpr.reshape(pr0.shape).to(pr0.dtype), galpha[0].to(ap0.dtype).view_as(ap0),
            galpha[1].to(aq0.dtype).view_as(aq0), galpha[2].to(ar0.dtype).view_as(ar0),
            gbp.to(bp0.dtype), gbq.to(bq0.dtype), gbr.to(br0.dtype))


class WrapperDynamicPreNormFunction(torch.autograd.Function):
    """The fused n = 4 wrapper forward together with the next branch's input
    RMSNorm (a pre-norm transformer block normalises the hidden state the
    wrapper returns before its attention / MLP).  The reference runs
    MHCResidualWrapper.forward (layer.py:287-316) and then the branch's
    rmsnorm (ops.py:87-136) as separate passes; here the wrapper's output pass
    writes both the hidden state and its normalised copy, so the hidden state
    is not read back to be normalised.  Backward: the norm's input gradient
    (mhc_rmsnorm_bwd) joins the hidden state's own gradient before the
    wrapper's fused backward."""

    @staticmethod
    def forward(ctx, residual, branch, residual_mode, norm_weight, norm_eps, rmsnorm_weight,
                phi_pre, phi_post, phi_res, alpha_pre, alpha_post, alpha_res, b_pre, b_post,
                b_res, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps):
        n = 4
        T, C = residual.shape
        sc = wrapper_stream_scales(n, residual_mode)
        w = _f32(rmsnorm_weight)
        w2 = _f32(norm_weight)
        pp, pq, pr = _f32(phi_pre), _f32(phi_post), _f32(phi_res).reshape(n * n, n * C)
        ap, aq, ar = (_as_scalar_tensor(a, residual) for a in (alpha_pre, alpha_post, alpha_res))
        bp, bq, br = _f32(b_pre), _f32(b_post), _f32(b_res)
        dev = residual.device
        mean = torch.empty(T, C, dtype=torch.float32, device=dev)
        normed = torch.empty(T, C, dtype=torch.float32, device=dev)
        rms2 = torch.empty(T, dtype=torch.float32, device=dev)
        state = torch.empty(T, token_state_stride(n), dtype=torch.float32, device=dev)
        ws = _workspace(_lib.mhc_layer_fwd_dynamic_workspace_bytes(T, n, C), dev)
        with _DevGuard(residual):
            rc = _lib.mhc_wrapper_fwd_dynamic_prenorm(
                residual.data_ptr(), branch.data_ptr(), sc, w.data_ptr(), pp.data_ptr(),
                pq.data_ptr(), pr.data_ptr(), ap.data_ptr(), aq.data_ptr(), ar.data_ptr(),
                bp.data_ptr(), bq.data_ptr(), br.data_ptr(), w2.data_ptr(), float(norm_eps),
                mean.data_ptr(), normed.data_ptr(), rms2.data_ptr(), state.data_ptr(),
                T, n, C, int(sinkhorn_iters), float(sinkhorn_eps), float(rmsnorm_eps),
                ws.data_ptr(), ws.numel(), _stream(dev))
        _C.check(rc, "mhc_wrapper_fwd_dynamic_prenorm")
        ctx.save_for_backward(residual, branch, rmsnorm_weight, phi_pre, phi_post, phi_res,
                              alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res, state,
                              mean, norm_weight, rms2)
        ctx.sc = sc
        ctx.hp = (sinkhorn_iters, sinkhorn_eps, rmsnorm_eps)
        return mean, normed

    @staticmethod
    def backward(ctx, grad_mean, grad_normed):
        saved = ctx.saved_tensors
        mean, w2, rms2 = saved[13:]
        g = _f32(grad_mean) if grad_mean is not None else torch.zeros_like(mean)
        gw2 = None
        if grad_normed is not None:
            gi, gw2 = rmsnorm_bwd(grad_normed, mean, w2, rms2)
            g = g + gi
            gw2 = gw2.to(w2.dtype)
        grads = _wrapper_dynamic_bwd(saved[:13], ctx.sc, ctx.hp, g)
        return (grads[0], grads[1], None, gw2, None, *grads[2:], None, None, None)


def wrapper_fused_dynamic_prenorm(residual, branch, residual_mode, norm_weight, norm_eps,
                                  rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                                  alpha_post, alpha_res, b_pre, b_post, b_res, sinkhorn_iters=20,
                                  sinkhorn_eps=1e-8, rmsnorm_eps=1e-5):
    """[tokens, C] residual and branch -> ([tokens, C] stream mean, its RMSNorm
    with norm_weight / norm_eps), n = 4 dynamic H, with autograd."""
    _require_cuda("wrapper_fused_dynamic_prenorm", residual, branch, norm_weight)
    return WrapperDynamicPreNormFunction.apply(residual, branch, residual_mode, norm_weight,
                                               norm_eps, rmsnorm_weight, phi_pre, phi_post,
                                               phi_res, alpha_pre, alpha_post, alpha_res, b_pre,
                                               b_post, b_res, sinkhorn_iters, sinkhorn_eps,
                                               rmsnorm_eps)


def wrapper_fused_dynamic(residual, branch, residual_mode, rmsnorm_weight, phi_pre, phi_post,
                          phi_res, alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                          sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5):
    """[tokens, C] residual and branch -> [tokens, C] stream mean of the n = 4
    dynamic-H layer over the packed streams, with autograd."""
    _require_cuda("wrapper_fused_dynamic", residual, branch)
    return WrapperDynamicFunction.apply(residual, branch, residual_mode, rmsnorm_weight, phi_pre,
                                        phi_post, phi_res, alpha_pre, alpha_post, alpha_res,
                                        b_pre, b_post, b_res, sinkhorn_iters, sinkhorn_eps,
                                        rmsnorm_eps)


# =============================================================================
# Fused static-H layer (the reference composes it from four ops: layer.py:142-170)
# =============================================================================

def mhc_layer_fwd_static(x, rmsnorm_weight, H_pre, H_post, H_res, sinkhorn_iters=20,
                         sinkhorn_eps=1e-8, rmsnorm_eps=1e-5, save_rms=True, bf16_io=False):
    """Fused static-H forward.  Returns (out, rms or None).  With bf16_io the
    input must be bf16 and the output is bf16 (fp32 arithmetic inside)."""
    _require_cuda("mhc_layer_fwd_static", x, rmsnorm_weight, H_pre, H_post, H_res)
    if x.dim() != 3:
        raise RuntimeError("x_expanded must be [B, n, C]")
    B, n, C = x.shape
    w, hp, hq, hr = (_f32(t) for t in (rmsnorm_weight, H_pre, H_post, H_res))
    dev = x.device
    rms = torch.empty(B, dtype=torch.float32, device=dev) if save_rms else None
    ws = _workspace(_lib.mhc_layer_static_workspace_bytes(B, n, C), dev)
    if bf16_io:
        xi = x.detach().to(torch.bfloat16).contiguous()
        out = torch.empty_like(xi)
        fn = _lib.mhc_layer_fwd_static_bf16
    else:
        xi = _f32(x)
        out = torch.empty_like(xi)
        fn = _lib.mhc_layer_fwd_static_f32
    with _DevGuard(xi):
        rc = fn(xi.data_ptr(), w.data_ptr(), hp.data_ptr(), hq.data_ptr(), hr.data_ptr(),
                out.data_ptr(), _ptr(rms), B, n, C, int(sinkhorn_iters), float(sinkhorn_eps),
                float(rmsnorm_eps), ws.data_ptr(), ws.numel(), _stream(dev))
    _C.check(rc, "mhc_layer_fwd_static")
    return out, rms


def mhc_layer_bwd_static(grad_output, x, rmsnorm_weight, H_pre, H_post, H_res, rms,
                         sinkhorn_iters=20, sinkhorn_eps=1e-8, rmsnorm_eps=1e-5):
    B, n, C = x.shape
    g, xf = _f32(grad_output), _f32(x)
    w, hp, hq, hr = (_f32(t) for t in (rmsnorm_weight, H_pre, H_post, H_res))
    dev = xf.device
    gx = torch.empty_like(xf)
    gw = torch.empty(C, dtype=torch.float32, device=dev)
    ghp = torch.empty(n, dtype=torch.float32, device=dev)
    ghq = torch.empty(n, dtype=torch.float32, device=dev)
    ghr = torch.empty(n, n, dtype=torch.float32, device=dev)
    ws = _workspace(_lib.mhc_layer_static_workspace_bytes(B, n, C), dev)
    with _DevGuard(xf):
        rc = _lib.mhc_layer_bwd_static(g.data_ptr(), xf.data_ptr(), w.data_ptr(), hp.data_ptr(),
                                       hq.data_ptr(), hr.data_ptr(), rms.data_ptr(),
                                       gx.data_ptr(), gw.data_ptr(), ghp.data_ptr(),
                                       ghq.data_ptr(), ghr.data_ptr(), B, n, C,
                                       int(sinkhorn_iters), float(sinkhorn_eps),
                                       float(rmsnorm_eps), ws.data_ptr(), ws.numel(),
                                       _stream(dev))
    _C.check(rc, "mhc_layer_bwd_static")
    return gx, gw, ghp, ghq, ghr


class MHCLayerStaticFunction(torch.autograd.Function):
    """Static-H mHC layer as one fused forward and one fused backward."""

    @staticmethod
    def forward(ctx, x, rmsnorm_weight, H_pre, H_post, H_res, sinkhorn_iters, sinkhorn_eps,
                rmsnorm_eps):
        out, rms = mhc_layer_fwd_static(x, rmsnorm_weight, H_pre, H_post, H_res, sinkhorn_iters,
                                        sinkhorn_eps, rmsnorm_eps, save_rms=True)
        ctx.save_for_backward(x, rmsnorm_weight, H_pre, H_post, H_res, rms)
        ctx.hp = (sinkhorn_iters, sinkhorn_eps, rmsnorm_eps)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        x, w, hp, hq, hr, rms = ctx.saved_tensors
        gx, gw, ghp, ghq, ghr = mhc_layer_bwd_static(grad_output, x, w, hp, hq, hr, rms, *ctx.hp)
        return (gx.to(x.dtype), gw.to(w.dtype), ghp.to(hp.dtype), ghq.to(hq.dtype),
                ghr.to(hr.dtype), None, None, None)
