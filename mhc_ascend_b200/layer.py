"""mHC layer modules (drop-in for the reference's ``src/python/mhc/layer.py``).

Same constructor arguments, parameter names and shapes as the reference, so
``state_dict``s interchange.  One deliberate difference: ``rmsnorm_weight`` is
an fp32 parameter (the reference keeps it bf16, layer.py:65); loading a
reference checkpoint casts it to fp32 automatically.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .ops import (
    MHCLayerStaticFunction,
    compute_rms,
    fused_rmsnorm_matmul,
    mhc_layer_fused_dynamic_inference,
    mhc_layer_fused_dynamic_training,
    mhc_layer_fwd_static,
    rmsnorm,
    sinkhorn_knopp,
    stream_aggregate,
    stream_distribute_mix_add,
    stream_mean,
    wrapper_fused_dynamic,
    wrapper_fused_dynamic_prenorm,
    wrapper_fused_supported,
    wrapper_pack,
)

__all__ = ["MHCLayer", "create_mhc_layer", "MHCResidualWrapper", "replace_residual_with_mhc"]


class MHCLayer(nn.Module):
    """Manifold-Constrained Hyper-Connections layer (reference layer.py:24-179).

    Args:
        hidden_dim: hidden size C
        expansion_rate: number of residual streams n (1..32; dynamic H: the
            fused kernels for small n, the wide-rate kernels for n >= 8 and
            for n = 6, 7 from 1024 tokens)
        num_sinkhorn_iters: Sinkhorn-Knopp iterations
        sinkhorn_eps: Sinkhorn epsilon
        rmsnorm_eps: epsilon of both RMS computations (dynamic-H rms and RMSNorm)
        use_dynamic_h: per-token H (True) or shared learnable H (False)
        alpha_init: initial value of the alpha scales (dynamic H) / scale of the
            H_res initialisation (static H)
        bf16_io: when the input is bf16, read bf16 and write bf16 (fp32
            arithmetic): static-H inference, and dynamic-H training and
            inference at n <= 4 (n == 4 for training), hidden % 64 == 0.  Off
            by default: like the reference, the layer then returns fp32.
    """

    def __init__(self, hidden_dim: int, expansion_rate: int = 4, num_sinkhorn_iters: int = 20,
                 sinkhorn_eps: float = 1e-8, rmsnorm_eps: float = 1e-5,
                 use_dynamic_h: bool = True, alpha_init: float = 0.01, bf16_io: bool = False):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.expansion_rate = expansion_rate
        self.num_sinkhorn_iters = num_sinkhorn_iters
        self.sinkhorn_eps = sinkhorn_eps
        self.rmsnorm_eps = rmsnorm_eps
        self.use_dynamic_h = use_dynamic_h
        self.bf16_io = bf16_io
        n, C = expansion_rate, hidden_dim
        nC = n * C
        self.rmsnorm_weight = nn.Parameter(torch.ones(hidden_dim, dtype=torch.float32))
        if use_dynamic_h:
            self.phi_pre = nn.Parameter(torch.randn(n, nC) * 0.02)
            self.phi_post = nn.Parameter(torch.randn(n, nC) * 0.02)
            self.phi_res = nn.Parameter(torch.randn(n * n, nC) * 0.02)
            self.b_pre = nn.Parameter(torch.zeros(n))
            self.b_post = nn.Parameter(torch.zeros(n))
            self.b_res = nn.Parameter(torch.zeros(n, n))
            self.alpha_pre = nn.Parameter(torch.tensor(alpha_init))
            self.alpha_post = nn.Parameter(torch.tensor(alpha_init))
            self.alpha_res = nn.Parameter(torch.tensor(alpha_init))
        else:
            self.H_pre = nn.Parameter(torch.zeros(n, dtype=torch.float32))
            self.H_post = nn.Parameter(torch.zeros(n, dtype=torch.float32))
            self.H_res = nn.Parameter((alpha_init * torch.randn(n, n)).float())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, n, C = x.shape
        assert n == self.expansion_rate, f"Expected expansion_rate={self.expansion_rate}, got {n}"
        assert C == self.hidden_dim, f"Expected hidden_dim={self.hidden_dim}, got {C}"
        if self.use_dynamic_h:
            args = (self.rmsnorm_weight, self.phi_pre, self.phi_post, self.phi_res,
                    self.alpha_pre, self.alpha_post, self.alpha_res, self.b_pre, self.b_post,
                    self.b_res, self.num_sinkhorn_iters, self.sinkhorn_eps, self.rmsnorm_eps)
            bf16 = self.bf16_io and x.dtype == torch.bfloat16
            xin = x if bf16 else x.float()
            if (not self.training) and (not torch.is_grad_enabled()):
                return mhc_layer_fused_dynamic_inference(xin, *args, bf16_io=bf16)
            return mhc_layer_fused_dynamic_training(xin, *args, bf16_io=bf16)
        hp = (self.num_sinkhorn_iters, self.sinkhorn_eps, self.rmsnorm_eps)
        if n > 8:
            # the fused static kernels cover n <= 8; wider rates run the
            # reference's own composition (layer.py:142-170) over this
            # library's CUDA operators, with one Sinkhorn for the shared H_res
            xf = x.float()
            M = sinkhorn_knopp(torch.exp(self.H_res.float()).unsqueeze(0), hp[0], hp[1])
            y = rmsnorm(stream_aggregate(xf, self.H_pre.unsqueeze(0).expand(B, -1)),
                        self.rmsnorm_weight, hp[2])
            return stream_distribute_mix_add(y, self.H_post.unsqueeze(0).expand(B, -1),
                                             M.expand(B, -1, -1), xf)
        if not torch.is_grad_enabled() or not (x.requires_grad or any(
                p.requires_grad for p in (self.rmsnorm_weight, self.H_pre, self.H_post,
                                          self.H_res))):
            bf16 = self.bf16_io and x.dtype == torch.bfloat16
            out, _ = mhc_layer_fwd_static(x if bf16 else x.float(), self.rmsnorm_weight,
                                          self.H_pre, self.H_post, self.H_res, *hp,
                                          save_rms=False, bf16_io=bf16)
            return out
        return MHCLayerStaticFunction.apply(x.float(), self.rmsnorm_weight, self.H_pre,
                                            self.H_post, self.H_res, *hp)

    def extra_repr(self) -> str:
        return (f"hidden_dim={self.hidden_dim}, expansion_rate={self.expansion_rate}, "
                f"num_sinkhorn_iters={self.num_sinkhorn_iters}, "
                f"use_dynamic_h={self.use_dynamic_h}")


def create_mhc_layer(hidden_dim: int, expansion_rate: int = 4, num_sinkhorn_iters: int = 20,
                     sinkhorn_eps: float = 1e-8, rmsnorm_eps: float = 1e-5,
                     use_dynamic_h: bool = True, alpha_init: float = 0.01) -> MHCLayer:
    """Create an MHC layer with the given configuration (reference layer.py:186-218)."""
    return MHCLayer(hidden_dim=hidden_dim, expansion_rate=expansion_rate,
                    num_sinkhorn_iters=num_sinkhorn_iters, sinkhorn_eps=sinkhorn_eps,
                    rmsnorm_eps=rmsnorm_eps, use_dynamic_h=use_dynamic_h,
                    alpha_init=alpha_init)


class MHCResidualWrapper(nn.Module):
    """Use MHCLayer in place of a residual connection (reference layer.py:225-329).

    Streams: [residual, branch_output, 0.1*residual, 0.01*residual, ...]
    ('decay') or zeros beyond the first two ('zero'); the mHC output is averaged
    over streams.  ``use_post_norm`` is accepted and, as in the reference
    (layer.py:261), forced off.
    """

    def __init__(self, hidden_dim: int, expansion_rate: int = 4, residual_mode: str = "decay",
                 use_post_norm: bool = True, **mhc_kwargs):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.expansion_rate = expansion_rate
        self.residual_mode = residual_mode
        self.use_post_norm = False
        self.mhc = MHCLayer(hidden_dim=hidden_dim, expansion_rate=expansion_rate, **mhc_kwargs)

    def forward(self, residual: torch.Tensor, branch_output: torch.Tensor) -> torch.Tensor:
        original_shape = residual.shape
        if len(original_shape) == 3:
            B, T, C = original_shape
            residual = residual.reshape(B * T, C)
            branch_output = branch_output.reshape(B * T, C)
        else:
            B, C = original_shape
            T = 1
        n = self.expansion_rate
        m = self.mhc
        if wrapper_fused_supported(residual, branch_output, n, C, m.use_dynamic_h) and \
                self.residual_mode in ("decay", "zero"):
            # n = 4, dynamic H: the streams are built inside the layer's kernels
            # and the mean is written by its output pass -- no [B*T, n, C]
            # tensor in either direction
            output = wrapper_fused_dynamic(
                residual, branch_output, self.residual_mode, m.rmsnorm_weight, m.phi_pre,
                m.phi_post, m.phi_res, m.alpha_pre, m.alpha_post, m.alpha_res, m.b_pre, m.b_post,
                m.b_res, m.num_sinkhorn_iters, m.sinkhorn_eps, m.rmsnorm_eps)
            return output.reshape(B, T, C) if T > 1 else output
        # one CUDA pass packs the streams, one averages them (the reference
        # runs n - 1 scalings, a stack and a mean as framework ops)
        mhc_input = wrapper_pack(residual, branch_output, n, self.residual_mode)
        output = stream_mean(self.mhc(mhc_input))
        if T > 1:
            output = output.reshape(B, T, C)
        return output

    def forward_prenorm(self, residual: torch.Tensor, branch_output: torch.Tensor,
                        norm_weight: torch.Tensor, norm_eps: float = 1e-5):
        """forward() followed by the next branch's input RMSNorm, as a pre-norm
        block uses them: returns (hidden, rmsnorm(hidden, norm_weight,
        norm_eps)).  For n = 4, dynamic H, fp32 the normalised copy is written
        by the same output pass as the hidden state (no second read of it);
        otherwise the two run back to back on this library's CUDA operators.
        The reference has no such entry: its model code would call
        MHCResidualWrapper.forward (layer.py:287-316) and then rmsnorm
        (ops.py:87-136)."""
        shape = residual.shape
        C = shape[-1]
        r2, b2 = residual.reshape(-1, C), branch_output.reshape(-1, C)
        m = self.mhc
        if wrapper_fused_supported(r2, b2, self.expansion_rate, C, m.use_dynamic_h) and \
                self.residual_mode in ("decay", "zero"):
            hidden, normed = wrapper_fused_dynamic_prenorm(
                r2, b2, self.residual_mode, norm_weight, norm_eps, m.rmsnorm_weight, m.phi_pre,
                m.phi_post, m.phi_res, m.alpha_pre, m.alpha_post, m.alpha_res, m.b_pre, m.b_post,
                m.b_res, m.num_sinkhorn_iters, m.sinkhorn_eps, m.rmsnorm_eps)
            return hidden.reshape(shape), normed.reshape(shape)
        hidden = self.forward(residual, branch_output)
        return hidden, rmsnorm(hidden.reshape(-1, C), norm_weight, norm_eps).reshape(shape)

    def extra_repr(self) -> str:
        return (f"hidden_dim={self.hidden_dim}, expansion_rate={self.expansion_rate}, "
                f"residual_mode={self.residual_mode}")


def replace_residual_with_mhc(hidden_dim: int, expansion_rate: int = 4, **kwargs):
    """Helper returning an MHCResidualWrapper (reference layer.py:332-353)."""
    return MHCResidualWrapper(hidden_dim=hidden_dim, expansion_rate=expansion_rate, **kwargs)
