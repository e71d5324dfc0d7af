"""mHC (Manifold-Constrained Hyper-Connections) layer for NVIDIA B200 (sm_100a).

Drop-in for the Python API of ParadoxZW/mHC_Ascend (``mhc``): the same
modules and operators, backed by hand-written sm_100a CUDA kernels reached
through the C-ABI library ``libmhc_b200.so`` (declared in include/mhc_b200.h).

Example:
    >>> import torch
    >>> from mhc_ascend_b200 import MHCLayer
    >>> layer = MHCLayer(hidden_dim=4096, expansion_rate=4).cuda()
    >>> out = layer(torch.randn(32, 4, 4096, device="cuda"))
"""

__version__ = "0.1.0"

from .layer import MHCLayer, create_mhc_layer, MHCResidualWrapper, replace_residual_with_mhc
from .ops import (
    sinkhorn_knopp,
    rmsnorm,
    stream_aggregate,
    stream_distribute_mix_add,
)

__all__ = [
    "MHCLayer",
    "MHCResidualWrapper",
    "create_mhc_layer",
    "replace_residual_with_mhc",
    "sinkhorn_knopp",
    "rmsnorm",
    "stream_aggregate",
    "stream_distribute_mix_add",
]
