"""The allocation-free forward entry point (collected last on purpose).

mhc_layer_fwd_dynamic_noalloc serves callers that cannot provide device
scratch memory -- hosts without their own device allocator, processes whose
device memory is fixed after start-up, paths that must not call cudaMalloc or
cudaFree because those can synchronise the device.  It takes its scratch from
a fixed 16 MiB array inside the library.  This test calls it through the
C-ABI twice in a row (the second call reuses the scratch the first one left
behind) and compares each result with the workspace-taking entry point
mhc_layer_fwd_dynamic on the same inputs.
"""
import pytest
import torch

from mhc_ascend_b200 import _C
from oracle import mhc_oracle as O
from tests.helpers import close

pytestmark = pytest.mark.gpu


def _inputs(seed, B, n, C, dev):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, n, C, generator=gen)
    p = O.make_dynamic_params(n, C, gen, alpha=0.5, bias_std=0.5, weight="rand")
    p = {k: v.reshape(-1).contiguous().to(dev) for k, v in p.items()}
    return x.to(dev), p


def _args(x, p):
    return [x.data_ptr(), p["rmsnorm_weight"].data_ptr(), p["phi_pre"].data_ptr(),
            p["phi_post"].data_ptr(), p["phi_res"].data_ptr(), p["alpha_pre"].data_ptr(),
            p["alpha_post"].data_ptr(), p["alpha_res"].data_ptr(), p["b_pre"].data_ptr(),
            p["b_post"].data_ptr(), p["b_res"].data_ptr()]


def test_noalloc_matches_workspace_entry_point(cuda):
    lib = _C.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for seed, (B, n, C) in ((1, (300, 4, 4096)), (2, (77, 4, 1000))):
        x, p = _inputs(seed, B, n, C, cuda)
        stride = lib.mhc_token_state_stride(n)
        out_a = torch.empty_like(x)
        st_a = torch.empty(B, stride, device=cuda)
        ws = torch.empty(lib.mhc_layer_fwd_dynamic_workspace_bytes(B, n, C), dtype=torch.uint8,
                         device=cuda)
        rc = lib.mhc_layer_fwd_dynamic(*_args(x, p), out_a.data_ptr(), st_a.data_ptr(), B, n, C,
                                       20, 1e-8, 1e-5, ws.data_ptr(), ws.numel(), stream)
        assert rc == 0, _C.last_error()
        out_b = torch.empty_like(x)
        st_b = torch.empty(B, stride, device=cuda)
        rc = lib.mhc_layer_fwd_dynamic_noalloc(*_args(x, p), out_b.data_ptr(), st_b.data_ptr(),
                                               B, n, C, 20, 1e-8, 1e-5, stream)
        assert rc == 0, _C.last_error()
        torch.cuda.synchronize()
        close(out_b, out_a, what="noalloc out")
        used = 2 + 2 * n + n * n + (n * n + 2 * n)  # record fields; the rest is padding
        close(st_b[:, :used], st_a[:, :used], what="noalloc token_state")


def test_noalloc_rejects_requests_beyond_its_scratch(cuda):
    lib = _C.load()
    x, p = _inputs(3, 4, 4, 64, cuda)
    out = torch.empty_like(x)
    rc = lib.mhc_layer_fwd_dynamic_noalloc(*_args(x, p), out.data_ptr(), None, 1 << 20, 4, 4096,
                                           20, 1e-8, 1e-5, None)
    assert rc == -2
    assert "16777216" in _C.last_error()
