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


SCRATCH = 16 << 20  # the entry point's fixed scratch capacity


def _run_pair(lib, cuda, stream, seed, B, n, C, keep_state):
    """One call of each entry point on the same inputs; the noalloc call with or
    without a caller-kept token_state (without it the record is scratch too)."""
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
    st_b = torch.empty(B, stride, device=cuda) if keep_state else None
    rc = lib.mhc_layer_fwd_dynamic_noalloc(*_args(x, p), out_b.data_ptr(),
                                           st_b.data_ptr() if keep_state else None,
                                           B, n, C, 20, 1e-8, 1e-5, stream)
    assert rc == 0, _C.last_error()
    torch.cuda.synchronize()
    # same kernels, same split plan: the results are bitwise equal
    assert torch.equal(out_b, out_a), "noalloc out differs from the workspace entry point"
    if keep_state:
        used = 2 + 2 * n + n * n + (n * n + 2 * n)  # record fields; the rest is padding
        assert torch.equal(st_b[:, :used], st_a[:, :used]), "noalloc token_state differs"


def test_noalloc_matches_workspace_entry_point(cuda):
    """Two calls in a row with a caller-kept token_state, then one without it
    (the record then lives in the shared scratch as well)."""
    lib = _C.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    _run_pair(lib, cuda, stream, 1, 300, 4, 4096, keep_state=True)
    _run_pair(lib, cuda, stream, 2, 77, 4, 1000, keep_state=True)
    _run_pair(lib, cuda, stream, 4, 513, 4, 4096, keep_state=False)


def _largest_batch_with_state(lib, n, C):
    """Largest batch whose scratch need, with the record kept by the caller,
    fits the fixed array: the workspace size minus the record block."""
    stride = lib.mhc_token_state_stride(n)

    def need(B):
        rec = (B * stride * 4 + 255) // 256 * 256
        return lib.mhc_layer_fwd_dynamic_workspace_bytes(B, n, C) - rec

    lo, hi = 1, 1
    while need(hi) <= SCRATCH:
        lo, hi = hi, hi * 2
    while hi - lo > 1:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if need(mid) <= SCRATCH else (lo, mid)
    return lo


def test_noalloc_near_its_limit(cuda):
    """At the largest batch that fits with a caller-kept token_state the call
    succeeds and matches; the same batch without token_state is rejected when
    its record no longer fits."""
    lib = _C.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    n, C = 4, 4096
    B = _largest_batch_with_state(lib, n, C)
    _run_pair(lib, cuda, stream, 5, B, n, C, keep_state=True)
    if lib.mhc_layer_fwd_dynamic_workspace_bytes(B, n, C) > SCRATCH:
        x, p = _inputs(6, 4, n, C, cuda)
        out = torch.empty(B, n, C, device=cuda)
        rc = lib.mhc_layer_fwd_dynamic_noalloc(*_args(x, p), out.data_ptr(), None, B, n, C,
                                               20, 1e-8, 1e-5, stream)
        assert rc == -2 and "16777216" in _C.last_error()


def test_noalloc_rejects_requests_beyond_its_scratch(cuda):
    lib = _C.load()
    x, p = _inputs(3, 4, 4, 64, cuda)
    out = torch.empty_like(x)
    rc = lib.mhc_layer_fwd_dynamic_noalloc(*_args(x, p), out.data_ptr(), None, 1 << 20, 4, 4096,
                                           20, 1e-8, 1e-5, None)
    assert rc == -2
    assert "16777216" in _C.last_error()
    # invalid arguments are reported as such, not as a size problem
    rc = lib.mhc_layer_fwd_dynamic_noalloc(*_args(x, p), out.data_ptr(), None, 4, 4, 0,
                                           20, 1e-8, 1e-5, None)
    assert rc == -1 and "hidden" in _C.last_error()
