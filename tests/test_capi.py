"""C-ABI library checks that need no GPU: it loads, exports every symbol the
header declares, the ctypes table matches the header, and argument
validation fails with the documented status codes before any launch."""
import ctypes
import os
import re

import pytest

from mhc_ascend_b200 import _C

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "mhc_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"MHC_API\s+[\w\s\*]+?\b(mhc_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert len(names) >= 20
    assert "mhc_layer_fwd_dynamic" in names and "mhc_layer_bwd_dynamic" in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_C.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_ctypes_table_covers_header():
    assert set(declared_symbols()) == set(_C.SIGNATURES)


def test_version():
    assert b"sm_100a" in _C.load().mhc_version()


ERR_INVALID, ERR_UNSUPPORTED, ERR_WORKSPACE = -1, -2, -4


def test_validation_errors_without_gpu():
    lib = _C.load()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    assert lib.mhc_sinkhorn_knopp_fwd(p, p, 4, 33, 20, 1e-8, None) == ERR_UNSUPPORTED
    assert "n must be in [1, 32]" in _C.last_error()
    assert lib.mhc_sinkhorn_knopp_fwd(p, p, 4, 4, -1, 1e-8, None) == ERR_INVALID
    assert lib.mhc_sinkhorn_knopp_fwd(None, p, 4, 4, 20, 1e-8, None) == ERR_INVALID
    assert lib.mhc_rmsnorm_fwd(p, p, p, None, 4, 8, 1e-5, None) == ERR_INVALID
    args = [p] * 13 + [8, 33, 64, 20, 1e-8, 1e-5, p, 1 << 30, None]
    assert lib.mhc_layer_fwd_dynamic(*args) == ERR_UNSUPPORTED
    assert "expansion_rate" in _C.last_error()
    args = [p] * 13 + [8, 9, 64, 20, 1e-8, 1e-5, p, 1 << 30, None]
    assert lib.mhc_layer_fwd_dynamic_bf16(*args) == ERR_UNSUPPORTED  # bf16 streams: n <= 8
    args = [p] * 13 + [8, 16, 64, 20, 1e-8, 1e-5, p, 0, None]
    assert lib.mhc_layer_fwd_dynamic(*args) == ERR_WORKSPACE  # wide rates plan a workspace too
    args = [p] * 13 + [8, 4, 64, 20, 1e-8, 1e-5, p, 0, None]
    assert lib.mhc_layer_fwd_dynamic(*args) == ERR_WORKSPACE
    assert "workspace" in _C.last_error()
    args = [p] * 24 + [8, 4, 64, 20, 1e-8, 1e-5, None, 0, None]
    assert lib.mhc_layer_bwd_dynamic(*args) == ERR_WORKSPACE


def test_wrapper_entry_points_validate_without_gpu():
    lib = _C.load()
    p = ctypes.c_void_p(16)
    sc = (ctypes.c_float * 65)(*([1.0] * 65))
    assert lib.mhc_wrapper_pack_fwd(p, p, p, sc, 4, 65, 8, None) == ERR_UNSUPPORTED
    assert "n must be in [1, 64]" in _C.last_error()
    assert lib.mhc_wrapper_pack_fwd(p, None, p, sc, 4, 2, 8, None) == ERR_INVALID
    assert "branch" in _C.last_error()
    assert lib.mhc_wrapper_pack_fwd(p, None, p, sc, 0, 1, 8, None) == 0  # n = 1 needs no branch
    assert lib.mhc_stream_mean_fwd(None, p, 4, 4, 8, None) == ERR_INVALID
    assert lib.mhc_stream_mean_bwd(p, p, -1, 4, 8, None) == ERR_INVALID
    assert lib.mhc_wrapper_pack_bwd(p, p, None, None, 4, 4, 8, None) == ERR_INVALID


def test_wrapper_prenorm_validates_without_gpu():
    """mhc_wrapper_fwd_dynamic_prenorm checks its extra arguments (the next
    branch's norm weight, eps and outputs) before any device work."""
    lib = _C.load()
    p, odd = ctypes.c_void_p(16), ctypes.c_void_p(20)
    sc = (ctypes.c_float * 4)(1.0, 0.0, 0.1, 0.01)

    def call(norm_w=p, eps=1e-5, normed=p, rms=p, tokens=8):
        return lib.mhc_wrapper_fwd_dynamic_prenorm(
            p, p, sc, p, p, p, p, p, p, p, p, p, p, norm_w, eps, p, normed, rms, p,
            tokens, 4, 64, 20, 1e-8, 1e-5, None, 0, None)

    assert call(eps=-1.0) == ERR_INVALID and "norm_eps" in _C.last_error()
    assert call(norm_w=None) == ERR_INVALID and "norm_weight" in _C.last_error()
    assert call(rms=None) == ERR_INVALID and "out_norm_rms" in _C.last_error()
    assert call(normed=odd) == -3 and "aligned" in _C.last_error()
    assert call(tokens=0) == 0


def test_empty_batch_is_a_noop():
    lib = _C.load()
    p = ctypes.c_void_p(16)
    assert lib.mhc_sinkhorn_knopp_fwd(p, p, 0, 4, 20, 1e-8, None) == 0
    args = [p] * 13 + [0, 4, 64, 20, 1e-8, 1e-5, None, 0, None]
    assert lib.mhc_layer_fwd_dynamic(*args) == 0


def test_workspace_queries():
    lib = _C.load()
    fwd = lib.mhc_layer_fwd_dynamic_workspace_bytes(8192, 4, 4096)
    bwd = lib.mhc_layer_bwd_dynamic_workspace_bytes(8192, 4, 4096)
    assert 0 < fwd < 64 << 20
    assert 0 < bwd < 512 << 20
    assert lib.mhc_token_state_stride(4) == 72  # 50 record floats + padding + fp64 Gram (10 doubles)
    assert lib.mhc_token_state_stride(32) == 2180  # 2 + 2n + n^2 + (n^2 + 2n) = 2178, 4-aligned; no Gram
    assert lib.mhc_layer_static_workspace_bytes(65536, 4, 4096) > 0
    assert lib.mhc_rmsnorm_bwd_workspace_bytes(1024, 4096) >= 4096 * 4
