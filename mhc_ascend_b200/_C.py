"""ctypes binding of the C-ABI library ``libmhc_b200.so`` (include/mhc_b200.h).

This module is the only place that talks to the native library.  It loads the
in-tree shared object and declares every entry point's signature.  There is no
CPU or PyTorch fallback: if the library is missing, importing ``lib`` raises.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmhc_b200.so")

c_float_p = ctypes.c_void_p  # device pointers are passed as raw addresses
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "mhc_version": (ctypes.c_char_p, []),
    "mhc_get_last_error_string": (ctypes.c_char_p, []),
    "mhc_sinkhorn_knopp_fwd": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _F, _P]),
    "mhc_sinkhorn_knopp_bwd": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I32, _F, _P]),
    "mhc_rmsnorm_fwd": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _F, _P]),
    "mhc_rmsnorm_bwd_workspace_bytes": (_SZ, [_I64, _I64]),
    "mhc_rmsnorm_bwd": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _P, _SZ, _P]),
    "mhc_stream_aggregate_fwd": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I64, _P]),
    "mhc_stream_aggregate_bwd": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _I32, _I64, _P]),
    "mhc_stream_distribute_mix_add_fwd": (ctypes.c_int,
                                          [_P, _P, _P, _P, _P, _P, _I64, _I32, _I64, _P]),
    "mhc_stream_distribute_mix_add_bwd": (ctypes.c_int,
                                          [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I32,
                                           _I64, _P]),
    "mhc_compute_rms_fwd": (ctypes.c_int, [_P, _P, _I64, _I64, _F, _P]),
    "mhc_fused_rmsnorm_matmul_fwd": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I32, _P]),
    "mhc_fused_rmsnorm_matmul_bwd_workspace_bytes": (_SZ, [_I64, _I64, _I32]),
    "mhc_fused_rmsnorm_matmul_bwd": (ctypes.c_int,
                                     [_P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _SZ, _P]),
    "mhc_wrapper_pack_fwd": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I64, _P]),
    "mhc_wrapper_pack_fwd_bf16": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I64, _P]),
    "mhc_wrapper_pack_bwd": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I64, _P]),
    "mhc_stream_mean_fwd": (ctypes.c_int, [_P, _P, _I64, _I32, _I64, _P]),
    "mhc_stream_mean_bwd": (ctypes.c_int, [_P, _P, _I64, _I32, _I64, _P]),
    "mhc_token_state_stride": (_I32, [_I32]),
    "mhc_layer_fwd_dynamic_workspace_bytes": (_SZ, [_I64, _I32, _I64]),
    "mhc_layer_fwd_dynamic": (ctypes.c_int,
                              [_P] * 13 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_layer_fwd_dynamic_noalloc": (ctypes.c_int,
                                      [_P] * 13 + [_I64, _I32, _I64, _I32, _F, _F, _P]),
    "mhc_layer_fwd_dynamic_bf16": (ctypes.c_int,
                                   [_P] * 13 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_wrapper_fwd_dynamic": (ctypes.c_int,
                                [_P] * 15 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_wrapper_fwd_dynamic_prenorm": (ctypes.c_int,
                                        [_P] * 14 + [_F] + [_P] * 4 +
                                        [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_wrapper_bwd_dynamic": (ctypes.c_int,
                                [_P] * 27 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_layer_bwd_dynamic_workspace_bytes": (_SZ, [_I64, _I32, _I64]),
    "mhc_layer_bwd_dynamic": (ctypes.c_int,
                              [_P] * 24 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_layer_bwd_dynamic_bf16": (ctypes.c_int,
                                   [_P] * 24 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_layer_static_workspace_bytes": (_SZ, [_I64, _I32, _I64]),
    "mhc_layer_fwd_static_f32": (ctypes.c_int,
                                 [_P] * 7 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_layer_fwd_static_bf16": (ctypes.c_int,
                                  [_P] * 7 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_layer_bwd_static": (ctypes.c_int,
                             [_P] * 12 + [_I64, _I32, _I64, _I32, _F, _F, _P, _SZ, _P]),
    "mhc_device_error_word": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32]),
    "mhc_profile_enable": (ctypes.c_int, [ctypes.c_int]),
    "mhc_profile_report": (ctypes.c_int, [ctypes.c_char_p, _SZ]),
}


def device_error_word(reset: bool = False) -> int:
    """Nonzero if a bounded device-side wait ran out (the kernel gave up)."""
    v = ctypes.c_int32(0)
    check(load().mhc_device_error_word(ctypes.byref(v), 1 if reset else 0), "mhc_device_error_word")
    return v.value


def profile_enable(on: bool) -> None:
    load().mhc_profile_enable(1 if on else 0)


def profile_report() -> dict:
    """Wait for the recorded kernel events; return {name: (launches, total_ms)}."""
    lib = load()
    cap = 1 << 16
    buf = ctypes.create_string_buffer(cap)
    n = lib.mhc_profile_report(buf, cap)
    if n < 0:
        raise RuntimeError("mhc_profile_report failed: " + last_error())
    out = {}
    for line in buf.value.decode().splitlines():
        name, cnt, ms = line.split()
        out[name] = (int(cnt), float(ms))
    return out

_lib = None


class NativeLibraryMissing(ImportError):
    pass


def load():
    """Load (once) and return the ctypes handle of libmhc_b200.so."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise NativeLibraryMissing(
            f"mhc_ascend_b200 native library not found at {LIB_PATH}. Build it first:\n"
            "  python -m mhc_ascend_b200.build")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().mhc_get_last_error_string()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed (status {rc}): {last_error()}")
