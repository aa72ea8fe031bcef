"""ctypes binding of the in-tree C-ABI library ``libvc_b200.so``.

There is no fallback: if the library is missing or the device is not
sm_100, calls raise.  Status codes map to exceptions:
VC_ERR_ARG / VC_ERR_WORKSPACE -> ValueError, others -> RuntimeError.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libvc_b200.so"

VC_OK, VC_ERR_ARG, VC_ERR_LAUNCH, VC_ERR_UNSUPPORTED, VC_ERR_WORKSPACE = 0, 1, 2, 3, 4
VC_DTYPE_F16, VC_DTYPE_BF16, VC_DTYPE_F32 = 0, 1, 2

_i64, _i32, _p, _f = C.c_int64, C.c_int, C.c_void_p, C.c_float

# name -> (restype, argtypes); mirrors include/vc_b200.h
SIGNATURES = {
    "vc_api_version": (_i32, []),
    "vc_build_info": (C.c_char_p, []),
    "vc_last_error": (C.c_char_p, []),
    "vc_error_read": (_i32, [_i32, C.POINTER(C.c_uint32), _i32]),
    "vc_expcast_codes": (_i32, [_p, _p, _i64, _p]),
    "vc_prep_qk_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "vc_prep_qk_int8": (_i32, [_p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                               _p, _p, _p, _i64, _i64, _p, _p, _p, _p, _p, _i64, _p]),
    "vc_prep_qk_hadamard_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "vc_prep_qk_hadamard_e4m3": (_i32, [_p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                        _i64, _p, _i32, _p, _p, _i64, _p, _p, _p, _p, _p, _i64, _p]),
    "vc_prep_v_channel_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "vc_prep_v_channel": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _p]),
    "vc_prep_v_channel_static": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "vc_prep_v_blocks_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "vc_prep_v_blocks": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i32, _i32, _p, _p, _p, _p,
                                _i64, _p]),
    "vc_group_values_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i32]),
    "vc_group_values": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _p,
                               _i64, _p]),
    "vc_attention_fwd": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                _i32, _i32, _i32, _f, _i64, _i64, _p]),
    "vc_attention_fwd_e4m3qk": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                       _i64, _i32, _i32, _i32, _i64, _f, _i64, _i64, _p]),
    "vc_kernel_resources": (_i32, [_i32, C.POINTER(C.c_int64)]),
    "vc_attention_plan": (_i32, [C.c_int64, C.c_int64, C.c_int64, _i32, C.POINTER(C.c_int64)]),
    "vc_tensor_peak": (_i32, [_i32, _i32, _i64, _i32, _i32, _i32, _p, _p]),
    "vc_selftest_wait_timeout": (_i32, [_i64, _p, _p]),
}

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def load(build_if_missing: bool = False):
    """Load (optionally building) the library; raise if unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists() and build_if_missing:
            from .build import build
            build()
        if not LIB_PATH.exists():
            raise NativeLibraryMissing(
                f"{LIB_PATH} is missing. Build it with `python -m vc_b200.build` (nvcc, sm_100a). "
                "There is no CPU or reference fallback.")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.vc_api_version() != 1:
            raise NativeLibraryMissing("libvc_b200.so API version mismatch; rebuild it")
        _lib = lib
        return lib


def last_error() -> str:
    return load().vc_last_error().decode(errors="replace")


def check(status: int, what: str) -> None:
    if status == VC_OK:
        return
    msg = f"{what}: {last_error()} (status {status})"
    if status in (VC_ERR_ARG, VC_ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def error_word(device: int = 0, clear: bool = True) -> int:
    code = C.c_uint32(0)
    check(load().vc_error_read(device, C.byref(code), int(clear)), "vc_error_read")
    return code.value
