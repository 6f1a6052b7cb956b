"""ctypes binding of the C ABI in include/b2q4nx.h (libb2q4nx.so, built in-tree).

The product path has no fallback: if the shared library is missing, importing
an op raises, naming the build command.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "_lib" / "libb2q4nx.so"
HEADER = PKG.parent / "include" / "b2q4nx.h"

_c = ctypes
_vp, _i32, _i64, _f32 = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_float

# name -> (restype, argtypes); must match include/b2q4nx.h
SIGNATURES: dict[str, tuple] = {
    "b2_version": (_i32, []),
    "b2_status_string": (_c.c_char_p, [_i32]),
    "b2_last_error_message": (_c.c_char_p, []),
    "b2_set_launch_options": (_i32, [_i32]),
    "b2_read_device_error": (_i32, [_c.POINTER(_i32), _vp]),
    "b2_q4_gemv": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _i32, _vp]),
    "b2_q8_gemv": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _i32, _vp]),
    "b2_q4_swiglu_gemv": (_i32, [_vp, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _i32, _vp]),
    "b2_q4_gemv_rmsnorm": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _i32, _vp]),
    "b2_q8_gemv_rmsnorm": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _i32, _vp]),
    "b2_q4_swiglu_gemv_rmsnorm": (_i32, [_vp, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _i32, _vp]),
    "b2_gqa_decode_workspace_size": (_i32, [_i32, _i32, _i32, _i32, _i32, _c.POINTER(_c.c_size_t)]),
    "b2_gqa_decode": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _f32,
                             _vp, _i32, _vp, _c.c_size_t, _i32, _vp]),
    "b2_gqa_decode_static": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32,
                                    _f32, _vp, _i32, _i32, _vp]),
    "b2_rmsnorm": (_i32, [_vp, _i32, _i32, _vp, _f32, _i32, _i32, _vp, _i32, _vp]),
    "b2_peer_alloc": (_i32, [_c.c_size_t, _c.POINTER(_vp), _c.c_char_p]),
    "b2_peer_free": (_i32, [_vp]),
    "b2_peer_open": (_i32, [_c.c_char_p, _c.POINTER(_vp)]),
    "b2_peer_close": (_i32, [_vp]),
    "b2_set_peer_timeout_ms": (_i32, [_i32]),
    "b2_tp_gather": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _i32, _i32, _c.c_longlong, _i32, _vp, _vp]),
    "b2_tp_allreduce": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _i32, _c.c_longlong, _vp, _i32, _vp]),
    "b2_gated_attn_decode_workspace_size": (_i32, [_i32, _i32, _i32, _i32, _i32, _c.POINTER(_c.c_size_t)]),
    "b2_gated_attn_decode": (_i32, [_vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _i32, _i32, _i32,
                                    _i32, _i32, _i32, _f32, _vp, _i32, _i32, _vp, _c.c_size_t, _vp]),
    "b2_gated_delta_step": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                   _i32, _i32, _f32, _vp, _i32, _i32, _vp]),
    "b2_q4_gemm_workspace_size": (_i32, [_i32, _i32, _c.POINTER(_c.c_size_t)]),
    "b2_q4_gemm": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _c.c_size_t, _vp]),
    "b2_q4_swiglu_gemm": (_i32, [_vp, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _c.c_size_t, _vp]),
    "b2_q4_gemm_rmsnorm": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _i32, _vp, _c.c_size_t,
                                  _vp]),
    "b2_q4_swiglu_gemm_rmsnorm": (_i32, [_vp, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _i32, _vp,
                                         _c.c_size_t, _vp]),
    "b2_q4_gemm_swiglu_in": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _c.c_size_t, _vp]),
    "b2_gemm_rmsnorm_seam": (_i32, [_i32, _vp, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _i32, _vp,
                                     _c.c_size_t, _vp, _i32, _i32, _c.c_longlong, _i32, _i32, _vp]),
    "b2_q4_gemm_pack": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "b2_q8_gemm_pack": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "b2_q8_gemm": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _i32, _vp, _c.c_size_t, _vp]),
    "b2_q8_gemm_rmsnorm": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _i32, _vp, _c.c_size_t,
                                  _vp]),
    "b2_q4_dequant_tiles": (_i32, [_vp, _i64, _vp, _vp]),
    "b2_q8_dequant_tiles": (_i32, [_vp, _i64, _vp, _vp]),
    "b2_q4_dequant_matrix": (_i32, [_vp, _i32, _i32, _vp, _i64, _vp]),
    "b2_q8_dequant_matrix": (_i32, [_vp, _i32, _i32, _vp, _i64, _vp]),
}

_LIB: ctypes.CDLL | None = None


class B2Error(RuntimeError):
    """A b2q4nx entry point returned a non-zero status."""

    def __init__(self, what: str, status: int, detail: str):
        super().__init__(f"{what} failed: status {status} ({detail})")
        self.status = status


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(b2_\w+)\s*\(", text, re.M)))


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"native library {LIB_PATH} is not built; run `python -m llmnputest_b200.build` "
                "(there is no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        detail = L.b2_last_error_message().decode() or L.b2_status_string(status).decode()
        raise B2Error(what, status, detail)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def read_device_error(stream: int = 0) -> int:
    code = _i32(0)
    check(lib().b2_read_device_error(ctypes.byref(code), _vp(stream)), "b2_read_device_error")
    return code.value
