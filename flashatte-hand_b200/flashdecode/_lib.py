"""ctypes binding of ``libflashdecode_sm100.so`` (declared in include/flashdecode.h).

The reference drove its operator through a pybind shim compiled on the fly
(scripts/evaluate_flashattn_submission.py:24-102); here the same
``extern "C"`` surface is bound with ctypes, so no compiler is needed at
import time.  There is no fallback: if the library is absent or cannot be
loaded, importing the operator raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libflashdecode_sm100.so"

# Every symbol include/flashdecode.h declares, with (restype, argtypes).
_c = ctypes
_vp, _i64, _i32, _f32, _sz = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_float, _c.c_size_t
SIGNATURES: dict[str, tuple] = {
    "run_kernel": (None, [_vp, _vp, _vp, _vp, _vp, _vp] + [_i64] * 9),
    "fd_decode_paged": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp] + [_i64] * 7
                        + [_i32, _i32, _f32, _i64, _vp, _sz, _vp]),
    "fd_decode_paged_mq": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp] + [_i64] * 8
                           + [_i32, _i32, _f32, _i32, _i64, _vp, _sz, _vp]),
    "fd_decode_workspace_size_mq": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "fd_decode_paged_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp] + [_i64] * 7
                                + [_i32, _i32, _f32, _i64, _vp]),
    "fd_decode_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "fd_append_kv_paged": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp] + [_i64] * 7 + [_i32, _vp]),
    "fd_decode_paged_fp8": (_i32, [_vp] * 7 + [_i64] + [_vp] * 4 + [_i64] * 8
                            + [_i32, _i32, _f32, _i32, _i64, _vp, _sz, _vp]),
    "fd_decode_workspace_size_fp8": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "fd_append_kv_paged_fp8": (_i32, [_vp] * 8 + [_i64] * 7 + [_i32, _vp]),
    "fd_decode_paged_kvappend": (_i32, [_vp] * 9 + [_i64] * 9 + [_i32, _i32, _f32, _i32, _i64, _vp,
                                                                _sz, _vp]),
    "fd_combine_lse": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _vp, _vp]),
    "fd_xgpu_buffer_size": (_sz, [_i64, _i64, _i64, _i32]),
    "fd_xgpu_alloc": (_i32, [_sz, _c.POINTER(_vp), _c.c_char_p]),
    "fd_xgpu_open": (_i32, [_c.c_char_p, _c.POINTER(_vp)]),
    "fd_xgpu_close": (_i32, [_vp]),
    "fd_xgpu_free": (_i32, [_vp]),
    "fd_decode_paged_xgpu": (_i32, [_vp, _vp, _vp, _vp, _vp] + [_i64] * 8
                             + [_i32, _i32, _f32, _i32, _i64, _i32, _i32, _c.POINTER(_vp),
                                _c.c_uint64, _vp, _vp, _vp, _sz, _vp]),
    "fd_decode_paged_fp8_xgpu": (_i32, [_vp] * 7 + [_i64] * 8
                                 + [_i32, _i32, _f32, _i32, _i64, _i32, _i32, _c.POINTER(_vp),
                                    _c.c_uint64, _vp, _vp, _vp, _sz, _vp]),
    "fd_last_error": (_i32, []),
    "fd_error_string": (_c.c_char_p, [_i32]),
    "fd_last_error_message": (_c.c_char_p, []),
    "fd_device_status": (_i32, []),
    "fd_library_workspace_bytes": (_sz, []),
    "fd_selftest_bounded_wait": (_i32, [_c.c_uint64, _c.POINTER(_c.c_uint64)]),
    "fd_version": (_c.c_char_p, []),
}

FD_DTYPE_BF16, FD_DTYPE_FP16, FD_DTYPE_FP32, FD_DTYPE_E4M3 = 0, 1, 2, 3
FD_OK = 0
STATUS_NAMES = {0: "FD_OK", 1: "FD_ERR_INVALID_ARG", 2: "FD_ERR_UNSUPPORTED",
                3: "FD_ERR_WORKSPACE", 4: "FD_ERR_CUDA", 5: "FD_ERR_DEVICE_TIMEOUT",
                6: "FD_ERR_BAD_PAGE"}

_lib = None


class FlashDecodeError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")
        self.code = code


def load_library(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and type the shared library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python -m flashdecode.build` "
            "(there is no CPU or Python fallback for this operator)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(status: int) -> None:
    if status != FD_OK:
        lib = load_library()
        raise FlashDecodeError(status, lib.fd_last_error_message().decode())
