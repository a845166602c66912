"""ctypes binding of libfl_b200.so (the C ABI declared in include/fl_b200.h).

This is the thin, torch-free view of the kernel library: every function takes
integer device addresses, sizes and a stream handle, exactly like the C
header.  ``call(name, *args)`` raises ``FlB200Error`` on a non-zero status.
The library must exist (``build.py``); there is no fallback.
"""

from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libfl_b200.so")

# dtype enum (fl_b200_dtype)
F32, BF16, F16, I32, I64 = 0, 1, 2, 3, 4
# rounding policy (fl_b200_rounding)
ROUND_FUSED, ROUND_CHAIN = 0, 1
# fl_b200_unary_op
UNARY_SILU, UNARY_RSQRT, UNARY_NEG, UNARY_COS, UNARY_SIN, UNARY_SQUARE, UNARY_CUBE, UNARY_POW = \
    range(8)

_p = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int
_f32 = C.c_float
_f64 = C.c_double
_sz = C.c_size_t
_pi64 = C.POINTER(C.c_int64)

# name -> (restype, argtypes); mirrors include/fl_b200.h one to one.
PROTOTYPES: dict[str, tuple] = {
    "fl_b200_version": (_i32, []),
    "fl_b200_status_string": (C.c_char_p, [_i32]),
    "fl_b200_last_cuda_error": (_i32, []),
    "fl_b200_set_pdl": (_i32, [_i32]),
    "fl_b200_rms_norm_fwd": (
        _i32, [_p, _i64, _p, _p, _i64, _i64, _i64, _f32, _i32, _i32, _p]),
    "fl_b200_add_rms_norm_fwd": (
        _i32, [_p, _p, _p, _p, _p, _i64, _i64, _f32, _i32, _i32, _p]),
    "fl_b200_rope_qk": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _p]),
    "fl_b200_rms_norm_rope": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p,
         _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p,
         _p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _p]),
    "fl_b200_swiglu": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i32, _i32, _p]),
    "fl_b200_swiglu_residual": (
        _i32, [_p, _p, _p, _i64, _p, _p, _p, _i64, _i64, _i32, _i32, _p]),
    "fl_b200_add": (_i32, [_p, _pi64, _p, _pi64, _p, _pi64, _i32, _f64, _i32, _p]),
    "fl_b200_mul": (_i32, [_p, _pi64, _p, _pi64, _p, _pi64, _i32, _i32, _p]),
    "fl_b200_binary_scalar": (_i32, [_p, _f64, _p, _i64, _i32, _f64, _i32, _p]),
    "fl_b200_cast": (_i32, [_p, _i32, _p, _i32, _i64, _p]),
    "fl_b200_unary": (_i32, [_p, _pi64, _pi64, _i32, _i64, _p, _i32, _f64, _i32, _p]),
    "fl_b200_cat": (_i32, [C.POINTER(_p), _pi64, _pi64, _i32, _pi64, _i32, _p, _i32, _p]),
    "fl_b200_softmax_lastdim": (
        _i32, [_p, _i64, _p, _i64, _i64, _i64, _i32, _i32, _i32, _i64, _i64, _p]),
    "fl_b200_softmax_middim": (_i32, [_p, _p, _i64, _i64, _i64, _i32, _i32, _p]),
    "fl_b200_softmax_masked": (
        _i32, [_p, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _f32,
               _i32, _i32, _i32, _p]),
    "fl_b200_reduce_workspace_size": (_sz, [_i64, _i64]),
    "fl_b200_reduce_sum_lastdim": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _i32, _p, _sz, _p]),
    "fl_b200_reduce_mean_lastdim": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _i32, _p, _sz, _p]),
    "fl_b200_reduce_amax_lastdim": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _p, _sz, _p]),
    "fl_b200_reduce_sum_all": (_i32, [_p, _i64, _p, _i32, _i32, _p, _sz, _p]),
    "fl_b200_reduce_mean_all": (_i32, [_p, _i64, _p, _i32, _i32, _p, _sz, _p]),
    "fl_b200_reduce_amax_all": (_i32, [_p, _i64, _p, _i32, _p, _sz, _p]),
    "fl_b200_reduce_middim": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _i32, _i32, _p]),
    "fl_b200_argmax_lastdim": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _p, _sz, _p]),
    "fl_b200_sum_i32_i64": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _p, _sz, _p]),
    "fl_b200_reduce_sum_all_noalloc": (_i32, [_p, _i64, _p, _i32, _i32, _p]),
    "fl_b200_rms_norm_bwd_workspace_size": (_sz, [_i64, _i64]),
    "fl_b200_rms_norm_bwd": (
        _i32, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _i64, _f32, _i32, _p, _sz, _p]),
    "fl_b200_swiglu_bwd": (_i32, [_p, _p, _p, _p, _p, _i64, _i32, _p]),
    "fl_b200_silu_bwd": (_i32, [_p, _p, _p, _i64, _i32, _p]),
    "fl_b200_softmax_bwd": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i32, _i32, _p]),
    "fl_b200_softmax_bwd_scaled": (
        _i32, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _f32, _i32, _i32, _p]),
}


class FlB200Error(RuntimeError):
    """A libfl_b200 entry point returned a non-zero fl_b200_status."""

    def __init__(self, name: str, status: int, cuda_error: int):
        self.status = status
        self.cuda_error = cuda_error
        msg = _LIB.fl_b200_status_string(status).decode() if _LIB else str(status)
        super().__init__(f"{name}: {msg} (status {status}, cuda error {cuda_error})")


_LIB: C.CDLL | None = None


def open_library(path: str) -> C.CDLL:
    """Open a libfl_b200.so and attach the prototypes; a missing file is an
    error (the b200 route has no fallback)."""
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with `python pytorch-plugin-fl_b200/build.py` "
            "(the b200 route has no fallback)"
        )
    lib = C.CDLL(path)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load the kernel library (once per process)."""
    global _LIB
    if _LIB is None:
        _LIB = open_library(path)
    return _LIB


def lib() -> C.CDLL:
    return load()


def call(name: str, *args) -> None:
    """Call entry point `name`; raise FlB200Error on a non-zero status."""
    lib_ = load()
    st = getattr(lib_, name)(*args)
    if st != 0:
        raise FlB200Error(name, st, lib_.fl_b200_last_cuda_error())


def set_pdl(enable: bool) -> bool:
    """Launch the library's kernels with programmatic dependent launch (the
    default) or without; returns the previous setting.  Results are the
    same either way."""
    return bool(load().fl_b200_set_pdl(1 if enable else 0))


def i64_array(vals) -> C.Array:
    arr = (C.c_int64 * max(1, len(vals)))()
    for i, v in enumerate(vals):
        arr[i] = int(v)
    return arr
