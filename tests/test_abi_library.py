"""The C-ABI library: it loads, exports every entry point that
include/fl_b200.h declares, and its host-side argument checks answer with the
documented status codes.  CPU only: nothing here launches a kernel."""

import ctypes
import os
import re

import pytest

from torch_fl import _abi

HEADER_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def declared_symbols():
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if fn.endswith(".h"):
            src = open(os.path.join(HEADER_DIR, fn)).read()
            names |= set(re.findall(r"FL_B200_API\s+[\w\s\*]+?\b(fl_b200_\w+)\s*\(", src))
    return sorted(names)


def test_header_declares_the_path():
    names = declared_symbols()
    for required in ["fl_b200_rms_norm_fwd", "fl_b200_rope_qk", "fl_b200_rms_norm_rope",
                     "fl_b200_swiglu", "fl_b200_swiglu_residual", "fl_b200_add", "fl_b200_mul",
                     "fl_b200_softmax_lastdim", "fl_b200_reduce_sum_lastdim",
                     "fl_b200_reduce_mean_lastdim", "fl_b200_reduce_amax_lastdim",
                     "fl_b200_reduce_sum_all", "fl_b200_reduce_mean_all",
                     "fl_b200_reduce_amax_all", "fl_b200_argmax_lastdim",
                     "fl_b200_sum_i32_i64"]:
        assert required in names, required


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_abi.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert set(declared_symbols()) == set(_abi.PROTOTYPES), \
        set(declared_symbols()) ^ set(_abi.PROTOTYPES)


def test_identity_and_status_strings():
    lib = _abi.load()
    assert lib.fl_b200_version() >= 100
    assert lib.fl_b200_status_string(0) == b"success"
    for st in range(1, 8):
        assert lib.fl_b200_status_string(st) != b"unknown fl_b200 status"
    assert lib.fl_b200_status_string(99) == b"unknown fl_b200 status"


def test_workspace_size_plan():
    lib = _abi.load()
    assert lib.fl_b200_reduce_workspace_size(65536, 8192) == 0   # enough rows: no split
    assert lib.fl_b200_reduce_workspace_size(1, 100) == 0        # tiny row: one CTA
    n = lib.fl_b200_reduce_workspace_size(1, 65536 * 8192)       # full-tensor sum
    # 27 chunks per SM of a 148-SM B200, 16-byte partials + a ticket; a
    # single row's split always fits the no-allocation entry's 64 KB scratch
    assert 2048 * 16 < n <= 148 * 27 * 16 + 64
    assert n <= 65536
    assert lib.fl_b200_reduce_workspace_size(0, 10) == 0


@pytest.mark.parametrize("call", [
    lambda: _abi.call("fl_b200_rms_norm_fwd", None, 0, None, None, 0, -1, 4, 1e-6, 1, 0, None),
    lambda: _abi.call("fl_b200_rms_norm_fwd", 8, 4, 8, 8, 4, 2, 4, 1e-6, 1, 7, None),
    lambda: _abi.call("fl_b200_swiglu", None, 0, None, 0, None, 0, -2, 8, 1, 0, None),
    lambda: _abi.call("fl_b200_cast", None, 0, None, 1, -5, None),
    lambda: _abi.call("fl_b200_add", None, None, None, None, None, None, 9, 1.0, 1, None),
    lambda: _abi.call("fl_b200_softmax_lastdim", None, 0, None, 0, -1, 4, 1, 1, 0, 1, 0, None),
    lambda: _abi.call("fl_b200_rope_qk", 8, 8, 1, 0, 0, 0, 0, 0, 0, None, None, 0, 0, 0, 0,
                      0, 0, 0, 8, 8, 0, 0, 1, 1, 3, 1, 0, None),  # odd head dim
    lambda: _abi.call("fl_b200_reduce_middim", None, 1, 1, 1, None, 5, 0, 0, None),
    # masked softmax: rows not a whole number of (heads x q_len) blocks, no
    # heads, an unknown rounding mode
    lambda: _abi.call("fl_b200_softmax_masked", 16, 8, None, 0, 0, 0, 16, 8, 6, 8, 2, 4, 1.0,
                      1, 1, 0, None),
    lambda: _abi.call("fl_b200_softmax_masked", 16, 8, None, 0, 0, 0, 16, 8, 8, 8, 0, 4, 1.0,
                      1, 1, 0, None),
    lambda: _abi.call("fl_b200_softmax_masked", 16, 8, None, 0, 0, 0, 16, 8, 8, 8, 2, 4, 1.0,
                      1, 1, 7, None),
    lambda: _abi.call("fl_b200_softmax_bwd_scaled", None, 0, None, 0, None, 0, -1, 4, 1.0, 1, 1,
                      None),
])
def test_bad_arguments_are_rejected_on_the_host(call):
    with pytest.raises(_abi.FlB200Error) as ei:
        call()
    assert ei.value.status == 1  # FL_B200_ERR_INVALID_ARGUMENT


def test_empty_inputs_are_no_ops():
    # zero-sized work returns success before touching any device
    _abi.call("fl_b200_rms_norm_fwd", None, 0, None, None, 0, 0, 4096, 1e-6, 1, 0, None)
    _abi.call("fl_b200_swiglu", None, 0, None, 0, None, 0, 0, 8, 1, 0, None)
    _abi.call("fl_b200_cast", None, 0, None, 1, 0, None)
    _abi.call("fl_b200_softmax_lastdim", None, 0, None, 0, 0, 4, 1, 1, 0, 1, 0, None)
    _abi.call("fl_b200_softmax_masked", None, 0, None, 0, 0, 0, None, 0, 0, 64, 4, 16, 0.125,
              1, 1, 0, None)
