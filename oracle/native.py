"""ctypes loader for oracle/_build/liboracle.so (TEST INFRASTRUCTURE ONLY)."""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        lib = C.CDLL(LIB)
        P, I = C.c_void_p, C.c_int64
        lib.oracle_sum_i32_i64_rows.argtypes = [P, I, I, I, P]
        lib.oracle_argmax_rows_bf16.argtypes = [P, I, I, I, P]
        lib.oracle_amax_rows_f32.argtypes = [P, I, I, I, P]
        _lib = lib
    return _lib


def sum_i32_i64_rows(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int32)
    rows, cols = x.shape
    out = np.empty(rows, np.int64)
    load().oracle_sum_i32_i64_rows(x.ctypes.data, rows, cols, cols, out.ctypes.data)
    return out


def argmax_rows_bf16(bits: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    rows, cols = bits.shape
    out = np.empty(rows, np.int64)
    load().oracle_argmax_rows_bf16(bits.ctypes.data, rows, cols, cols, out.ctypes.data)
    return out


def amax_rows_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(rows, np.float32)
    load().oracle_amax_rows_f32(x.ctypes.data, rows, cols, cols, out.ctypes.data)
    return out
