"""Comparison helpers shared by the parity tests.

Tolerances (stated once, used everywhere):
  * integer / index results: bit-exact;
  * bf16 / f16 results: at most 1 ulp from the fp64-evaluated formula rounded
    once (the "fp32-accumulated result"), ``assert_ulp``;
  * fp32 elementwise / row-normalised results: relative error <= 1e-5
    (``assert_rel``);
  * fp32 sums: |got - exact| <= 1e-5 * max(|exact|, sum|x| / sqrt(n)), i.e.
    1e-5 relative to the scale a sum of n terms of that size has
    (``assert_sum``) -- a plain relative bound is meaningless for sums that
    cancel to nearly zero (torch's own CPU sum misses it there).
"""

from __future__ import annotations

import os

import numpy as np

from oracle import ops

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")

ULP_TOL = 1
REL_TOL = 1e-5
SUM_TOL = 1e-5


class Golden:
    """Access to tests/golden/golden.npz: get(key) returns float32 values for
    float arrays (bf16 decoded from its bit patterns) or the integer array."""

    def __init__(self, path: str = GOLDEN):
        self.z = np.load(path)

    def get(self, key: str) -> np.ndarray:
        z = self.z
        if key + ":bf16" in z:
            return ops.bf16_from_bits(z[key + ":bf16"])
        if key + ":f16" in z:
            return z[key + ":f16"].astype(np.float32)
        if key + ":f32" in z:
            return z[key + ":f32"]
        if key + ":int" in z:
            return z[key + ":int"]
        raise KeyError(key)

    def dtype(self, key: str) -> str:
        for suf in ("bf16", "f16", "f32"):
            if f"{key}:{suf}" in self.z:
                return suf
        return "int"


def assert_ulp(got, ref, dtype: str, max_ulp: int = ULP_TOL, what: str = "") -> np.ndarray:
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    d = ops.ulp_diff(got, ref, dtype)
    worst = int(d.max()) if d.size else 0
    if worst > max_ulp:
        i = np.unravel_index(int(np.argmax(d)), d.shape)
        raise AssertionError(
            f"{what}: {worst} ulp ({dtype}) > {max_ulp} at {i}: got {got[i]!r} want {ref[i]!r}; "
            f"{int(np.sum(d > max_ulp))} of {d.size} elements over"
        )
    return d


def assert_exact(got, ref, what: str = "") -> None:
    got = np.asarray(got)
    ref = np.asarray(ref)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    if got.dtype.kind == "f":
        same = (got == ref) | (np.isnan(got) & np.isnan(ref))
    else:
        same = got == ref
    if not np.all(same):
        i = np.argwhere(~same)[0]
        raise AssertionError(f"{what}: mismatch at {tuple(i)}: got {got[tuple(i)]} want {ref[tuple(i)]}")


def assert_rel(got, ref, rtol: float = REL_TOL, atol: float = 0.0, what: str = "") -> None:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    both_nan = np.isnan(got) & np.isnan(ref)
    err = np.abs(got - ref)
    bad = ~both_nan & ~(err <= atol + rtol * np.abs(ref))
    if np.any(bad):
        i = tuple(np.argwhere(bad)[0])
        raise AssertionError(f"{what}: rel err {err[i] / max(abs(ref[i]), 1e-300):.3g} at {i}: "
                             f"got {got[i]!r} want {ref[i]!r}")


# Gradients whose terms can cancel (RMSNorm dx = r (w dy - n m), softmax
# dx = y (dy - sum dy y)) are checked against an elementwise bound scaled by
# the magnitude of the terms: an fp32 evaluation is within a few 2^-24 of
# that magnitude, however small the result.  BWD_TERM_TOL is that factor;
# the storage rounding (1 ulp of the output dtype) comes on top.
BWD_TERM_TOL = 64 * 2.0 ** -24


def ulp_of(ref, dtype: str) -> np.ndarray:
    """Spacing of the storage dtype at |ref| (its unit in the last place)."""
    r = np.abs(np.asarray(ref, np.float64)).astype(np.float32)
    if dtype == "f16":
        return np.spacing(r.astype(np.float16)).astype(np.float64)
    sp = np.spacing(r).astype(np.float64)
    return sp * 2.0 ** 16 if dtype == "bf16" else sp


def assert_within(got, ref, tol, what: str = "", dtype: str | None = None) -> None:
    """|got - ref| <= tol elementwise (tol broadcasts); with a 16-bit `dtype`
    the final rounding adds 1 ulp of ref to the tolerance."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    err = np.abs(got - ref)
    lim = np.broadcast_to(tol, err.shape).astype(np.float64)
    if dtype in ("bf16", "f16"):
        lim = lim + ulp_of(ref, dtype)
    ok = (err <= lim) | (np.isnan(got) & np.isnan(ref))
    if not np.all(ok):
        i = tuple(np.argwhere(~ok)[0])
        t = lim[i]
        raise AssertionError(f"{what}: err {err[i]:.3g} > tol {t:.3g} at {i}: "
                             f"got {got[i]!r} want {ref[i]!r}")


def assert_sum(got, x, axis, what: str = "", tol: float = SUM_TOL) -> None:
    x64 = np.asarray(x, np.float64)
    exact = np.sum(x64, axis=axis)
    n = x64.size if axis is None else x64.shape[axis]
    scale = np.maximum(np.abs(exact), np.sum(np.abs(x64), axis=axis) / np.sqrt(max(n, 1)))
    err = np.abs(np.asarray(got, np.float64) - exact)
    bad = err > tol * scale
    if np.any(bad):
        i = tuple(np.argwhere(np.atleast_1d(bad))[0])
        raise AssertionError(f"{what}: sum error {np.atleast_1d(err)[i]:.3g} > "
                             f"{tol} * {np.atleast_1d(scale)[i]:.3g}")


# ------------------------------------------------ torch <-> oracle arrays ---
def to_np(t) -> np.ndarray:
    """A torch tensor (any device) as numpy: float types as float32 values."""
    import torch

    t = t.detach().to("cpu")
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.numpy()


def from_np(a: np.ndarray, dtype, device):
    """Upload float32 values (already representable in dtype) as a tensor."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


DT_NAME = {"float32": "f32", "bfloat16": "bf16", "float16": "f16"}


def dname(dtype) -> str:
    return DT_NAME[str(dtype).replace("torch.", "")]
