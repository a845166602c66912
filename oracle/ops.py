"""numpy restatement of the non-GEMM op path (TEST INFRASTRUCTURE ONLY).

Two flavours per floating-point op:

* ``*_golden`` -- fp64 math with ONE final rounding to the storage dtype: the
  "fp32-accumulated result" that the bf16/f16 tolerance (1 ulp) is stated
  against.
* ``*_chain``  -- fp32 math rounded to the storage dtype after every step,
  exactly where the reference's op-by-op chain on the flagos device rounds
  (every aten op returns a tensor of the input dtype; PyTorch computes each
  op in fp32 "opmath" for bf16/f16 -- csrc/aten/backends/cuda/add.cu:48-84,
  mul.cu:28-52, silu.cu:27-29, pow.cu:29-32, mean.cu:17-28, rsqrt.cu:14-32).

Integer and index work (int32 -> int64 sums, amax, argmax) is exact.

Arrays in: float32 arrays holding values already representable in the
storage dtype (``round_to``), or integer arrays.  Storage dtypes are named
'f32', 'bf16', 'f16'.
"""

from __future__ import annotations

import numpy as np

# ----------------------------------------------------------- number formats --


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest-even), return the 16-bit
    patterns.  Restates c10::BFloat16's round_to_nearest_even: NaN -> 0x7FC0,
    otherwise (bits + 0x7FFF + lsb) >> 16."""
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)).astype(np.uint16)
    r = np.where(np.isnan(f), np.uint16(0x7FC0), r)
    return r


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_to(a, dtype: str) -> np.ndarray:
    """Round to the storage dtype; returns float32 values (exactly
    representable in `dtype`)."""
    a = np.asarray(a)
    if dtype == "f32":
        return a.astype(np.float32)
    f = a.astype(np.float32)  # f64 -> f32 first (nearest-even)
    if dtype == "bf16":
        return bf16_from_bits(bf16_bits(f))
    if dtype == "f16":
        return f.astype(np.float16).astype(np.float32)
    raise ValueError(dtype)


def to_bits(a: np.ndarray, dtype: str) -> np.ndarray:
    """Storage bit patterns of values representable in `dtype`."""
    if dtype == "bf16":
        return bf16_bits(a)
    if dtype == "f16":
        return np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)
    if dtype == "f32":
        return np.asarray(a, dtype=np.float32).view(np.uint32)
    raise ValueError(dtype)


def ulp_diff(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """Distance in units of the last place of `dtype` between a and b (both
    representable in dtype).  Equal NaNs count 0, a NaN against a number a
    huge distance."""
    ba = to_bits(a, dtype).astype(np.int64)
    bb = to_bits(b, dtype).astype(np.int64)
    width = 32 if dtype == "f32" else 16
    sign = np.int64(1) << np.int64(width - 1)
    mag = sign - 1

    def key(x):
        return np.where(x & sign, -(x & mag), x & mag)

    d = np.abs(key(ba) - key(bb))
    na, nb = np.isnan(np.asarray(a, np.float32)), np.isnan(np.asarray(b, np.float32))
    d = np.where(na & nb, 0, d)
    d = np.where(na ^ nb, np.int64(1) << 40, d)
    return d


# ----------------------------------------------------------------- RMSNorm ---


def rms_norm_golden(x, w, eps: float, dtype: str) -> np.ndarray:
    """w * x * rsqrt(mean(x^2) + eps) over the last dim, fp64, one rounding.
    Formula: transformers models/qwen3/modeling_qwen3.py:59-64."""
    x64 = np.asarray(x, np.float64)
    r = 1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + eps)
    return round_to(np.asarray(w, np.float64) * (x64 * r), dtype)


def rms_norm_chain(x, w, eps: float, dtype: str) -> np.ndarray:
    """The HF formula rounded where the reference's aten chain rounds:
    h32 = x.to(f32); var = h32.pow(2).mean(-1); h = h32 * rsqrt(var + eps);
    out = w * h.to(dtype)   (modeling_qwen3.py:59-64 over pow.cu, mean.cu,
    add.cu, rsqrt.cu, mul.cu and the _to_copy casts of copy_ops.cc:225-240)."""
    h = np.asarray(x, np.float32)
    var = np.mean(h * h, axis=-1, keepdims=True, dtype=np.float32)
    r = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    y = round_to(h * r, dtype)
    return round_to(np.asarray(w, np.float32) * y, dtype)


def add_rms_norm_golden(x, y, w, eps: float, dtype: str):
    h = round_to(np.asarray(x, np.float64) + np.asarray(y, np.float64), dtype)
    return rms_norm_golden(h, w, eps, dtype), h


def add_rms_norm_chain(x, y, w, eps: float, dtype: str):
    h = round_to(np.asarray(x, np.float32) + np.asarray(y, np.float32), dtype)
    return rms_norm_chain(h, w, eps, dtype), h


# -------------------------------------------------------------------- RoPE ---


def _rotate_half(x):
    """cat(-x2, x1) over the last dim (modeling_qwen3.py:151-155)."""
    d = x.shape[-1] // 2
    return np.concatenate([-x[..., d:], x[..., :d]], axis=-1)


def rope_golden(x, cos, sin, dtype: str) -> np.ndarray:
    """x*cos + rotate_half(x)*sin in fp64, one rounding
    (apply_rotary_pos_emb, modeling_qwen3.py:158-181).  cos/sin broadcast
    against x."""
    x64 = np.asarray(x, np.float64)
    return round_to(x64 * np.asarray(cos, np.float64) + _rotate_half(x64) * np.asarray(sin, np.float64), dtype)


def rope_chain(x, cos, sin, dtype: str) -> np.ndarray:
    """Rounded after each aten op: mul, (neg, cat: exact), mul, add."""
    x = np.asarray(x, np.float32)
    t1 = round_to(x * np.asarray(cos, np.float32), dtype)
    t2 = round_to(_rotate_half(x) * np.asarray(sin, np.float32), dtype)
    return round_to(t1 + t2, dtype)


def rms_norm_rope_golden(x, w, cos, sin, eps: float, dtype: str) -> np.ndarray:
    """Qwen3 q_norm/k_norm over the head dim then RoPE (modeling_qwen3.py:
    248-249, 263-268), fp64 end to end, one rounding."""
    x64 = np.asarray(x, np.float64)
    r = 1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + eps)
    n = np.asarray(w, np.float64) * (x64 * r)
    return round_to(n * np.asarray(cos, np.float64) + _rotate_half(n) * np.asarray(sin, np.float64), dtype)


def rms_norm_rope_chain(x, w, cos, sin, eps: float, dtype: str) -> np.ndarray:
    return rope_chain(rms_norm_chain(x, w, eps, dtype), cos, sin, dtype)


def rope_tables(positions, dim: int, theta: float, dtype: str):
    """cos/sin tables as HF builds them (Qwen3RotaryEmbedding,
    modeling_qwen3.py:86-148): inv_freq = 1/theta^(arange(0,D,2)/D) in fp32,
    freqs = pos * inv_freq (fp32), emb = cat(freqs, freqs), cos/sin in fp32,
    then cast to the activation dtype.

    The fp32 steps run on torch CPU aten -- the kernels the reference's CPU
    path uses -- because the table is defined by them: numpy's float32 power
    and cos/sin differ from torch's in the last bit for some exponents and
    angles, and a last-bit difference in inv_freq times a position near
    131072 moves cos/sin by up to ~145 bf16 ulp.  The position product is an
    elementwise fp32 multiply, which is what HF's [D/2, 1] @ [1, S] matmul
    computes (one product per output, no sum)."""
    import torch

    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(torch.float32) / dim))
    pos = torch.as_tensor(np.asarray(positions, np.int64)).to(torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    c, s = emb.cos().numpy(), emb.sin().numpy()
    return round_to(c, dtype), round_to(s, dtype)


# ------------------------------------------------------------------ SwiGLU ---


def swiglu_golden(g, u, dtype: str) -> np.ndarray:
    g64 = np.asarray(g, np.float64)
    return round_to(g64 / (1.0 + np.exp(-g64)) * np.asarray(u, np.float64), dtype)


def swiglu_chain(g, u, dtype: str) -> np.ndarray:
    """silu (silu.cu:27-29: x / (1 + exp(-x)) in fp32) rounded, then mul."""
    g = np.asarray(g, np.float32)
    with np.errstate(over="ignore"):
        s = round_to(g / (np.float32(1.0) + np.exp(-g)), dtype)
    return round_to(s * np.asarray(u, np.float32), dtype)


# ------------------------------------------------------------- elementwise ---


def add_golden(a, b, alpha: float, dtype: str) -> np.ndarray:
    return round_to(np.asarray(a, np.float64) + alpha * np.asarray(b, np.float64), dtype)


def mul_golden(a, b, dtype: str) -> np.ndarray:
    return round_to(np.asarray(a, np.float64) * np.asarray(b, np.float64), dtype)


def add_int(a, b, alpha: int, bits: int) -> np.ndarray:
    """Integer add with two's-complement wrap in `bits` bits."""
    t = np.int32 if bits == 32 else np.int64
    with np.errstate(over="ignore"):
        return (np.asarray(a, t) + t(alpha) * np.asarray(b, t)).astype(t)


# ----------------------------------------------------------------- softmax ---


def causal_mask(rows_shape, cols: int, offset: int = 0) -> np.ndarray:
    """Boolean [q_len, cols] mask of visible keys: j <= i + offset."""
    q_len = rows_shape
    i = np.arange(q_len)[:, None]
    j = np.arange(cols)[None, :]
    return j <= i + offset


def softmax_golden(x, out_dtype: str, causal: bool = False, offset: int = 0) -> np.ndarray:
    """softmax over the last dim in fp64 (torch._softmax semantics: an all
    -inf row gives NaN).  causal: x is [..., q_len, cols], masked to
    j <= i + offset before the softmax."""
    x64 = np.asarray(x, np.float64).copy()
    if causal:
        m = causal_mask(x64.shape[-2], x64.shape[-1], offset)
        x64 = np.where(m, x64, -np.inf)
    with np.errstate(invalid="ignore"):
        mx = np.max(x64, axis=-1, keepdims=True)
        e = np.exp(x64 - mx)
        s = np.sum(e, axis=-1, keepdims=True)
        return round_to(e / s, out_dtype)


def masked_logits_chain(x, mask, scale: float, dtype: str) -> np.ndarray:
    """The logits HF's eager attention hands its softmax
    (transformers models/qwen3/modeling_qwen3.py eager_attention_forward):
    `attn_weights * scaling` (mul with a scalar, fp32 opmath, rounded to the
    dtype: csrc/aten/backends/cuda/mul.cu:28-52), then `+ attention_mask`
    (add.cu:48-84, rounded again).  mask None: the scale only."""
    t = round_to(np.asarray(x, np.float32) * np.float32(scale), dtype)
    if mask is not None:
        t = round_to(t + np.asarray(mask, np.float32), dtype)
    return t


def masked_softmax_chain(x, mask, scale: float, dtype: str, out_dtype: str) -> np.ndarray:
    """The whole tail op by op: the logits above, softmax(dtype=float32)
    (rounded to fp32) and `.to(query.dtype)` (rounded again to out_dtype)."""
    z = masked_logits_chain(x, mask, scale, dtype)
    return round_to(softmax_golden(z, "f32"), out_dtype)


def masked_softmax_golden(x, mask, scale: float, out_dtype: str) -> np.ndarray:
    """The fused formula: logits x * scale + mask rounded once to fp32 (one
    FMA; fp64 holds x * scale exactly, so this is the FMA's rounding up to a
    double-rounding tie), then the softmax in fp64
    with one rounding to out_dtype.  A row whose keys are all masked with the
    lowest finite value is uniform, as the reference's softmax makes it; with
    an f16 mask (-65504) the fp32 logits keep x * scale to 2^-8, so such a
    row is the softmax of those quantised logits."""
    z = np.asarray(x, np.float64) * float(np.float32(scale))
    if mask is not None:
        z = z + np.asarray(mask, np.float64)
    return softmax_golden(z.astype(np.float32), out_dtype)


def softmax_dim_golden(x, dim: int, out_dtype: str) -> np.ndarray:
    x64 = np.asarray(x, np.float64)
    mx = np.max(x64, axis=dim, keepdims=True)
    e = np.exp(x64 - mx)
    return round_to(e / np.sum(e, axis=dim, keepdims=True), out_dtype)


# -------------------------------------------------------------- reductions ---


def sum_golden(x, axis, out_dtype: str) -> np.ndarray:
    return round_to(np.sum(np.asarray(x, np.float64), axis=axis), out_dtype)


def mean_golden(x, axis, out_dtype: str) -> np.ndarray:
    return round_to(np.mean(np.asarray(x, np.float64), axis=axis), out_dtype)


def amax(x, axis) -> np.ndarray:
    """Exact max; NaN propagates (torch.amax)."""
    x = np.asarray(x, np.float32)
    return np.max(x, axis=axis)


def argmax_first(x, axis=-1) -> np.ndarray:
    """Index of the first maximum; the first NaN wins (torch.argmax)."""
    x = np.asarray(x, np.float32)
    return np.argmax(x, axis=axis).astype(np.int64)


def sum_i32_i64(x, axis=None) -> np.ndarray:
    return np.sum(np.asarray(x, np.int32).astype(np.int64), axis=axis)


# ---------------------------------------------------------------- helpers ---


def sum_abs(x, axis) -> np.ndarray:
    """sum(|x|): the scale fp32 summation error is measured against."""
    return np.sum(np.abs(np.asarray(x, np.float64)), axis=axis)


# --------------------------------------------------------------- backward ---
# The gradients of the fused formulas, fp64 math, one rounding.  They restate
# what torch autograd computes through the HF modules (the reference trains
# through those: pow/mean/rsqrt/mul backward for RMSNorm, silu_backward
# csrc/aten/backends/cuda/silu_backward.cu:15-35, softmax backward).


def rms_norm_bwd_golden(x, w, dy, eps: float, dtype: str):
    """(dx, dw) of out = w * x * r, r = 1/sqrt(mean(x^2) + eps) over the last
    dim: dx = r (w dy - n mean(w dy n)), n = x r; dw = sum over rows dy n."""
    x64 = np.asarray(x, np.float64)
    w64 = np.asarray(w, np.float64)
    g64 = np.asarray(dy, np.float64)
    r = 1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + eps)
    n = x64 * r
    m = np.mean(w64 * g64 * n, axis=-1, keepdims=True)
    dx = r * (w64 * g64 - n * m)
    dw = np.sum((g64 * n).reshape(-1, x64.shape[-1]), axis=0)
    return round_to(dx, dtype), round_to(dw, dtype)


def rms_norm_bwd_bound(x, w, dy, eps: float) -> np.ndarray:
    """Magnitude of the terms of dx, r (|w dy| + |n| mean(|w dy n|)): an fp32
    evaluation is within a few 2^-24 of this (the mean is a sum that can
    cancel, so its error scales with the sum of magnitudes), so tests scale
    their absolute tolerance by it."""
    x64 = np.asarray(x, np.float64)
    w64 = np.asarray(w, np.float64)
    g64 = np.asarray(dy, np.float64)
    r = 1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + eps)
    n = x64 * r
    m_abs = np.mean(np.abs(w64 * g64 * n), axis=-1, keepdims=True)
    return r * (np.abs(w64 * g64) + np.abs(n) * m_abs)


def _sigmoid64(g):
    return 1.0 / (1.0 + np.exp(-g))


def swiglu_bwd_golden(dout, g, u, dtype: str):
    """(dgate, dup) of silu(g) * u: dup = dout silu(g),
    dgate = dout u s (1 + g (1 - s)), s = sigmoid(g)."""
    d64 = np.asarray(dout, np.float64)
    g64 = np.asarray(g, np.float64)
    u64 = np.asarray(u, np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        s = _sigmoid64(g64)
        dg = d64 * u64 * s * (1.0 + g64 * (1.0 - s))
        du = d64 * g64 * s
    return round_to(dg, dtype), round_to(du, dtype)


def silu_bwd_golden(dout, x, dtype: str):
    """silu_backward: dout * s * (1 + x (1 - s)) (silu_backward.cu:27-31)."""
    d64 = np.asarray(dout, np.float64)
    x64 = np.asarray(x, np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        s = _sigmoid64(x64)
        return round_to(d64 * s * (1.0 + x64 * (1.0 - s)), dtype)


def softmax_bwd_golden(dy, y, dtype: str, scale: float = 1.0):
    """dx = scale y (dy - sum(dy y)) over the last dim (scale != 1: the
    gradient of softmax(x * scale + mask) with respect to x)."""
    g64 = np.asarray(dy, np.float64)
    y64 = np.asarray(y, np.float64)
    return round_to(float(scale) * y64 * (g64 - np.sum(g64 * y64, axis=-1, keepdims=True)),
                    dtype)


def softmax_bwd_bound(dy, y) -> np.ndarray:
    """Magnitude of the terms of the softmax gradient, |y| (|dy| + sum |dy y|)
    (the sum can cancel, so its error scales with the sum of magnitudes)."""
    g64 = np.asarray(dy, np.float64)
    y64 = np.asarray(y, np.float64)
    return np.abs(y64) * (np.abs(g64) + np.sum(np.abs(g64 * y64), axis=-1, keepdims=True))


def rope_bwd_golden(dq_out, cos, sin, dtype: str):
    """Gradient of x cos + rotate_half(x) sin w.r.t. x: dq_out cos +
    rotate_half^T(dq_out sin), rotate_half^T(v) = cat(v2, -v1)."""
    d64 = np.asarray(dq_out, np.float64)
    c64 = np.asarray(cos, np.float64)
    s64 = np.asarray(sin, np.float64)
    t = d64 * s64
    h = t.shape[-1] // 2
    rt = np.concatenate([t[..., h:], -t[..., :h]], axis=-1)
    return round_to(d64 * c64 + rt, dtype)
