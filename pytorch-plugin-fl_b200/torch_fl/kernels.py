"""Tensor-level entry points of the B200 kernels (libfl_b200.so through ctypes).

Each function validates its tensors, allocates the outputs with
``torch.empty_like``-style calls on the input's device, and launches on the
current CUDA stream of that device.  Tensors may live on ``cuda`` or on the
``flagos`` PrivateUse1 device (both are plain device memory of the same GPU).
There is no CPU path: a CPU tensor is an error.

The fused-op semantics follow the HF formulas the reference runs op by op:
``rms_norm`` (transformers models/qwen3/modeling_qwen3.py:59-64),
``rope_qk`` (modeling_qwen3.py:138-169), ``swiglu`` (modeling_qwen3.py:81-82).
"""

from __future__ import annotations

import torch

from . import _abi

_DT = {
    torch.float32: _abi.F32,
    torch.bfloat16: _abi.BF16,
    torch.float16: _abi.F16,
    torch.int32: _abi.I32,
    torch.int64: _abi.I64,
}
_ROUND = {"fused": _abi.ROUND_FUSED, "chain": _abi.ROUND_CHAIN}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"b200 kernels do not support dtype {t.dtype}") from None


def _device_index(t: torch.Tensor) -> int:
    if t.device.type == "cpu":
        raise RuntimeError("b200 kernels need device tensors, got a CPU tensor")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(_device_index(t)).cuda_stream


class _on_device:
    """Make the tensor's GPU current for the launch (kernels launch there)."""

    def __init__(self, t: torch.Tensor):
        self.idx = _device_index(t)
        self.prev = None

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.prev != self.idx:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None and self.prev != self.idx:
            torch.cuda.set_device(self.prev)
        return False


def _rows_view(x: torch.Tensor) -> tuple[int, int, int]:
    """(rows, cols, leading stride) of x viewed as [rows, cols] over its last
    dim; requires a unit last-dim stride and rows evenly spaced."""
    if x.dim() == 0:
        return 1, 1, 1
    cols = x.shape[-1]
    rows = 1
    for s in x.shape[:-1]:
        rows *= s
    if x.stride(-1) != 1 and cols > 1:
        raise ValueError("last dim must be contiguous")
    if x.dim() == 1 or rows <= 1:
        return rows, cols, max(cols, 1)
    ld = x.stride(-2)
    # all leading dims must collapse onto one stride
    expect = ld
    for d in range(x.dim() - 2, -1, -1):
        if x.shape[d] != 1 and x.stride(d) != expect:
            raise ValueError("leading dims do not collapse to one row stride")
        expect *= x.shape[d]
    return rows, cols, ld


def _rows_or_contig(x: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    try:
        r, c, ld = _rows_view(x)
        return x, r, c, ld
    except ValueError:
        x = x.contiguous()
        r, c, ld = _rows_view(x)
        return x, r, c, ld


# --------------------------------------------------------------------- RMSNorm
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, rounding: str = "fused",
             out: torch.Tensor | None = None) -> torch.Tensor:
    x, rows, cols, ld = _rows_or_contig(x)
    if weight.dtype != x.dtype or weight.numel() != cols or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [cols] tensor of x's dtype")
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _, _, ldo = _rows_view(out)
    with _on_device(x):
        _abi.call("fl_b200_rms_norm_fwd", x.data_ptr(), ld, weight.data_ptr(), out.data_ptr(),
                  ldo, rows, cols, float(eps), dtype_code(x), _ROUND[rounding], _stream(x))
    return out


def add_rms_norm(x: torch.Tensor, y: torch.Tensor, weight: torch.Tensor, eps: float,
                 rounding: str = "fused", h_out: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """h = x + y; returns (rmsnorm(h) * weight, h).  Dense tensors only."""
    if x.shape != y.shape or x.dtype != y.dtype:
        raise ValueError("x and y must match")
    x = x.contiguous()
    y = y.contiguous()
    cols = x.shape[-1]
    rows = x.numel() // cols
    h = torch.empty_like(x) if h_out is None else h_out
    o = torch.empty_like(x) if out is None else out
    with _on_device(x):
        _abi.call("fl_b200_add_rms_norm_fwd", x.data_ptr(), y.data_ptr(), h.data_ptr(),
                  weight.data_ptr(), o.data_ptr(), rows, cols, float(eps), dtype_code(x),
                  _ROUND[rounding], _stream(x))
    return o, h


# ------------------------------------------------------------------------ RoPE
def _bhsd(t: torch.Tensor, layout: str) -> tuple[int, int, int, int, tuple[int, int, int]]:
    """Sizes (B, H, S, D) and strides over (b, h, s) for a q/k tensor."""
    if t.stride(-1) != 1:
        raise ValueError("head dim must be contiguous")
    if layout == "bhsd":
        B, H, S, D = t.shape
        return B, H, S, D, (t.stride(0), t.stride(1), t.stride(2))
    if layout == "bshd":
        B, S, H, D = t.shape
        return B, H, S, D, (t.stride(0), t.stride(2), t.stride(1))
    raise ValueError(layout)


def _cos_strides(cos: torch.Tensor, B: int, S: int, D: int) -> tuple[int, int]:
    """Strides (b, s) of a cos/sin table given as [S, D], [B, S, D] or
    [B, 1, S, D] (HF unsqueezes dim 1)."""
    if cos.stride(-1) != 1:
        raise ValueError("cos/sin last dim must be contiguous")
    if cos.dim() == 4:
        cos = cos.squeeze(1)
    if cos.dim() == 2:
        if tuple(cos.shape) != (S, D):
            raise ValueError("cos/sin shape mismatch")
        return 0, cos.stride(0)
    if cos.dim() == 3:
        if cos.shape[1] != S or cos.shape[2] != D or cos.shape[0] not in (1, B):
            raise ValueError("cos/sin shape mismatch")
        return (cos.stride(0) if cos.shape[0] == B and B > 1 else 0), cos.stride(1)
    raise ValueError("cos/sin must be 2-D, 3-D or 4-D")


def rope_qk(q: torch.Tensor, k: torch.Tensor | None, cos: torch.Tensor, sin: torch.Tensor,
            layout: str = "bhsd", rounding: str = "fused", inplace: bool = False,
            q_weight: torch.Tensor | None = None, k_weight: torch.Tensor | None = None,
            eps: float = 1e-6, q_out: torch.Tensor | None = None,
            k_out: torch.Tensor | None = None):
    """q_embed, k_embed = apply_rotary_pos_emb(q, k, cos, sin); with q_weight /
    k_weight given, Qwen3's per-head RMSNorm is applied first (fused).
    Outputs go to q_out / k_out when given (same shape and layout as q / k)."""
    B, Hq, S, D, sq = _bhsd(q, layout)
    qo = q if inplace else (q_out if q_out is not None else torch.empty_like(q))
    _, _, _, _, soq = _bhsd(qo, layout)
    if k is not None:
        Bk, Hk, Sk, Dk, sk = _bhsd(k, layout)
        if (Bk, Sk, Dk) != (B, S, D) or k.dtype != q.dtype:
            raise ValueError("q and k disagree")
        ko = k if inplace else (k_out if k_out is not None else torch.empty_like(k))
        _, _, _, _, sok = _bhsd(ko, layout)
        kp, kop = k.data_ptr(), ko.data_ptr()
    else:
        Hk, sk, sok, ko, kp, kop = 0, (0, 0, 0), (0, 0, 0), None, None, None
    if cos.dtype != q.dtype or sin.dtype != q.dtype:
        raise ValueError("cos/sin dtype must match q")
    scb, scs = _cos_strides(cos, B, S, D)
    if _cos_strides(sin, B, S, D) != (scb, scs):
        raise ValueError("cos and sin must share a layout")
    with _on_device(q):
        if q_weight is None:
            _abi.call("fl_b200_rope_qk", q.data_ptr(), qo.data_ptr(), Hq, *sq, *soq,
                      kp, kop, Hk, *sk, *sok, cos.data_ptr(), sin.data_ptr(), scb, scs,
                      B, S, D, dtype_code(q), _ROUND[rounding], _stream(q))
        else:
            wk = k_weight.data_ptr() if (k is not None and k_weight is not None) else None
            _abi.call("fl_b200_rms_norm_rope", q.data_ptr(), qo.data_ptr(), Hq, *sq, *soq,
                      q_weight.data_ptr(), kp, kop, Hk, *sk, *sok, wk, cos.data_ptr(),
                      sin.data_ptr(), scb, scs, B, S, D, float(eps), dtype_code(q),
                      _ROUND[rounding], _stream(q))
    return qo, ko


# ---------------------------------------------------------------------- SwiGLU
def swiglu(gate: torch.Tensor, up: torch.Tensor, rounding: str = "fused",
           out: torch.Tensor | None = None) -> torch.Tensor:
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError("gate and up must match")
    gate, rows, cols, ldg = _rows_or_contig(gate)
    up, _, _, ldu = _rows_or_contig(up)
    if out is None:
        out = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    _, _, ldo = _rows_view(out)
    with _on_device(gate):
        _abi.call("fl_b200_swiglu", gate.data_ptr(), ldg, up.data_ptr(), ldu, out.data_ptr(),
                  ldo, rows, cols, dtype_code(gate), _ROUND[rounding], _stream(gate))
    return out


def swiglu_residual(gate, up, x, y, rounding: str = "fused", act_out=None, h_out=None):
    """(silu(gate) * up, x + y) in one launch.  Dense, 16-byte aligned tensors."""
    rows = gate.shape[0]
    act = torch.empty_like(gate) if act_out is None else act_out
    h = torch.empty_like(x) if h_out is None else h_out
    with _on_device(gate):
        _abi.call("fl_b200_swiglu_residual", gate.data_ptr(), up.data_ptr(), act.data_ptr(),
                  gate.numel() // rows, x.data_ptr(), y.data_ptr(), h.data_ptr(),
                  x.numel() // rows, rows, dtype_code(gate), _ROUND[rounding], _stream(gate))
    return act, h


# ---------------------------------------------------------------- elementwise
def _broadcast(a: torch.Tensor, b: torch.Tensor):
    shape = torch.broadcast_shapes(a.shape, b.shape)
    ea, eb = a.expand(shape), b.expand(shape)
    if len(shape) > 8:
        raise ValueError("at most 8 dims")
    return shape, ea.stride(), eb.stride()


def _binary_out(out, shape, a):
    if out is None:
        return torch.empty(shape, dtype=a.dtype, device=a.device)
    if tuple(out.shape) != tuple(shape) or out.dtype != a.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor of the broadcast shape and dtype")
    return out


def add(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0,
        out: torch.Tensor | None = None) -> torch.Tensor:
    if a.dtype != b.dtype:
        raise TypeError("add: operands must share a dtype (promote first)")
    shape, sa, sb = _broadcast(a, b)
    out = _binary_out(out, shape, a)
    with _on_device(a):
        _abi.call("fl_b200_add", a.data_ptr(), _abi.i64_array(sa), b.data_ptr(),
                  _abi.i64_array(sb), out.data_ptr(), _abi.i64_array(shape), len(shape),
                  float(alpha), dtype_code(a), _stream(a))
    return out


def mul(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if a.dtype != b.dtype:
        raise TypeError("mul: operands must share a dtype (promote first)")
    shape, sa, sb = _broadcast(a, b)
    out = _binary_out(out, shape, a)
    with _on_device(a):
        _abi.call("fl_b200_mul", a.data_ptr(), _abi.i64_array(sa), b.data_ptr(),
                  _abi.i64_array(sb), out.data_ptr(), _abi.i64_array(shape), len(shape),
                  dtype_code(a), _stream(a))
    return out


def binary_scalar(a: torch.Tensor, s: float, op: str, alpha: float = 1.0) -> torch.Tensor:
    a = a.contiguous()
    out = torch.empty_like(a)
    with _on_device(a):
        _abi.call("fl_b200_binary_scalar", a.data_ptr(), float(s), out.data_ptr(), a.numel(),
                  {"add": 0, "mul": 1}[op], float(alpha), dtype_code(a), _stream(a))
    return out


def cast(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    with _on_device(x):
        _abi.call("fl_b200_cast", x.data_ptr(), dtype_code(x), out.data_ptr(),
                  _DT[dtype], x.numel(), _stream(x))
    return out


# --------------------------------------------------------------------- softmax
def softmax(x: torch.Tensor, dim: int = -1, out_dtype: torch.dtype | None = None,
            causal: bool = False, causal_offset: int = 0) -> torch.Tensor:
    """softmax over `dim` in fp32; out_dtype None = x.dtype (or float32 for
    half_to_float).  causal applies the mask of query row i (the second-last
    dim) over keys j <= i + causal_offset in the kernel."""
    out_dtype = out_dtype or x.dtype
    dim = dim % max(x.dim(), 1)
    if x.dim() == 0:
        return torch.ones((), dtype=out_dtype, device=x.device)
    if dim != x.dim() - 1:
        if causal:
            raise ValueError("causal softmax is over the last dim")
        xc = x.contiguous()
        outer = 1
        for s in x.shape[:dim]:
            outer *= s
        inner = 1
        for s in x.shape[dim + 1:]:
            inner *= s
        out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
        with _on_device(x):
            _abi.call("fl_b200_softmax_middim", xc.data_ptr(), out.data_ptr(), outer,
                      x.shape[dim], inner, dtype_code(x), _DT[out_dtype], _stream(x))
        return out
    x, rows, cols, ld = _rows_or_contig(x)
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    q_len = x.shape[-2] if x.dim() >= 2 else 1
    with _on_device(x):
        _abi.call("fl_b200_softmax_lastdim", x.data_ptr(), ld, out.data_ptr(), cols, rows,
                  cols, dtype_code(x), _DT[out_dtype], int(causal), q_len,
                  int(causal_offset), _stream(x))
    return out


def _as_bhqk(x: torch.Tensor) -> torch.Tensor:
    if not 2 <= x.dim() <= 4:
        raise ValueError("x must be [Q, K], [H, Q, K] or [B, H, Q, K]")
    while x.dim() < 4:
        x = x.unsqueeze(0)
    return x


def masked_softmax(x: torch.Tensor, mask: torch.Tensor | None = None, scale: float = 1.0,
                   out_dtype: torch.dtype | None = None, rounding: str = "fused") -> torch.Tensor:
    """softmax(x * scale + mask) over the last dim, HF eager attention's tail
    (modeling_qwen3.py eager_attention_forward: scale, mask add,
    softmax(dtype=float32), cast back) in one launch.  x is [B, H, Q, K] (or
    fewer leading dims); mask has x's dtype and broadcasts to x; out_dtype
    None = x.dtype (the cast back fused), or float32."""
    out_dtype = out_dtype or x.dtype
    x4 = _as_bhqk(x)
    B, H, Q, K = x4.shape
    x4, rows, cols, ld = _rows_or_contig(x4)
    mp, sb, sh, sq = 0, 0, 0, 0
    if mask is not None:
        if mask.dtype != x.dtype:
            raise TypeError("mask must have x's dtype")
        m = mask.expand(x4.shape)
        if K > 1 and m.stride(3) != 1:
            m = m.contiguous()
        mask = m
        mp, sb, sh, sq = m.data_ptr(), m.stride(0), m.stride(1), m.stride(2)
    out = torch.empty(x4.shape, dtype=out_dtype, device=x.device)
    if out.numel():
        with _on_device(x):
            _abi.call("fl_b200_softmax_masked", x4.data_ptr(), ld, mp, sb, sh, sq,
                      out.data_ptr(), cols, rows, cols, H, Q, float(scale), dtype_code(x),
                      _DT[out_dtype], _ROUND[rounding], _stream(x))
    return out.view(x.shape)


# --------------------------------------------- the other HF formula ops
_UNARY = {"silu": _abi.UNARY_SILU, "rsqrt": _abi.UNARY_RSQRT, "neg": _abi.UNARY_NEG,
          "cos": _abi.UNARY_COS, "sin": _abi.UNARY_SIN}


def _outer(x: torch.Tensor, split: int):
    """(sizes, strides) of x's dims before `split` when its dims from `split`
    on are contiguous, else None."""
    expect = 1
    for d in range(x.dim() - 1, split - 1, -1):
        if x.size(d) != 1 and x.stride(d) != expect:
            return None
        expect *= x.size(d)
    return list(x.shape[:split]), list(x.stride()[:split])


def unary(x: torch.Tensor, op: str, exponent: float = 0.0) -> torch.Tensor:
    """silu / rsqrt / neg / cos / sin of x, or pow(x, exponent) (op "pow";
    the exponent rounded to x's dtype first, 2 and 3 as products, as the
    reference's cuda route computes them) through fl_b200_unary.  x's rows of
    the last dim may be strided (any outer dims); the result is dense."""
    if op == "pow":
        e = float(torch.tensor(exponent, dtype=x.dtype)) if x.is_floating_point() else exponent
        code = _abi.UNARY_SQUARE if e == 2.0 else (_abi.UNARY_CUBE if e == 3.0 else _abi.UNARY_POW)
    else:
        e, code = 0.0, _UNARY[op]
    view = _outer(x, x.dim() - 1) if x.dim() else ([], [])
    if view is None:
        x = x.contiguous()
        view = _outer(x, x.dim() - 1)
    sizes, strides = view
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if out.numel():
        with _on_device(x):
            _abi.call("fl_b200_unary", x.data_ptr(), _abi.i64_array(sizes),
                      _abi.i64_array(strides), len(sizes), x.shape[-1] if x.dim() else 1,
                      out.data_ptr(), code, float(e), dtype_code(x), _stream(x))
    return out


def cat(tensors, dim: int = 0) -> torch.Tensor:
    """torch.cat(tensors, dim) for tensors of one dtype through fl_b200_cat
    (row blocks; each input's dims from `dim` on contiguous, any outer
    strides)."""
    t0 = tensors[0]
    d = dim % t0.dim()
    shape = list(t0.shape)
    shape[d] = sum(t.shape[d] for t in tensors)
    out = torch.empty(shape, dtype=t0.dtype, device=t0.device)
    srcs, strides, widths, keep = [], [], [], []
    for t in tensors:
        v = _outer(t, d)
        if v is None:
            t = t.contiguous()
            keep.append(t)
            v = _outer(t, d)
        srcs.append(t.data_ptr())
        strides += v[1]
        widths.append(int(torch.tensor(t.shape[d:]).prod()) if d < t.dim() else 1)
    if out.numel():
        import ctypes as C
        arr = (C.c_void_p * len(srcs))(*srcs)
        with _on_device(t0):
            _abi.call("fl_b200_cat", arr, _abi.i64_array(strides), _abi.i64_array(widths),
                      len(srcs), _abi.i64_array(shape[:d]), d, out.data_ptr(),
                      t0.element_size(), _stream(t0))
    return out


# ------------------------------------------------------------------ reductions
def _workspace(rows: int, cols: int, device) -> torch.Tensor | None:
    n = _abi.lib().fl_b200_reduce_workspace_size(rows, cols)
    if n == 0:
        return None
    return torch.empty(n, dtype=torch.uint8, device=device)


def _reduce_lastdim(name: str, x: torch.Tensor, out_dtype: torch.dtype, keepdim: bool,
                    with_out_dtype: bool = True) -> torch.Tensor:
    x, rows, cols, ld = _rows_or_contig(x)
    shape = list(x.shape[:-1]) + ([1] if keepdim else [])
    out = torch.empty(shape, dtype=out_dtype, device=x.device)
    ws = _workspace(rows, cols, x.device)
    wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    with _on_device(x):
        if with_out_dtype:
            _abi.call(name, x.data_ptr(), ld, rows, cols, out.data_ptr(), dtype_code(x),
                      _DT[out_dtype], wsp, wsn, _stream(x))
        else:
            _abi.call(name, x.data_ptr(), ld, rows, cols, out.data_ptr(), dtype_code(x),
                      wsp, wsn, _stream(x))
    return out


def _reduce_all(name: str, x: torch.Tensor, out_dtype: torch.dtype,
                with_out_dtype: bool = True) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty((), dtype=out_dtype, device=x.device)
    ws = _workspace(1, x.numel(), x.device)
    wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    with _on_device(x):
        if with_out_dtype:
            _abi.call(name, x.data_ptr(), x.numel(), out.data_ptr(), dtype_code(x),
                      _DT[out_dtype], wsp, wsn, _stream(x))
        else:
            _abi.call(name, x.data_ptr(), x.numel(), out.data_ptr(), dtype_code(x), wsp, wsn,
                      _stream(x))
    return out


def _sum_dtype(x: torch.Tensor, dtype) -> torch.dtype:
    if dtype is not None:
        return dtype
    return torch.int64 if x.dtype in (torch.int32, torch.int64) else x.dtype


def sum_lastdim(x, keepdim=False, dtype=None):
    return _reduce_lastdim("fl_b200_reduce_sum_lastdim", x, _sum_dtype(x, dtype), keepdim)


def mean_lastdim(x, keepdim=False, dtype=None):
    return _reduce_lastdim("fl_b200_reduce_mean_lastdim", x, dtype or x.dtype, keepdim)


def amax_lastdim(x, keepdim=False):
    return _reduce_lastdim("fl_b200_reduce_amax_lastdim", x, x.dtype, keepdim,
                           with_out_dtype=False)


def sum_all(x, dtype=None):
    return _reduce_all("fl_b200_reduce_sum_all", x, _sum_dtype(x, dtype))


def mean_all(x, dtype=None):
    return _reduce_all("fl_b200_reduce_mean_all", x, dtype or x.dtype)


def amax_all(x):
    return _reduce_all("fl_b200_reduce_amax_all", x, x.dtype, with_out_dtype=False)


def reduce_middim(x: torch.Tensor, dim: int, op: str, keepdim=False, dtype=None):
    x = x.contiguous()
    dim = dim % x.dim()
    outer = 1
    for s in x.shape[:dim]:
        outer *= s
    inner = 1
    for s in x.shape[dim + 1:]:
        inner *= s
    shape = list(x.shape)
    if keepdim:
        shape[dim] = 1
    else:
        shape.pop(dim)
    out_dtype = dtype or x.dtype
    out = torch.empty(shape, dtype=out_dtype, device=x.device)
    with _on_device(x):
        _abi.call("fl_b200_reduce_middim", x.data_ptr(), outer, x.shape[dim], inner,
                  out.data_ptr(), {"sum": 0, "mean": 1, "amax": 2}[op], dtype_code(x),
                  _DT[out_dtype], _stream(x))
    return out


def argmax_lastdim(x: torch.Tensor, keepdim: bool = False) -> torch.Tensor:
    x, rows, cols, ld = _rows_or_contig(x)
    shape = list(x.shape[:-1]) + ([1] if keepdim else [])
    out = torch.empty(shape, dtype=torch.int64, device=x.device)
    ws = _workspace(rows, cols, x.device)
    wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    with _on_device(x):
        _abi.call("fl_b200_argmax_lastdim", x.data_ptr(), ld, rows, cols, out.data_ptr(),
                  dtype_code(x), wsp, wsn, _stream(x))
    return out


def sum_i32_i64(x: torch.Tensor, full: bool) -> torch.Tensor:
    if x.dtype != torch.int32:
        raise TypeError("sum_i32_i64 takes int32")
    x, rows, cols, ld = _rows_or_contig(x)
    if full:
        x = x.contiguous()
        rows, cols, ld = 1, x.numel(), x.numel()
    out = torch.empty(() if full else x.shape[:-1], dtype=torch.int64, device=x.device)
    ws = _workspace(rows, cols, x.device)
    wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    with _on_device(x):
        _abi.call("fl_b200_sum_i32_i64", x.data_ptr(), ld, rows, cols, out.data_ptr(),
                  int(full), wsp, wsn, _stream(x))
    return out


# -------------------------------------------------------------------- backward
def rms_norm_backward(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, eps: float,
                      need_dw: bool = True) -> tuple[torch.Tensor, torch.Tensor | None]:
    """(dx, dw) of out = weight * x * rsqrt(mean(x^2) + eps) over the last dim;
    dw is None when not need_dw.  fp32 math, deterministic dw."""
    if dy.shape != x.shape or dy.dtype != x.dtype:
        raise ValueError("dy and x must match")
    x, rows, cols, ldx = _rows_or_contig(x)
    dy, _, _, lddy = _rows_or_contig(dy)
    if weight.dtype != x.dtype or weight.numel() != cols or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [cols] tensor of x's dtype")
    dx = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _, _, lddx = _rows_view(dx)
    dw = torch.empty(cols, dtype=x.dtype, device=x.device) if need_dw else None
    with _on_device(x):
        ws, nws = None, 0
        if need_dw:
            nws = _abi.lib().fl_b200_rms_norm_bwd_workspace_size(rows, cols)
            ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=x.device) if nws else None
        _abi.call("fl_b200_rms_norm_bwd", dy.data_ptr(), lddy, x.data_ptr(), ldx,
                  weight.data_ptr(), dx.data_ptr(), lddx, dw.data_ptr() if need_dw else None,
                  rows, cols, float(eps), dtype_code(x), ws.data_ptr() if ws is not None else None,
                  nws, _stream(x))
    return dx, dw


def swiglu_backward(dout: torch.Tensor, gate: torch.Tensor,
                    up: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(dgate, dup) of out = silu(gate) * up."""
    if not (dout.shape == gate.shape == up.shape) or not (dout.dtype == gate.dtype == up.dtype):
        raise ValueError("dout, gate and up must match")
    dout, gate, up = dout.contiguous(), gate.contiguous(), up.contiguous()
    dg, du = torch.empty_like(gate), torch.empty_like(up)
    with _on_device(gate):
        _abi.call("fl_b200_swiglu_bwd", dout.data_ptr(), gate.data_ptr(), up.data_ptr(),
                  dg.data_ptr(), du.data_ptr(), gate.numel(), dtype_code(gate), _stream(gate))
    return dg, du


def silu_backward(dout: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """d silu(x) = dout * s * (1 + x (1 - s)), s = sigmoid(x)."""
    if dout.shape != x.shape or dout.dtype != x.dtype:
        raise ValueError("dout and x must match")
    dout, x = dout.contiguous(), x.contiguous()
    dx = torch.empty_like(x)
    with _on_device(x):
        _abi.call("fl_b200_silu_bwd", dout.data_ptr(), x.data_ptr(), dx.data_ptr(), x.numel(),
                  dtype_code(x), _stream(x))
    return dx


def softmax_backward(dy: torch.Tensor, y: torch.Tensor,
                     out_dtype: torch.dtype | None = None, scale: float = 1.0) -> torch.Tensor:
    """dx = scale * y * (dy - sum(dy * y)) over the last dim; out_dtype
    defaults to y's dtype (a 16-bit dtype with fp32 dy/y: half_to_float's
    backward).  scale != 1 is the backward of masked_softmax."""
    if dy.shape != y.shape or dy.dtype != y.dtype:
        raise ValueError("dy and y must match")
    out_dtype = out_dtype or y.dtype
    if y.dim() == 0:
        return torch.zeros((), dtype=out_dtype, device=y.device)
    y, rows, cols, ldy = _rows_or_contig(y)
    dy, _, _, lddy = _rows_or_contig(dy)
    dx = torch.empty(y.shape, dtype=out_dtype, device=y.device)
    with _on_device(y):
        _abi.call("fl_b200_softmax_bwd_scaled", dy.data_ptr(), lddy, y.data_ptr(), ldy,
                  dx.data_ptr(), cols, rows, cols, float(scale), dtype_code(y), _DT[out_dtype],
                  _stream(y))
    return dx
