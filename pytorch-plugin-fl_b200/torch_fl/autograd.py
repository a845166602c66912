"""Autograd formulas of the flagos:: fused ops, so training runs through them.

Each formula calls the backward kernels (flagos::rms_norm_backward,
swiglu_backward, softmax_backward; RoPE needs none, see below).  The
gradients are the fused formulas in fp32 with one rounding, whatever
rounding the forward used.

* rms_norm(x, w):   dx, dw = rms_norm_backward(dy, x, w, eps)
* add_rms_norm(x, res, w) -> (out, h = x + res):
                    d(x) = d(res) = rms_norm_backward(d_out, h, w)[0] + d_h
* rope_qk(q, k, cos, sin): the rotation is orthogonal and, with cos/sin
  built as cat(freqs, freqs) (the HF construction, modeling_qwen3.py:
  96-116), its adjoint is the same rotation with -sin:
                    dq, dk = rope_qk(dq_out, dk_out, cos, -sin)
  cos and sin get no gradient (HF computes them without one).
* rms_norm_rope: the RoPE adjoint, then rms_norm_backward over the head dim.
* swiglu(g, u):     dg, du = swiglu_backward(d_act, g, u)
* swiglu_residual(g, u, x, y) -> (act, h = x + y): the SwiGLU part as above,
                    d(x) = d(y) = d_h
* causal_softmax(x): dx = softmax_backward(dy, y, x.dtype) (masked keys have
  y = 0, so their gradient is 0)
* masked_softmax(x, mask, scale): dx = softmax_backward(dy, y, x.dtype, scale);
  a mask that needs a gradient gets the unscaled product summed over the
  dims it broadcasts (HF's mask needs none)
"""

from __future__ import annotations

import torch

_F = torch.ops.flagos


def _meta(t):
    return (t.shape, t.dtype, t.device)


def _or_zeros(g, meta):
    """g, or zeros of the recorded shape when that output got no gradient."""
    if g is not None:
        return g
    shape, dtype, device = meta
    return torch.zeros(shape, dtype=dtype, device=device)


# ---------------------------------------------------------------- RMSNorm
def _rms_setup(ctx, inputs, output):
    x, weight, eps, _ = inputs
    ctx.save_for_backward(x, weight)
    ctx.eps = eps


def _rms_backward(ctx, dy):
    x, w = ctx.saved_tensors
    dx, dw = _F.rms_norm_backward(dy, x, w, ctx.eps)
    return (dx if ctx.needs_input_grad[0] else None,
            dw if ctx.needs_input_grad[1] else None, None, None)


def _add_rms_setup(ctx, inputs, output):
    _, _, weight, eps, _ = inputs
    ctx.save_for_backward(output[1], weight)
    ctx.eps = eps


def _add_rms_backward(ctx, d_out, d_h):
    h, w = ctx.saved_tensors
    dsum, dw = _F.rms_norm_backward(_or_zeros(d_out, _meta(h)), h, w, ctx.eps)
    if d_h is not None:
        dsum = dsum + d_h
    return (dsum if ctx.needs_input_grad[0] else None,
            dsum if ctx.needs_input_grad[1] else None,
            dw if ctx.needs_input_grad[2] else None, None, None)


# ------------------------------------------------------------------- RoPE
def _rope_setup(ctx, inputs, output):
    q, k, cos, sin, unsqueeze_dim, _ = inputs
    ctx.save_for_backward(cos, sin)
    ctx.unsqueeze_dim = unsqueeze_dim
    ctx.metas = (_meta(output[0]), _meta(output[1]))


def _rope_backward(ctx, dqo, dko):
    cos, sin = ctx.saved_tensors
    mq, mk = ctx.metas
    dq, dk = _F.rope_qk(_or_zeros(dqo, mq), _or_zeros(dko, mk), cos, -sin, ctx.unsqueeze_dim,
                        "fused")
    return (dq if ctx.needs_input_grad[0] else None,
            dk if ctx.needs_input_grad[1] else None, None, None, None, None)


def _rms_rope_setup(ctx, inputs, output):
    q, k, qw, kw, cos, sin, eps, unsqueeze_dim, _ = inputs
    ctx.save_for_backward(q, k, qw, kw, cos, sin)
    ctx.eps = eps
    ctx.unsqueeze_dim = unsqueeze_dim


def _rms_rope_backward(ctx, dqo, dko):
    q, k, qw, kw, cos, sin = ctx.saved_tensors
    dqn, dkn = _F.rope_qk(_or_zeros(dqo, _meta(q)), _or_zeros(dko, _meta(k)), cos, -sin,
                          ctx.unsqueeze_dim, "fused")
    dq, dqw = _F.rms_norm_backward(dqn, q, qw, ctx.eps)
    dk, dkw = _F.rms_norm_backward(dkn, k, kw, ctx.eps)
    g = ctx.needs_input_grad
    return (dq if g[0] else None, dk if g[1] else None, dqw if g[2] else None,
            dkw if g[3] else None, None, None, None, None, None)


# ----------------------------------------------------------------- SwiGLU
def _swiglu_setup(ctx, inputs, output):
    gate, up, _ = inputs
    ctx.save_for_backward(gate, up)


def _swiglu_backward(ctx, dact):
    gate, up = ctx.saved_tensors
    dg, du = _F.swiglu_backward(dact, gate, up)
    return (dg if ctx.needs_input_grad[0] else None,
            du if ctx.needs_input_grad[1] else None, None)


def _swiglu_res_setup(ctx, inputs, output):
    gate, up, x, _, _ = inputs
    ctx.save_for_backward(gate, up)
    ctx.x_meta = _meta(x)


def _swiglu_res_backward(ctx, dact, dh):
    gate, up = ctx.saved_tensors
    dg = du = None
    if dact is not None:
        dg, du = _F.swiglu_backward(dact, gate, up)
    dxy = _or_zeros(dh, ctx.x_meta)
    g = ctx.needs_input_grad
    return (dg if g[0] else None, du if g[1] else None, dxy if g[2] else None,
            dxy if g[3] else None, None)


# ---------------------------------------------------------------- softmax
def _softmax_setup(ctx, inputs, output):
    x, _, _ = inputs
    ctx.save_for_backward(output)
    ctx.in_dtype = x.dtype


def _softmax_backward(ctx, dy):
    (y,) = ctx.saved_tensors
    dx = _F.softmax_backward(dy, y, ctx.in_dtype)
    return dx if ctx.needs_input_grad[0] else None, None, None


def _masked_softmax_setup(ctx, inputs, output):
    x, mask, scale, _, _ = inputs
    ctx.save_for_backward(output)
    ctx.in_dtype = x.dtype
    ctx.scale = scale
    ctx.mask_meta = None if mask is None else (mask.shape, mask.dtype)


def _masked_softmax_backward(ctx, dy):
    (y,) = ctx.saved_tensors
    dx = dmask = None
    if ctx.needs_input_grad[0]:
        dx = _F.softmax_backward(dy, y, ctx.in_dtype, ctx.scale)
    if ctx.mask_meta is not None and ctx.needs_input_grad[1]:
        shape, dtype = ctx.mask_meta
        dmask = _F.softmax_backward(dy, y, None, 1.0).sum_to_size(shape).to(dtype)
    return dx, dmask, None, None, None


def register() -> None:
    """Attach the formulas to the flagos:: ops (once per process)."""
    reg = torch.library.register_autograd
    reg("flagos::rms_norm", _rms_backward, setup_context=_rms_setup)
    reg("flagos::add_rms_norm", _add_rms_backward, setup_context=_add_rms_setup)
    reg("flagos::rope_qk", _rope_backward, setup_context=_rope_setup)
    reg("flagos::rms_norm_rope", _rms_rope_backward, setup_context=_rms_rope_setup)
    reg("flagos::swiglu", _swiglu_backward, setup_context=_swiglu_setup)
    reg("flagos::swiglu_residual", _swiglu_res_backward, setup_context=_swiglu_res_setup)
    reg("flagos::causal_softmax", _softmax_backward, setup_context=_softmax_setup)
    reg("flagos::masked_softmax", _masked_softmax_backward, setup_context=_masked_softmax_setup)
