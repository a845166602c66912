"""Parity of the backward kernels (RMSNorm, SwiGLU, SiLU, softmax) with the
oracle's fp64 gradients, and of autograd through the flagos:: fused ops.

Tolerances (tests/parity.py): fp32 evaluation error within BWD_TERM_TOL times
the magnitude of the formula's terms (the terms of dx = r (w dy - n m) and
dx = y (dy - sum dy y) can cancel), plus 1 ulp of the output for 16-bit
dtypes; dw (a sum over rows) within 1e-5 of the sum of |dy n|.
"""

import numpy as np
import pytest
import torch

import torch_fl  # noqa: F401  (registers the flagos:: ops and their autograd)
from oracle import ops
from tests import parity
from torch_fl import kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def rnd(shape, dtype, seed, scale=1.0, loc=0.0, device=DEV):
    g = torch.Generator().manual_seed(seed)
    return (loc + scale * torch.randn(*shape, generator=g)).to(dtype).to(device)


def _none16(dt):
    return dt if dt in ("bf16", "f16") else None


# ------------------------------------------------------------------ RMSNorm
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 8), (3, 7), (5, 96), (127, 4096), (16, 8192),
                                   (33, 1000), (2, 65536 + 8), (4096, 512), (3, 2, 256), (4, 16384)])
def test_rms_norm_backward(dtype, shape):
    x = rnd(shape, dtype, 60)
    w = rnd(shape[-1:], dtype, 61, scale=0.1, loc=1.0)
    dy = rnd(shape, dtype, 62)
    dx, dw = K.rms_norm_backward(dy, x, w, 1e-6)
    dt = parity.dname(dtype)
    xn, wn, gn = parity.to_np(x), parity.to_np(w), parity.to_np(dy)
    rdx, rdw = ops.rms_norm_bwd_golden(xn, wn, gn, 1e-6, dt)
    bound = ops.rms_norm_bwd_bound(xn, wn, gn, 1e-6)
    parity.assert_within(parity.to_np(dx), rdx, parity.BWD_TERM_TOL * bound, f"dx {shape}",
                         _none16(dt))
    r = 1.0 / np.sqrt(np.mean(xn.astype(np.float64) ** 2, -1, keepdims=True) + 1e-6)
    terms = np.sum(np.abs(gn * xn * r).reshape(-1, shape[-1]), axis=0)
    parity.assert_within(parity.to_np(dw), rdw, 1e-5 * terms, f"dw {shape}", _none16(dt))


def test_rms_norm_backward_strided_no_dw_and_deterministic():
    base = rnd((64, 4096 + 64), torch.bfloat16, 63)
    x = base[:, :4096]                                  # leading stride 4160
    w = rnd((4096,), torch.bfloat16, 64, scale=0.1, loc=1.0)
    dy = rnd((64, 4096), torch.bfloat16, 65)
    dx1, dw1 = K.rms_norm_backward(dy, x, w, 1e-5)
    dx2, dw2 = K.rms_norm_backward(dy, x.contiguous(), w, 1e-5)
    assert torch.equal(dx1, dx2) and torch.equal(dw1, dw2)   # same rows, same order
    dx3, none = K.rms_norm_backward(dy, x, w, 1e-5, need_dw=False)
    assert none is None and torch.equal(dx3, dx1)
    xu = rnd((9, 4097), torch.bfloat16, 66)[:, 1:]       # misaligned rows -> looped kernel
    dyu = rnd((9, 4096), torch.bfloat16, 67)
    dxu, dwu = K.rms_norm_backward(dyu, xu, w, 1e-5)
    rdx, rdw = ops.rms_norm_bwd_golden(parity.to_np(xu), parity.to_np(w), parity.to_np(dyu),
                                       1e-5, "bf16")
    bound = ops.rms_norm_bwd_bound(parity.to_np(xu), parity.to_np(w), parity.to_np(dyu), 1e-5)
    parity.assert_within(parity.to_np(dxu), rdx, parity.BWD_TERM_TOL * bound, "looped dx", "bf16")
    e = torch.empty(0, 4096, dtype=torch.bfloat16, device=DEV)
    dxe, dwe = K.rms_norm_backward(e, e, w, 1e-5)
    assert dxe.shape == (0, 4096) and torch.equal(dwe.cpu(), torch.zeros(4096, dtype=torch.bfloat16))


# ----------------------------------------------------------- SwiGLU / SiLU
def _silu_scale(d, g, u):
    d, g, u = (np.asarray(a, np.float64) for a in (d, g, u))
    s = 1.0 / (1.0 + np.exp(-np.clip(g, -80, 80)))
    return np.abs(d) * (np.abs(u) * s * (1 + np.abs(g) * (1 - s)) + np.abs(g) * s)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 7, 4096, 14336 * 3, 1_000_003])
def test_swiglu_and_silu_backward(dtype, n):
    g = rnd((n,), dtype, 70, scale=3.0)
    u = rnd((n,), dtype, 71)
    d = rnd((n,), dtype, 72)
    dt = parity.dname(dtype)
    dg, du = K.swiglu_backward(d, g, u)
    gn, un, dn = parity.to_np(g), parity.to_np(u), parity.to_np(d)
    rdg, rdu = ops.swiglu_bwd_golden(dn, gn, un, dt)
    tol = 2.0 ** -18 * _silu_scale(dn, gn, un)
    parity.assert_within(parity.to_np(dg), rdg, tol, f"dgate {n}", _none16(dt))
    parity.assert_within(parity.to_np(du), rdu, tol, f"dup {n}", _none16(dt))
    dx = K.silu_backward(d, g)
    parity.assert_within(parity.to_np(dx), ops.silu_bwd_golden(dn, gn, dt),
                         2.0 ** -18 * _silu_scale(dn, gn, np.ones_like(gn)), f"silu {n}",
                         _none16(dt))


def test_swiglu_backward_2d_and_extremes():
    g = torch.tensor([[-100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 100.0, float("inf")]],
                     device=DEV).repeat(3, 1)
    u = torch.ones_like(g)
    d = torch.ones_like(g)
    dg, du = K.swiglu_backward(d, g, u)
    ref_g, ref_u = ops.swiglu_bwd_golden(parity.to_np(d), parity.to_np(g), parity.to_np(u), "f32")
    finite = np.isfinite(ref_g)
    np.testing.assert_allclose(parity.to_np(dg)[finite], ref_g[finite], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(parity.to_np(du)[:, :7], ref_u[:, :7], rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------------ softmax
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 10), (128, 256), (2, 8, 64), (5, 1001), (3, 40000),
                                   (64, 4096), (37, 2048)])
def test_softmax_backward(dtype, shape):
    x = rnd(shape, dtype, 80, scale=3.0)
    dt = parity.dname(dtype)
    y = K.softmax(x)
    dy = rnd(shape, dtype, 81)
    dx = K.softmax_backward(dy, y)
    yn, gn = parity.to_np(y), parity.to_np(dy)
    parity.assert_within(parity.to_np(dx), ops.softmax_bwd_golden(gn, yn, dt),
                         parity.BWD_TERM_TOL * ops.softmax_bwd_bound(gn, yn), f"dx {shape}",
                         _none16(dt))
    if dtype != torch.float32:   # half_to_float: fp32 probabilities and grads -> 16-bit dx
        y32 = K.softmax(x, out_dtype=torch.float32)
        dy32 = rnd(shape, torch.float32, 82)
        dx16 = K.softmax_backward(dy32, y32, out_dtype=dtype)
        assert dx16.dtype == dtype
        y32n, g32n = parity.to_np(y32), parity.to_np(dy32)
        parity.assert_within(parity.to_np(dx16), ops.softmax_bwd_golden(g32n, y32n, dt),
                             parity.BWD_TERM_TOL * ops.softmax_bwd_bound(g32n, y32n),
                             f"half_to_float {shape}", dt)


def test_backward_golden_fixtures(golden):
    """The kernels against torch CPU autograd of the transformers modules."""
    x, w, dy = (parity.from_np(golden.get(f"rmsnorm_bwd_f32/{k}"), torch.float32, DEV)
                for k in ("x", "w", "dy"))
    dx, dw = K.rms_norm_backward(dy, x, w, 1e-6)
    bound = ops.rms_norm_bwd_bound(*(golden.get(f"rmsnorm_bwd_f32/{k}") for k in ("x", "w", "dy")),
                                   1e-6)
    parity.assert_within(parity.to_np(dx), golden.get("rmsnorm_bwd_f32/dx"),
                         4 * parity.BWD_TERM_TOL * bound, "rmsnorm dx")
    parity.assert_rel(parity.to_np(dw), golden.get("rmsnorm_bwd_f32/dw"), rtol=1e-4, atol=1e-4,
                      what="rmsnorm dw")
    g, u, d = (parity.from_np(golden.get(f"swiglu_bwd_f32/{k}"), torch.float32, DEV)
               for k in ("gate", "up", "dout"))
    dg, du = K.swiglu_backward(d, g, u)
    scale = _silu_scale(*(golden.get(f"swiglu_bwd_f32/{k}") for k in ("dout", "gate", "up")))
    parity.assert_within(parity.to_np(dg), golden.get("swiglu_bwd_f32/dgate"), 2.0 ** -18 * scale,
                         "dgate")
    parity.assert_within(parity.to_np(du), golden.get("swiglu_bwd_f32/dup"), 2.0 ** -18 * scale,
                         "dup")
    y = parity.from_np(golden.get("softmax_bwd_half_to_float/y"), torch.float32, DEV)
    dyh = parity.from_np(golden.get("softmax_bwd_half_to_float/dy"), torch.float32, DEV)
    dxh = K.softmax_backward(dyh, y, out_dtype=torch.bfloat16)
    parity.assert_within(parity.to_np(dxh), golden.get("softmax_bwd_half_to_float/dx"),
                         4 * parity.BWD_TERM_TOL * ops.softmax_bwd_bound(parity.to_np(dyh),
                                                                        parity.to_np(y)),
                         "softmax half_to_float", "bf16")


# ------------------------------------------------- autograd through flagos::
def _grads(fn, inputs, grad_out):
    ins = [t.detach().clone().requires_grad_(True) for t in inputs]
    out = fn(*ins)
    outs = out if isinstance(out, tuple) else (out,)
    torch.autograd.backward(outs, grad_out)
    return [t.grad for t in ins]


def _cpu64(t):
    return t.detach().cpu().double()


# Autograd runs on flagos tensors: once the flagos PrivateUse1 backend is
# registered PyTorch treats it as the accelerator, and its autograd engine
# tracks streams for that device type only (plain cuda tensors hit an
# internal assert in the engine in such a process, with or without these ops).
@pytest.mark.parametrize("device", ["flagos"])
def test_autograd_rms_norm_swiglu_softmax(device):
    F = torch.ops.flagos
    x = rnd((8, 512), torch.float32, 90, device=device)
    w = rnd((512,), torch.float32, 91, scale=0.1, loc=1.0, device=device)
    dy = rnd((8, 512), torch.float32, 92, device=device)
    gx, gw = _grads(lambda a, b: F.rms_norm(a, b, 1e-6), [x, w], [dy])
    rx, rw = _grads(lambda a, b: b * (a * torch.rsqrt(a.pow(2).mean(-1, keepdim=True) + 1e-6)),
                    [_cpu64(x), _cpu64(w)], [_cpu64(dy)])
    torch.testing.assert_close(gx.cpu().double(), rx, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(gw.cpu().double(), rw, rtol=1e-4, atol=1e-4)

    g = rnd((8, 704), torch.float32, 93, scale=3.0, device=device)
    u = rnd((8, 704), torch.float32, 94, device=device)
    da = rnd((8, 704), torch.float32, 95, device=device)
    gg, gu = _grads(lambda a, b: F.swiglu(a, b), [g, u], [da])
    rg, ru = _grads(lambda a, b: torch.nn.functional.silu(a) * b, [_cpu64(g), _cpu64(u)],
                    [_cpu64(da)])
    torch.testing.assert_close(gg.cpu().double(), rg, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(gu.cpu().double(), ru, rtol=1e-4, atol=1e-5)

    s = rnd((2, 4, 64, 64), torch.float32, 96, scale=3.0, device=device)
    ds = rnd((2, 4, 64, 64), torch.float32, 97, device=device)
    (gs,) = _grads(lambda a: F.causal_softmax(a), [s], [ds])
    mask = torch.triu(torch.ones(64, 64, dtype=torch.bool), 1)
    (rs,) = _grads(lambda a: torch.softmax(a.masked_fill(mask, float("-inf")), -1), [_cpu64(s)],
                   [_cpu64(ds)])
    torch.testing.assert_close(gs.cpu().double(), rs, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("device", ["flagos"])
def test_autograd_rope_and_residual_ops(device):
    F = torch.ops.flagos
    B, S, Hq, Hk, D = 2, 16, 4, 2, 64
    pos = np.arange(S)
    ct, st = ops.rope_tables(pos, D, 1e4, "f32")
    cos = parity.from_np(np.broadcast_to(ct, (B, S, D)), torch.float32, device)
    sin = parity.from_np(np.broadcast_to(st, (B, S, D)), torch.float32, device)
    q = rnd((B, S, Hq, D), torch.float32, 100, device=device).transpose(1, 2)
    k = rnd((B, S, Hk, D), torch.float32, 101, device=device).transpose(1, 2)
    dqo = rnd((B, Hq, S, D), torch.float32, 102, device=device)
    dko = rnd((B, Hk, S, D), torch.float32, 103, device=device)

    def hf_rope(a, b, c, s):
        def rot(t):
            return torch.cat((-t[..., D // 2:], t[..., :D // 2]), -1)
        c, s = c.unsqueeze(1), s.unsqueeze(1)
        return a * c + rot(a) * s, b * c + rot(b) * s

    gq, gk = _grads(lambda a, b: F.rope_qk(a, b, cos, sin), [q, k], [dqo, dko])
    rq, rk = _grads(lambda a, b: hf_rope(a, b, _cpu64(cos), _cpu64(sin)), [_cpu64(q), _cpu64(k)],
                    [_cpu64(dqo), _cpu64(dko)])
    torch.testing.assert_close(gq.cpu().double(), rq, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(gk.cpu().double(), rk, rtol=1e-5, atol=1e-5)

    # q/k norm then RoPE
    wq = rnd((D,), torch.float32, 104, scale=0.1, loc=1.0, device=device)
    wk = rnd((D,), torch.float32, 105, scale=0.1, loc=1.0, device=device)

    def hf_norm(t, w):
        return w * (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6))

    got = _grads(lambda a, b, c, d: F.rms_norm_rope(a, b, c, d, cos, sin, 1e-6),
                 [q, k, wq, wk], [dqo, dko])
    ref = _grads(lambda a, b, c, d: hf_rope(hf_norm(a, c), hf_norm(b, d), _cpu64(cos), _cpu64(sin)),
                 [_cpu64(q), _cpu64(k), _cpu64(wq), _cpu64(wk)], [_cpu64(dqo), _cpu64(dko)])
    for a, b in zip(got, ref):
        torch.testing.assert_close(a.cpu().double(), b, rtol=1e-4, atol=1e-4)

    # add + RMSNorm and SwiGLU + residual
    x = rnd((8, 256), torch.float32, 106, device=device)
    r = rnd((8, 256), torch.float32, 107, device=device)
    w = rnd((256,), torch.float32, 108, scale=0.1, loc=1.0, device=device)
    do, dh = rnd((8, 256), torch.float32, 109, device=device), rnd((8, 256), torch.float32, 110,
                                                                   device=device)
    got = _grads(lambda a, b, c: F.add_rms_norm(a, b, c, 1e-6), [x, r, w], [do, dh])
    ref = _grads(lambda a, b, c: (hf_norm(a + b, c), a + b), [_cpu64(x), _cpu64(r), _cpu64(w)],
                 [_cpu64(do), _cpu64(dh)])
    for a, b in zip(got, ref):
        torch.testing.assert_close(a.cpu().double(), b, rtol=1e-4, atol=1e-4)
    g = rnd((8, 512), torch.float32, 111, device=device)
    u = rnd((8, 512), torch.float32, 112, device=device)
    da = rnd((8, 512), torch.float32, 113, device=device)
    got = _grads(lambda a, b, c, d: F.swiglu_residual(a, b, c, d), [g, u, x, r], [da, dh])
    ref = _grads(lambda a, b, c, d: (torch.nn.functional.silu(a) * b, c + d),
                 [_cpu64(g), _cpu64(u), _cpu64(x), _cpu64(r)], [_cpu64(da), _cpu64(dh)])
    for a, b in zip(got, ref):
        torch.testing.assert_close(a.cpu().double(), b, rtol=1e-4, atol=1e-5)


def test_routed_backward_ops_on_flagos():
    """_softmax_backward_data and silu_backward on the flagos device run the
    b200 kernels (backends.conf) and match torch CPU."""
    x = torch.randn(16, 300, generator=torch.Generator().manual_seed(120)) * 3
    dy = torch.randn(16, 300, generator=torch.Generator().manual_seed(121))
    xd = x.to("flagos").requires_grad_(True)
    torch.softmax(xd, -1).backward(dy.to("flagos"))
    xc = x.clone().requires_grad_(True)
    torch.softmax(xc, -1).backward(dy)
    torch.testing.assert_close(xd.grad.cpu(), xc.grad, rtol=1e-4, atol=1e-6)
    # non-last dim and half_to_float
    y = torch.softmax(x.to(torch.bfloat16), 0, dtype=torch.float32)
    dxd = torch.ops.aten._softmax_backward_data(dy.to("flagos"), y.to("flagos"), 0, torch.bfloat16)
    dxc = torch.ops.aten._softmax_backward_data(dy, y, 0, torch.bfloat16)
    torch.testing.assert_close(dxd.cpu().float(), dxc.float(), rtol=2e-2, atol=1e-3)
    g = torch.randn(4, 1000, generator=torch.Generator().manual_seed(122))
    got = torch.ops.aten.silu_backward(dy[:4, :1].expand(4, 1000).to("flagos"), g.to("flagos"))
    ref = torch.ops.aten.silu_backward(dy[:4, :1].expand(4, 1000), g)
    torch.testing.assert_close(got.cpu(), ref, rtol=1e-5, atol=1e-6)
    routes = torch_fl.routes()
    assert routes.get("_softmax_backward_data") == "b200" and routes.get("silu_backward") == "b200"
