"""The remaining ops of the HF formulas on the b200 route: silu, rsqrt, neg,
cos, sin, pow.Tensor_Scalar and cat (the reference registers them at
csrc/aten/register.cc:405-417 and runs them with its cuda route,
csrc/aten/backends/cuda/{silu,rsqrt,neg,cos,sin,pow}.cu and cat.cc).

Each op runs on flagos tensors through the aten registration (routed to b200
by backends.conf) and through the C ABI (torch_fl.kernels), on contiguous
tensors, on the strided halves HF's rotate_half slices from a transposed q,
and on widths that 16-byte packs do not fit; the result is compared with the
same op on torch CPU (the reference's own CPU semantics): within 1 ulp for
bf16/f16, 1e-5 relative for fp32 (CUDA's rsqrtf, cosf and sinf are within 2
fp32 ulp), exact for neg and cat."""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import torch_fl  # noqa: F401
from torch_fl import kernels as K
from tests import parity

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def _inputs(dtype, op):
    """Contiguous, strided (rotate_half's halves of a transposed q), odd width."""
    g = torch.Generator().manual_seed(hash((str(dtype), op)) % 1000)
    scale = 3.0 if op in ("silu", "neg", "cos", "sin") else 1.0
    q = (scale * torch.randn(2, 9, 4, 128, generator=g)).to(dtype)   # [B, S, H, D]
    qt = q.transpose(1, 2)                                            # [B, H, S, D] view
    base = [("contiguous", (scale * torch.randn(33, 256, generator=g)).to(dtype)),
            ("transposed", qt),
            ("half_slice", qt[..., 64:]),
            ("odd_width", (scale * torch.randn(7, 37, generator=g)).to(dtype)),
            ("scalar", (scale * torch.randn((), generator=g)).to(dtype))]
    if op in ("rsqrt", "pow"):
        base = [(n, t.abs() + 0.05) for n, t in base]   # a real power of a positive base
    return base


def _check(got, ref, dtype, what):
    assert got.shape == ref.shape, what
    g = got.float().numpy()
    r = ref.float().numpy()
    if dtype == torch.float32:
        parity.assert_rel(g, r, rtol=1e-5, atol=1e-6, what=what)
    else:
        parity.assert_ulp(g, r, parity.dname(dtype), 1, what)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("op", ["silu", "rsqrt", "neg", "cos", "sin"])
def test_unary_ops_match_torch_cpu(op, dtype):
    fn = {"silu": torch.nn.functional.silu, "rsqrt": torch.rsqrt, "neg": torch.neg,
          "cos": torch.cos, "sin": torch.sin}[op]
    for name, x in _inputs(dtype, op):
        ref = fn(x)
        got = fn(x.to("flagos")).cpu()       # aten registration -> b200 route
        _check(got, ref, dtype, f"{op} {name} flagos")
        if op == "neg":
            assert torch.equal(got, ref), name
        abi = K.unary(x.cuda(), op).cpu()    # the C ABI directly
        _check(abi, ref, dtype, f"{op} {name} abi")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("e", [2, 3, 2.0, 0.5, -1, 2.5, 0.3])
def test_pow_tensor_scalar_matches_torch_cpu(e, dtype):
    for name, x in _inputs(dtype, "pow"):
        ref = torch.pow(x, e)
        got = torch.pow(x.to("flagos"), e).cpu()
        _check(got, ref, dtype, f"pow {e} {name}")
        _check(K.unary(x.cuda(), "pow", e).cpu(), ref, dtype, f"pow {e} {name} abi")


def test_pow_follows_the_reference_arithmetic():
    # exponent 2 is one rounded product; a bf16 cube rounds the square first
    # (pow.cu:29-36: b*b*b in the tensor's dtype); other exponents are first
    # rounded to the dtype (0.3 -> 0.30078125 in bf16)
    x = torch.tensor([1.0078125, 3.0, 1.5, 0.7], dtype=torch.bfloat16)
    sq = torch.pow(x.to("flagos"), 2).cpu()
    assert torch.equal(sq, (x.float() * x.float()).to(torch.bfloat16))
    cube = torch.pow(x.to("flagos"), 3).cpu()
    assert torch.equal(cube, ((x.float() * x.float()).to(torch.bfloat16).float()
                              * x.float()).to(torch.bfloat16))
    p = torch.pow(x.to("flagos"), 0.3).cpu()
    e = float(torch.tensor(0.3, dtype=torch.bfloat16))
    assert torch.equal(p, torch.pow(x.float(), e).to(torch.bfloat16))


def test_integer_tensors():
    xi = torch.randint(-2**31, 2**31 - 1, (5, 9), dtype=torch.int32)
    xi[0, 0] = -2**31                                  # two's complement: maps to itself
    assert torch.equal(torch.neg(xi.to("flagos")).cpu(), torch.neg(xi))
    xl = torch.randint(-1000, 1000, (3, 4), dtype=torch.int64)
    assert torch.equal(torch.neg(xl.to("flagos")).cpu(), torch.neg(xl))
    assert torch.equal(torch.pow(xl.to("flagos"), 2).cpu(), torch.pow(xl, 2))   # cuda route


@pytest.mark.parametrize("dtype", DTYPES + [torch.int64, torch.bool])
def test_cat_matches_torch_cpu(dtype):
    g = torch.Generator().manual_seed(3)

    def r(*s):
        t = torch.randn(*s, generator=g)
        return (t > 0) if dtype == torch.bool else t.to(dtype)

    q = r(2, 9, 4, 128).transpose(1, 2)                # [B, H, S, D] view
    x1, x2 = q[..., :64], q[..., 64:]
    cases = [((-x2 if dtype != torch.bool else ~x2, x1), -1),   # HF rotate_half
             ((r(3, 5), r(4, 5), r(1, 5)), 0),
             ((r(2, 3, 7), r(2, 1, 7), r(2, 4, 7)), 1),
             ((r(6, 3), r(6, 5)), -1),                  # widths 16-byte packs do not fit
             ((r(2, 3), torch.empty(0, dtype=r(1).dtype), r(2, 3)), 0)]   # legacy empty
    for i, (ts, d) in enumerate(cases):
        ref = torch.cat(ts, d)
        got = torch.cat([t.to("flagos") for t in ts], d).cpu()
        assert torch.equal(got, ref), i
        kept = [t for t in ts if not (t.dim() == 1 and t.numel() == 0)]
        assert torch.equal(K.cat([t.cuda() for t in kept], d).cpu(), ref), i


def test_cat_mixed_dtypes_promote_like_torch():
    a = torch.randn(2, 3)
    b = torch.randn(2, 3).to(torch.bfloat16)
    ref = torch.cat([a, b])
    got = torch.cat([a.to("flagos"), b.to("flagos")]).cpu()
    assert got.dtype == ref.dtype and torch.equal(got, ref)


def test_rotate_half_chain_on_flagos_matches_cpu():
    # the whole HF RoPE formula op by op (hooks off): mul, neg, cat, mul, add
    from oracle import hf_chain

    g = torch.Generator().manual_seed(8)
    q = torch.randn(1, 16, 4, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(1, 16, 2, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    cos, sin = hf_chain.rope_tables(torch.arange(16)[None], 128, 1e4, torch.bfloat16)
    ref = hf_chain.rope(q, k, cos, sin)
    got = hf_chain.rope(q.to("flagos"), k.to("flagos"), cos.to("flagos"), sin.to("flagos"))
    for a, b in zip(got, ref):
        assert torch.equal(a.cpu(), b)


def test_dispatch_log_names_b200_for_the_formula_ops():
    code = ("import torch_fl, torch; x = torch.randn(4, 8, device='flagos:0'); "
            "torch.nn.functional.silu(x); torch.rsqrt(x.abs() + 1); torch.neg(x); torch.cos(x); "
            "torch.sin(x); x.pow(2); torch.cat([x, x], -1); torch.flagos.synchronize()")
    e = os.environ.copy()
    e["FLAGOS_LOG_DISPATCH"] = "1"
    e["PYTHONPATH"] = os.pathsep.join([ROOT, os.path.join(ROOT, "pytorch-plugin-fl_b200"),
                                       e.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", code], env=e, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    for op in ("silu", "rsqrt", "neg", "cos", "sin", "pow.Tensor_Scalar", "cat"):
        assert f"[flagos dispatch] {op} -> b200" in r.stderr, op


def test_unary_large_dense_and_strided_rows_exact_vs_oracle():
    # a size well past one wave of CTAs: both kernels cover every row
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(4096, 1000, generator=g, device="cuda").to(torch.bfloat16)
    ref = torch.neg(x)
    assert torch.equal(K.unary(x, "neg"), ref)
    xs = x[:, 8:1000]                                   # strided rows, 16-byte aligned starts
    assert torch.equal(K.unary(xs, "neg"), ref[:, 8:1000])
    xo = x[:, 1:999]                                    # unaligned starts: element path
    assert torch.equal(K.unary(xo, "neg"), ref[:, 1:999])
    np.testing.assert_array_equal(K.unary(x[::2], "neg").cpu().float().numpy(),
                                  ref[::2].cpu().float().numpy())
