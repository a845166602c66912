"""Parity of the B200 kernels (through the C ABI of libfl_b200.so) with the
oracle, on seeded inputs.  Tolerances are the ones stated in tests/parity.py:
bf16/f16 within 1 ulp of the fp64 formula rounded once ("fused" rounding),
fp32 within 1e-5 relative, integer and index results bit-exact; the "chain"
rounding mode must reproduce the reference's op-by-op result (bit-exact for
RoPE and the golden fixtures where the reference's steps are exactly rounded).
"""

import numpy as np
import pytest
import torch

from oracle import native, ops
from tests import parity
from torch_fl import kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def rnd(shape, dtype, seed, scale=1.0, loc=0.0, device=DEV):
    g = torch.Generator().manual_seed(seed)
    return (loc + scale * torch.randn(*shape, generator=g)).to(dtype).to(device)


def check_float(got, ref, dt, what=""):
    if dt == "f32":
        parity.assert_rel(parity.to_np(got), ref, rtol=1e-5, atol=1e-30, what=what)
    else:
        parity.assert_ulp(parity.to_np(got), ref, dt, 1, what)


# ------------------------------------------------------------------- RMSNorm
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 1), (3, 7), (5, 96), (127, 4096), (16, 8192),
                                   (4, 32768), (2, 65536 + 8), (33, 1000)])
def test_rms_norm_fused(dtype, shape):
    x = rnd(shape, dtype, 1)
    w = rnd(shape[-1:], dtype, 2, scale=0.1, loc=1.0)
    out = K.rms_norm(x, w, 1e-5)
    dt = parity.dname(dtype)
    ref = ops.rms_norm_golden(parity.to_np(x), parity.to_np(w), 1e-5, dt)
    check_float(out, ref, dt, f"rms_norm {shape}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rms_norm_chain_matches_reference_chain(dtype):
    x = rnd((64, 4096), dtype, 3)
    w = rnd((4096,), dtype, 4, scale=0.1, loc=1.0)
    out = K.rms_norm(x, w, 1e-5, rounding="chain")
    dt = parity.dname(dtype)
    ref = ops.rms_norm_chain(parity.to_np(x), parity.to_np(w), 1e-5, dt)
    # Differs only where the fp32 sum order flips the intermediate rounding of
    # x*r; the weight multiply can carry that 1-ulp flip into a 2-ulp one.
    d = parity.assert_ulp(parity.to_np(out), ref, dt, 2, "chain")
    assert np.mean(d == 0) > 0.999


def test_rms_norm_golden_fixtures(golden):
    x = parity.from_np(golden.get("rmsnorm_f32/x"), torch.float32, DEV)
    w = parity.from_np(golden.get("rmsnorm_f32/w"), torch.float32, DEV)
    parity.assert_rel(parity.to_np(K.rms_norm(x, w, 1e-6)), golden.get("rmsnorm_f32/out"),
                      rtol=1e-5, what="f32 fixture")
    x = parity.from_np(golden.get("rmsnorm_bf16/x"), torch.bfloat16, DEV)
    w = parity.from_np(golden.get("rmsnorm_bf16/w"), torch.bfloat16, DEV)
    d = parity.assert_ulp(parity.to_np(K.rms_norm(x, w, 1e-5, rounding="chain")),
                          golden.get("rmsnorm_bf16/out"), "bf16", 1, "bf16 fixture chain")
    assert np.mean(d == 0) > 0.999
    parity.assert_ulp(parity.to_np(K.rms_norm(x, w, 1e-5)),
                      ops.rms_norm_golden(golden.get("rmsnorm_bf16/x"), golden.get("rmsnorm_bf16/w"),
                                          1e-5, "bf16"), "bf16", 1, "bf16 fixture fused")


def test_rms_norm_strided_and_inplace():
    base = rnd((64, 4096 + 64), torch.bfloat16, 5)
    x = base[:, :4096]                      # leading stride 4160
    w = rnd((4096,), torch.bfloat16, 6, scale=0.1, loc=1.0)
    ref = ops.rms_norm_golden(parity.to_np(x), parity.to_np(w), 1e-6, "bf16")
    parity.assert_ulp(parity.to_np(K.rms_norm(x, w, 1e-6)), ref, "bf16", 1, "strided")
    y = x.clone()
    K.rms_norm(y, w, 1e-6, out=y)
    parity.assert_ulp(parity.to_np(y), ref, "bf16", 1, "in place")
    xu = rnd((9, 4097), torch.bfloat16, 7)[:, 1:]   # misaligned base -> looped kernel
    ref = ops.rms_norm_golden(parity.to_np(xu), parity.to_np(w), 1e-6, "bf16")
    parity.assert_ulp(parity.to_np(K.rms_norm(xu, w, 1e-6)), ref, "bf16", 1, "misaligned")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("cols", [4096, 8192, 16384, 1024, 2048, 4104, 40])
def test_add_rms_norm(dtype, cols):
    # 32-byte path: one pack per thread (4096, 8192, 16384 16-bit wide), the
    # two-pack ladder (1024, 2048; fp32 40); 4104 and 40 16-bit values are
    # not whole 32-byte packs: the 16-byte kernel
    x = rnd((48, cols), dtype, 8)
    y = rnd((48, cols), dtype, 9)
    w = rnd((cols,), dtype, 10, scale=0.1, loc=1.0)
    dt = parity.dname(dtype)
    xn, yn, wn = parity.to_np(x), parity.to_np(y), parity.to_np(w)
    out, h = K.add_rms_norm(x, y, w, 1e-5)
    ref_o, ref_h = ops.add_rms_norm_golden(xn, yn, wn, 1e-5, dt)
    check_float(h, ref_h, dt, "h")
    # the norm is taken over the stored (rounded) h
    check_float(out, ops.rms_norm_golden(parity.to_np(h), wn, 1e-5, dt), dt, "out")
    # chain rounding: h exact, the norm rounded where the reference's chain
    # rounds (16-bit: differs only where the fp32 sum order flips the
    # intermediate rounding of h*r, as for RMSNorm alone; fp32 has no
    # intermediate rounding, so the fused bound holds)
    out_c, h_c = K.add_rms_norm(x, y, w, 1e-5, rounding="chain")
    ref_oc, ref_hc = ops.add_rms_norm_chain(xn, yn, wn, 1e-5, dt)
    check_float(h_c, ref_hc, dt, "h chain")
    if dt == "f32":
        check_float(out_c, ref_oc, dt, "out chain")
    else:
        d = parity.assert_ulp(parity.to_np(out_c), ref_oc, dt, 2, "out chain")
        assert np.mean(d == 0) > 0.99


def test_add_rms_norm_unaligned_rows_take_the_other_paths():
    # a base offset of one element (16-byte but not 32-byte aligned rows
    # would need 8-element offsets): the looped kernel; 8 elements: the
    # 16-byte kernel; both must give the 32-byte kernel's values
    base_x = rnd((16, 4096 + 8), torch.bfloat16, 11)
    base_y = rnd((16, 4096 + 8), torch.bfloat16, 12)
    w = rnd((4096,), torch.bfloat16, 13, scale=0.1, loc=1.0)
    ref_o, ref_h = K.add_rms_norm(base_x[:, :4096].contiguous(), base_y[:, :4096].contiguous(), w,
                                  1e-5)
    for off in (8, 1):
        xs = base_x.flatten()[off:off + 16 * 4096].view(16, 4096)
        ys = base_y.flatten()[off:off + 16 * 4096].view(16, 4096)
        o, h = K.add_rms_norm(xs, ys, w, 1e-5)
        ro, rh = K.add_rms_norm(xs.contiguous() * 1, ys.contiguous() * 1, w, 1e-5)
        parity.assert_ulp(parity.to_np(h), parity.to_np(rh), "bf16", 0, f"h offset {off}")
        parity.assert_ulp(parity.to_np(o), parity.to_np(ro), "bf16", 1, f"out offset {off}")


# ---------------------------------------------------------------------- RoPE
def _fixture_rope(golden, dtype=torch.bfloat16):
    q = parity.from_np(golden.get("rope_bf16/q"), dtype, DEV)
    k = parity.from_np(golden.get("rope_bf16/k"), dtype, DEV)
    cos = parity.from_np(golden.get("rope_bf16/cos"), dtype, DEV)
    sin = parity.from_np(golden.get("rope_bf16/sin"), dtype, DEV)
    return q, k, cos, sin


def test_rope_chain_bit_exact_with_reference(golden):
    q, k, cos, sin = _fixture_rope(golden)
    qo, ko = K.rope_qk(q, k, cos, sin, rounding="chain")
    parity.assert_ulp(parity.to_np(qo), golden.get("rope_bf16/q_out"), "bf16", 0, "q")
    parity.assert_ulp(parity.to_np(ko), golden.get("rope_bf16/k_out"), "bf16", 0, "k")


def test_rope_fused_within_1ulp_of_golden(golden):
    q, k, cos, sin = _fixture_rope(golden)
    qo, ko = K.rope_qk(q, k, cos, sin)
    c, s = golden.get("rope_bf16/cos")[:, None], golden.get("rope_bf16/sin")[:, None]
    parity.assert_ulp(parity.to_np(qo), ops.rope_golden(golden.get("rope_bf16/q"), c, s, "bf16"), "bf16", 1)
    parity.assert_ulp(parity.to_np(ko), ops.rope_golden(golden.get("rope_bf16/k"), c, s, "bf16"), "bf16", 1)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D", [128, 64, 96, 256])
def test_rope_layouts(dtype, D):
    B, S, Hq, Hk = 2, 24, 4, 2
    # HF layout: projections are [B, S, H, D] viewed as [B, H, S, D]
    q = rnd((B, S, Hq, D), dtype, 11).transpose(1, 2)
    k = rnd((B, S, Hk, D), dtype, 12).transpose(1, 2)
    pos = np.arange(S) + 1000
    ct, st = ops.rope_tables(pos, D, 1e4, parity.dname(dtype))
    cos = parity.from_np(np.broadcast_to(ct, (B, S, D)), dtype, DEV)
    sin = parity.from_np(np.broadcast_to(st, (B, S, D)), dtype, DEV)
    dt = parity.dname(dtype)
    for rounding in ("fused", "chain"):
        qo, ko = K.rope_qk(q, k, cos, sin, rounding=rounding)
        c, s = ct[None, None], st[None, None]
        f = ops.rope_golden if rounding == "fused" else ops.rope_chain
        tol = 1 if rounding == "fused" else 0
        if dt == "f32":
            parity.assert_rel(parity.to_np(qo), ops.rope_golden(parity.to_np(q), c, s, dt),
                              rtol=1e-5, atol=1e-6, what=f"q {rounding}")
            parity.assert_rel(parity.to_np(ko), ops.rope_golden(parity.to_np(k), c, s, dt),
                              rtol=1e-5, atol=1e-6, what=f"k {rounding}")
        else:
            parity.assert_ulp(parity.to_np(qo), f(parity.to_np(q), c, s, dt), dt, tol, f"q {rounding}")
            parity.assert_ulp(parity.to_np(ko), f(parity.to_np(k), c, s, dt), dt, tol, f"k {rounding}")


def test_rope_inplace_bshd_and_no_k():
    B, S, H, D = 1, 33, 8, 128
    q = rnd((B, S, H, D), torch.bfloat16, 13)
    ct, st = ops.rope_tables(np.arange(S), D, 1e4, "bf16")
    cos = parity.from_np(ct, torch.bfloat16, DEV)   # [S, D] table
    sin = parity.from_np(st, torch.bfloat16, DEV)
    ref = ops.rope_chain(parity.to_np(q), ct[None, :, None], st[None, :, None], "bf16")
    q2 = q.clone()
    K.rope_qk(q2, None, cos, sin, layout="bshd", rounding="chain", inplace=True)
    parity.assert_ulp(parity.to_np(q2), ref, "bf16", 0, "in place bshd")


def test_rope_full_decoder_shape():
    T = 8192
    q = rnd((T, 32, 128), torch.bfloat16, 14).unsqueeze(0)   # [1, T, Hq, D] = bshd
    k = rnd((T, 8, 128), torch.bfloat16, 15).unsqueeze(0)
    ct, st = ops.rope_tables(np.arange(T), 128, 1e4, "bf16")
    cos, sin = parity.from_np(ct, torch.bfloat16, DEV), parity.from_np(st, torch.bfloat16, DEV)
    qo, ko = K.rope_qk(q, k, cos, sin, layout="bshd")
    c, s = ct[None, :, None], st[None, :, None]
    parity.assert_ulp(parity.to_np(qo), ops.rope_golden(parity.to_np(q), c, s, "bf16"), "bf16", 1, "q")
    parity.assert_ulp(parity.to_np(ko), ops.rope_golden(parity.to_np(k), c, s, "bf16"), "bf16", 1, "k")


def test_rms_norm_rope_fixture(golden):
    q, k, cos, sin = _fixture_rope(golden)
    wq = parity.from_np(golden.get("qknorm_rope_bf16/wq"), torch.bfloat16, DEV)
    wk = parity.from_np(golden.get("qknorm_rope_bf16/wk"), torch.bfloat16, DEV)
    qo, ko = K.rope_qk(q, k, cos, sin, rounding="chain", q_weight=wq, k_weight=wk, eps=1e-6)
    d = parity.assert_ulp(parity.to_np(qo), golden.get("qknorm_rope_bf16/q_out"), "bf16", 1, "q")
    assert np.mean(d == 0) > 0.999
    parity.assert_ulp(parity.to_np(ko), golden.get("qknorm_rope_bf16/k_out"), "bf16", 1, "k")
    qf, kf = K.rope_qk(q, k, cos, sin, q_weight=wq, k_weight=wk, eps=1e-6)
    c, s = golden.get("rope_bf16/cos")[:, None], golden.get("rope_bf16/sin")[:, None]
    parity.assert_ulp(parity.to_np(qf), ops.rms_norm_rope_golden(
        golden.get("rope_bf16/q"), golden.get("qknorm_rope_bf16/wq"), c, s, 1e-6, "bf16"), "bf16", 1, "q fused")
    parity.assert_ulp(parity.to_np(kf), ops.rms_norm_rope_golden(
        golden.get("rope_bf16/k"), golden.get("qknorm_rope_bf16/wk"), c, s, 1e-6, "bf16"), "bf16", 1, "k fused")


@pytest.mark.parametrize("D", [128, 80])
def test_rms_norm_rope_dtypes(D):
    for dtype in DTYPES:
        B, S, H = 2, 9, 3
        q = rnd((B, H, S, D), dtype, 16)
        w = rnd((D,), dtype, 17, scale=0.1, loc=1.0)
        ct, st = ops.rope_tables(np.arange(S), D, 1e4, parity.dname(dtype))
        cos, sin = parity.from_np(ct, dtype, DEV), parity.from_np(st, dtype, DEV)
        qo, _ = K.rope_qk(q, None, cos, sin, q_weight=w, eps=1e-6)
        dt = parity.dname(dtype)
        ref = ops.rms_norm_rope_golden(parity.to_np(q), parity.to_np(w), ct[None, None], st[None, None], 1e-6, dt)
        if dt == "f32":
            parity.assert_rel(parity.to_np(qo), ref, rtol=1e-5, atol=1e-6)
        else:
            parity.assert_ulp(parity.to_np(qo), ref, dt, 1, f"{dtype} D={D}")


# -------------------------------------------------------------------- SwiGLU
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 8), (16, 1024), (7, 1001), (64, 14336)])
def test_swiglu(dtype, shape):
    g, u = rnd(shape, dtype, 18), rnd(shape, dtype, 19)
    dt = parity.dname(dtype)
    check_float(K.swiglu(g, u), ops.swiglu_golden(parity.to_np(g), parity.to_np(u), dt), dt, "fused")
    if dt != "f32":
        # CUDA's expf and the host's differ in the last fp32 bit; where that
        # flips the rounding of silu, the multiply by `up` can make it 2 ulp.
        d = parity.assert_ulp(parity.to_np(K.swiglu(g, u, rounding="chain")),
                              ops.swiglu_chain(parity.to_np(g), parity.to_np(u), dt), dt, 2, "chain")
        assert np.mean(d == 0) > 0.999


def test_swiglu_fixture_and_extremes(golden):
    g = parity.from_np(golden.get("swiglu_bf16/gate"), torch.bfloat16, DEV)
    u = parity.from_np(golden.get("swiglu_bf16/up"), torch.bfloat16, DEV)
    d = parity.assert_ulp(parity.to_np(K.swiglu(g, u, rounding="chain")), golden.get("swiglu_bf16/out"),
                          "bf16", 1, "fixture chain")
    assert np.mean(d == 0) > 0.999
    ext = torch.tensor([[-200.0, -90.0, -20.0, 0.0, 20.0, 90.0, 200.0, 1e30]], dtype=torch.float32)
    ones = torch.ones_like(ext)
    got = parity.to_np(K.swiglu(ext.to(DEV), ones.to(DEV)))
    ref = ops.swiglu_golden(ext.numpy(), ones.numpy(), "f32")
    parity.assert_rel(got, ref, rtol=1e-5, atol=1e-30, what="extremes")


def test_swiglu_strided_and_inplace():
    base = rnd((32, 2048), torch.bfloat16, 20)
    g, u = base[:, :1024], base[:, 1024:]           # the fused gate_up projection layout
    ref = ops.swiglu_golden(parity.to_np(g), parity.to_np(u), "bf16")
    parity.assert_ulp(parity.to_np(K.swiglu(g, u)), ref, "bf16", 1, "strided halves")
    g2 = g.contiguous()
    K.swiglu(g2, u.contiguous(), out=g2)
    parity.assert_ulp(parity.to_np(g2), ref, "bf16", 1, "in place")


@pytest.mark.parametrize("dtype", DTYPES)
def test_swiglu_residual(dtype):
    T = 40
    g, u = rnd((T, 14336), dtype, 21), rnd((T, 14336), dtype, 22)
    x, y = rnd((T, 4096), dtype, 23), rnd((T, 4096), dtype, 24)
    a, h = K.swiglu_residual(g, u, x, y)
    dt = parity.dname(dtype)
    check_float(a, ops.swiglu_golden(parity.to_np(g), parity.to_np(u), dt), dt, "act")
    check_float(h, ops.add_golden(parity.to_np(x), parity.to_np(y), 1.0, dt), dt, "h")


def test_swiglu_full_size_rows():
    g, u = rnd((8192, 14336), torch.bfloat16, 25), rnd((8192, 14336), torch.bfloat16, 26)
    a = K.swiglu(g, u)
    rows = [0, 1, 4095, 8190, 8191]
    ref = ops.swiglu_golden(parity.to_np(g[rows]), parity.to_np(u[rows]), "bf16")
    parity.assert_ulp(parity.to_np(a[rows]), ref, "bf16", 1, "sampled rows")
    # every row: same kernel result as the row-sliced call (position independence)
    b = K.swiglu(g[4096:], u[4096:])
    assert torch.equal(a[4096:], b)


# --------------------------------------------------------------- elementwise
def test_add_mul_fixtures(golden):
    a = parity.from_np(golden.get("add_bf16/a"), torch.bfloat16, DEV)
    b = parity.from_np(golden.get("add_bf16/b"), torch.bfloat16, DEV)
    parity.assert_ulp(parity.to_np(K.add(a, b)), golden.get("add_bf16/out"), "bf16", 0, "add")
    parity.assert_ulp(parity.to_np(K.add(a, b, alpha=2.5)), golden.get("add_bf16/out_alpha"), "bf16", 1,
                      "alpha")
    x = parity.from_np(golden.get("residual_bf16/x"), torch.bfloat16, DEV)
    y = parity.from_np(golden.get("residual_bf16/y"), torch.bfloat16, DEV)
    parity.assert_ulp(parity.to_np(K.add(x, y)), golden.get("residual_bf16/out"), "bf16", 0, "residual")
    w = parity.from_np(golden.get("mul_bf16/w"), torch.bfloat16, DEV)
    h = parity.from_np(golden.get("mul_bf16/h"), torch.bfloat16, DEV)
    c = parity.from_np(golden.get("mul_bf16/c"), torch.bfloat16, DEV)
    parity.assert_ulp(parity.to_np(K.mul(w, h)), golden.get("mul_bf16/w_h"), "bf16", 0, "w*h")
    parity.assert_ulp(parity.to_np(K.mul(h, c)), golden.get("mul_bf16/h_c"), "bf16", 0, "h*c")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("sa,sb", [((64, 4096), (64, 4096)), ((64, 4096), (4096,)),
                                   ((4096,), (64, 4096)), ((8, 1, 16), (1, 5, 16)),
                                   ((3, 7), (3, 1)), ((2, 3, 4, 5), (5,)), ((1,), (9, 9)),
                                   # dense, not whole 32-byte packs: the 16-byte kernel
                                   ((3, 1000), (3, 1000)),
                                   # one value per row, second or first operand,
                                   # whole and partial 8-row tiles, long rows
                                   ((64, 4096), (64, 1)), ((64, 1), (64, 4096)),
                                   ((13, 1024), (13, 1)), ((3, 8192), (1024 * 8,)),
                                   # per-row values of a 3-d tensor (leading dims
                                   # collapse to one stride) and ones that do not
                                   # collapse (the N-d path)
                                   ((4, 16, 256), (4, 16, 1)), ((4, 16, 256), (4, 1, 1))])
def test_add_mul_broadcast(dtype, sa, sb):
    a, b = rnd(sa, dtype, 27), rnd(sb, dtype, 28)
    dt = parity.dname(dtype)
    na, nb = parity.to_np(a), parity.to_np(b)
    check_float(K.add(a, b, alpha=0.5), ops.add_golden(na, nb, 0.5, dt), dt, "add")
    check_float(K.mul(a, b), ops.mul_golden(na, nb, dt), dt, "mul")


@pytest.mark.parametrize("tdtype,bits", [(torch.int32, 32), (torch.int64, 64)])
def test_add_int(tdtype, bits):
    g = torch.Generator().manual_seed(29)
    a = torch.randint(-2**30, 2**30, (100, 33), generator=g, dtype=tdtype)
    b = torch.randint(-2**30, 2**30, (33,), generator=g, dtype=tdtype)
    got = K.add(a.to(DEV), b.to(DEV), alpha=3).cpu().numpy()
    parity.assert_exact(got, ops.add_int(a.numpy(), b.numpy(), 3, bits), "int add")
    got = K.mul(a.to(DEV), b.to(DEV)).cpu().numpy()
    with np.errstate(over="ignore"):
        ref = (a.numpy() * b.numpy()).astype(a.numpy().dtype)
    parity.assert_exact(got, ref, "int mul")


def test_binary_scalar_keeps_opmath():
    x = rnd((1000,), torch.bfloat16, 30)
    got = parity.to_np(K.binary_scalar(x, 1e-5, "add"))
    # the scalar is not rounded to bf16 first (aten wrapped-number semantics)
    ref = ops.round_to(parity.to_np(x).astype(np.float32) + np.float32(1e-5), "bf16")
    parity.assert_ulp(got, ref, "bf16", 0, "add scalar")
    got = parity.to_np(K.binary_scalar(x, 3.0, "mul"))
    parity.assert_ulp(got, ops.mul_golden(parity.to_np(x), 3.0, "bf16"), "bf16", 0, "mul scalar")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [4096 * 3 + 16, 1000, 1 << 20])
def test_binary_scalar_vector_paths(dtype, n):
    # whole 32-byte packs: two per thread in 512-thread CTAs (a partial last
    # CTA at 12304 elements); 1000 16-bit values: the 16-byte kernel
    x = rnd((n,), dtype, 34)
    dt = parity.dname(dtype)
    xn = parity.to_np(x).astype(np.float32)
    got = parity.to_np(K.binary_scalar(x, 0.37, "add"))
    parity.assert_ulp(got, ops.round_to(xn + np.float32(0.37), dt), dt, 0, "add scalar")
    got = parity.to_np(K.binary_scalar(x, -1.7, "mul"))
    parity.assert_ulp(got, ops.round_to(xn * np.float32(-1.7), dt), dt, 0, "mul scalar")


@pytest.mark.parametrize("n", [12000, 8 * 1024 * 2, 1 << 20])
def test_cast_vector_paths(n):
    # n % 8 == 0 with 16-byte aligned tensors: two units of 8 per thread
    # (a partial last CTA at 12000); every pair against torch's CPU cast
    base = torch.randn(n, generator=torch.Generator().manual_seed(33)) * 1000
    kinds = [torch.float32, torch.bfloat16, torch.float16, torch.int32, torch.int64]
    for s in kinds:
        src = base.to(s)
        for d in kinds:
            if d == s:
                continue
            got = K.cast(src.to(DEV), d).cpu()
            assert torch.equal(got, src.to(d)), (n, s, d)


def test_cast_all_pairs():
    vals = torch.tensor([0.0, -0.0, 1.0, -2.5, 65504.0, 1e-8, 3.14159, -1000.75, 7.0, 2**24 + 1.0])
    for s in [torch.float32, torch.bfloat16, torch.float16, torch.int32, torch.int64]:
        src = vals.to(s)
        for d in [torch.float32, torch.bfloat16, torch.float16, torch.int32, torch.int64]:
            got = K.cast(src.to(DEV), d).cpu()
            ref = src.to(d)    # torch CPU cast semantics
            if s.is_floating_point and not d.is_floating_point:
                # float -> int of inf / out-of-range values is unspecified (C
                # semantics; x86 and the GPU saturate differently): skip those
                ok = torch.isfinite(src.float())
                got, ref = got[ok], ref[ok]
            assert torch.equal(got, ref), (s, d, got, ref)
    x = rnd((1 << 20,), torch.float32, 31)
    assert torch.equal(K.cast(x, torch.bfloat16).cpu(), x.cpu().to(torch.bfloat16))
    nan_inf = torch.tensor([float("nan"), float("inf"), -float("inf"), 1e39], dtype=torch.float32)
    got = K.cast(nan_inf.to(DEV), torch.bfloat16).cpu().float()
    assert torch.isnan(got[0]) and got[1] == float("inf") and got[2] == -float("inf")


# ------------------------------------------------------------------- softmax
def test_softmax_fixtures(golden):
    x = parity.from_np(golden.get("softmax_causal_bf16/x"), torch.bfloat16, DEV)
    parity.assert_rel(parity.to_np(K.softmax(x, out_dtype=torch.float32)),
                      golden.get("softmax_causal_bf16/out_f32"), rtol=1e-5, atol=1e-30, what="f32 out")
    parity.assert_ulp(parity.to_np(K.softmax(x)), golden.get("softmax_causal_bf16/out_bf16"), "bf16", 1)
    # in-kernel causal mask on unmasked logits gives the same probabilities
    xu = torch.where(torch.isinf(x), torch.zeros_like(x), x)
    parity.assert_ulp(parity.to_np(K.softmax(xu, causal=True)), golden.get("softmax_causal_bf16/out_bf16"),
                      "bf16", 1, "causal in kernel")
    x16 = parity.from_np(golden.get("softmax_f16/x"), torch.float16, DEV)
    parity.assert_ulp(parity.to_np(K.softmax(x16)), golden.get("softmax_f16/out"), "f16", 1)
    x32 = parity.from_np(golden.get("softmax_f32/x"), torch.float32, DEV)
    parity.assert_rel(parity.to_np(K.softmax(x32)), golden.get("softmax_f32/out"), what="f32")
    parity.assert_rel(parity.to_np(K.softmax(x32, dim=0)), golden.get("softmax_f32/out_dim0"), what="dim0")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 10), (128, 256), (2, 8, 64), (5, 1001), (3, 40000), (64, 4096)])
def test_softmax_shapes(dtype, shape):
    x = rnd(shape, dtype, 32, scale=3.0)
    dt = parity.dname(dtype)
    check_float(K.softmax(x), ops.softmax_golden(parity.to_np(x), dt), dt, f"{shape}")
    if dtype != torch.float32:
        parity.assert_rel(parity.to_np(K.softmax(x, out_dtype=torch.float32)),
                          ops.softmax_golden(parity.to_np(x), "f32"), rtol=1e-5, atol=1e-30)


@pytest.mark.parametrize("L,offset", [(64, 0), (2048, 0), (37, 0), (16, 5), (16, -3)])
def test_causal_softmax(L, offset):
    x = rnd((2, 3, L, L + max(offset, 0)), torch.bfloat16, 33, scale=3.0)
    got = K.softmax(x, causal=True, causal_offset=offset)
    ref = ops.softmax_golden(parity.to_np(x), "bf16", causal=True, offset=offset)
    parity.assert_ulp(parity.to_np(got), ref, "bf16", 1, f"L={L} off={offset}")
    if offset < 0:  # rows with no visible key are all NaN, like softmax of an all -inf row
        assert torch.isnan(got[..., 0, :]).all()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("cols", [512, 1024, 2048, 4096, 8192, 16384, 65536])
def test_softmax_row_rungs(dtype, cols):
    """Every rung of the register-row ladder from 512 to 16384 keys (4..128
    threads per row, up to 8 packs per thread) and the two-pass kernel beyond,
    a ragged last group of rows, causal rows with a partly visible last pack
    and a history offset (the causal kernel runs only its visible pack
    iterations), fp32 output, and rows with a leading stride."""
    dt = parity.dname(dtype)
    x = rnd((37, cols), dtype, 50 + cols, scale=3.0)
    check_float(K.softmax(x), ops.softmax_golden(parity.to_np(x), dt), dt, f"plain {cols}")
    wide = rnd((37, cols + 64), dtype, 51 + cols, scale=3.0)[:, :cols]   # ld = cols + 64
    check_float(K.softmax(wide), ops.softmax_golden(parity.to_np(wide), dt), dt, f"strided {cols}")
    if dtype != torch.float32:
        parity.assert_rel(parity.to_np(K.softmax(x, out_dtype=torch.float32)),
                          ops.softmax_golden(parity.to_np(x), "f32"), rtol=1e-5, atol=1e-30)
    xc = rnd((2, 19, cols), dtype, 52 + cols, scale=3.0)
    for off in (cols // 3 + 1, cols - 19):
        got = K.softmax(xc, causal=True, causal_offset=off)
        ref = ops.softmax_golden(parity.to_np(xc), dt, causal=True, offset=off)
        check_float(got, ref, dt, f"causal {cols} off={off}")
    # rows with no visible key (a negative offset) are all NaN
    got = K.softmax(xc, causal=True, causal_offset=-3)
    assert torch.isnan(got[:, :3]).all() and not torch.isnan(got[:, 3:]).any()


@pytest.mark.parametrize("cols", [2048, 4096])
@pytest.mark.parametrize("causal", [False, True])
def test_softmax_f32_out_both_store_widths(causal, cols):
    """fp32 output of 16-bit rows goes out as 32-byte stores when the output
    is 32-byte aligned and as 16-byte stores otherwise; both match the oracle
    (4096 keys: the causal rows run two warps a row, staged one row ahead)."""
    from torch_fl import _abi

    rows = 96
    x = rnd((rows, cols), torch.bfloat16, 41, scale=3.0)
    ref = ops.softmax_golden(parity.to_np(x).reshape(1, rows, cols), "f32", causal=causal)
    ref = ref.reshape(rows, cols)
    for shift in (0, 4):                                 # 4 floats = 16 bytes off
        buf = torch.full((rows * cols + 8,), float("nan"), device=DEV)
        out = buf[shift:shift + rows * cols]
        assert (out.data_ptr() % 32 == 0) == (shift == 0)
        _abi.call("fl_b200_softmax_lastdim", x.data_ptr(), cols, out.data_ptr(), cols, rows, cols,
                  _abi.BF16, _abi.F32, int(causal), rows, 0,
                  torch.cuda.current_stream().cuda_stream)
        parity.assert_rel(parity.to_np(out).reshape(rows, cols), ref, rtol=1e-5, atol=1e-30,
                          what=f"shift {shift}")
        assert torch.isnan(buf[:shift]).all() and torch.isnan(buf[shift + rows * cols:]).all()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("cols", [40000, 128256, 131072, 40001])
def test_softmax_long_rows_special_values(dtype, cols):
    """Rows over 4096 packs: one thread-block cluster of 3..8 CTAs per row
    up to 16384 packs (40000, 128256 and 131072 16-bit keys; 40000 fp32
    keys), the two-pass kernel beyond (131072 fp32 keys), the unaligned
    loop kernel for 40001 columns (two passes) -- with -inf
    keys, keys far below the max, a one-hot row, a row at the format's
    lowest finite value (fp16 -65504: pass 2 must use the argument pass 1
    summed, else the rounding of m*log2e scales every output by up to
    2^(|m| * 2^-24)), and a NaN or an all -inf row, which come out all NaN."""
    dt = parity.dname(dtype)
    g = torch.Generator().manual_seed(cols + 7)
    x = 3.0 * torch.randn(8, cols, generator=g)
    x[0, ::7] = float("-inf")
    x[1] = -60.0 * torch.rand(cols, generator=g)
    x[1, ::5] = -150.0
    x[2] = float("-inf")
    x[2, cols // 3] = 1.5
    x[3] = torch.finfo(dtype).min
    x[4, 12345] = float("nan")
    x[5] = float("-inf")
    x[6, : cols // 2] = float("-inf")          # the first half of the row masked
    x = x.to(dtype).to(DEV)
    got = K.softmax(x)
    ref = ops.softmax_golden(parity.to_np(x), dt)
    ok = [0, 1, 2, 3, 6, 7]
    check_float(got[ok], ref[ok], dt, f"long {cols}")
    assert torch.isnan(got[4]).all() and torch.isnan(got[5]).all()
    assert got[2, cols // 3].item() == 1.0 and (got[2].float().sum() == 1.0).item()
    if dtype != torch.float32:
        got32 = K.softmax(x, out_dtype=torch.float32)
        ref32 = ops.softmax_golden(parity.to_np(x), "f32")
        parity.assert_rel(parity.to_np(got32[ok]), ref32[ok], rtol=1e-5, atol=1e-30)


@pytest.mark.parametrize("dtype,cols", [(torch.bfloat16, 128256), (torch.float32, 32000),
                                        (torch.float16, 50000)])
def test_softmax_cluster_rows_walk(dtype, cols):
    """Many more rows than resident clusters: each cluster walks several rows
    with the next rows' slices in flight, and the last pass of the walk is
    partial (333 rows)."""
    dt = parity.dname(dtype)
    g = torch.Generator().manual_seed(cols)
    x = (4.0 * torch.randn(333, cols, generator=g)).to(dtype)
    x[7, : cols // 3] = float("-inf")          # a CTA's whole slice masked
    xd = x.to(DEV)
    got = K.softmax(xd)
    check_float(got, ops.softmax_golden(parity.to_np(xd), dt), dt, f"walk {cols}")
    if dtype != torch.float32:
        got32 = K.softmax(xd, out_dtype=torch.float32)
        ref32 = ops.softmax_golden(parity.to_np(xd), "f32")
        parity.assert_rel(parity.to_np(got32), ref32, rtol=1e-5, atol=1e-30)


def test_softmax_infinities():
    x = torch.tensor([[float("-inf")] * 8, [0.0, float("-inf"), 1.0, float("-inf"), 2, 3, 4, 5],
                      [1.0, float("nan"), 2, 3, 4, 5, 6, 7], [float("inf"), 1, 2, 3, 4, 5, 6, 7]])
    for dtype in DTYPES:
        got = parity.to_np(K.softmax(x.to(dtype).to(DEV)))
        ref = torch.softmax(x.to(dtype).float(), -1).numpy()   # torch's own special-value rules
        assert np.array_equal(np.isnan(got), np.isnan(ref)), dtype
        m = ~np.isnan(ref)
        np.testing.assert_allclose(got[m], ref[m], rtol=1e-2, atol=1e-3)


@pytest.mark.slow
def test_causal_softmax_full_size():
    B, H, L = 8, 32, 2048
    g = torch.Generator(device=DEV).manual_seed(34)
    x = (3.0 * torch.randn(B, H, L, L, generator=g, device=DEV)).to(torch.bfloat16)
    plain_in = x.masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool, device=DEV), 1), float("-inf"))
    a = K.softmax(plain_in)
    b = K.softmax(x, causal=True)
    assert torch.equal(a, b)   # reading only the visible keys changes nothing
    idx = [(0, 0), (7, 31), (3, 17)]
    for bi, hi in idx:
        ref = ops.softmax_golden(parity.to_np(x[bi, hi]), "bf16", causal=True)
        parity.assert_ulp(parity.to_np(b[bi, hi]), ref, "bf16", 1, f"slice {bi},{hi}")
    s = b.float().sum(-1)
    assert torch.allclose(s, torch.ones_like(s), atol=2e-2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_causal_softmax_4096_keys(dtype):
    """Causal rows of 4096 16-bit keys (two warps a row, one (max, sum)
    exchange, the visible packs staged one row ahead): every query of 2 x 8
    heads against the oracle, and the in-kernel mask against the same
    logits masked beforehand."""
    B, H, L = 2, 8, 4096
    dt = parity.dname(dtype)
    g = torch.Generator(device=DEV).manual_seed(35)
    x = (3.0 * torch.randn(B, H, L, L, generator=g, device=DEV)).to(dtype)
    got = K.softmax(x, causal=True)
    for bi, hi in [(0, 0), (1, 7), (0, 5)]:
        ref = ops.softmax_golden(parity.to_np(x[bi, hi]), dt, causal=True)
        parity.assert_ulp(parity.to_np(got[bi, hi]), ref, dt, 1, f"slice {bi},{hi}")
    masked = torch.triu(torch.ones(L, L, dtype=torch.bool, device=DEV), 1)
    assert (got[:, :, masked] == 0).all()            # masked keys: exact zeros
    plain = K.softmax(x.masked_fill(masked, float("-inf")))
    # probabilities are >= 0, so 16-bit patterns order like the values: the
    # ulp distance is the difference of the patterns
    d = (got.view(torch.int16).int() - plain.view(torch.int16).int()).abs().max().item()
    assert d <= 1, d


# ---------------------------------------------------------------- reductions
def test_reduction_fixtures(golden):
    xn = golden.get("reduce_f32/x")
    x = parity.from_np(xn, torch.float32, DEV)
    parity.assert_sum(parity.to_np(K.sum_lastdim(x)), xn, -1, "sum_last")
    parity.assert_sum(parity.to_np(K.sum_all(x)), xn, None, "sum_all")
    parity.assert_sum(parity.to_np(K.reduce_middim(x, 0, "sum")), xn, 0, "sum_dim0")
    parity.assert_rel(parity.to_np(K.mean_lastdim(x)), golden.get("reduce_f32/mean_last"), rtol=1e-4,
                      atol=1e-6)
    parity.assert_exact(parity.to_np(K.amax_lastdim(x)), golden.get("reduce_f32/amax_last"), "amax_last")
    parity.assert_exact(parity.to_np(K.amax_all(x)), golden.get("reduce_f32/amax_all"), "amax_all")
    xa = parity.from_np(golden.get("argmax_bf16/x"), torch.bfloat16, DEV)
    parity.assert_exact(K.argmax_lastdim(xa).cpu().numpy(), golden.get("argmax_bf16/out"), "argmax")
    xi = torch.from_numpy(golden.get("sum_i32/x")).to(DEV)
    parity.assert_exact(K.sum_i32_i64(xi, False).cpu().numpy(), golden.get("sum_i32/sum_last"), "int")
    assert int(K.sum_i32_i64(xi, True)) == int(golden.get("sum_i32/sum_all"))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 1), (7, 13), (300, 4096), (3, 1_000_003), (1, 50_000_000)])
def test_float_reductions(dtype, shape):
    x = rnd(shape, dtype, 35)
    xn = parity.to_np(x)
    dt = parity.dname(dtype)
    got = parity.to_np(K.sum_lastdim(x, dtype=torch.float32))
    parity.assert_sum(got, xn, -1, f"sum {shape}", tol=1e-5)
    parity.assert_sum(parity.to_np(K.sum_all(x, dtype=torch.float32)), xn, None, "sum_all")
    if dt != "f32":  # sum returned in the input dtype: fp32 accumulation, one rounding
        parity.assert_sum(parity.to_np(K.sum_lastdim(x)), xn, -1, "sum in dtype",
                          tol=2.0 ** -8 if dt == "bf16" else 2.0 ** -11)
    parity.assert_exact(parity.to_np(K.amax_lastdim(x)), ops.amax(xn, -1), "amax")
    parity.assert_exact(parity.to_np(K.amax_all(x)), ops.amax(xn, None), "amax_all")
    m = parity.to_np(K.mean_lastdim(x, dtype=torch.float32))
    exact = np.mean(xn.astype(np.float64), axis=-1)
    assert np.all(np.abs(m - exact) <= 1e-5 * np.maximum(np.abs(exact),
                                                         np.mean(np.abs(xn), -1) / np.sqrt(shape[-1])))


def test_reductions_are_deterministic():
    x = rnd((2, 20_000_000), torch.float32, 36)    # split across CTAs
    a = K.sum_lastdim(x)
    b = K.sum_lastdim(x)
    assert torch.equal(a, b)
    c = K.sum_all(x)
    assert torch.equal(c, K.sum_all(x))


def test_reductions_nan_and_empty():
    x = torch.zeros(4, 100, device=DEV)
    x[1, 50] = float("nan")
    x[2, :] = float("-inf")
    am = K.amax_lastdim(x).cpu()
    assert torch.isnan(am[1]) and am[2] == float("-inf") and am[0] == 0
    assert torch.isnan(K.amax_all(x).cpu())
    assert int(K.argmax_lastdim(x)[1]) == 50
    e = torch.empty(3, 0, device=DEV)
    assert torch.equal(K.sum_lastdim(e).cpu(), torch.zeros(3))
    assert torch.isnan(K.mean_lastdim(e).cpu()).all()


@pytest.mark.parametrize("cols", [1, 7, 32000, 3_000_001])
def test_argmax_ties_nan_split(cols):
    rows = 5
    g = torch.Generator().manual_seed(37)
    x = torch.randn(rows, cols, generator=g).to(torch.bfloat16)
    if cols > 10:
        x[1, cols // 3] = 50.0
        x[1, cols - 1] = 50.0            # tie across chunks: first wins
        x[2, cols // 2] = float("nan")
        x[2, cols - 2] = float("nan")    # first NaN wins
        x[3, :] = float("-inf")
        x[4, cols // 5] = 4.0            # a max early in the row ...
        x[4, cols // 5 + 1] = 4.0        # ... tied right after it
    got = K.argmax_lastdim(x.to(DEV)).cpu().numpy()
    parity.assert_exact(got, native.argmax_rows_bf16(x.view(torch.int16).numpy().view(np.uint16)), "C oracle")
    parity.assert_exact(got, x.argmax(-1).numpy(), "torch CPU")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("cols", [8, 37, 4096, 100_003])
def test_argmax_dense_ties_all_dtypes(dtype, cols):
    """Ties inside one 16-byte pack and across packs, +-0, NaN and inf
    mixes: the kernel folds whole packs (packed max, then a search of the
    winning pack), and must still return the first index of the maximum."""
    g = torch.Generator().manual_seed(41 + cols)
    x = torch.randint(-3, 4, (7, cols), generator=g).to(dtype)   # many exact ties
    x[1] = 0.0
    x[1, : cols // 2] = -0.0                 # -0 == +0: the first zero wins
    x[2, cols // 3] = float("nan")
    x[3] = float("-inf")
    x[4, 1::3] = float("inf")
    x[4, cols - 1] = float("nan")            # NaN beats inf
    x[5, cols - 1] = 3.5                     # the max in the last element
    x[6] = -1.0
    x[6, cols // 2] = float("-inf")
    got = K.argmax_lastdim(x.to(DEV)).cpu()
    assert torch.equal(got, x.argmax(-1)), (got, x.argmax(-1))


def test_sum_i32_full_size_exact():
    g = torch.Generator().manual_seed(38)
    x = torch.randint(-1000, 1001, (65536, 8192), generator=g, dtype=torch.int32)
    xd = x.to(DEV)
    rows = K.sum_i32_i64(xd, False).cpu().numpy()
    full = int(K.sum_i32_i64(xd, True))
    ref_rows = native.sum_i32_i64_rows(x.numpy())
    parity.assert_exact(rows, ref_rows, "rows")
    assert full == int(ref_rows.sum()) == int(x.numpy().astype(np.int64).sum())


@pytest.mark.slow
def test_argmax_full_size_exact():
    g = torch.Generator(device=DEV).manual_seed(39)
    x = torch.randn(65536, 32000, generator=g, device=DEV).to(torch.bfloat16)
    got = K.argmax_lastdim(x).cpu().numpy()
    ref = native.argmax_rows_bf16(x.cpu().view(torch.int16).numpy().view(np.uint16))
    parity.assert_exact(got, ref, "full-size argmax")


def test_full_size_f32_reductions_properties():
    g = torch.Generator(device=DEV).manual_seed(40)
    x = torch.randn(65536, 8192, generator=g, device=DEV)
    rows_sum = K.sum_lastdim(x)
    total = K.sum_all(x)
    amax_rows = K.amax_lastdim(x)
    # checksum of checksums: the full sum equals the sum of the row sums
    rs = rows_sum.double().sum().item()
    assert abs(total.item() - rs) <= 1e-5 * max(abs(rs), (x.numel() ** 0.5) * 0.8)
    assert K.amax_all(x).item() == amax_rows.max().item()
    sample = [0, 1, 777, 65535]
    xn = x[sample].cpu().numpy()
    parity.assert_sum(rows_sum[sample].cpu().numpy(), xn, -1, "sampled rows")
    parity.assert_exact(amax_rows[sample].cpu().numpy(), ops.amax(xn, -1), "sampled amax")
    # amax of each row is attained in that row (argmax points at it)
    idx = K.argmax_lastdim(x)
    assert torch.equal(x.gather(1, idx[:, None])[:, 0], amax_rows)
