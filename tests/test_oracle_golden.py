"""Pins the oracle (oracle/ops.py) to the golden vectors of the reference's
own path (tests/golden/golden.npz, produced by tests/golden/make_golden.py
from the transformers 5.5.0 modules on torch 2.11 CPU).  CPU only.

The chain flavour must reproduce the reference bit for bit where the
reference's result is determined by exactly-rounded steps (RMSNorm bf16,
RoPE, SwiGLU, softmax); the golden flavour must sit within the stated
tolerance of it.
"""

import numpy as np
import pytest

from oracle import native, ops
from tests import parity


def test_rmsnorm_f32(golden):
    x, w, y = golden.get("rmsnorm_f32/x"), golden.get("rmsnorm_f32/w"), golden.get("rmsnorm_f32/out")
    parity.assert_rel(ops.rms_norm_chain(x, w, 1e-6, "f32"), y, rtol=1e-6, what="chain")
    parity.assert_rel(ops.rms_norm_golden(x, w, 1e-6, "f32"), y, rtol=1e-6, what="golden")


def test_rmsnorm_bf16_chain_bit_exact(golden):
    x, w, y = golden.get("rmsnorm_bf16/x"), golden.get("rmsnorm_bf16/w"), golden.get("rmsnorm_bf16/out")
    parity.assert_ulp(ops.rms_norm_chain(x, w, 1e-5, "bf16"), y, "bf16", max_ulp=0, what="chain")


def test_rmsnorm_bf16_golden_within_1ulp_of_reference(golden):
    x, w, y = golden.get("rmsnorm_bf16/x"), golden.get("rmsnorm_bf16/w"), golden.get("rmsnorm_bf16/out")
    parity.assert_ulp(ops.rms_norm_golden(x, w, 1e-5, "bf16"), y, "bf16", max_ulp=1, what="golden")


def _rope_inputs(golden):
    q, k = golden.get("rope_bf16/q"), golden.get("rope_bf16/k")
    cos, sin = golden.get("rope_bf16/cos")[:, None], golden.get("rope_bf16/sin")[:, None]
    return q, k, cos, sin


def test_rope_chain_bit_exact(golden):
    q, k, cos, sin = _rope_inputs(golden)
    parity.assert_ulp(ops.rope_chain(q, cos, sin, "bf16"), golden.get("rope_bf16/q_out"), "bf16", 0, "q")
    parity.assert_ulp(ops.rope_chain(k, cos, sin, "bf16"), golden.get("rope_bf16/k_out"), "bf16", 0, "k")


@pytest.mark.parametrize("fixture", ["rope_bf16", "rope_bf16_far"])
def test_rope_tables_are_hf_tables(golden, fixture):
    # The oracle's cos/sin must be the transformers module's own tables, bit
    # for bit, at the 8192-token config's positions and at stack-scale ones
    # (up to 131071, where one ulp of inv_freq moves cos by ~145 bf16 ulp).
    pos = golden.get(f"{fixture}/pos")[0]
    c, s = ops.rope_tables(pos, 128, 1e4, "bf16")
    parity.assert_ulp(c, golden.get(f"{fixture}/cos")[0], "bf16", 0, "cos")
    parity.assert_ulp(s, golden.get(f"{fixture}/sin")[0], "bf16", 0, "sin")
    if fixture == "rope_bf16_far":
        c32, s32 = ops.rope_tables(pos, 128, 1e4, "f32")
        assert np.array_equal(c32, golden.get(f"{fixture}/cos_f32")[0])
        assert np.array_equal(s32, golden.get(f"{fixture}/sin_f32")[0])


def test_rope_chain_bit_exact_far_positions(golden):
    q, k = golden.get("rope_bf16_far/q"), golden.get("rope_bf16_far/k")
    pos = golden.get("rope_bf16_far/pos")[0]
    c, s = ops.rope_tables(pos, 128, 1e4, "bf16")
    cos, sin = c[None, None], s[None, None]
    parity.assert_ulp(ops.rope_chain(q, cos, sin, "bf16"), golden.get("rope_bf16_far/q_out"),
                      "bf16", 0, "q")
    parity.assert_ulp(ops.rope_chain(k, cos, sin, "bf16"), golden.get("rope_bf16_far/k_out"),
                      "bf16", 0, "k")


def test_rope_golden_is_the_single_rounding(golden):
    # The reference rounds three times (two products, one sum), so where the
    # sum cancels it is far, in ulps of the result, from the single-rounded
    # value (up to ~15k ulp on these inputs); the single-rounded value is
    # within 1 ulp of the exact one by construction.  Where the result keeps
    # at least half the magnitude of its terms the two agree within 2 ulp.
    q, k, cos, sin = _rope_inputs(golden)
    g = ops.rope_golden(q, cos, sin, "bf16")
    ref = golden.get("rope_bf16/q_out")
    big = np.abs(q * cos) + np.abs(ops._rotate_half(q) * sin)
    no_cancel = np.abs(ref) > 0.5 * big
    d = ops.ulp_diff(g[no_cancel], ref[no_cancel], "bf16")
    assert d.max() <= 2


def test_qknorm_rope_chain(golden):
    q, k, cos, sin = _rope_inputs(golden)
    wq, wk = golden.get("qknorm_rope_bf16/wq"), golden.get("qknorm_rope_bf16/wk")
    d = parity.assert_ulp(ops.rms_norm_rope_chain(q, wq, cos, sin, 1e-6, "bf16"),
                          golden.get("qknorm_rope_bf16/q_out"), "bf16", 1, "q")
    assert np.mean(d == 0) > 0.999
    parity.assert_ulp(ops.rms_norm_rope_chain(k, wk, cos, sin, 1e-6, "bf16"),
                      golden.get("qknorm_rope_bf16/k_out"), "bf16", 1, "k")


def test_swiglu(golden):
    g, u, y = golden.get("swiglu_bf16/gate"), golden.get("swiglu_bf16/up"), golden.get("swiglu_bf16/out")
    parity.assert_ulp(ops.swiglu_chain(g, u, "bf16"), y, "bf16", 0, "chain")
    parity.assert_ulp(ops.swiglu_golden(g, u, "bf16"), y, "bf16", 1, "golden")


def test_softmax(golden):
    x = golden.get("softmax_causal_bf16/x")
    parity.assert_rel(ops.softmax_golden(x, "f32"), golden.get("softmax_causal_bf16/out_f32"),
                      rtol=1e-5, atol=1e-30, what="causal f32")
    parity.assert_ulp(ops.softmax_golden(x, "bf16"), golden.get("softmax_causal_bf16/out_bf16"),
                      "bf16", 0, "causal bf16")
    # The in-kernel mask formulation equals softmax of the pre-masked logits.
    unmasked = np.where(np.isinf(x), 0.0, x)
    parity.assert_ulp(ops.softmax_golden(unmasked, "bf16", causal=True),
                      golden.get("softmax_causal_bf16/out_bf16"), "bf16", 0, "mask")
    parity.assert_ulp(ops.softmax_golden(golden.get("softmax_f16/x"), "f16"),
                      golden.get("softmax_f16/out"), "f16", 0, "f16")
    x32 = golden.get("softmax_f32/x")
    parity.assert_rel(ops.softmax_golden(x32, "f32"), golden.get("softmax_f32/out"), what="f32")
    parity.assert_rel(ops.softmax_dim_golden(x32, 0, "f32"), golden.get("softmax_f32/out_dim0"),
                      what="dim0")


def test_softmax_special_rows_match_torch():
    """The oracle's softmax on the rows the long-row GPU test uses, against
    torch's own fp64 softmax: -inf keys, keys far below the max, one-hot,
    a row at each format's lowest finite value (uniform), and NaN / all -inf
    rows (all NaN)."""
    import torch

    for dtype, dt in ((torch.float32, "f32"), (torch.bfloat16, "bf16"), (torch.float16, "f16")):
        g = torch.Generator().manual_seed(3)
        x = 3.0 * torch.randn(7, 4096, generator=g)
        x[0, ::7] = float("-inf")
        x[1] = -60.0 * torch.rand(4096, generator=g)
        x[1, ::5] = -150.0
        x[2] = float("-inf")
        x[2, 100] = 1.5
        x[3] = torch.finfo(dtype).min
        x[4, 123] = float("nan")
        x[5] = float("-inf")
        x = x.to(dtype)
        xn = parity.to_np(x)
        ref = torch.softmax(x.double(), -1).numpy()
        got = ops.softmax_golden(xn, "f32")
        assert np.array_equal(np.isnan(got), np.isnan(ref)), dt
        assert np.isnan(got[4]).all() and np.isnan(got[5]).all()
        ok = [0, 1, 2, 3, 6]
        parity.assert_rel(got[ok], ref[ok].astype(np.float32), rtol=1e-6, atol=1e-38, what=dt)
        assert got[2, 100] == 1.0 and np.all(got[3] == np.float32(1.0 / 4096))


def test_float_reductions(golden):
    x = golden.get("reduce_f32/x")
    # torch's own fp32 sums meet the stated sum tolerance against fp64
    parity.assert_sum(golden.get("reduce_f32/sum_last"), x, -1, "torch sum_last")
    parity.assert_sum(golden.get("reduce_f32/sum_all"), x, None, "torch sum_all")
    parity.assert_sum(golden.get("reduce_f32/sum_dim0"), x, 0, "torch sum_dim0")
    parity.assert_sum(ops.sum_golden(x, -1, "f32"), x, -1, "oracle sum_last")
    parity.assert_rel(ops.mean_golden(x, None, "f32"), golden.get("reduce_f32/mean_all"), rtol=1e-5)
    parity.assert_exact(ops.amax(x, -1), golden.get("reduce_f32/amax_last"), "amax_last")
    parity.assert_exact(ops.amax(x, None), golden.get("reduce_f32/amax_all"), "amax_all")


def test_argmax_exact(golden):
    x = golden.get("argmax_bf16/x")
    ref = golden.get("argmax_bf16/out")
    parity.assert_exact(ops.argmax_first(x, -1), ref, "numpy oracle")
    parity.assert_exact(native.argmax_rows_bf16(ops.bf16_bits(x)), ref, "C oracle")
    assert ref[3] == 100 and ref[5] == 7 and ref[6] == 0  # planted tie / NaN / all -inf


def test_int_sums_exact(golden):
    x = golden.get("sum_i32/x")
    parity.assert_exact(ops.sum_i32_i64(x, -1), golden.get("sum_i32/sum_last"), "numpy")
    parity.assert_exact(native.sum_i32_i64_rows(x), golden.get("sum_i32/sum_last"), "C")
    assert int(ops.sum_i32_i64(x)) == int(golden.get("sum_i32/sum_all"))


def test_add_mul(golden):
    a, b = golden.get("add_bf16/a"), golden.get("add_bf16/b")
    parity.assert_ulp(ops.add_golden(a, b, 1.0, "bf16"), golden.get("add_bf16/out"), "bf16", 0)
    parity.assert_ulp(ops.add_golden(a, b, 2.5, "bf16"), golden.get("add_bf16/out_alpha"), "bf16", 1)
    x, y = golden.get("residual_bf16/x"), golden.get("residual_bf16/y")
    parity.assert_ulp(ops.add_golden(x, y, 1.0, "bf16"), golden.get("residual_bf16/out"), "bf16", 0)
    w, h, c = golden.get("mul_bf16/w"), golden.get("mul_bf16/h"), golden.get("mul_bf16/c")
    parity.assert_ulp(ops.mul_golden(w, h, "bf16"), golden.get("mul_bf16/w_h"), "bf16", 0)
    parity.assert_ulp(ops.mul_golden(h, c, "bf16"), golden.get("mul_bf16/h_c"), "bf16", 0)


def test_amax_c_oracle_nan():
    x = np.array([[1.0, np.nan, 5.0], [-np.inf, -np.inf, -np.inf], [2.0, 3.0, 1.0]], np.float32)
    out = native.amax_rows_f32(x)
    assert np.isnan(out[0]) and out[1] == -np.inf and out[2] == 3.0
    parity.assert_exact(ops.amax(x, -1), out)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_ulp_distance(dtype):
    a = ops.round_to(np.array([1.0, -1.0, 0.0, 3.0], np.float32), dtype)
    step = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    b = ops.round_to(np.array([1.0 + step, -1.0 - step, -0.0, 3.0], np.float32), dtype)
    assert list(ops.ulp_diff(a, b, dtype)) == [1, 1, 0, 0]


# --------------------------------------------------------------- backward ---
# torch CPU autograd of the transformers modules (fp32) against the oracle's
# fp64 gradients: agreement to fp32 accuracy, scaled by the magnitude of the
# terms where they cancel.


def test_rmsnorm_backward_oracle_matches_autograd(golden):
    x, w, dy = (golden.get(f"rmsnorm_bwd_f32/{k}") for k in ("x", "w", "dy"))
    dx, dw = ops.rms_norm_bwd_golden(x, w, dy, 1e-6, "f32")
    bound = ops.rms_norm_bwd_bound(x, w, dy, 1e-6)
    parity.assert_within(dx, golden.get("rmsnorm_bwd_f32/dx"), 4 * parity.BWD_TERM_TOL * bound,
                         "dx")
    r = 1.0 / np.sqrt(np.mean(x.astype(np.float64) ** 2, -1, keepdims=True) + 1e-6)
    terms = np.sum(np.abs(dy * x * r), axis=0)
    parity.assert_within(dw, golden.get("rmsnorm_bwd_f32/dw"), 1e-5 * terms, "dw")


def test_swiglu_backward_oracle_matches_autograd(golden):
    g, u, d = (golden.get(f"swiglu_bwd_f32/{k}") for k in ("gate", "up", "dout"))
    dg, du = ops.swiglu_bwd_golden(d, g, u, "f32")
    scale = np.abs(d) * (np.abs(u) * (1 + np.abs(g)) + np.abs(g))
    parity.assert_within(dg, golden.get("swiglu_bwd_f32/dgate"), 1e-6 * scale, "dgate")
    parity.assert_within(du, golden.get("swiglu_bwd_f32/dup"), 1e-6 * scale, "dup")
    # the silu part alone is silu_backward (dout * u as its incoming grad)
    parity.assert_within(ops.silu_bwd_golden(d * u, g, "f32"),
                         golden.get("swiglu_bwd_f32/dgate"), 1e-6 * scale, "silu_backward")


def test_softmax_backward_oracle_matches_autograd(golden):
    x, dy = golden.get("softmax_bwd_f32/x"), golden.get("softmax_bwd_f32/dy")
    y = ops.softmax_golden(x, "f32")
    parity.assert_within(ops.softmax_bwd_golden(dy, y, "f32"), golden.get("softmax_bwd_f32/dx"),
                         4 * parity.BWD_TERM_TOL * ops.softmax_bwd_bound(dy, y), "dx")
    # half_to_float: fp32 probabilities and grads back to bf16 logits
    y, dy = golden.get("softmax_bwd_half_to_float/y"), golden.get("softmax_bwd_half_to_float/dy")
    parity.assert_within(ops.softmax_bwd_golden(dy, y, "bf16"),
                         golden.get("softmax_bwd_half_to_float/dx"),
                         4 * parity.BWD_TERM_TOL * ops.softmax_bwd_bound(dy, y), "dx bf16",
                         dtype="bf16")


def test_rope_backward_oracle_matches_autograd(golden):
    cos, sin = golden.get("rope_bwd_f32/cos")[:, None], golden.get("rope_bwd_f32/sin")[:, None]
    for name in ("q", "k"):
        d = golden.get(f"rope_bwd_f32/d{name}_out")
        got = ops.rope_bwd_golden(d, cos, sin, "f32")
        parity.assert_rel(got, golden.get(f"rope_bwd_f32/d{name}"), rtol=1e-6, atol=1e-6, what=name)
        # the adjoint is the forward rotation with -sin (cos/sin halves repeat)
        parity.assert_rel(ops.rope_golden(d, cos, -sin, "f32"), got, rtol=1e-7, atol=1e-7,
                          what=f"{name} via -sin")


def _masked_inputs(golden):
    s = float(golden.get("masked_softmax_bf16/scaling")[0])
    return golden.get("masked_softmax_bf16/w"), golden.get("masked_softmax_bf16/mask"), s


def test_masked_softmax_logits_chain_bit_exact(golden):
    # HF eager attention: `w * scaling + mask` as two rounded bf16 ops
    w, mask, s = _masked_inputs(golden)
    parity.assert_exact(ops.masked_logits_chain(w, mask, s, "bf16"),
                        golden.get("masked_softmax_bf16/z32"), "logits")


def test_masked_softmax_oracle_matches_hf_eager_attention(golden):
    w, mask, s = _masked_inputs(golden)
    ref = golden.get("masked_softmax_bf16/attn_weights")
    # the padding queries of batch 1 see no key: uniform rows, not NaN
    np.testing.assert_array_equal(ref[1, :, :5, :], np.float32(1.0 / 64))
    # The chain flavour is pinned to the reference.  (The fused flavour is
    # not: the reference rounds each logit to bf16 after the scale, a 2^-9
    # relative change of the logit that alone moves exp by about one ulp.)
    parity.assert_ulp(ops.masked_softmax_chain(w, mask, s, "bf16", "bf16"), ref, "bf16", 1, "chain")
    d = ops.ulp_diff(ops.masked_softmax_chain(w, mask, s, "bf16", "bf16"), ref, "bf16")
    assert np.mean(d == 0) > 0.99
    z = golden.get("masked_softmax_bf16/z32")
    parity.assert_rel(ops.softmax_golden(z, "f32"), golden.get("masked_softmax_bf16/z32_softmax"),
                      what="softmax of the masked fp32 logits")
    wf, mf = golden.get("masked_softmax_f32/w"), golden.get("masked_softmax_f32/mask")
    assert mf.min() == np.finfo(np.float32).min
    parity.assert_rel(ops.masked_softmax_golden(wf, mf, s, "f32"), golden.get("masked_softmax_f32/out"),
                      what="f32")


def test_masked_softmax_backward_oracle_matches_autograd(golden):
    w, mask, s = _masked_inputs(golden)
    dy = golden.get("masked_softmax_bf16/dy")
    y = ops.masked_softmax_chain(w, mask, s, "bf16", "f32")
    # The reference's backward uses its own fp32 probabilities (of the
    # bf16-rounded logits) and rounds the softmax's input gradient to bf16
    # before the scale: one more bf16 rounding than the fused formula.
    parity.assert_within(ops.softmax_bwd_golden(dy, y, "bf16", s), golden.get("masked_softmax_bf16/dw"),
                         s * (4 * parity.BWD_TERM_TOL * ops.softmax_bwd_bound(dy, y)
                              + parity.ulp_of(ops.softmax_bwd_golden(dy, y, "f32"), "bf16")),
                         "dw", dtype="bf16")
