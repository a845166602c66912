"""Parity of flagos::masked_softmax (HF eager attention's scale + mask +
softmax + cast tail in one launch) and of the softmax kernels on rows masked
with the lowest finite value.

Tolerances (tests/parity.py): chain rounding against the reference's own
output (tests/golden, transformers' eager_attention_forward on torch CPU)
within 1 ulp; fused rounding within 1 ulp of the fp64 formula for 16-bit
outputs, 1e-5 relative for fp32 outputs; gradients within BWD_TERM_TOL of
the magnitude of their terms plus 1 ulp of a 16-bit output.
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


def rnd(shape, dtype, seed, scale=1.0, device=DEV):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).to(dtype).to(device)


def hf_mask(B, Q, Kn, dtype, pad=(), device=DEV):
    """HF's eager mask: 0 where visible (causal, keys not padding), the
    dtype's lowest value elsewhere; `pad[b]` left-padding tokens in batch b."""
    i = torch.arange(Q)[:, None] + (Kn - Q)
    j = torch.arange(Kn)[None, :]
    vis = (j <= i)[None].repeat(B, 1, 1)
    for b, p in enumerate(pad):
        vis[b, :, :p] = False
    lo = torch.finfo(dtype).min
    m = torch.where(vis, torch.tensor(0.0), torch.tensor(lo))
    return m[:, None].to(dtype).to(device)


def _check(y, x, mask, scale, out_dt, what):
    xn = parity.to_np(x)
    mn = None if mask is None else parity.to_np(mask)
    ref = ops.masked_softmax_golden(xn, mn, scale, out_dt)
    if out_dt == "f32":
        parity.assert_rel(parity.to_np(y), ref, what=what)
    else:
        parity.assert_ulp(parity.to_np(y), ref, out_dt, 1, what)


def test_masked_softmax_matches_hf_eager_attention(golden):
    """The golden fixture: transformers' eager mask with a left-padded batch,
    the bf16 logits of q @ k^T; chain rounding reproduces the reference's
    attention weights within 1 ulp, and the padding queries' rows (no
    visible key) are uniform like the reference's."""
    w = torch.from_numpy(golden.get("masked_softmax_bf16/w")).to(torch.bfloat16).to(DEV)
    mask = torch.from_numpy(golden.get("masked_softmax_bf16/mask")).to(torch.bfloat16).to(DEV)
    s = float(golden.get("masked_softmax_bf16/scaling")[0])
    ref = golden.get("masked_softmax_bf16/attn_weights")
    y = K.masked_softmax(w, mask, s, rounding="chain")
    assert y.dtype == torch.bfloat16 and y.shape == w.shape
    got = parity.to_np(y)
    parity.assert_ulp(got, ref, "bf16", 1, "chain vs reference")
    np.testing.assert_array_equal(got[1, :, :5, :], np.float32(1.0 / 64))
    yf = K.masked_softmax(w, mask, s)                       # fused rounding
    _check(yf, w, mask, s, "bf16", "fused")
    # fp32 model: the mask holds float32's lowest value
    wf = torch.from_numpy(golden.get("masked_softmax_f32/w")).to(DEV)
    mf = torch.from_numpy(golden.get("masked_softmax_f32/mask")).to(DEV)
    parity.assert_rel(parity.to_np(K.masked_softmax(wf, mf, s)),
                      golden.get("masked_softmax_f32/out"), what="f32")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape,mask_kind", [
    ((2, 4, 64, 64), "hf"),            # HF [B, 1, Q, K]
    ((1, 8, 100, 100), "hf"),          # ragged width: the looped kernel for 16-bit
    ((2, 2, 16, 2048), "hf"),          # decode-like: few queries, long keys
    ((1, 2, 8, 5001), "full"),         # ragged long rows: the looped kernel
    ((1, 1, 4, 40000), "full"),        # past the row ladder
    ((2, 3, 24, 256), "full"),         # a mask per head
    ((2, 2, 32, 128), "pad"),          # [B, 1, 1, K] padding-only mask
    ((1, 4, 32, 512), "none"),
    ((32, 256), "shared"),             # [Q, K] logits, [Q, K] mask
    # rows of 257..512 packs: one warp per row, staged in shared memory
    ((2, 4, 16, 4096), "hf"),          # HF mask, padding queries at the lowest value
    ((1, 5, 8, 4096), "hf"),           # 5 heads: head-inner order across CTA warps
    ((1, 3, 8, 2056), "full"),         # 257 packs (16-bit), a mask per head
    ((2, 2, 8, 4096), "pad"),          # [B, 1, 1, K]: mask shared by heads and queries
    ((1, 2, 8, 4096), "none"),
])
def test_masked_softmax_fused_vs_oracle(dtype, shape, mask_kind):
    x = rnd(shape, dtype, 70, scale=4.0)
    B, H, Q, Kn = (1,) * (4 - len(shape)) + shape
    if mask_kind == "hf":
        mask = hf_mask(B, Q, Kn, dtype, pad=(3,) if B > 1 else ())
    elif mask_kind == "full":
        mask = rnd((B, H, Q, Kn), dtype, 71, scale=2.0)
    elif mask_kind == "pad":
        mask = hf_mask(B, 1, Kn, dtype, pad=(0, 9))[:, :, :1, :]
        mask[:, :, :, Kn // 2:] = 0
    elif mask_kind == "shared":
        mask = rnd((Q, Kn), dtype, 72, scale=2.0)
    else:
        mask = None
    s = 0.0883883476
    dt = parity.dname(dtype)
    y = K.masked_softmax(x, mask, s)
    _check(y, x, mask, s, dt, f"{shape} {mask_kind}")
    if dtype != torch.float32:
        y32 = K.masked_softmax(x, mask, s, out_dtype=torch.float32)
        assert y32.dtype == torch.float32
        _check(y32, x, mask, s, "f32", f"{shape} {mask_kind} f32 out")
    # chain rounding: the op-by-op logits, then the fp32 softmax rounded once
    yc = K.masked_softmax(x, mask, s, rounding="chain")
    mn = None if mask is None else parity.to_np(mask)
    z = ops.masked_logits_chain(parity.to_np(x), mn, s, dt)
    ref = ops.softmax_golden(z, dt)
    if dt == "f32":
        parity.assert_rel(parity.to_np(yc), ref, what="chain")
    else:
        parity.assert_ulp(parity.to_np(yc), ref, dt, 1, "chain")


def test_masked_softmax_strided_rows_and_flagos_op():
    # logits with a leading stride (a slice of wider rows), through the aten op
    base = rnd((2, 4, 64, 128 + 64), torch.bfloat16, 73, scale=3.0)
    x = base[..., :128]
    mask = hf_mask(2, 64, 128, torch.bfloat16, pad=(0, 7))
    y = torch.ops.flagos.masked_softmax(x, mask, 0.125, None, "fused")
    _check(y, x, mask, 0.125, "bf16", "strided")
    assert torch.equal(y, K.masked_softmax(x.contiguous(), mask, 0.125))
    xf = torch_fl.kernels.masked_softmax(x.to("flagos"), mask.to("flagos"), 0.125)
    assert xf.device.type == "flagos" and torch.equal(xf.cpu(), y.cpu())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_softmax_rows_at_the_lowest_finite_value(golden, dtype):
    """_softmax on logits HF masked op by op (the flagos path without the
    attention hook): rows whose keys all hold the lowest finite value come
    out uniform, as in the reference, not NaN."""
    z = torch.from_numpy(golden.get("masked_softmax_bf16/z32")).to(DEV)
    parity.assert_rel(parity.to_np(K.softmax(z)), golden.get("masked_softmax_bf16/z32_softmax"),
                      what="f32 logits")
    lo = torch.finfo(dtype).min
    dt = parity.dname(dtype)
    # row ladder rungs (64, 2048, 4096 keys), the 16-pack rung (4096 f16-wide
    # rows are bf16 here: 512 packs), the looped kernel (ragged, long rows)
    for cols in (64, 2048, 4096, 100, 9000):
        x = torch.full((4, cols), lo, dtype=dtype, device=DEV)
        x[1, 3] = 0.5                                   # one row with a visible key
        y = parity.to_np(K.softmax(x, out_dtype=torch.float32))
        parity.assert_rel(y, ops.softmax_golden(parity.to_np(x), "f32"), what=f"{cols} keys")
        y = parity.to_np(K.softmax(x))
        ref = ops.softmax_golden(parity.to_np(x), dt)
        if dt == "f32":
            parity.assert_rel(y, ref, what=f"{cols} keys, {dt} out")
        else:
            parity.assert_ulp(y, ref, dt, 1, f"{cols} keys, {dt} out")
    # the causal kernel too: causal rows whose visible keys are all masked
    x = torch.full((2, 8, 64), lo, dtype=dtype, device=DEV)
    y = parity.to_np(K.softmax(x, causal=True))
    ref = ops.softmax_golden(parity.to_np(x), dt, causal=True)
    if dt == "f32":
        parity.assert_rel(y, ref, what="causal")
    else:
        parity.assert_ulp(y, ref, dt, 1, "causal")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(64, 64), (2, 4, 64, 2048), (3, 100), (2, 5000)])
def test_softmax_backward_scaled(dtype, shape):
    y = torch.softmax(rnd(shape, torch.float32, 74, scale=3.0), -1).to(dtype)
    dy = rnd(shape, dtype, 75)
    s = 0.0883883476
    dx = K.softmax_backward(dy, y, scale=s)
    dt = parity.dname(dtype)
    yn, gn = parity.to_np(y), parity.to_np(dy)
    parity.assert_within(parity.to_np(dx), ops.softmax_bwd_golden(gn, yn, dt, s),
                         s * parity.BWD_TERM_TOL * ops.softmax_bwd_bound(gn, yn), f"dx {shape}",
                         dt if dt != "f32" else None)
    # scale 1 is the plain backward; same inputs, same bits
    assert torch.equal(K.softmax_backward(dy, y, scale=1.0), K.softmax_backward(dy, y))


def test_masked_softmax_autograd_on_flagos(golden):
    """Gradient of the fused op on flagos tensors against the reference's
    autograd through the HF chain (tests/golden: torch CPU)."""
    from torch_fl import ops as fops

    s = float(golden.get("masked_softmax_bf16/scaling")[0])
    w = torch.from_numpy(golden.get("masked_softmax_bf16/w")).to(torch.bfloat16).to("flagos")
    mask = torch.from_numpy(golden.get("masked_softmax_bf16/mask")).to(torch.bfloat16).to("flagos")
    dy = torch.from_numpy(golden.get("masked_softmax_bf16/dy")).to(torch.bfloat16).to("flagos")
    wg = w.clone().requires_grad_(True)
    y = fops.masked_softmax(wg, mask, s, rounding="chain")
    y.backward(dy)
    dyn = golden.get("masked_softmax_bf16/dy")
    yc = ops.masked_softmax_chain(golden.get("masked_softmax_bf16/w"),
                                  golden.get("masked_softmax_bf16/mask"), s, "bf16", "f32")
    ref = golden.get("masked_softmax_bf16/dw")
    # fused gradient from the bf16-rounded probabilities vs the reference's
    # fp32 ones: the probability rounding (2^-9 relative) enters through y
    # and through sum(dy y); the reference adds one bf16 rounding before the
    # scale
    bound = ops.softmax_bwd_bound(dyn, yc)
    tol = s * (2.0 ** -8 * bound + parity.ulp_of(ops.softmax_bwd_golden(dyn, yc, "f32"), "bf16"))
    parity.assert_within(parity.to_np(wg.grad), ref, tol, "dw", "bf16")
    # and the mask's gradient when it asks for one: the unscaled product
    # summed over the heads it broadcasts to
    mg = mask.clone().requires_grad_(True)
    y2 = fops.masked_softmax(w, mg, s)
    y2.backward(dy)
    y2n = parity.to_np(y2)
    dz = ops.softmax_bwd_golden(dyn, y2n, "f32").sum(axis=1, keepdims=True)
    parity.assert_within(parity.to_np(mg.grad), dz,
                         2.0 ** -7 * ops.softmax_bwd_bound(dyn, y2n).sum(axis=1, keepdims=True),
                         "dmask", "bf16")
