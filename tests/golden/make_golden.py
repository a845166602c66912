"""Generate tests/golden/golden.npz: golden vectors of the reference's own path.

The reference computes RMSNorm, RoPE and SwiGLU as the HuggingFace formulas
(transformers models/qwen3/modeling_qwen3.py) over aten ops, and softmax /
sum / mean / amax / argmax / add / mul as aten ops.  This script runs exactly
that on torch CPU (PyTorch 2.11, the version the reference pins), using the
transformers 5.5.0 modules themselves where they exist (Qwen3RMSNorm,
Qwen3RotaryEmbedding, apply_rotary_pos_emb, ACT2FN["silu"]), on seeded
inputs with the distributions of the benchmark configs, and stores inputs and
outputs.  It also checks that oracle/hf_chain.py (the restated formulas used
as the CPU baseline) reproduces the transformers modules bit for bit.

Run from the repository root:  python tests/golden/make_golden.py
bf16 arrays are stored as uint16 bit patterns under keys ending in ':bf16'.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import hf_chain  # noqa: E402

OUT = os.path.join(HERE, "golden.npz")


def _store(d: dict, key: str, t: torch.Tensor) -> None:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        d[key + ":bf16"] = t.view(torch.int16).numpy().view(np.uint16)
    elif t.dtype == torch.float16:
        d[key + ":f16"] = t.numpy()
    elif t.dtype == torch.float32:
        d[key + ":f32"] = t.numpy()
    elif t.dtype in (torch.int32, torch.int64):
        d[key + ":int"] = t.numpy()
    else:
        raise TypeError(t.dtype)


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def main() -> None:
    from transformers.activations import ACT2FN
    from transformers.models.qwen3 import modeling_qwen3 as mq
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    d: dict[str, np.ndarray] = {}

    # --- RMSNorm, fp32, the CPU-oracle config's distribution (eps 1e-6, seed 0)
    g = _gen(0)
    x = torch.randn(16, 4096, generator=g)
    w = 1 + 0.1 * torch.randn(4096, generator=g)
    mod = mq.Qwen3RMSNorm(4096, eps=1e-6)
    with torch.no_grad():
        mod.weight.copy_(w)
        y = mod(x)
    assert torch.equal(y, hf_chain.rms_norm(x, w, 1e-6))
    _store(d, "rmsnorm_f32/x", x)
    _store(d, "rmsnorm_f32/w", w)
    _store(d, "rmsnorm_f32/out", y)

    # --- RMSNorm, bf16, the decoder-chain config (eps 1e-5)
    g = _gen(1)
    x = torch.randn(16, 4096, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    mod = mq.Qwen3RMSNorm(4096, eps=1e-5).to(torch.bfloat16)
    with torch.no_grad():
        mod.weight.copy_(w)
        y = mod(x)
    assert torch.equal(y, hf_chain.rms_norm(x, w, 1e-5))
    _store(d, "rmsnorm_bf16/x", x)
    _store(d, "rmsnorm_bf16/w", w)
    _store(d, "rmsnorm_bf16/out", y)

    # --- RoPE tables + apply, bf16, theta 1e4, head dim 128; positions cover
    # the start and the end of the 8192-token config.
    cfg = Qwen3Config(head_dim=128, hidden_size=4096, num_attention_heads=32,
                      num_key_value_heads=8, max_position_embeddings=8192,
                      rope_parameters={"rope_type": "default", "rope_theta": 10000.0})
    rot = mq.Qwen3RotaryEmbedding(cfg)
    pos = torch.tensor([list(range(0, 8)) + list(range(8184, 8192))], dtype=torch.int64)
    S = pos.shape[1]
    g = _gen(2)
    q = torch.randn(1, S, 32, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(1, S, 8, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    with torch.no_grad():
        cos, sin = rot(q, pos)
    c2, s2 = hf_chain.rope_tables(pos, 128, 10000.0, torch.bfloat16)
    assert torch.equal(cos, c2) and torch.equal(sin, s2)
    qe, ke = mq.apply_rotary_pos_emb(q, k, cos, sin)
    qe2, ke2 = hf_chain.rope(q, k, cos, sin)
    assert torch.equal(qe, qe2) and torch.equal(ke, ke2)
    _store(d, "rope_bf16/pos", pos)
    _store(d, "rope_bf16/q", q.contiguous())       # [B, H, S, D]
    _store(d, "rope_bf16/k", k.contiguous())
    _store(d, "rope_bf16/cos", cos)                # [B, S, D]
    _store(d, "rope_bf16/sin", sin)
    _store(d, "rope_bf16/q_out", qe.contiguous())
    _store(d, "rope_bf16/k_out", ke.contiguous())

    # --- Qwen3 q_norm / k_norm (RMSNorm over the head dim, eps 1e-6) then RoPE
    wq = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    qn_mod = mq.Qwen3RMSNorm(128, eps=1e-6).to(torch.bfloat16)
    kn_mod = mq.Qwen3RMSNorm(128, eps=1e-6).to(torch.bfloat16)
    with torch.no_grad():
        qn_mod.weight.copy_(wq)
        kn_mod.weight.copy_(wk)
        qn = qn_mod(q)
        kn = kn_mod(k)
    qe, ke = mq.apply_rotary_pos_emb(qn, kn, cos, sin)
    _store(d, "qknorm_rope_bf16/wq", wq)
    _store(d, "qknorm_rope_bf16/wk", wk)
    _store(d, "qknorm_rope_bf16/q_out", qe.contiguous())
    _store(d, "qknorm_rope_bf16/k_out", ke.contiguous())

    # --- RoPE at stack-scale positions (the 131072-token stack's last rows and
    # the 2^16 boundary), where a last-bit difference in inv_freq is magnified
    # by the position; tables from the transformers module itself.
    pos_far = torch.tensor([[8191, 16383, 32767, 65535, 65536, 98304, 114688, 131070, 131071]],
                           dtype=torch.int64)
    Sf = pos_far.shape[1]
    g = _gen(15)
    qf_ = torch.randn(1, Sf, 32, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    kf_ = torch.randn(1, Sf, 8, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    with torch.no_grad():
        cos_f, sin_f = rot(qf_, pos_far)
        cos_f32, sin_f32 = rot(qf_.float(), pos_far)
    c2, s2 = hf_chain.rope_tables(pos_far, 128, 10000.0, torch.bfloat16)
    assert torch.equal(cos_f, c2) and torch.equal(sin_f, s2)
    qe, ke = mq.apply_rotary_pos_emb(qf_, kf_, cos_f, sin_f)
    _store(d, "rope_bf16_far/pos", pos_far)
    _store(d, "rope_bf16_far/q", qf_.contiguous())
    _store(d, "rope_bf16_far/k", kf_.contiguous())
    _store(d, "rope_bf16_far/cos", cos_f)
    _store(d, "rope_bf16_far/sin", sin_f)
    _store(d, "rope_bf16_far/cos_f32", cos_f32)
    _store(d, "rope_bf16_far/sin_f32", sin_f32)
    _store(d, "rope_bf16_far/q_out", qe.contiguous())
    _store(d, "rope_bf16_far/k_out", ke.contiguous())

    # --- SwiGLU, bf16 (act_fn = silu)
    g = _gen(3)
    gate = torch.randn(16, 1024, generator=g).to(torch.bfloat16)
    up = torch.randn(16, 1024, generator=g).to(torch.bfloat16)
    a = ACT2FN["silu"](gate) * up
    assert torch.equal(a, hf_chain.swiglu(gate, up))
    _store(d, "swiglu_bf16/gate", gate)
    _store(d, "swiglu_bf16/up", up)
    _store(d, "swiglu_bf16/out", a)

    # --- causal softmax, bf16 logits ~ N(0, 3^2), upper triangle -inf
    g = _gen(4)
    L = 64
    logits = (3.0 * torch.randn(2, 4, L, L, generator=g)).to(torch.bfloat16)
    mask = torch.triu(torch.ones(L, L, dtype=torch.bool), diagonal=1)
    logits = logits.masked_fill(mask, float("-inf"))
    p32 = torch.softmax(logits, dim=-1, dtype=torch.float32)   # HF eager attention
    p16 = torch.softmax(logits, dim=-1)                        # _softmax, bf16 out
    _store(d, "softmax_causal_bf16/x", logits)
    _store(d, "softmax_causal_bf16/out_f32", p32)
    _store(d, "softmax_causal_bf16/out_bf16", p16)

    # --- softmax, fp16 and fp32 (the reference's own test shapes)
    g = _gen(5)
    x16 = torch.randn(4, 8, 128, generator=g).to(torch.float16)
    _store(d, "softmax_f16/x", x16)
    _store(d, "softmax_f16/out", torch.softmax(x16, dim=-1))
    x32 = torch.randn(16, 32, generator=g)
    _store(d, "softmax_f32/x", x32)
    _store(d, "softmax_f32/out", torch.softmax(x32, dim=-1))
    _store(d, "softmax_f32/out_dim0", torch.softmax(x32, dim=0))

    # --- reductions, fp32 ~ N(0,1)
    g = _gen(6)
    xr = torch.randn(16, 8192, generator=g)
    _store(d, "reduce_f32/x", xr)
    _store(d, "reduce_f32/sum_last", xr.sum(-1))
    _store(d, "reduce_f32/mean_last", xr.mean(-1))
    _store(d, "reduce_f32/amax_last", xr.amax(-1))
    _store(d, "reduce_f32/sum_all", xr.sum())
    _store(d, "reduce_f32/mean_all", xr.mean())
    _store(d, "reduce_f32/amax_all", xr.amax())
    _store(d, "reduce_f32/sum_dim0", xr.sum(0))

    # --- argmax, bf16 ~ N(0,1) [8, 32000], with planted ties and NaNs
    g = _gen(7)
    xa = torch.randn(8, 32000, generator=g).to(torch.bfloat16)
    xa[3, 100] = 9.0
    xa[3, 31999] = 9.0                   # tie: the first index wins
    xa[5, 7] = float("nan")
    xa[5, 20000] = float("nan")          # first NaN wins
    xa[6, :] = float("-inf")             # all -inf: index 0
    _store(d, "argmax_bf16/x", xa)
    _store(d, "argmax_bf16/out", xa.argmax(-1))

    # --- int32 -> int64 sums, U[-1000, 1000]
    g = _gen(8)
    xi = torch.randint(-1000, 1001, (16, 8192), generator=g, dtype=torch.int32)
    _store(d, "sum_i32/x", xi)
    _store(d, "sum_i32/sum_last", xi.sum(-1))
    _store(d, "sum_i32/sum_all", xi.sum())

    # --- broadcast add / mul (the reference's own test shapes + the chain's)
    g = _gen(9)
    a = torch.randn(4, 8, generator=g).to(torch.bfloat16)
    b = torch.randn(8, generator=g).to(torch.bfloat16)
    _store(d, "add_bf16/a", a)
    _store(d, "add_bf16/b", b)
    _store(d, "add_bf16/out", a + b)
    _store(d, "add_bf16/out_alpha", torch.add(a, b, alpha=2.5))
    xr_ = torch.randn(16, 4096, generator=g).to(torch.bfloat16)
    yr_ = torch.randn(16, 4096, generator=g).to(torch.bfloat16)
    _store(d, "residual_bf16/x", xr_)
    _store(d, "residual_bf16/y", yr_)
    _store(d, "residual_bf16/out", xr_ + yr_)
    wv = (1 + 0.1 * torch.randn(512, generator=g)).to(torch.bfloat16)
    hv = torch.randn(8, 512, generator=g).to(torch.bfloat16)
    cv = torch.randn(8, 1, generator=g).to(torch.bfloat16)
    _store(d, "mul_bf16/w", wv)
    _store(d, "mul_bf16/h", hv)
    _store(d, "mul_bf16/c", cv)
    _store(d, "mul_bf16/w_h", wv * hv)
    _store(d, "mul_bf16/h_c", hv * cv)

    # --- backward: torch CPU autograd of the same modules, fp32 -------------
    # RMSNorm (Qwen3RMSNorm: dx and the weight gradient)
    g = _gen(10)
    x = torch.randn(16, 512, generator=g)
    w = 1 + 0.1 * torch.randn(512, generator=g)
    dy = torch.randn(16, 512, generator=g)
    mod = mq.Qwen3RMSNorm(512, eps=1e-6)
    with torch.no_grad():
        mod.weight.copy_(w)
    xg = x.clone().requires_grad_(True)
    mod(xg).backward(dy)
    for k_, t in (("x", x), ("w", w), ("dy", dy), ("dx", xg.grad), ("dw", mod.weight.grad)):
        _store(d, f"rmsnorm_bwd_f32/{k_}", t)

    # SwiGLU: act_fn(gate) * up
    g = _gen(11)
    gate = 3.0 * torch.randn(16, 1024, generator=g)
    up = torch.randn(16, 1024, generator=g)
    dact = torch.randn(16, 1024, generator=g)
    gg, ug = gate.clone().requires_grad_(True), up.clone().requires_grad_(True)
    (ACT2FN["silu"](gg) * ug).backward(dact)
    for k_, t in (("gate", gate), ("up", up), ("dout", dact), ("dgate", gg.grad),
                  ("dup", ug.grad)):
        _store(d, f"swiglu_bwd_f32/{k_}", t)

    # softmax over the last dim, fp32; and the half_to_float variant (bf16
    # logits, fp32 probabilities as HF eager attention computes them)
    g = _gen(12)
    xs = 3.0 * torch.randn(8, 256, generator=g)
    dys = torch.randn(8, 256, generator=g)
    xsg = xs.clone().requires_grad_(True)
    torch.softmax(xsg, dim=-1).backward(dys)
    for k_, t in (("x", xs), ("dy", dys), ("dx", xsg.grad)):
        _store(d, f"softmax_bwd_f32/{k_}", t)
    xh = (3.0 * torch.randn(8, 256, generator=g)).to(torch.bfloat16)
    dyh = torch.randn(8, 256, generator=g)
    xhg = xh.clone().requires_grad_(True)
    yh = torch.softmax(xhg, dim=-1, dtype=torch.float32)
    yh.backward(dyh)
    for k_, t in (("x", xh), ("y", yh.detach()), ("dy", dyh), ("dx", xhg.grad)):
        _store(d, f"softmax_bwd_half_to_float/{k_}", t)

    # RoPE: apply_rotary_pos_emb, fp32 q/k, the fp32 HF tables
    g = _gen(13)
    cosf, sinf = hf_chain.rope_tables(pos, 128, 10000.0, torch.float32)
    qf = torch.randn(1, 4, S, 128, generator=g)
    kf = torch.randn(1, 2, S, 128, generator=g)
    dq_o = torch.randn(1, 4, S, 128, generator=g)
    dk_o = torch.randn(1, 2, S, 128, generator=g)
    qg, kg = qf.clone().requires_grad_(True), kf.clone().requires_grad_(True)
    qo_, ko_ = mq.apply_rotary_pos_emb(qg, kg, cosf, sinf)
    torch.autograd.backward([qo_, ko_], [dq_o, dk_o])
    for k_, t in (("q", qf), ("k", kf), ("cos", cosf), ("sin", sinf), ("dq_out", dq_o),
                  ("dk_out", dk_o), ("dq", qg.grad), ("dk", kg.grad)):
        _store(d, f"rope_bwd_f32/{k_}", t)

    # HF eager attention (modeling_qwen3.eager_attention_forward) with the
    # mask transformers itself builds (masking_utils.eager_mask: causal, and
    # batch 1 left-padded by 5 tokens, so its first 5 queries see no key and
    # the reference's softmax makes their rows uniform).  `w` is the bf16
    # q @ repeat_kv(k)^T the function computes before its softmax tail.
    import types

    from transformers import masking_utils

    g = _gen(14)
    B, Hq, Hk, L, D = 2, 4, 2, 64, 32
    scaling = D ** -0.5
    q = torch.randn(B, Hq, L, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hk, L, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hk, L, D, generator=g).to(torch.bfloat16)
    keep = torch.ones(B, L, dtype=torch.bool)
    keep[1, :5] = False
    mask = masking_utils.eager_mask(batch_size=B, q_length=L, kv_length=L, attention_mask=keep,
                                    dtype=torch.bfloat16)
    module = types.SimpleNamespace(num_key_value_groups=Hq // Hk, training=False)
    attn_out, attn_w = mq.eager_attention_forward(module, q, k, v, mask, scaling)
    w = torch.matmul(q, mq.repeat_kv(k, Hq // Hk).transpose(2, 3))
    wg = w.clone().requires_grad_(True)
    y = torch.softmax(wg * scaling + mask, dim=-1, dtype=torch.float32).to(torch.bfloat16)
    assert torch.equal(y.detach(), attn_w)
    dy = torch.randn(B, Hq, L, L, generator=g).to(torch.bfloat16)
    y.backward(dy)
    z32 = (w * scaling + mask).float()  # what _softmax(float32) receives op by op
    for k_, t in (("w", w), ("mask", mask), ("attn_weights", attn_w), ("dy", dy),
                  ("dw", wg.grad), ("z32", z32), ("z32_softmax", torch.softmax(z32, dim=-1))):
        _store(d, f"masked_softmax_bf16/{k_}", t)
    d["masked_softmax_bf16/scaling:f32"] = np.array([scaling], np.float32)
    # fp32 model: the mask holds float32's lowest value
    wf = torch.randn(B, Hq, L, L, generator=g)
    maskf = masking_utils.eager_mask(batch_size=B, q_length=L, kv_length=L, attention_mask=keep,
                                     dtype=torch.float32)
    yf = torch.softmax(wf * scaling + maskf, dim=-1, dtype=torch.float32)
    for k_, t in (("w", wf), ("mask", maskf), ("out", yf)):
        _store(d, f"masked_softmax_f32/{k_}", t)

    np.savez_compressed(OUT, **d)
    print(f"wrote {OUT}: {len(d)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
