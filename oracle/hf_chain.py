"""The reference's own CPU path for the op set (TEST INFRASTRUCTURE ONLY).

On the flagos device the reference runs the HuggingFace formulas op by op
through its aten registrations; on CPU the same formulas run on torch's CPU
aten kernels (PyTorch 2.11.0, the version the reference pins in README.md).
These functions are those formulas, op for op, on torch CPU tensors:

* rms_norm    transformers 5.5.0 models/qwen3/modeling_qwen3.py:59-64
* rotate_half modeling_qwen3.py:151-155
* rope        apply_rotary_pos_emb, modeling_qwen3.py:158-181
* rope_tables Qwen3RotaryEmbedding.forward, modeling_qwen3.py:86-148
* swiglu      Qwen3MLP.forward's act_fn(gate) * up, modeling_qwen3.py:81-82
* softmax     torch.softmax (aten _softmax, csrc/aten/softmax.h:10)

tests/golden/make_golden.py checks these against the transformers modules
themselves before writing fixtures; bench.py times them as the CPU baseline.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    input_dtype = x.dtype
    h = x.to(torch.float32)
    variance = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    return weight * h.to(input_dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def rope(q, k, cos, sin, unsqueeze_dim: int = 1):
    cos = cos.unsqueeze(unsqueeze_dim)
    sin = sin.unsqueeze(unsqueeze_dim)
    q_embed = (q * cos) + (rotate_half(q) * sin)
    k_embed = (k * cos) + (rotate_half(k) * sin) if k is not None else None
    return q_embed, k_embed


def rope_tables(position_ids: torch.Tensor, dim: int, theta: float, dtype: torch.dtype):
    """cos, sin of shape [B, S, D] for int64 position_ids [B, S]."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim))
    inv_freq_expanded = inv_freq[None, :, None].float().expand(position_ids.shape[0], -1, 1)
    position_ids_expanded = position_ids[:, None, :].float()
    freqs = (inv_freq_expanded.float() @ position_ids_expanded.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = emb.cos() * 1.0
    sin = emb.sin() * 1.0
    return cos.to(dtype=dtype), sin.to(dtype=dtype)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate) * up


def decoder_chain(x, w, q, k, cos, sin, gate, up, y, eps: float):
    """One decoder layer's non-GEMM chain (RMSNorm -> RoPE on q/k -> SwiGLU ->
    residual add), each step as the HF formula.  Returns all outputs."""
    n = rms_norm(x, w, eps)
    qe, ke = rope(q, k, cos, sin)
    a = swiglu(gate, up)
    h = x + y
    return n, qe, ke, a, h
