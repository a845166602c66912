"""Python entry points of the flagos:: fused ops (torch.ops.flagos.*).

They take flagos or cuda tensors and return tensors on the same device.
`rounding` is "fused" (compute in fp32, round once: within 1 ulp of the
fp32-accumulated result) or "chain" (round where the reference's op-by-op HF
chain rounds); the default comes from FLAGOS_B200_ROUNDING, else "fused".
"""

from __future__ import annotations

import os

import torch


def default_rounding() -> str:
    r = os.environ.get("FLAGOS_B200_ROUNDING", "fused")
    if r not in ("fused", "chain"):
        raise ValueError(f"FLAGOS_B200_ROUNDING must be 'fused' or 'chain', got {r!r}")
    return r


def rms_norm(x, weight, eps: float, rounding: str | None = None):
    """weight * (x * rsqrt(mean(x^2) + eps)) over the last dim
    (transformers models/qwen3/modeling_qwen3.py:59-64)."""
    return torch.ops.flagos.rms_norm(x, weight, float(eps), rounding or default_rounding())


def add_rms_norm(x, residual, weight, eps: float, rounding: str | None = None):
    """(rms_norm(x + residual), x + residual) in one pass."""
    return torch.ops.flagos.add_rms_norm(x, residual, weight, float(eps),
                                         rounding or default_rounding())


def rope_qk(q, k, cos, sin, unsqueeze_dim: int = 1, rounding: str | None = None):
    """apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim)
    (modeling_qwen3.py:158-181); q/k are [B,H,S,D] (unsqueeze_dim=1) or
    [B,S,H,D] (unsqueeze_dim=2), cos/sin [B,S,D] or [S,D]."""
    return torch.ops.flagos.rope_qk(q, k, cos, sin, int(unsqueeze_dim),
                                    rounding or default_rounding())


def rms_norm_rope(q, k, q_weight, k_weight, cos, sin, eps: float, unsqueeze_dim: int = 1,
                  rounding: str | None = None):
    """Qwen3's q_norm / k_norm over the head dim followed by RoPE, one pass
    (modeling_qwen3.py:248-249, 263-268)."""
    return torch.ops.flagos.rms_norm_rope(q, k, q_weight, k_weight, cos, sin, float(eps),
                                          int(unsqueeze_dim), rounding or default_rounding())


def swiglu(gate, up, rounding: str | None = None):
    """silu(gate) * up (Qwen3MLP, modeling_qwen3.py:81-82)."""
    return torch.ops.flagos.swiglu(gate, up, rounding or default_rounding())


def swiglu_residual(gate, up, x, y, rounding: str | None = None):
    """(silu(gate) * up, x + y) in one launch."""
    return torch.ops.flagos.swiglu_residual(gate, up, x, y, rounding or default_rounding())


def causal_softmax(x, offset: int = 0, dtype: torch.dtype | None = None):
    """softmax over the last dim of x [..., q_len, k_len] with the causal mask
    applied in the kernel: query i sees keys j <= i + offset; masked entries
    are exact zeros and are never read."""
    return torch.ops.flagos.causal_softmax(x, int(offset), dtype)


def masked_softmax(x, mask=None, scale: float = 1.0, dtype: torch.dtype | None = None,
                   rounding: str | None = None):
    """softmax(x * scale + mask) over the last dim in one launch: the tail of
    HF's eager attention (modeling_qwen3.py eager_attention_forward,
    `attn_weights * scaling + attention_mask`, softmax(dtype=float32), then
    `.to(query.dtype)`).  x is [B, H, Q, K] (or fewer leading dims); mask has
    x's dtype and broadcasts to x; dtype None = x's dtype (the cast back
    fused) or float32."""
    return torch.ops.flagos.masked_softmax(x, mask, float(scale), dtype,
                                           rounding or default_rounding())
