"""Operator registration helpers and the HuggingFace fused-op hooks.

`register_flagos_operator` keeps the reference's API
(torch_fl/integration.py:33-49 there): register a Python implementation of an
aten op for the flagos device.

`enable_hf_fused_ops()` is the site the reference lacks (it has no HF hooks):
it replaces, in the installed transformers, the forward of the RMSNorm
modules, the module-level `apply_rotary_pos_emb`, the SwiGLU MLP forward and
the module-level `eager_attention_forward` (its scale + mask + softmax +
cast tail becomes one flagos::masked_softmax launch; the two matmuls stay
torch's) of the Qwen3 / Qwen2 / Llama / Mistral model files with the
flagos:: fused kernels.  Two forwards are replaced so that neighbouring ops
run as one kernel: the decoder layer's (the residual add after attention and
`post_attention_layernorm` become one flagos::add_rms_norm), and Qwen3's
attention (`q_norm` / `k_norm` and `apply_rotary_pos_emb` become one
flagos::rms_norm_rope; the projections, the KV cache update and the
attention interface are HF's own).  The hooks act on device tensors (flagos
or cuda), in inference and in training (the fused ops carry autograd
formulas, torch_fl/autograd.py); CPU tensors, RoPE tables that themselves
need a gradient, and attention with dropout active, run the original HF code
unchanged.  `disable_hf_fused_ops()` restores the originals.
"""

from __future__ import annotations

import importlib
from typing import Callable, Optional

import torch

from . import ops

_registered_ops: set = set()
_libs: list = []


def register_flagos_operator(op_name: str, impl_func: Callable, schema: Optional[str] = None) -> None:
    """Register `impl_func` as the flagos (PrivateUse1) kernel of aten op
    `op_name` (e.g. "add.Tensor"); with `schema`, define it first."""
    lib = torch.library.Library("aten", "IMPL") if schema is None else torch.library.Library(
        "aten", "FRAGMENT")
    if schema is not None:
        lib.define(schema)
    lib.impl(op_name, impl_func, "PrivateUse1")
    _registered_ops.add(op_name)
    _libs.append(lib)


def get_registered_ops() -> list:
    return sorted(_registered_ops)


# ------------------------------------------------------------- HF fused hooks
_MODEL_FILES = {
    # RMSNorm, MLP, decoder layer, attention with q/k norms (Qwen3 only)
    "qwen3": ("Qwen3RMSNorm", "Qwen3MLP", "Qwen3DecoderLayer", "Qwen3Attention"),
    "qwen2": ("Qwen2RMSNorm", "Qwen2MLP", "Qwen2DecoderLayer", None),
    "llama": ("LlamaRMSNorm", "LlamaMLP", "LlamaDecoderLayer", None),
    "mistral": ("MistralRMSNorm", "MistralMLP", "MistralDecoderLayer", None),
}
_saved: dict = {}
_rounding: Optional[str] = None


def _fusable(*tensors) -> bool:
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type not in ("flagos", "privateuseone",
                                                                     "cuda"):
            return False
        if t.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            return False
    return True


def _rms_forward(orig):
    def forward(self, hidden_states):
        w = self.weight
        if _fusable(hidden_states, w) and w.dtype == hidden_states.dtype:
            return ops.rms_norm(hidden_states, w, self.variance_epsilon, _rounding)
        return orig(self, hidden_states)

    forward.__wrapped__ = orig
    return forward


def _rope_fn(orig):
    def apply_rotary_pos_emb(q, k, cos, sin, *args, **kwargs):
        unsqueeze_dim = kwargs.get("unsqueeze_dim", args[-1] if args and isinstance(args[-1], int) else 1)
        tables_need_grad = torch.is_grad_enabled() and (cos.requires_grad or sin.requires_grad)
        if (_fusable(q, k, cos, sin) and q.dim() == 4 and q.dtype == cos.dtype == k.dtype
                and unsqueeze_dim in (1, 2) and not tables_need_grad):
            return ops.rope_qk(q, k, cos, sin, unsqueeze_dim, _rounding)
        return orig(q, k, cos, sin, *args, **kwargs)

    apply_rotary_pos_emb.__wrapped__ = orig
    return apply_rotary_pos_emb


def _mlp_forward(orig):
    def forward(self, x):
        act = getattr(self, "act_fn", None)
        is_silu = isinstance(act, torch.nn.SiLU) or type(act).__name__ in ("SiLUActivation", "SiLU")
        if is_silu and _fusable(x):
            return self.down_proj(ops.swiglu(self.gate_proj(x), self.up_proj(x), _rounding))
        return orig(self, x)

    forward.__wrapped__ = orig
    return forward


def _attention_fn(orig):
    repeat_kv = getattr(importlib.import_module(orig.__module__), "repeat_kv", None)

    def eager_attention_forward(module, query, key, value, attention_mask, scaling,
                                dropout=0.0, **kwargs):
        mask = attention_mask
        mask_ok = mask is None or (_fusable(mask) and mask.dtype == query.dtype
                                   and mask.dim() == 4 and mask.shape[-1] == key.shape[-2])
        dropping = bool(dropout) and module.training
        if (repeat_kv is None or dropping or not mask_ok or query.dim() != 4
                or not _fusable(query, key, value)):
            return orig(module, query, key, value, attention_mask, scaling, dropout, **kwargs)
        groups = module.num_key_value_groups
        key_states = repeat_kv(key, groups)
        value_states = repeat_kv(value, groups)
        w = torch.matmul(query, key_states.transpose(2, 3))
        w = ops.masked_softmax(w, mask, float(scaling), None, _rounding)
        out = torch.matmul(w, value_states).transpose(1, 2).contiguous()
        return out, w

    eager_attention_forward.__wrapped__ = orig
    return eager_attention_forward


def _norm_weight(norm, like: torch.Tensor):
    """The weight of an HF RMSNorm module when the b200 kernel can take it,
    else None (another norm class, or a weight of another dtype/device)."""
    w = getattr(norm, "weight", None)
    eps = getattr(norm, "variance_epsilon", None)
    if (eps is None or not isinstance(w, torch.Tensor) or w.dim() != 1
            or w.dtype != like.dtype or not _fusable(w, like)):
        return None
    return w


def _decoder_forward(orig):
    """The decoder layer of Qwen3 / Qwen2 / Llama / Mistral (one forward in
    all four files: residual -> input_layernorm -> self_attn -> residual add
    -> post_attention_layernorm -> mlp -> residual add) with the residual add
    after attention and post_attention_layernorm as one add_rms_norm."""

    def forward(self, hidden_states, attention_mask=None, position_ids=None,
                past_key_values=None, use_cache=False, position_embeddings=None, **kwargs):
        post = self.post_attention_layernorm
        w = _norm_weight(post, hidden_states)
        if w is None or hidden_states.shape[-1] != w.shape[0]:
            return orig(self, hidden_states, attention_mask=attention_mask,
                        position_ids=position_ids, past_key_values=past_key_values,
                        use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
        residual = hidden_states
        hidden_states = self.input_layernorm(hidden_states)
        hidden_states, _ = self.self_attn(
            hidden_states=hidden_states, attention_mask=attention_mask,
            position_ids=position_ids, past_key_values=past_key_values, use_cache=use_cache,
            position_embeddings=position_embeddings, **kwargs)
        if hidden_states.dtype == residual.dtype and hidden_states.shape == residual.shape:
            # (residual + attn) and its norm in one pass; x + y == y + x bit for bit
            normed, hidden_states = ops.add_rms_norm(hidden_states, residual, w,
                                                     post.variance_epsilon, _rounding)
        else:
            hidden_states = residual + hidden_states
            normed = post(hidden_states)
        residual = hidden_states
        hidden_states = self.mlp(normed)
        return residual + hidden_states

    forward.__wrapped__ = orig
    return forward


def _qwen3_attention_forward(orig):
    """Qwen3Attention.forward (modeling_qwen3.py) with q_norm / k_norm and
    apply_rotary_pos_emb as one rms_norm_rope over the projections' [B, S,
    H, D] views; everything else is the original's code path."""
    mod = importlib.import_module(orig.__module__)

    def forward(self, hidden_states, position_embeddings, attention_mask,
                past_key_values=None, **kwargs):
        cos, sin = position_embeddings
        qn, kn = self.q_norm, self.k_norm
        wq, wk = _norm_weight(qn, hidden_states), _norm_weight(kn, hidden_states)
        tables_need_grad = torch.is_grad_enabled() and (cos.requires_grad or sin.requires_grad)
        if (wq is None or wk is None or qn.variance_epsilon != kn.variance_epsilon
                or tables_need_grad or not _fusable(cos, sin) or cos.dtype != hidden_states.dtype
                or sin.dtype != cos.dtype):
            return orig(self, hidden_states, position_embeddings, attention_mask,
                        past_key_values, **kwargs)
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, self.head_dim)
        q = self.q_proj(hidden_states).view(hidden_shape)          # [B, S, Hq, D]
        k = self.k_proj(hidden_states).view(hidden_shape)          # [B, S, Hkv, D]
        value_states = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        q, k = ops.rms_norm_rope(q, k, wq, wk, cos, sin, qn.variance_epsilon, 2, _rounding)
        query_states, key_states = q.transpose(1, 2), k.transpose(1, 2)
        if past_key_values is not None:
            key_states, value_states = past_key_values.update(key_states, value_states,
                                                              self.layer_idx)
        attention_interface = mod.ALL_ATTENTION_FUNCTIONS.get_interface(
            self.config._attn_implementation, mod.eager_attention_forward)
        attn_output, attn_weights = attention_interface(
            self, query_states, key_states, value_states, attention_mask,
            dropout=0.0 if not self.training else self.attention_dropout,
            scaling=self.scaling, sliding_window=self.sliding_window, **kwargs)
        attn_output = attn_output.reshape(*input_shape, -1).contiguous()
        return self.o_proj(attn_output), attn_weights

    forward.__wrapped__ = orig
    return forward


def enable_hf_fused_ops(models=tuple(_MODEL_FILES), rounding: Optional[str] = None) -> list:
    """Patch the installed transformers model files; returns what was patched."""
    global _rounding
    _rounding = rounding
    patched = []
    for name in models:
        try:
            mod = importlib.import_module(f"transformers.models.{name}.modeling_{name}")
        except Exception:
            continue
        norm_cls, mlp_cls, layer_cls, attn_cls = _MODEL_FILES[name]
        targets = [(getattr(mod, norm_cls, None), "forward", _rms_forward),
                   (getattr(mod, mlp_cls, None), "forward", _mlp_forward),
                   (mod, "apply_rotary_pos_emb", _rope_fn),
                   (mod, "eager_attention_forward", _attention_fn),
                   (getattr(mod, layer_cls, None), "forward", _decoder_forward)]
        if attn_cls is not None:
            targets.append((getattr(mod, attn_cls, None), "forward", _qwen3_attention_forward))
        for owner, attr, make in targets:
            if owner is None or not hasattr(owner, attr):
                continue
            key = (id(owner), attr)
            if key in _saved:
                continue
            orig = getattr(owner, attr)
            _saved[key] = (owner, attr, orig)
            setattr(owner, attr, make(orig))
            patched.append(f"{getattr(owner, '__name__', owner)}.{attr}")
    return patched


def disable_hf_fused_ops() -> None:
    for owner, attr, orig in _saved.values():
        setattr(owner, attr, orig)
    _saved.clear()
