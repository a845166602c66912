"""HuggingFace models on the flagos device, with and without the fused-op
hooks (torch_fl.enable_hf_fused_ops).  A small random-init Qwen3 (the
reference's e2e tests use Qwen3-0.6B weights, which are not available here)
runs its forward on flagos:0 and is compared with the same model on the CPU.
"""

import pytest
import torch

import torch_fl
from torch_fl import integration

pytestmark = pytest.mark.gpu


def tiny_qwen3(dtype):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=704,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, max_position_embeddings=256, rms_norm_eps=1e-6,
                      attn_implementation="eager")
    torch.manual_seed(0)
    m = Qwen3ForCausalLM(cfg).to(dtype).eval()
    return m


@pytest.fixture(autouse=True)
def _no_hooks_after():
    yield
    torch_fl.disable_hf_fused_ops()


def test_qwen3_forward_on_flagos_matches_cpu():
    model = tiny_qwen3(torch.float32)
    ids = torch.randint(0, 512, (2, 48), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model(ids).logits
        model_d = model.to("flagos:0")
        out = model_d(ids.to("flagos:0")).logits
    assert out.device.type == "flagos"
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-3, atol=1e-3)


def _count_fused_calls(monkeypatch):
    calls = {n: 0 for n in ("rms_norm", "rope_qk", "swiglu", "masked_softmax", "add_rms_norm",
                            "rms_norm_rope")}
    for name in calls:
        orig = getattr(torch_fl.ops, name)

        def counted(*a, _orig=orig, _name=name, **k):
            calls[_name] += 1
            return _orig(*a, **k)

        monkeypatch.setattr(torch_fl.ops, name, counted)
    return calls


def test_qwen3_forward_with_fused_hooks(monkeypatch):
    calls = _count_fused_calls(monkeypatch)
    model = tiny_qwen3(torch.float32)
    ids = torch.randint(0, 512, (2, 48), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = model(ids).logits
        model_d = model.to("flagos:0")
        patched = torch_fl.enable_hf_fused_ops()
        assert any("apply_rotary_pos_emb" in p for p in patched)
        assert any("Qwen3Attention" in p for p in patched)
        out = model_d(ids.to("flagos:0")).logits
    # per layer: input_layernorm; q_norm + k_norm + RoPE as one rms_norm_rope;
    # the residual add + post_attention_layernorm as one add_rms_norm; the
    # MLP's SwiGLU; the eager attention tail.  Plus the final norm.
    assert calls["rms_norm_rope"] == 2 and calls["rope_qk"] == 0, calls
    assert calls["add_rms_norm"] == 2 and calls["rms_norm"] == 3, calls
    assert calls["swiglu"] == 2 and calls["masked_softmax"] == 2, calls
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-3, atol=1e-3)


def tiny_llama(dtype):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=704,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, max_position_embeddings=256, rms_norm_eps=1e-5,
                      attn_implementation="eager")
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(dtype).eval()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_llama_forward_with_fused_hooks(monkeypatch, dtype):
    """Llama has no q/k norms: RoPE stays one rope_qk per layer, the residual
    add + post_attention_layernorm is one add_rms_norm."""
    calls = _count_fused_calls(monkeypatch)
    model = tiny_llama(dtype)
    ids = torch.randint(0, 512, (2, 40), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        model_d = model.to("flagos:0")
        ref = model_d(ids.to("flagos:0")).logits.float().cpu()   # unhooked, on flagos
        torch_fl.enable_hf_fused_ops(rounding="chain")
        out = model_d(ids.to("flagos:0")).logits.float().cpu()
    assert calls["rope_qk"] == 2 and calls["rms_norm_rope"] == 0, calls
    assert calls["add_rms_norm"] == 2 and calls["rms_norm"] == 3, calls
    if dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-3)
    else:
        assert (out - ref).abs().max() <= 0.05 * ref.abs().max()


@pytest.mark.parametrize("hooks", [True, False])
def test_qwen3_left_padded_batch_matches_cpu(hooks):
    """A left-padded batch: HF's eager mask leaves the padding queries with
    no visible key (every logit at float32's lowest value), which the
    reference's softmax turns into uniform rows.  With the hooks the
    attention tail is flagos::masked_softmax; without them HF's op chain
    runs on flagos (mask add, then _softmax on the b200 route)."""
    model = tiny_qwen3(torch.float32)
    ids = torch.randint(0, 512, (2, 40), generator=torch.Generator().manual_seed(4))
    am = torch.ones(2, 40, dtype=torch.long)
    am[1, :6] = 0
    with torch.no_grad():
        ref = model(ids, attention_mask=am).logits
        model_d = model.to("flagos:0")
        if hooks:
            torch_fl.enable_hf_fused_ops()
        out = model_d(ids.to("flagos:0"), attention_mask=am.to("flagos:0")).logits
    assert torch.isfinite(out.cpu()).all()
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-3, atol=1e-3)


def test_qwen3_bf16_hooks_match_unhooked():
    model = tiny_qwen3(torch.bfloat16).to("flagos:0")
    ids = torch.randint(0, 512, (1, 64), generator=torch.Generator().manual_seed(3)).to("flagos:0")
    with torch.no_grad():
        plain = model(ids).logits.float().cpu()
        torch_fl.enable_hf_fused_ops(rounding="chain")
        chain = model(ids).logits.float().cpu()
        torch_fl.disable_hf_fused_ops()
        torch_fl.enable_hf_fused_ops(rounding="fused")
        fused = model(ids).logits.float().cpu()
    scale = plain.abs().max()
    assert (chain - plain).abs().max() <= 0.05 * scale
    assert (fused - plain).abs().max() <= 0.05 * scale


def test_hooks_leave_cpu_paths_alone():
    model = tiny_qwen3(torch.float32)
    torch_fl.enable_hf_fused_ops()
    ids = torch.randint(0, 512, (1, 16))
    out = model(ids).logits          # CPU tensors: the original HF code runs
    out.sum().backward()             # and autograd works
    assert model.model.norm.weight.grad is not None
    integration.disable_hf_fused_ops()


@pytest.mark.parametrize("hooks", [True, False])
def test_qwen3_training_step_on_flagos_matches_cpu(hooks):
    """One forward + backward of a causal-LM loss on flagos:0: with the hooks
    the fused ops and their backward kernels run (RMSNorm, RoPE, SwiGLU);
    without them the aten ops do (silu_backward and _softmax_backward_data on
    the b200 route).  Loss and every parameter gradient match the same model
    on the CPU."""
    import copy

    cpu = tiny_qwen3(torch.float32).train()
    dev = copy.deepcopy(cpu).to("flagos")
    ids = torch.randint(0, 512, (2, 32), generator=torch.Generator().manual_seed(3))
    if hooks:
        torch_fl.enable_hf_fused_ops()
    loss_d = dev(ids.to("flagos"), labels=ids.to("flagos")).loss
    loss_d.backward()
    loss_c = cpu(ids, labels=ids).loss       # CPU tensors: the original HF code
    loss_c.backward()
    torch.testing.assert_close(loss_d.cpu(), loss_c, rtol=1e-5, atol=1e-5)
    n = 0
    for (name, pd), (_, pc) in zip(dev.named_parameters(), cpu.named_parameters()):
        assert pd.grad is not None, name
        scale = pc.grad.abs().max().item() + 1e-12
        torch.testing.assert_close(pd.grad.cpu(), pc.grad, rtol=1e-3, atol=1e-4 * scale,
                                   msg=lambda m, name=name: f"{name}: {m}")
        n += 1
    assert n > 10
