"""The flagos device end to end: tensors created, copied and cast on
`flagos:0`, the routed aten ops on the b200 route compared with torch CPU
(the reference's own tests compare flagos results with torch CPU:
tests/integration/ops/test_*_dispatch.py), routing checked through the
dispatch log in a subprocess (FLAGOS_LOG_DISPATCH / FLAGOS_OP_*), and the hot
ops checked to run on registered flagos kernels rather than the fallback."""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import torch_fl  # noqa: F401
from oracle import hf_chain, ops
from tests import parity

pytestmark = pytest.mark.gpu
DEV = "flagos:0"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def cpu_rand(*shape, dtype=torch.float32, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).to(dtype)


# --------------------------------------------------------------- plumbing --
def test_device_basics():
    assert torch.flagos.is_available() and torch.flagos.device_count() >= 1
    x = torch.randn(4, 8, device=DEV)
    assert x.device.type == "flagos" and x.is_flagos
    c = cpu_rand(5, 7)
    assert torch.equal(c.to(DEV).cpu(), c)
    # strided copies, slices, transposes
    t = c.to(DEV).t()
    assert torch.equal(t.cpu(), c.t())
    assert torch.equal(t.contiguous().cpu(), c.t().contiguous())
    assert torch.equal(c.to(DEV)[1:4, ::2].cpu(), c[1:4, ::2])
    # item / scalars
    assert c.to(DEV)[2, 3].item() == c[2, 3].item()
    # factory ops through the fallback
    assert torch.equal(torch.zeros(3, 4, device=DEV).cpu(), torch.zeros(3, 4))
    assert torch.equal(torch.arange(10, device=DEV).cpu(), torch.arange(10))
    torch.flagos.synchronize()


def test_on_device_dtype_casts_match_cpu():
    c = cpu_rand(64, 33, scale=100.0)
    d = c.to(DEV)
    for dt in (torch.bfloat16, torch.float16, torch.int32, torch.int64):
        assert torch.equal(d.to(dt).cpu(), c.to(dt)), dt
        assert torch.equal(d.to(dt).float().cpu(), c.to(dt).float()), dt
    # flagos -> flagos casts no longer go through host memory: compare with the kernel
    assert torch.equal(d.to(torch.bfloat16).cpu(), c.to(torch.bfloat16))


def test_streams_events_and_allocator():
    s = torch.flagos.Stream()
    e0, e1 = torch.flagos.Event(enable_timing=True), torch.flagos.Event(enable_timing=True)
    with torch.flagos.stream(s):
        e0.record()
        x = torch.randn(1024, 1024, device=DEV)
        y = x * 2.0
        e1.record()
    e1.synchronize()
    assert e0.elapsed_time(e1) >= 0.0
    y.record_stream(torch.flagos.current_stream())
    before = torch.flagos.memory_stats()
    z = torch.empty(1 << 20, device=DEV)
    mid = torch.flagos.memory_stats()
    assert mid["allocations"] == before["allocations"] + 1
    assert mid["bytes_in_use"] >= before["bytes_in_use"] + (1 << 22)
    del z
    assert torch.flagos.memory_stats()["frees"] >= before["frees"] + 1


def test_recorded_block_waits_for_the_other_stream():
    """A block freed while another stream (recorded with record_stream) still
    has work queued goes back to the pool only after that stream passes the
    free: allocations in between get other memory, however many there are,
    and no stream is made to wait for another."""
    user = torch.flagos.Stream()
    n = 1 << 20
    x = torch.empty(n, device=DEV)
    x_ptr = x.data_ptr()
    with torch.flagos.stream(user):
        torch.cuda._sleep(400_000_000)           # keeps `user` busy ~0.2 s (a bounded spin)
    x.record_stream(user)
    del x
    assert torch.flagos.memory_stats()["pending_frees"] >= 1
    held = []
    for _ in range(4):                           # each allocation polls the pending frees
        y = torch.empty(n, device=DEV)
        assert y.data_ptr() != x_ptr
        held.append(y)
    assert not user.query()                      # the block was held while `user` ran
    user.synchronize()
    torch.flagos.synchronize()
    del held
    torch.empty(n, device=DEV)                   # polls again: the block is released
    assert torch.flagos.memory_stats()["pending_frees"] == 0


# ------------------------------------------------------- routed aten ops --
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_add_mul_match_cpu(dtype):
    a, b = cpu_rand(4, 8, dtype=dtype, seed=1), cpu_rand(8, dtype=dtype, seed=2)
    tol = {} if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
    torch.testing.assert_close((a.to(DEV) + b.to(DEV)).cpu(), a + b, **tol)
    torch.testing.assert_close(torch.add(a.to(DEV), b.to(DEV), alpha=2.5).cpu(),
                               torch.add(a, b, alpha=2.5), **tol)
    torch.testing.assert_close((a.to(DEV) * b.to(DEV)).cpu(), a * b, **tol)
    torch.testing.assert_close((a.to(DEV) + 1e-5).cpu(), a + 1e-5, **tol)
    torch.testing.assert_close((a.to(DEV) * 3).cpu(), a * 3, **tol)
    torch.testing.assert_close((2.0 + a.to(DEV)).cpu(), 2.0 + a, **tol)
    # bf16 results are bit-identical to torch CPU's single-op rounding
    if dtype == torch.bfloat16:
        assert torch.equal((a.to(DEV) + b.to(DEV)).cpu(), a + b)
        assert torch.equal((a.to(DEV) * b.to(DEV)).cpu(), a * b)


def test_mixed_dtype_promotion():
    a, b = cpu_rand(16, 32, dtype=torch.bfloat16, seed=3), cpu_rand(32, seed=4)
    got = (a.to(DEV) + b.to(DEV)).cpu()
    assert got.dtype == torch.float32
    torch.testing.assert_close(got, a + b)
    i = torch.arange(12, dtype=torch.int32).reshape(3, 4)
    assert torch.equal((i.to(DEV) + i.to(DEV) * 2).cpu(), i + i * 2)


@pytest.mark.parametrize("shape", [(128, 256), (1, 10), (2, 8, 64)])
def test_softmax_matches_cpu(shape):
    x = cpu_rand(*shape, seed=5)
    torch.testing.assert_close(torch.softmax(x.to(DEV), dim=-1).cpu(), torch.softmax(x, -1),
                               rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(torch.softmax(x.to(DEV), dim=0).cpu(), torch.softmax(x, 0),
                               rtol=1e-5, atol=1e-6)
    h = x.to(torch.float16)
    out = torch.softmax(h.to(DEV), dim=-1)
    assert out.dtype == torch.float16
    parity.assert_ulp(parity.to_np(out), ops.softmax_golden(parity.to_np(h), "f16"), "f16", 1)
    # half_to_float (the HF eager-attention softmax(dtype=float32) on CUDA)
    o32 = torch._softmax(h.to(DEV), -1, True)
    assert o32.dtype == torch.float32
    parity.assert_rel(parity.to_np(o32), ops.softmax_golden(parity.to_np(h), "f32"), atol=1e-30)


@pytest.mark.parametrize("dim,keepdim", [(0, False), (1, False), (-1, True), ([0, 2], False),
                                         (None, False), ([], True)])
def test_sum_mean_amax_match_cpu(dim, keepdim):
    x = cpu_rand(8, 16, 32, seed=6)
    d = x.to(DEV)
    if dim is None:
        torch.testing.assert_close(d.sum().cpu(), x.sum(), rtol=1e-5, atol=1e-4)
        torch.testing.assert_close(d.mean().cpu(), x.mean(), rtol=1e-5, atol=1e-6)
        assert torch.equal(d.amax().cpu(), x.amax())
        return
    torch.testing.assert_close(d.sum(dim, keepdim=keepdim).cpu(), x.sum(dim, keepdim=keepdim),
                               rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(d.mean(dim, keepdim=keepdim).cpu(), x.mean(dim, keepdim=keepdim),
                               rtol=1e-5, atol=1e-6)
    assert torch.equal(d.amax(dim, keepdim=keepdim).cpu(), x.amax(dim, keepdim=keepdim))


def test_sum_dtypes():
    x = cpu_rand(16, 16, dtype=torch.bfloat16, seed=7)
    torch.testing.assert_close(x.to(DEV).sum(0).cpu().float(), x.float().sum(0), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(x.to(DEV).sum(1, dtype=torch.float32).cpu(), x.float().sum(1),
                               rtol=1e-5, atol=1e-5)
    i = torch.randint(-1000, 1001, (64, 8192), dtype=torch.int32)
    assert torch.equal(i.to(DEV).sum(-1).cpu(), i.sum(-1))
    assert i.to(DEV).sum().item() == i.sum().item()
    l = torch.randint(-2**40, 2**40, (33, 1000), dtype=torch.int64)
    assert torch.equal(l.to(DEV).sum(1).cpu(), l.sum(1))
    m = torch.rand(100, 100) > 0.5
    assert m.to(DEV).sum().item() == m.sum().item()


def test_argmax_matches_cpu(golden):
    xa = torch.from_numpy(ops.bf16_bits(golden.get("argmax_bf16/x")).view(np.int16)).view(torch.bfloat16)
    assert torch.equal(xa.to(DEV).argmax(-1).cpu(), xa.argmax(-1))
    assert torch.equal(xa.to(DEV).argmax(-1, keepdim=True).cpu(), xa.argmax(-1, keepdim=True))
    x = cpu_rand(7, 9, 11, seed=8)
    assert torch.equal(x.to(DEV).argmax().cpu(), x.argmax())
    assert torch.equal(x.to(DEV).argmax(1).cpu(), x.argmax(1))
    assert torch.equal(x.to(DEV).argmax(0, keepdim=True).cpu(), x.argmax(0, keepdim=True))


def test_unsupported_dtype_errors_name_the_route():
    x = torch.randn(4, 4, dtype=torch.float64).to(DEV)
    with pytest.raises(RuntimeError, match="b200 route"):
        torch.softmax(x, -1)


# ------------------------------------------------- HF formulas on flagos --
def test_hf_rmsnorm_chain_on_flagos_matches_cpu(golden):
    """The unfused HF RMSNorm on flagos tensors: _to_copy casts on the device,
    pow/rsqrt on the cuda route, mean/add/mul on b200."""
    x = torch.from_numpy(ops.bf16_bits(golden.get("rmsnorm_bf16/x")).view(np.int16)).view(torch.bfloat16)
    w = torch.from_numpy(ops.bf16_bits(golden.get("rmsnorm_bf16/w")).view(np.int16)).view(torch.bfloat16)
    got = hf_chain.rms_norm(x.to(DEV), w.to(DEV), 1e-5).cpu()
    d = parity.assert_ulp(got.float().numpy(), golden.get("rmsnorm_bf16/out"), "bf16", 2, "hf chain")
    assert np.mean(d == 0) > 0.999


def test_fused_ops_on_flagos(golden):
    q = torch.from_numpy(golden.get("rope_bf16/q")).to(torch.bfloat16).to(DEV)
    k = torch.from_numpy(golden.get("rope_bf16/k")).to(torch.bfloat16).to(DEV)
    cos = torch.from_numpy(golden.get("rope_bf16/cos")).to(torch.bfloat16).to(DEV)
    sin = torch.from_numpy(golden.get("rope_bf16/sin")).to(torch.bfloat16).to(DEV)
    qo, ko = torch_fl.ops.rope_qk(q, k, cos, sin, 1, "chain")
    assert qo.device.type == "flagos"
    parity.assert_ulp(qo.cpu().float().numpy(), golden.get("rope_bf16/q_out"), "bf16", 0)
    parity.assert_ulp(ko.cpu().float().numpy(), golden.get("rope_bf16/k_out"), "bf16", 0)
    g = torch.from_numpy(golden.get("swiglu_bf16/gate")).to(torch.bfloat16).to(DEV)
    u = torch.from_numpy(golden.get("swiglu_bf16/up")).to(torch.bfloat16).to(DEV)
    parity.assert_ulp(torch_fl.ops.swiglu(g, u).cpu().float().numpy(),
                      ops.swiglu_golden(golden.get("swiglu_bf16/gate"), golden.get("swiglu_bf16/up"),
                                        "bf16"), "bf16", 1)
    x = torch.from_numpy(golden.get("rmsnorm_bf16/x")).to(torch.bfloat16).to(DEV)
    w = torch.from_numpy(golden.get("rmsnorm_bf16/w")).to(torch.bfloat16).to(DEV)
    parity.assert_ulp(torch_fl.ops.rms_norm(x, w, 1e-5).cpu().float().numpy(),
                      ops.rms_norm_golden(golden.get("rmsnorm_bf16/x"), golden.get("rmsnorm_bf16/w"),
                                          1e-5, "bf16"), "bf16", 1)
    xl = torch.from_numpy(golden.get("softmax_causal_bf16/x")).to(torch.bfloat16)
    xu = torch.where(torch.isinf(xl), torch.zeros_like(xl), xl).to(DEV)
    parity.assert_ulp(torch_fl.ops.causal_softmax(xu).cpu().float().numpy(),
                      golden.get("softmax_causal_bf16/out_bf16"), "bf16", 1)


# ---------------------------------------------------------------- routing --
def _run(code, env):
    e = os.environ.copy()
    e.update(env)
    e["PYTHONPATH"] = os.pathsep.join([ROOT, os.path.join(ROOT, "pytorch-plugin-fl_b200"),
                                       e.get("PYTHONPATH", "")])
    return subprocess.run([sys.executable, "-c", code], env=e, capture_output=True, text=True,
                          timeout=300)


SOFTMAX = "import torch_fl, torch; x = torch.randn(4, 8, device='flagos:0'); torch.softmax(x, dim=-1); torch.flagos.synchronize()"


def test_dispatch_log_b200():
    r = _run(SOFTMAX, {"FLAGOS_LOG_DISPATCH": "1"})
    assert r.returncode == 0, r.stderr
    assert "[flagos dispatch] _softmax -> b200" in r.stderr


def test_dispatch_log_cuda_override():
    r = _run(SOFTMAX, {"FLAGOS_LOG_DISPATCH": "1", "FLAGOS_OP__softmax": "cuda"})
    assert r.returncode == 0, r.stderr
    assert "[flagos dispatch] _softmax -> cuda" in r.stderr


def test_pinned_host_tensors_report_pinned():
    a = torch.empty(1024, pin_memory=True)
    assert a.is_pinned()
    b = torch.randn(256).pin_memory()
    assert b.is_pinned() and not torch.randn(8).is_pinned()
    # a non-blocking copy from pinned memory into flagos and back
    x = b.to("flagos:0", non_blocking=True)
    out = torch.empty(256, pin_memory=True)
    out.copy_(x, non_blocking=True)
    torch.flagos.synchronize()
    assert torch.equal(out, b)


def test_first_op_through_the_cuda_fallback_in_a_fresh_process():
    # an op with no flagos kernel (abs, cumsum) as the process's first op on
    # flagos: PyTorch's CUDA kernel runs on aliases and must find CUDA set up
    code = ("import torch_fl, torch; x = torch.randn(4, 8).to('flagos:0'); "
            "y = x.abs().cumsum(-1); torch.flagos.synchronize(); "
            "assert torch.allclose(y.cpu(), x.cpu().abs().cumsum(-1), rtol=1e-5, atol=1e-6); "
            "print('ok')")
    r = _run(code, {})
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr


def test_unbuilt_backend_is_an_error():
    r = _run(SOFTMAX, {"FLAGOS_OP__softmax": "flaggems"})
    assert r.returncode != 0
    assert "not registered" in r.stderr


def test_hot_ops_have_flagos_kernels():
    """No hot op of the path reaches the fallback (the reference's
    test_fallback_trace.py:325-393 checks the same with
    _dispatch_has_kernel_for_dispatch_key)."""
    for op in ["aten::add.Tensor", "aten::mul.Tensor", "aten::_softmax", "aten::sum.dim_IntList",
               "aten::mean.dim", "aten::amax", "aten::argmax", "aten::_copy_from",
               "flagos::rms_norm", "flagos::rope_qk", "flagos::rms_norm_rope", "flagos::swiglu",
               "flagos::swiglu_residual", "flagos::add_rms_norm", "flagos::causal_softmax"]:
        assert torch._C._dispatch_has_kernel_for_dispatch_key(op, "PrivateUse1"), op
