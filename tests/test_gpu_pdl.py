"""Programmatic dependent launch (PDL): every kernel of the stack's files is
launched so that it may start while the previous kernel in the stream
finishes, and waits on the device before its first memory access.  These
tests run producer -> consumer chains (each launch reads what the launch
before it wrote, or overwrites what it read) with PDL on and off, eager and
replayed from a CUDA graph, and require bit-identical results."""

import pytest
import torch

from torch_fl import _abi
from torch_fl import kernels as K

pytestmark = pytest.mark.gpu

H, HQ, HKV, D, I = 1024, 8, 2, 128, 2816


def _inputs(T, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)

    def rn(*s, scale=1.0, loc=0.0):
        return (loc + scale * torch.randn(*s, generator=g, device=dev)).to(torch.bfloat16)

    pos = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (1e4 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    fr = pos[:, None] * inv[None]
    emb = torch.cat([fr, fr], -1)
    return dict(x=rn(T, H), y=rn(T, H), w=rn(H, scale=0.1, loc=1.0), q=rn(1, T, HQ, D),
                k=rn(1, T, HKV, D), g=rn(T, I), u=rn(T, I), wq=rn(D, scale=0.1, loc=1.0),
                wk=rn(D, scale=0.1, loc=1.0), cos=emb.cos().to(torch.bfloat16).to(dev),
                sin=emb.sin().to(torch.bfloat16).to(dev))


def _chain(t, layers=3):
    """Each launch depends on the one before it: h feeds the next
    add_rms_norm, the norm output feeds the mul, RoPE runs in place twice on
    the same buffers, SwiGLU's output is the next add's operand."""
    h, n = t["x"], None
    q, k = t["q"].clone(), t["k"].clone()
    outs = []
    for _ in range(layers):
        n, h = K.add_rms_norm(h, t["y"], t["w"], 1e-5)
        K.rope_qk(q, k, t["cos"], t["sin"], layout="bshd", inplace=True)
        K.rope_qk(q, k, t["cos"], t["sin"], layout="bshd", inplace=True, q_weight=t["wq"],
                  k_weight=t["wk"], eps=1e-6)
        a = K.swiglu(t["g"], t["u"])
        a2, h = K.swiglu_residual(t["g"], a, h, n)
        n = K.rms_norm(h, t["w"], 1e-5)
        h = K.add(h, K.mul(n, t["w"]))
        outs += [n, h, a2]
    return outs + [q, k]


@pytest.fixture
def pdl_restore():
    prev = _abi.set_pdl(True)
    yield
    _abi.set_pdl(prev)


@pytest.mark.parametrize("T", [8, 4096])
def test_pdl_chain_matches_serial_launches(pdl_restore, T):
    dev = torch.device("cuda", 0)
    t = _inputs(T, dev)
    _abi.set_pdl(False)
    ref = [o.clone() for o in _chain(t)]
    torch.cuda.synchronize()
    _abi.set_pdl(True)
    got = _chain(t)
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(got, ref)):
        assert torch.equal(a, b), i


def test_pdl_chain_in_cuda_graph(pdl_restore):
    dev = torch.device("cuda", 0)
    t = _inputs(2048, dev, seed=3)
    _abi.set_pdl(False)
    ref = [o.clone() for o in _chain(t)]
    torch.cuda.synchronize()
    _abi.set_pdl(True)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _chain(t)
    torch.cuda.current_stream().wait_stream(side)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        outs = _chain(t)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(outs, ref)):
        assert torch.equal(a, b), i
    del gr
