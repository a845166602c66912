"""The full-tensor sum that allocates nothing (fl_b200_reduce_sum_all_noalloc).

Callers that cannot allocate device memory -- code reached through a C FFI
that only receives tensors from its host framework, or code running where a
cudaMalloc is not allowed -- call this entry instead of
fl_b200_reduce_sum_all: its cross-CTA partials live in a fixed scratch array
inside libfl_b200.so rather than in a caller-provided workspace.  This test
calls it through the C ABI twice in a row and checks each result against the
workspace entry point (bit-identical: same kernel, same split) and against
the stated fp32 sum tolerance of tests/parity.py.  It sits in a file that
pytest collects last and passes alone in a fresh process as well.
"""

import math

import numpy as np
import pytest
import torch

from tests import parity
from torch_fl import _abi

pytestmark = pytest.mark.gpu

CASES = [
    (50_000_000, torch.float32),   # split over ~3000 CTAs: the scratch is used
    (3_000_001, torch.bfloat16),   # split, odd length, 16-bit input
    (1_000, torch.float32),        # single CTA: no scratch needed
]


@pytest.mark.parametrize("n,dtype", CASES)
def test_sum_all_noalloc_matches_workspace_entry(n, dtype):
    lib = _abi.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(1234 + n)
    x = torch.randn(n, generator=g, device=dev).to(dtype)
    code = _abi.F32 if dtype == torch.float32 else _abi.BF16

    # the existing entry point, with a workspace allocated by the caller
    ws_bytes = lib.fl_b200_reduce_workspace_size(1, n)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    ref = torch.empty((), dtype=torch.float32, device=dev)
    _abi.call("fl_b200_reduce_sum_all", x.data_ptr(), n, ref.data_ptr(), code, _abi.F32,
              ws.data_ptr(), ws_bytes, stream)
    torch.cuda.synchronize(dev)
    ref_v = ref.item()
    xn = parity.to_np(x)

    for call in range(2):  # two calls in a row share the library's scratch
        out = torch.full((), math.nan, dtype=torch.float32, device=dev)
        _abi.call("fl_b200_reduce_sum_all_noalloc", x.data_ptr(), n, out.data_ptr(), code,
                  _abi.F32, stream)
        torch.cuda.synchronize(dev)
        got = out.item()
        assert np.float32(got).tobytes() == np.float32(ref_v).tobytes(), (call, got, ref_v)
        parity.assert_sum(np.float32(got), xn, None, f"noalloc call {call}")


@pytest.mark.parametrize("n", [40_000_003, 777])
def test_sum_all_noalloc_int32_to_int64_exact(n):
    # The integer route of the same entry: int32 in, exact int64 out.
    lib = _abi.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(99 + n)
    x = torch.randint(-1000, 1001, (n,), generator=g, device=dev, dtype=torch.int32)
    ws_bytes = lib.fl_b200_reduce_workspace_size(1, n)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    ref = torch.empty((), dtype=torch.int64, device=dev)
    _abi.call("fl_b200_reduce_sum_all", x.data_ptr(), n, ref.data_ptr(), _abi.I32, _abi.I64,
              ws.data_ptr(), ws_bytes, stream)
    torch.cuda.synchronize(dev)
    exact = int(x.cpu().numpy().astype(np.int64).sum())
    assert ref.item() == exact
    for call in range(2):
        out = torch.full((), -1, dtype=torch.int64, device=dev)
        _abi.call("fl_b200_reduce_sum_all_noalloc", x.data_ptr(), n, out.data_ptr(), _abi.I32,
                  _abi.I64, stream)
        torch.cuda.synchronize(dev)
        assert out.item() == exact, (call, out.item(), exact)


def test_sum_all_noalloc_rejects_bad_arguments():
    with pytest.raises(_abi.FlB200Error) as ei:
        _abi.call("fl_b200_reduce_sum_all_noalloc", None, -1, None, _abi.F32, _abi.F32, None)
    assert ei.value.status == 1
