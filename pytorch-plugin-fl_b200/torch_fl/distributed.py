"""torch.distributed on flagos tensors (NCCL over NVLink).

As in the reference (torch_fl/distributed.py:36-170): collectives take flagos
tensors by passing zero-copy CUDA views of them to the NCCL process group
(flagos memory is CUDA memory of the same GPU).  The b200 op path shards by
token rows and needs no collective on the hot path; these wrappers serve the
final correctness gathers and any user collectives.
"""

from __future__ import annotations

import functools

import torch
import torch.distributed as dist

from . import _C

_patched = False


def _view(t):
    if isinstance(t, torch.Tensor) and t.device.type in ("flagos", "privateuseone"):
        return _C._flagos_to_cuda_view(t)
    if isinstance(t, (list, tuple)):
        return type(t)(_view(x) for x in t)
    return t


def _wrap(fn):
    @functools.wraps(fn)
    def inner(*args, **kwargs):
        args = tuple(_view(a) for a in args)
        kwargs = {k: _view(v) for k, v in kwargs.items()}
        return fn(*args, **kwargs)

    inner.__wrapped__ = fn
    return inner


_COLLECTIVES = ("all_reduce", "broadcast", "reduce", "all_gather", "all_gather_into_tensor",
                "reduce_scatter_tensor", "all_to_all_single", "send", "recv", "barrier")


def patch_collectives() -> None:
    """Let dist.<collective> take flagos tensors (idempotent)."""
    global _patched
    if _patched:
        return
    for name in _COLLECTIVES:
        if hasattr(dist, name):
            setattr(dist, name, _wrap(getattr(dist, name)))
    _patched = True


def init_process_group(backend: str = "nccl", **kwargs) -> None:
    """dist.init_process_group + flagos-aware collectives.  The rank's GPU
    (LOCAL_RANK) must be current; NCCL runs on it."""
    patch_collectives()
    if not dist.is_initialized():
        dist.init_process_group(backend=backend, **kwargs)
