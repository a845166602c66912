"""torch.flagos: the device module of the flagos PrivateUse1 device.

Same surface as the reference's torch_fl/flagos/__init__.py:11-229 (device,
device_count, current_device, set_device, synchronize, Stream, Event,
current_stream, stream, RNG state, get_amp_supported_dtype).  flagos device i
is CUDA device i and flagos streams are CUDA streams, so Stream and Event are
the CUDA ones; Event measures device time (the reference's Event is a host
timestamp taken after a device synchronize).
"""

import torch

from .. import _C

_initialized = False


class device:
    """Context manager that makes `device` (index or torch.device) current."""

    def __init__(self, device):
        self.idx = torch.accelerator._get_device_index(device, optional=True)
        self.prev_idx = -1

    def __enter__(self):
        self.prev_idx = _C._exchangeDevice(self.idx)

    def __exit__(self, *exc):
        _C._set_device(self.prev_idx)
        return False


def is_available() -> bool:
    return _C._get_device_count() > 0


def device_count() -> int:
    return _C._get_device_count()


def current_device() -> int:
    return _C._get_device()


def set_device(device) -> None:
    _C._set_device(torch.accelerator._get_device_index(device, optional=True))


def synchronize(device=None) -> None:
    """Wait for all work on a flagos device (default: the current one)."""
    idx = -1 if device is None else torch.accelerator._get_device_index(device, optional=True)
    _C._synchronize(idx)


def init() -> None:
    _lazy_init()


def is_initialized() -> bool:
    return _initialized


def _lazy_init() -> None:
    global _initialized
    if not _initialized:
        _C._init()
        _initialized = True


def _is_in_bad_fork() -> bool:
    return torch.cuda._is_in_bad_fork()


class Stream(torch.cuda.Stream):
    """A flagos stream is a CUDA stream of the same GPU."""

    def __new__(cls, device=None, priority=0, **kwargs):
        if device is None:
            device = current_device()
        if isinstance(device, torch.device):
            device = device.index if device.index is not None else current_device()
        return super().__new__(cls, device=device, priority=priority, **kwargs)


class Event(torch.cuda.Event):
    """A device event (CUDA event) usable with flagos streams."""


def current_stream(device=None):
    if device is None:
        device = current_device()
    if isinstance(device, torch.device):
        device = device.index if device.index is not None else current_device()
    return torch.cuda.current_stream(device)


def default_stream(device=None):
    if device is None:
        device = current_device()
    return torch.cuda.default_stream(device)


def stream(s):
    return torch.cuda.stream(s)


# ---- RNG: flagos ops draw from the CUDA generator of the same GPU -----------
def manual_seed(seed) -> None:
    torch.cuda.manual_seed(seed)


def manual_seed_all(seed) -> None:
    torch.cuda.manual_seed_all(seed)


def seed() -> None:
    torch.cuda.seed()


def initial_seed() -> int:
    return torch.cuda.initial_seed()


def get_rng_state(device="cuda"):
    return torch.cuda.get_rng_state(_cuda_index(device))


def set_rng_state(state, device="cuda") -> None:
    torch.cuda.set_rng_state(state, _cuda_index(device))


def _cuda_index(device):
    if isinstance(device, torch.device):
        return device.index if device.index is not None else current_device()
    if isinstance(device, str):
        d = torch.device(device.replace("flagos", "cuda"))
        return d.index if d.index is not None else current_device()
    return device


class _DefaultGenerators:
    def __getitem__(self, i):
        return _C._get_default_generator(i)

    def __len__(self):
        return device_count()


default_generators = _DefaultGenerators()


def get_amp_supported_dtype():
    return [torch.float16, torch.bfloat16]


# ---- memory -----------------------------------------------------------------
def memory_stats() -> dict:
    """Counters of the stream-ordered caching allocator behind flagos tensors."""
    return dict(_C._allocator_stats())


def memory_allocated(device=None) -> int:
    return int(_C._allocator_stats()["bytes_in_use"])


def empty_cache() -> None:
    """Return cached, unused flagos memory to the driver."""
    _C._empty_cache()


__all__ = [
    "device", "device_count", "current_device", "set_device", "synchronize", "init",
    "is_initialized", "is_available", "Stream", "Event", "current_stream", "default_stream",
    "stream", "manual_seed", "manual_seed_all", "seed", "initial_seed", "get_rng_state",
    "set_rng_state", "default_generators", "get_amp_supported_dtype", "memory_stats",
    "memory_allocated", "empty_cache",
]
