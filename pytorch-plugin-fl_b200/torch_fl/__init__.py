"""torch_fl -- the flagos PrivateUse1 device with a B200-native `b200` route.

`import torch_fl` does what the reference's plugin entry does
(torch_fl/__init__.py:33-54 there): loads the native library (here
libfl_b200.so, the sm_100a kernels, and torch_fl/_C, the device runtime and
aten registrations), renames PrivateUse1 to "flagos" and registers the device
module, so `torch.randn(..., device="flagos")` and every aten op on flagos
tensors dispatch through torch_fl.  The route of each hot op (b200 or cuda)
comes from torch_fl/backends.conf.  Nothing falls back to the CPU: a missing
native library is an ImportError.
"""

import torch

from . import _abi

_abi.load()

from . import _C  # noqa: E402  (registers the device runtime and aten kernels)
from . import flagos  # noqa: E402

torch.utils.rename_privateuse1_backend("flagos")
torch._register_device_module("flagos", flagos)
torch.utils.generate_methods_for_privateuse1_backend(for_storage=True)

from . import kernels, ops  # noqa: E402
from . import autograd as _autograd  # noqa: E402

_autograd.register()  # backward formulas of the flagos:: fused ops
from .integration import (  # noqa: E402
    disable_hf_fused_ops,
    enable_hf_fused_ops,
    register_flagos_operator,
)


def routes() -> dict:
    """Effective backend of every routed aten op, e.g. {"_softmax": "b200"}."""
    return dict(_C._routes())


def config_path() -> str:
    """The backends.conf that was loaded ("" if none)."""
    return _C._config_path()


__all__ = [
    "flagos",
    "kernels",
    "ops",
    "routes",
    "config_path",
    "enable_hf_fused_ops",
    "disable_hf_fused_ops",
    "register_flagos_operator",
]
