"""torch_fl -- B200-native backend of the flagos PrivateUse1 device.

`import torch_fl` loads libfl_b200.so (the kernels) and, once built, the
torch extension that registers the flagos device and its aten routes.
"""

from . import _abi  # noqa: F401

_abi.load()
