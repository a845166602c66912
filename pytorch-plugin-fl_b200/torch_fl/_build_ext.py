"""Build recipe of torch_fl/_C (the flagos PrivateUse1 device); see build.py."""

import os

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose: bool = False):
    src_dir = os.path.join(os.path.dirname(HERE), "csrc", "aten")
    if not os.path.isdir(src_dir):
        return None
    raise NotImplementedError
