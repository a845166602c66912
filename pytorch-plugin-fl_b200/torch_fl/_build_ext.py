"""Build recipe of torch_fl/_C (the flagos PrivateUse1 device layer).

Compiles csrc/module.cc, csrc/runtime/*.cc and csrc/aten/*.cc against the
installed torch with torch.utils.cpp_extension (ninja), links them to
lib/libfl_b200.so through an $ORIGIN rpath and copies the module to
torch_fl/_C.so.  The compile runs in a fresh interpreter: cpp_extension
imports what it built, and a process that already imported torch_fl._C must
not register the flagos op library a second time.  A content hash of the
sources, headers and flags decides whether anything is stale.
"""

from __future__ import annotations

import glob
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(HERE)
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
BUILD_DIR = os.path.join(PKG_DIR, "_build", "torch_ext")
TARGET = os.path.join(HERE, "_C.so")
STAMP = TARGET + ".stamp"

CFLAGS = ["-O2", "-std=c++17", "-fvisibility=hidden"]
# $$ for ninja, single quotes for the shell ninja runs the link in
LDFLAGS = [f"-L{LIB_DIR}", "-lfl_b200", "'-Wl,-rpath,$$ORIGIN/lib'", "-lcudart"]


def sources() -> list[str]:
    return sorted([os.path.join(CSRC, "module.cc")]
                  + glob.glob(os.path.join(CSRC, "runtime", "*.cc"))
                  + glob.glob(os.path.join(CSRC, "aten", "*.cc")))


def _fingerprint() -> str:
    h = hashlib.sha256()
    deps = (sources() + sorted(glob.glob(os.path.join(CSRC, "runtime", "*.h")))
            + sorted(glob.glob(os.path.join(CSRC, "aten", "*.h")))
            + [os.path.join(REPO_DIR, "include", "fl_b200.h")])
    for d in deps:
        h.update(os.path.relpath(d, PKG_DIR).encode())
        with open(d, "rb") as f:
            h.update(f.read())
    h.update(repr((CFLAGS, LDFLAGS[1:])).encode())
    import torch

    h.update(torch.__version__.encode())
    return h.hexdigest()


def build(verbose: bool = False) -> str:
    fp = _fingerprint()
    if os.path.exists(TARGET) and os.path.exists(STAMP) and open(STAMP).read() == fp:
        return TARGET
    os.makedirs(BUILD_DIR, exist_ok=True)
    code = (
        "import ctypes\n"
        f"ctypes.CDLL({os.path.join(LIB_DIR, 'libfl_b200.so')!r}, mode=ctypes.RTLD_GLOBAL)\n"
        "from torch.utils import cpp_extension\n"
        f"cpp_extension.load(name='_C', sources={sources()!r}, "
        f"extra_include_paths={[CSRC, REPO_DIR]!r}, extra_cflags={CFLAGS!r}, "
        f"extra_ldflags={LDFLAGS!r}, with_cuda=True, build_directory={BUILD_DIR!r}, "
        f"verbose={verbose!r}, is_python_module=True)\n"
    )
    proc = subprocess.run([sys.executable, "-c", code], capture_output=not verbose, text=True)
    if proc.returncode != 0:
        raise RuntimeError("building torch_fl/_C failed:\n" + (proc.stdout or "") + (proc.stderr or ""))
    shutil.copy2(os.path.join(BUILD_DIR, "_C.so"), TARGET)
    with open(STAMP, "w") as f:
        f.write(fp)
    return TARGET
