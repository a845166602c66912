"""Build steps of the B200 backend (run in-tree; outputs stay inside the package).

* ``build_kernels()``  -- nvcc, sm_100a: ``csrc/b200/*.cu`` -> ``torch_fl/lib/libfl_b200.so``
  (the C-ABI declared in ``include/fl_b200.h``; no torch dependency).
* ``build_torch_ext()`` -- the PrivateUse1 ``flagos`` device and its aten
  registrations: ``csrc/{runtime,aten}/*.cc`` + ``csrc/module.cc`` ->
  ``torch_fl/_C*.so`` (linked against libfl_b200.so through an $ORIGIN rpath).
* ``build_all()`` -- both.

Every step is incremental: a target is rebuilt only when a source or header
it depends on is newer than it.
"""

from __future__ import annotations

import concurrent.futures as _cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
KERNEL_DIR = os.path.join(CSRC, "b200")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")
LIB_DIR = os.path.join(PKG_DIR, "torch_fl", "lib")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
KERNEL_LIB = os.path.join(LIB_DIR, "libfl_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-diag-suppress=177",
]


def _nvcc() -> str:
    cand = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cand, "bin", "nvcc")
    if os.path.exists(path):
        return path
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: the B200 kernels need the CUDA toolkit to build")
    return found


def _newer(target: str, deps: list[str]) -> bool:
    """True if target is missing or older than any dependency."""
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "build command failed:\n" + " ".join(cmd) + "\n" + proc.stdout + proc.stderr
        )


def build_kernels(verbose: bool = False, jobs: int | None = None) -> str:
    """Compile every kernel source for sm_100a and link libfl_b200.so."""
    nvcc = _nvcc()
    os.makedirs(LIB_DIR, exist_ok=True)
    obj_dir = os.path.join(BUILD_DIR, "b200")
    os.makedirs(obj_dir, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(KERNEL_DIR, "*.cu")))
    headers = sorted(glob.glob(os.path.join(KERNEL_DIR, "*.cuh"))) + [
        os.path.join(INCLUDE_DIR, "fl_b200.h")
    ]
    objs = []
    todo = []
    for src in sources:
        obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if _newer(obj, [src] + headers):
            todo.append(
                [nvcc, *NVCC_FLAGS, "-I", INCLUDE_DIR, "-c", src, "-o", obj]
            )
    if todo:
        n = jobs or min(len(todo), os.cpu_count() or 4)
        with _cf.ThreadPoolExecutor(max_workers=n) as ex:
            for cmd, fut in [(c, ex.submit(_run, c)) for c in todo]:
                fut.result()
                if verbose:
                    print("[build] " + os.path.basename(cmd[-3]))
    if _newer(KERNEL_LIB, objs):
        _run([nvcc, *ARCH_FLAGS, "-shared", "-o", KERNEL_LIB, *objs])
        if verbose:
            print("[build] linked " + KERNEL_LIB)
    return KERNEL_LIB


def build_torch_ext(verbose: bool = False) -> str | None:
    """Build the torch extension (flagos PrivateUse1 device) if its sources exist."""
    sys.path.insert(0, PKG_DIR)
    try:
        from torch_fl import _build_ext  # noqa: WPS433 (local import by design)
    finally:
        sys.path.pop(0)
    return _build_ext.build(verbose=verbose)


def build_all(verbose: bool = False) -> None:
    build_kernels(verbose=verbose)
    build_torch_ext(verbose=verbose)


if __name__ == "__main__":
    build_all(verbose=True)
