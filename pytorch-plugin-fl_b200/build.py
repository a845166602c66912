"""Build steps of the B200 backend (run in-tree; outputs stay inside the package).

* ``build_kernels()``  -- nvcc, sm_100a: ``csrc/b200/*.cu`` -> ``torch_fl/lib/libfl_b200.so``
  (the C-ABI declared in ``include/fl_b200.h``; no torch dependency).
* ``build_torch_ext()`` -- the PrivateUse1 ``flagos`` device and its aten
  registrations: ``csrc/{runtime,aten}/*.cc`` + ``csrc/module.cc`` ->
  ``torch_fl/_C*.so`` (linked against libfl_b200.so through an $ORIGIN rpath).
* ``build_all()`` -- both.

Every step is incremental: a target is rebuilt only when the content of a
source, header or flag it depends on changed (hash stamps next to it).
"""

from __future__ import annotations

import concurrent.futures as _cf
import glob
import hashlib
import importlib.util
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


def _digest(paths: list[str], extra: str = "") -> str:
    h = hashlib.sha256(extra.encode())
    for p in paths:
        h.update(os.path.basename(p).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def _stale(target: str, digest: str) -> bool:
    """True unless `target` exists and was built from inputs with `digest`
    (content hashes, so copies of the tree that lose mtimes stay valid)."""
    stamp = target + ".stamp"
    if not (os.path.exists(target) and os.path.exists(stamp)):
        return True
    with open(stamp) as f:
        return f.read() != digest


def _stamp(target: str, digest: str) -> None:
    with open(target + ".stamp", "w") as f:
        f.write(digest)


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
    flags = " ".join(NVCC_FLAGS)
    objs, todo = [], []
    for src in sources:
        obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        dg = _digest([src] + headers, flags)
        if _stale(obj, dg):
            todo.append((obj, dg, [nvcc, *NVCC_FLAGS, "-I", INCLUDE_DIR, "-c", src, "-o", obj]))
    if todo:
        n = jobs or min(len(todo), os.cpu_count() or 4)
        with _cf.ThreadPoolExecutor(max_workers=n) as ex:
            futs = [(obj, dg, cmd, ex.submit(_run, cmd)) for obj, dg, cmd in todo]
            for obj, dg, cmd, fut in futs:
                fut.result()
                _stamp(obj, dg)
                if verbose:
                    print("[build] " + os.path.basename(cmd[-3]))
    link_dg = _digest(objs, "link")
    if _stale(KERNEL_LIB, link_dg):
        _run([nvcc, *ARCH_FLAGS, "-shared", "-Xlinker", "-soname=libfl_b200.so", "-o",
              KERNEL_LIB, *objs])
        _stamp(KERNEL_LIB, link_dg)
        if verbose:
            print("[build] linked " + KERNEL_LIB)
    return KERNEL_LIB


def build_torch_ext(verbose: bool = False) -> str | None:
    """Build torch_fl/_C (the flagos PrivateUse1 device layer).  The recipe is
    loaded by path so that the torch_fl package itself is not imported."""
    spec = importlib.util.spec_from_file_location(
        "_fl_b200_build_ext", os.path.join(PKG_DIR, "torch_fl", "_build_ext.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(verbose=verbose)


def build_all(verbose: bool = False) -> None:
    build_kernels(verbose=verbose)
    build_torch_ext(verbose=verbose)


if __name__ == "__main__":
    build_all(verbose=True)
