"""Builds libddtree_b200.so (the C-ABI library) from csrc/*.cu for sm_100a with nvcc.

The library is built in-tree, next to this file, so it travels with the repository.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libddtree_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: the ddtree_b200 CUDA library cannot be built")
    return found


def library_path() -> str:
    return os.path.join(HERE, LIB_NAME)


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def headers() -> list[str]:
    return (sorted(glob.glob(os.path.join(HERE, "csrc", "*.cuh"))) +
            sorted(glob.glob(os.path.join(HERE, "..", "include", "*.h"))))


def needs_build() -> bool:
    lib = library_path()
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    return any(os.path.getmtime(f) > t for f in sources() + headers())


def build(force: bool = False, verbose: bool = False) -> str:
    lib = library_path()
    if not force and not needs_build():
        return lib
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src).replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{out.decode()}")
        if verbose and out:
            print(out.decode())
    tmp = lib + ".tmp"
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs]
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
