"""Build recipe for the in-tree CUDA library ``libwl_attn.so`` (sm_100a).

The library is one translation unit (``csrc/wl_attn.cu``) compiled with nvcc
for ``sm_100a`` only, linked against the CUDA runtime (shared, so it shares the
process's primary context with PyTorch) and NCCL. The output lands next to
this file so that it travels with the source tree.

Usage: ``python -m windlass_b200.build`` (or ``build()`` from Python).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libwl_attn.so")
SOURCES = [os.path.join(CSRC, "wl_attn.cu")]
DEPS = SOURCES + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(ROOT, "include", "wl_attn.h")]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libwl_attn.so")


def _nccl_dirs() -> tuple[str, str]:
    """(include dir, lib dir) of the NCCL shipped with the Python environment."""
    try:
        import nvidia.nccl  # type: ignore

        base = list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(d) > t for d in DEPS if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    inc, libdir = _nccl_dirs()
    cmd = [
        _nvcc(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-shared", "-Xcompiler", "-fPIC", "-cudart", "shared",
        "-I", os.path.join(ROOT, "include"), "-I", inc,
        *SOURCES,
        "-L", libdir, "-l:libnccl.so.2",
        "-Xlinker", f"-rpath,{libdir}", "-Xlinker", "-rpath,/usr/local/cuda/lib64",
        "-o", LIB + ".tmp",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
