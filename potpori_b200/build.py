"""Compile the sm_100a CUDA library in-tree (potpori_b200/libpotpori_b200.so).

nvcc cross-compiles for sm_100a without a GPU. The CUDA runtime is linked statically so the
library does not depend on which libcudart another package (torch) has loaded; the driver
API entry point it needs (tensor-map encoding) is fetched at run time.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libpotpori_b200.so")
SOURCES = [os.path.join(HERE, "csrc", "pp_shard.cu"), os.path.join(HERE, "csrc", "pp_static_gemv.cu"),
           os.path.join(HERE, "csrc", "pp_prefill.cu")]
DEPS = SOURCES + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + [
    os.path.join(ROOT, "include", "potpori_b200.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-o", LIB + ".tmp", *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    env = dict(os.environ)
    env.pop("CC", None)  # the image's CC points at a gcc without the host runtime nvcc wants
    subprocess.run(cmd, check=True, env=env)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    import sys
    build(force=True, verbose="-v" in sys.argv)
    print(LIB)
