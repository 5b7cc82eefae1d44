"""Builds libazb200.so in place: every CUDA source of csrc/ compiled for
sm_100a only (SASS, no PTX) with the CUDA runtime linked statically, so the
library loads on a machine without a GPU (the driver API is reached at run
time through cudaGetDriverEntryPoint).

    python alphazero-go_b200/build_ext.py [--force]
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libazb200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo", "-shared",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-Wall",
    "--cudart", "static",
    "-Xlinker", "-z,defs",   # an unresolved symbol fails the build, not the first load
    "-ccbin", "g++",
]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp", ".cuh", ".hpp")))


def kernel_hash() -> str:
    """8 hex digits over the sources, the compiler's version and the flags
    (the role of the reference's AZGO_CUDA_KERNEL_HASH, cmake/azgo_cuda.cmake:55-74)."""
    h = hashlib.sha256()
    for path in sources() + [os.path.join(INCLUDE, "azb200.h")]:
        h.update(os.path.basename(path).encode())
        with open(path, "rb") as f:
            h.update(f.read())
    try:
        h.update(subprocess.run([NVCC, "--version"], capture_output=True, text=True, check=True).stdout.encode())
    except (OSError, subprocess.CalledProcessError):
        pass
    h.update(" ".join(FLAGS).encode())
    return h.hexdigest()[:8]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = sources() + [os.path.join(INCLUDE, "azb200.h"), os.path.abspath(__file__)]
    return all(os.path.getmtime(p) <= t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cu = [p for p in sources() if p.endswith((".cu", ".cpp"))]
    cmd = [NVCC, *FLAGS, f"-DAZB_KERNEL_HASH=\"{kernel_hash()}\"", "-I", CSRC, "-I", INCLUDE, "-o", OUT + ".tmp", *cu]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
