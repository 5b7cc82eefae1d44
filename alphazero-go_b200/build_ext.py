"""Builds libazb200.so in place: every CUDA source of csrc/ compiled for
sm_100a only (SASS, no PTX) with the CUDA runtime linked statically, so the
library loads on a machine without a GPU (the driver API is reached at run
time through cudaGetDriverEntryPoint). Translation units compile in
parallel into _build/ (git-ignored), then link.

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


OBJ = os.path.join(HERE, "_build")
COMPILE = [f for f in FLAGS if f != "-shared"]


def _object(src: str, khash: str) -> tuple[list[str], str]:
    """The compile command of one translation unit and its object path. The
    object's key covers the unit, every header, the flags and the compiler;
    only engine.cu, which prints the kernel hash, also depends on the others."""
    h = hashlib.sha256()
    for path in [src] + [p for p in sources() if p.endswith((".cuh", ".hpp"))] + [os.path.join(INCLUDE, "azb200.h")]:
        with open(path, "rb") as f:
            h.update(f.read())
    h.update(" ".join(COMPILE).encode())
    defs = []
    if os.path.basename(src) == "engine.cu":
        defs = [f"-DAZB_KERNEL_HASH=\"{khash}\""]
        h.update(khash.encode())
    obj = os.path.join(OBJ, f"{os.path.basename(src)}.{h.hexdigest()[:12]}.o")
    cmd = [NVCC, *COMPILE, "-c", *defs, "-I", CSRC, "-I", INCLUDE, "-o", obj + ".tmp", src]
    return cmd, obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the translation units in parallel into _build/, then links."""
    if not force and up_to_date():
        return OUT
    from concurrent.futures import ThreadPoolExecutor

    khash = kernel_hash()
    os.makedirs(OBJ, exist_ok=True)
    units = [_object(p, khash) for p in sources() if p.endswith((".cu", ".cpp"))]

    def compile_one(unit):
        cmd, obj = unit
        if os.path.exists(obj) and not force:
            return None
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            return f"{os.path.basename(cmd[-1])}: nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}"
        os.replace(obj + ".tmp", obj)
        return None

    with ThreadPoolExecutor(max_workers=min(len(units), os.cpu_count() or 4)) as pool:
        failures = [f for f in pool.map(compile_one, units) if f]
    if failures:
        raise RuntimeError("\n".join(failures))
    link = [NVCC, *FLAGS, "-o", OUT + ".tmp", *[obj for _, obj in units]]
    if verbose:
        print(" ".join(link), flush=True)
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(OUT + ".tmp", OUT)
    keep = {os.path.basename(obj) for _, obj in units}
    for f in os.listdir(OBJ):   # objects of earlier sources
        if f.endswith(".o") and f not in keep:
            os.remove(os.path.join(OBJ, f))
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
