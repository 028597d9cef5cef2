"""Build libaideen_b200.so in-tree with nvcc for sm_100a.

    python -m aideen_b200.build

Links the CUDA runtime and NCCL (the wheel that
ships with the interpreter's torch, found under site-packages/nvidia/nccl).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libaideen_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dir() -> str:
    for p in sys.path:
        cand = os.path.join(p, "nvidia", "nccl")
        if os.path.isdir(os.path.join(cand, "include")):
            return cand
    raise RuntimeError("NCCL headers not found under site-packages/nvidia/nccl")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps.append(os.path.join(HERE, "..", "include", "aideen_b200.h"))
    return any(os.path.getmtime(f) > t for f in deps)


def build(verbose: bool = False, force: bool = False, out: str | None = None,
          defines: tuple = ()) -> str:
    """Compile every csrc/*.cu into one shared library (default: in-tree LIB)."""
    if out is None and not force and not needs_build():
        return LIB
    target = out or LIB
    nccl = nccl_dir()
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    cmd = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", os.path.join(nccl, "include"), *[f"-D{x}" for x in defines],
           "-o", target + ".tmp", *sources(),
           "-L", os.path.join(nccl, "lib"), "-l:libnccl.so.2",
           "-Xlinker", "-rpath," + os.path.join(nccl, "lib")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(target + ".tmp", target)
    return target


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force=True)
    print(LIB)
