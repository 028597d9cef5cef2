"""Build the C restatements under oracle/ (test infrastructure: the checker and
the timed CPU baseline, never the product path).

    python -m oracle.build_c

gcc -O3 -fopenmp-simd -pthread; the hot loops carry target_clones (avx512f / avx2 / default),
so the library built here picks the widest vector ISA of whichever x86-64 host
loads it.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "adjoint_c.c")
LIB = os.path.join(HERE, "liboracle_c.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cc = os.environ.get("CC", "gcc")
    subprocess.run([cc, "-O3", "-std=c11", "-fopenmp-simd", "-pthread", "-fPIC", "-shared", "-o", LIB + ".tmp", SRC, "-lm"],
                   check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def load():
    """ctypes handle of the built library (built on first use)."""
    import ctypes as C
    lib = C.CDLL(build())
    f = lib.oracle_adjoint_c
    P = C.c_void_p
    f.argtypes = [P, P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, P, P, C.c_int]
    f.restype = C.c_int
    return lib


if __name__ == "__main__":
    print(build(force=True))
