"""Build libmssample.so in place with nvcc for sm_100a (B200).

    python -m miniserve_b200.build

The library is a plain C-ABI shared object (no torch types in its
signatures); it links the CUDA runtime statically so it does not depend on
which libcudart the host process loaded.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmssample.so")
SOURCES = ["ms_sample.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmssample.so")
    return path


def build(verbose: bool = False, extra_flags=None) -> str:
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "mssample.h"))
    if os.path.exists(LIB) and not extra_flags:
        lib_m = os.path.getmtime(LIB)
        if all(os.path.getmtime(d) <= lib_m for d in deps):
            return LIB
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-Xptxas", "-v" if verbose else "-O3", "-o", LIB + ".tmp",
           *[os.path.join(CSRC, s) for s in SOURCES], *(extra_flags or [])]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
