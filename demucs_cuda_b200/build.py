"""Build libdc_b200.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

    python -m demucs_cuda_b200.build [--verbose]

The library is one translation unit (csrc/all.cu) linked against the static CUDA runtime,
so it does not depend on which libcudart a host process (e.g. PyTorch) has loaded.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libdc_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=default",
    "-shared", "-cudart", "static",
]


def sources():
    return sorted(os.path.join(SRC, f) for f in os.listdir(SRC)
                  if f.endswith((".cu", ".cuh")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    srcs = sources() + [os.path.join(HERE, "..", "include", "dc_b200.h"), __file__]
    return all(os.path.getmtime(s) <= t for s in srcs if os.path.exists(s))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [NVCC] + FLAGS + ["-o", OUT + ".tmp", os.path.join(SRC, "all.cu")]
    if verbose:
        cmd += ["-Xptxas", "-v"]
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libdc_b200.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
