"""Build libqqt_b200.so for sm_100a in-tree (qqt_b200/_lib/).

    python qqt-gpu-sim_b200/build.py [--force]

nvcc cross-compiles without a GPU.  -fmad=false keeps the simulator's float
arithmetic in the reference's exact operation order.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "qqt_b200", "_lib", "libqqt_b200.so")
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-fmad=false",
         "-std=c++17", "-shared", "-Xcompiler", "-fPIC"]


def sources():
    return [os.path.join(SRC, f) for f in sorted(os.listdir(SRC))
            if f.endswith((".cu", ".cuh"))] + [os.path.join(HERE, "..", "include", "qqt_b200.h")]


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if force or needs_build():
        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + \
            ["-o", OUT, os.path.join(SRC, "qqt_b200.cu")]
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
