"""Build libqqt_b200.so for sm_100a in-tree (qqt_b200/_lib/).

    python qqt-gpu-sim_b200/build.py [--force] [--phase-stamps]

--phase-stamps builds libqqt_b200_phase.so instead: the same kernels with
their phase-boundary time stamps compiled in (QQT_PHASE_STAMPS), read by
`bench.py --phase-stamps`; the regular library is left as it is.

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
OUT_PHASE = os.path.join(HERE, "qqt_b200", "_lib", "libqqt_b200_phase.so")
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-fmad=false",
         "-std=c++17", "-shared", "-Xcompiler", "-fPIC"]


def sources():
    return [os.path.join(SRC, f) for f in sorted(os.listdir(SRC))
            if f.endswith((".cu", ".cuh"))] + [os.path.join(HERE, "..", "include", "qqt_b200.h")]


def needs_build(out: str = OUT) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False, phase_stamps: bool = False) -> str:
    out = OUT_PHASE if phase_stamps else OUT
    if force or needs_build(out):
        os.makedirs(os.path.dirname(out), exist_ok=True)
        cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + \
            (["-DQQT_PHASE_STAMPS"] if phase_stamps else []) + \
            ["-o", out, os.path.join(SRC, "qqt_b200.cu")]
        subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                phase_stamps="--phase-stamps" in sys.argv))
