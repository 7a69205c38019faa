"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device and the built C-ABI library; the CPU
suite (`-m "not gpu"`) checks the oracle against the golden vectors, the host
logic, and that the library loads and exports every declared symbol.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "qqt-gpu-sim_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")
