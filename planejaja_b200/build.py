"""Build libnsq.so in-tree:  python -m planejaja_b200.build

Runs `make` in planejaja_b200/csrc (nvcc -gencode arch=compute_100a,code=sm_100a).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", os.path.join(HERE, "csrc")], check=True)
    return os.path.join(HERE, "libnsq.so")


if __name__ == "__main__":
    print(build())
    sys.exit(0)
