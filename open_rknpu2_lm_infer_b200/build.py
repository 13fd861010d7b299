"""Build step for the CUDA library (nvcc cross-compiles sm_100a; no GPU needed)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build_library(force: bool = False, jobs: int = 8) -> str:
    """Compile csrc/*.cu into lib/libqlinear_b200.so with
    ``-gencode arch=compute_100a,code=sm_100a -lineinfo`` (see csrc/Makefile)."""
    cmd = ["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")]
    if force:
        cmd.append("-B")
    subprocess.run(cmd, check=True)
    path = os.path.join(HERE, "lib", "libqlinear_b200.so")
    if not os.path.exists(path):
        raise RuntimeError(f"build did not produce {path}")
    return path


if __name__ == "__main__":
    print(build_library())
