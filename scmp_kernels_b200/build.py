"""Build ``libscmp_b200.so`` from ``csrc/`` with nvcc for sm_100a.

Usage: ``python -m scmp_kernels_b200.build [--force]``. The library is built
in the package directory so that it travels with the source tree.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
OUT = os.path.join(HERE, "libscmp_b200.so")
MAIN = os.path.join(HERE, "csrc", "scmp_b200.cu")

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared", "-Xptxas", "-v"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*")) +
                  glob.glob(os.path.join(REPO, "include", "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", os.path.join(REPO, "include"), "-o", OUT, MAIN]
    r = subprocess.run(cmd, capture_output=True, text=True)
    # the compiler's report (ptxas registers, spills, shared memory per kernel)
    os.makedirs(os.path.join(HERE, "_build"), exist_ok=True)
    with open(os.path.join(HERE, "_build", "nvcc.log"), "w") as f:
        f.write(r.stdout + r.stderr)
    if verbose or r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode:
        raise RuntimeError(f"nvcc failed ({r.returncode}): {' '.join(cmd)}")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
