"""Build the C part of the oracle (test infrastructure): oracle/_build/libsc_oracle.so."""
from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_build", "libsc_oracle.so")
SRC = os.path.join(HERE, "sc_enable_sum.c")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cc = shutil.which("gcc") or "cc"
    subprocess.run([cc, "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-o", OUT, SRC],
                   check=True)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
