"""Build ``oracle/_lib/libcp_cpu.so`` (the C++ restatement of the CP loop) with g++.

Oracle (test and baseline infrastructure).  Generic x86-64-v2 code, OpenMP over
samples, ``-ffp-contract=off`` so products and sums round separately.  The
library is built in tree so it travels with the repository to the GPU host,
where bench.py times it on the host cores.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "_lib" / "libcp_cpu.so"
SOURCE = HERE / "cp_cpu.cpp"
FLAGS = ["-O3", "-std=c++17", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off",
         "-fno-fast-math", "-fPIC", "-shared"]


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB
    compiler = shutil.which("g++") or shutil.which("c++")
    if compiler is None:
        raise RuntimeError("g++ not found")
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    proc = subprocess.run([compiler, *FLAGS, "-o", str(tmp), str(SOURCE)], capture_output=True,
                          text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("g++ failed building libcp_cpu.so")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
