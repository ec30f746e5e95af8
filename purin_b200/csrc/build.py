"""Build ``purin_b200/_lib/libpurin_cp.so`` for sm_100a with nvcc.

Usage: ``python -m purin_b200.csrc.build [--verbose]``.  The library is built in
tree so it travels with the repository snapshot to the GPU host.  Every kernel
is compiled with ``-fmad=false`` so that products and sums round separately,
matching the reference's elementwise arithmetic one operation at a time.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PACKAGE = HERE.parent
ROOT = PACKAGE.parent
LIB_DIR = PACKAGE / "_lib"
LIB = LIB_DIR / "libpurin_cp.so"
SOURCES = ["capi.cu", "cp_forward.cu", "cp_adjoint.cu", "cp_gmres_cluster.cu", "cp_post.cu",
           "sell_order.cu", "admm_forward.cu"]
# cp_forward.cu is also compiled once per (dtype, shared values, QP) combination
# of its kernels, so that the heavy template instantiations build in parallel.
FORWARD_PARTS = [(t, sh, qp) for t in ("double", "float") for sh in ("true", "false")
                 for qp in ("true", "false")]
HEADERS = ["common.cuh", "plan.cuh", "cp_kernels.cuh", "sell.cuh", "sell_order.h",
           "adjoint_common.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-O3"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found; set CUDA_HOME")


def _inputs():
    files = [HERE / s for s in SOURCES] + [HERE / h for h in HEADERS]
    files.append(ROOT / "include" / "purin_cp.h")
    return files


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    stamp = LIB.stat().st_mtime
    return all(f.stat().st_mtime <= stamp for f in _inputs())


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every source to an object in parallel (one nvcc per file), then link."""
    from concurrent.futures import ThreadPoolExecutor
    import tempfile

    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    with tempfile.TemporaryDirectory(prefix="purin_build_") as objdir:
        def compile_one(job):
            src, defines, stem = job
            obj = str(Path(objdir) / (stem + ".o"))
            cmd = [nvcc(), *ARCH, *FLAGS, *defines, "-c", "-o", obj, str(HERE / src)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            return obj, subprocess.run(cmd, cwd=str(HERE), capture_output=True, text=True)

        jobs = [(src, [], Path(src).stem) for src in SOURCES]
        jobs += [("cp_forward.cu", [f"-DPURIN_FWD_PART_T={t}", f"-DPURIN_FWD_PART_SHARED={sh}",
                                    f"-DPURIN_FWD_PART_QP={qp}"], f"cp_forward_{t}_{sh}_{qp}")
                 for t, sh, qp in FORWARD_PARTS]
        workers = min(len(jobs), max(os.cpu_count() or 1, 1))
        with ThreadPoolExecutor(max_workers=workers) as pool:
            results = list(pool.map(compile_one, jobs))
        for _, proc in results:
            if proc.returncode != 0:
                sys.stderr.write(proc.stdout + proc.stderr)
                raise RuntimeError("nvcc failed building libpurin_cp.so")
            if verbose:
                sys.stderr.write(proc.stdout + proc.stderr)
        link = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[obj for obj, _ in results]]
        proc = subprocess.run(link, cwd=str(HERE), capture_output=True, text=True)
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError("nvcc failed linking libpurin_cp.so")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(verbose=args.verbose, force=args.force))


if __name__ == "__main__":
    main()
