"""Build the CUDA library libfold_b200.so in place (sm_100a only).

    python -m fold_b200.build [--verbose]

Compiles every fold_b200/csrc/*.cu with nvcc for compute_100a/sm_100a into one shared library
next to this file, with the CUDA runtime linked statically so that the library loads on a host
without a GPU (the C-ABI symbols can be listed there; kernels only run on a B200).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libfold_b200.so"
INCLUDE = PKG.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and not _stale():
        return LIB
    out_dir = PKG / "_build"
    out_dir.mkdir(exist_ok=True)
    objs = []
    procs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    for src in sources():
        obj = out_dir / (src.stem + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if out and (verbose or ptxas_verbose or p.returncode):
            print(out, file=sys.stderr)
        if p.returncode:
            failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
            *map(str, objs), "-ldl", "-o", str(tmp)]
    if verbose:
        print(" ".join(link), flush=True)
    r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode:
        print(r.stdout, file=sys.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print register/shared-memory use (-Xptxas -v)")
    a = ap.parse_args()
    print(build(force=a.force or a.ptxas, verbose=a.verbose, ptxas_verbose=a.ptxas))


if __name__ == "__main__":
    main()
