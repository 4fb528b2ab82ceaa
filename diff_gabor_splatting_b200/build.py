"""Build libgabor_b200.so (sm_100a) in-tree with nvcc.

    python -m diff_gabor_splatting_b200.build [--force] [--verbose]

The library is plain CUDA C++ behind a C ABI (include/gabor_b200.h); it links
only the CUDA runtime.  Objects are compiled in parallel and the shared library
is written next to this file, where the Python package loads it from.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCES = ["capi.cu", "project.cu", "sh.cu", "binning.cu", "composite.cu", "adam.cu"]
LIBRARY = PACKAGE / "libgabor_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]


def nvcc() -> str:
    """Locate nvcc (CUDA_HOME, /usr/local/cuda, or PATH)."""
    for candidate in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if candidate and (Path(candidate) / "bin" / "nvcc").exists():
            return str(Path(candidate) / "bin" / "nvcc")
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > mtime for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every source to an object in _build/ and link the shared library."""
    csrc = PACKAGE / "csrc"
    out = ROOT / "_build"
    out.mkdir(exist_ok=True)
    headers = list(csrc.glob("*.cuh")) + [ROOT / "include" / "gabor_b200.h"]
    compiler = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(name: str) -> Path:
        src = csrc / name
        obj = out / (Path(name).stem + ".o")
        if force or ptxas_info or _stale(obj, [src, *headers]):
            cmd = [compiler, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            result = subprocess.run(cmd, capture_output=True, text=True)
            if result.returncode != 0:
                raise RuntimeError(f"nvcc failed on {name}:\n{result.stderr}")
            if ptxas_info or verbose:
                sys.stderr.write(result.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        objects = list(pool.map(compile_one, SOURCES))
    if force or _stale(LIBRARY, objects):
        cmd = [compiler, *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stderr}")
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v resource usage")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
