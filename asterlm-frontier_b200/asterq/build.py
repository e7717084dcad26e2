"""Build recipe for ``libasterq.so`` (the C-ABI CUDA library), in-tree.

``python -m asterq.build`` (with ``asterlm-frontier_b200`` on ``sys.path``) or
``__graft_entry__.build()`` compiles every ``csrc/*.cu`` for sm_100a with nvcc
and links one shared library next to this file.  The library depends only on
the CUDA runtime (linked statically), so it loads without PyTorch.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
PROJECT_DIR = PKG_DIR.parent
CSRC = PROJECT_DIR / "csrc"
INCLUDE = PROJECT_DIR.parent / "include"
LIB_NAME = "libasterq.so"
LIB_PATH = PKG_DIR / LIB_NAME
BUILD_DIR = PROJECT_DIR / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    # IEEE division/sqrt and no flush-to-zero: the write path is bit-exact.
    "-prec-div=true",
    "-prec-sqrt=true",
    "-ftz=false",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    for root in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if root and Path(root, "bin", "nvcc").exists():
            return str(Path(root, "bin", "nvcc"))
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the CUDA sources (incrementally) and link ``libasterq.so``."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    objects = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if force or ptxas_verbose or _stale(obj, [src, *headers]):
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0 or ptxas_verbose:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}")
    if force or _stale(LIB_PATH, objects):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("linking libasterq.so failed")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB_PATH)
