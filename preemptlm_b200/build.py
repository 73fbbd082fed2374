"""Build libsg_b200.so (every CUDA source of the package) for sm_100a, in-tree.

    python -m preemptlm_b200.build          # or __graft_entry__.build()

nvcc cross-compiles without a GPU.  Objects go to ``_build/`` at the repo root;
the shared library goes to ``preemptlm_b200/lib/libsg_b200.so``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB_PATH = LIB_DIR / "libsg_b200.so"
BUILD_DIR = ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", "-DSG_BUILT_ARCH=1000",
    f"-I{ROOT / 'include'}", f"-I{CSRC}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsg_b200.so")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _newest_input_mtime() -> float:
    files = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    files.append(Path(__file__))
    return max(f.stat().st_mtime for f in files)


def is_stale() -> bool:
    return not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < _newest_input_mtime()


def build_library(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    if not force and not is_stale():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    cc = nvcc()
    flags = ARCH_FLAGS + COMMON_FLAGS + list(extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [cc, *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [cc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp), "-lcuda"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
