"""Build the sm_100a shared library ``tileops/libtileops_b200.so``.

Each ``*.cu`` file in this directory is compiled by nvcc for
``-gencode arch=compute_100a,code=sm_100a`` (Blackwell B200, architecture-
specific features such as tcgen05 / TMEM enabled) into ``_build/`` next to
this directory, and the objects are linked into one shared library with the
CUDA runtime linked statically, so the library has no dependency beyond the
driver.  Objects are rebuilt only when their source or a header changed.

Usage:  python csrc/build.py [--verbose] [--ptxas-info] [-j N]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
REPO_ROOT = PKG_ROOT.parent
BUILD_DIR = PKG_ROOT / "_build"
LIB_PATH = PKG_ROOT / "tileops" / "libtileops_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    f"-I{REPO_ROOT / 'include'}",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build tileops")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + [REPO_ROOT / "include" / "tileops_c.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers(), Path(__file__)])


def _compile(src: Path, verbose: bool, ptxas_info: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    if not _stale(obj, src):
        return obj
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if ptxas_info or verbose:
        sys.stdout.write(res.stderr)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False, jobs: int = 0) -> Path:
    """Compile every CUDA source and link the shared library; return its path."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_info), sources))
    if LIB_PATH.exists() and all(LIB_PATH.stat().st_mtime >= o.stat().st_mtime for o in objs):
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v resource usage")
    ap.add_argument("-j", type=int, default=0)
    args = ap.parse_args()
    path = build(args.verbose, args.ptxas_info, args.j)
    print(path)


if __name__ == "__main__":
    main()
