"""Build the sm_100a CUDA library ``ppu_b200/_lib/libqwen35_b200.so`` in-tree.

Each ``csrc/*.cu`` is compiled to an object in parallel with ``nvcc -gencode
arch=compute_100a,code=sm_100a``, then linked into one shared library that exports the C ABI
declared in ``include/qwen35_b200.h``. Incremental: objects newer than their source and the
headers are reused.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libqwen35_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build ppu_b200")
    return cand


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip():
        sys.stderr.write(f"[{src.name}] {res.stderr}")
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra or []), srcs))
    if LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:])
