"""Build the CUDA extension in-tree: csrc/*.cu -> lib/libbt_b200.so (sm_100a).

The library is a plain shared object with the C ABI of include/bt_b200.h; it
links the CUDA runtime statically and is loaded with ctypes.  Objects are
compiled in parallel and only rebuilt when a source or header is newer.

    python -m breezetoken_b200.build [--force] [--ptxas-verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libbt_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I",
    str(INCLUDE),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the B200 extension cannot be built")


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.inc")) + [
        INCLUDE / "bt_b200.h"
    ]


def _compile(src: Path, obj: Path, extra: list[str]) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    if proc.stderr.strip():
        sys.stderr.write(proc.stderr)


def build(force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link lib/libbt_b200.so."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    dep_mtime = max(p.stat().st_mtime for p in _deps())
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_verbose or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, dep_mtime):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            futs = [ex.submit(_compile, s, o, extra) for s, o in jobs]
            for f in futs:
                f.result()
    if force or jobs or not LIB.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, ptxas_verbose=args.ptxas_verbose))


if __name__ == "__main__":
    main()
