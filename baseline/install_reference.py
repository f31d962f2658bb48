"""Install the reference (xushuxun/breezetoken) into baseline/_ref.

    python baseline/install_reference.py /path/to/breezetoken-checkout

The reference is pure Python on torch + numpy.  Its wheel cannot be built
offline here (its build backend, hatchling, is not in the offline
wheelhouse), so this recipe installs it the way pip's --target leaves a
pure-Python package: the ``breezetoken`` package directory copied unchanged
into ``baseline/_ref/breezetoken``.  Its runtime dependencies (torch, numpy)
are already installed; tilelang (its GPU kernels) is not needed by the torch
CPU path or by the drop-in test.  baseline/_ref is git-ignored and travels
to the GPU box with the working tree.

Used by ``bench.py --impl reference`` (the reference's own torch CPU decode
path) and by tests/test_gpu_dropin.py (the reference's unchanged model layer
over this library's backend).
"""

from __future__ import annotations

import argparse
import shutil
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"


def install(reference: Path) -> Path:
    src = reference / "breezetoken"
    if not (src / "__init__.py").is_file() or not (src / "model" / "qwen36_moe.py").is_file():
        raise SystemExit(f"{reference} does not look like a breezetoken checkout")
    dst = TARGET / "breezetoken"
    if dst.exists():
        shutil.rmtree(dst)
    TARGET.mkdir(parents=True, exist_ok=True)
    shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    return dst


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("reference", type=Path, help="a checkout of xushuxun/breezetoken")
    print(install(ap.parse_args().reference))


if __name__ == "__main__":
    main()
