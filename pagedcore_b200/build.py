"""Build the native library ``libpagedkv.so`` in-tree for sm_100a.

The library holds the C++ block ledger and the CUDA kernels behind the C ABI
declared in ``include/pagedkv.h``.  It is compiled with nvcc for
``arch=compute_100a,code=sm_100a`` and links the CUDA runtime statically, so
it loads (and the ledger runs) on machines without a GPU.

Usage: ``python -m pagedcore_b200.build [--force]``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
LIBRARY = PACKAGE_DIR / "libpagedkv.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def _inputs() -> list[Path]:
    return [*sources(), *CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in _inputs())


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    if default.exists():
        return str(default)
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libpagedkv.so")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every source into ``libpagedkv.so`` (skipped when up to date)."""
    if not force and up_to_date():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    command = [
        nvcc(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC,-O3",
        "-shared",
        "-cudart",
        "static",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
        "-o",
        str(tmp),
        *[str(path) for path in sources()],
    ]
    if verbose:
        command.insert(1, "-Xptxas=-v")
        print(" ".join(command), file=sys.stderr)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"building libpagedkv.so failed:\n{result.stdout}\n{result.stderr}")
    if verbose and result.stderr:
        print(result.stderr, file=sys.stderr)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
