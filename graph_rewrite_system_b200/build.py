"""Build ``libgrs_b200.so`` in-tree from ``csrc/*.cu`` with nvcc for sm_100a.

The library is a plain C-ABI shared object (see ``include/grs_b200.h``); it
links only the CUDA runtime, so it loads through ``ctypes`` without any torch
C++ ABI coupling.  Objects are compiled in parallel into ``_build/`` and
relinked only when a source or header is newer than the library.
"""
from __future__ import annotations

import concurrent.futures as futures
import os
from pathlib import Path
import shutil
import subprocess
import sys

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libgrs_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgrs_b200.so")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def _compile(src: Path, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-I", str(CSRC),
           "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile every kernel source and link the in-tree shared library."""
    extra = list(extra or [])
    if not force and not _stale():
        return LIBRARY
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    with futures.ThreadPoolExecutor(max_workers=min(8, len(srcs) or 1)) as pool:
        objs = list(pool.map(lambda s: _compile(s, extra), srcs))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objs),
           "-o", str(tmp), "-lcudart"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stderr}")
    os.replace(tmp, LIBRARY)
    if verbose:
        print(f"built {LIBRARY}")
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
