"""Build libqrb200.so in-tree with nvcc for sm_100a.

The shared library is written next to this file (``gpumode_qr_b200/libqrb200.so``)
so that it travels with the source tree; object files go to ``_build/``.
Run as ``python -m gpumode_qr_b200.build`` or call :func:`build_library`.
"""

from __future__ import annotations

import concurrent.futures as cf
import fcntl
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libqrb200.so"
INCLUDE_DIR = PKG_DIR.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE_DIR}",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libqrb200")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cu*")) + sorted(INCLUDE_DIR.glob("*.h"))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libqrb200.so``.

    Concurrent callers (several ranks starting at once) serialise on a lock
    file; whoever gets it second finds the library fresh and returns.
    """
    if not force and not needs_build():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    with open(BUILD_DIR / ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and not needs_build():
                return LIB_PATH
            return _build_locked(verbose)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)


def _build_locked(verbose: bool) -> Path:
    nvcc = _nvcc()
    srcs = _sources()

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
        if verbose and res.stderr:
            print(res.stderr)
        return obj

    workers = min(len(srcs), os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    p = build_library(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
