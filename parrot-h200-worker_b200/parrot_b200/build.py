"""Compile ``libparrot_b200.so`` in-tree with nvcc for sm_100a.

``python -m parrot_b200.build`` (or ``__graft_entry__.build()``) compiles each
``csrc/*.cu`` to an object under ``_build/`` in parallel and links the shared
library next to this file, where ``parrot_b200._lib`` loads it.  nvcc
cross-compiles, so this runs on a machine without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import fcntl
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_DIR = PKG_DIR.parent / "csrc"
INCLUDE_DIR = PKG_DIR.parent.parent / "include"
BUILD_DIR = PKG_DIR.parent / "_build"
LIB_PATH = PKG_DIR / "libparrot_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                "--expt-relaxed-constexpr", f"-I{INCLUDE_DIR}", f"-I{SRC_DIR}"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build parrot_b200")


def _sources() -> list[Path]:
    return sorted(SRC_DIR.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(SRC_DIR.glob("*.cuh")) + sorted(SRC_DIR.glob("*.h")) + \
        sorted(INCLUDE_DIR.glob("*.h"))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Build the library if any source is newer than it; return its path.

    Processes that call this at once (the ranks of a torchrun job) take turns
    on a lock file: the first builds, the others then find it up to date.
    Without it they overwrote each other's objects and one loaded a library
    linked from a half-written set."""
    if not force and up_to_date():
        return LIB_PATH
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    with open(BUILD_DIR / "build.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and up_to_date():
                return LIB_PATH
            return _build_locked(verbose, ptxas_info)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)


def _build_locked(verbose: bool, ptxas_info: bool) -> Path:
    exe = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [exe, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        return obj, res.stdout + res.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_one, _sources()))
    logs = "".join(log for _, log in results)
    tmp = LIB_PATH.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [exe, *ARCH_FLAGS, "-shared", "-o", str(tmp), *[str(o) for o, _ in results],
           "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    if verbose or ptxas_info:
        sys.stdout.write(logs)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
