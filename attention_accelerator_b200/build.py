"""In-tree build of the sm_100a CUDA library ``lib/libgqa_b200.so``.

``nvcc`` cross-compiles without a GPU, so this runs on the build host; the built
``.so`` is not committed (``.gitignore``) but travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "lib" / "libgqa_b200.so"
SOURCES = [CSRC / "gqa_abi.cu", CSRC / "gqa_decode.cu", CSRC / "gqa_noalloc.cu", CSRC / "gqa_chunked.cu", CSRC / "gqa_peer.cu",
           CSRC / "gqa_memfile.cu", CSRC / "gqa_rtl.cu"]
HEADERS = [INCLUDE / "gqa_b200.h", CSRC / "gqa_device.cuh", CSRC / "gqa_internal.h"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).is_file():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def is_stale() -> bool:
    if not LIB.is_file():
        return True
    built = LIB.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``lib/libgqa_b200.so`` for sm_100a if it is missing or older than its sources.

    Processes that call this at the same time (the ranks of a torchrun job)
    serialise on a lock file: one compiles, the others then find it fresh."""
    if not force and not is_stale():
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    import fcntl
    with open(LIB.parent / ".build.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and not is_stale():
                return LIB
            return _compile(verbose)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)


def _compile(verbose: bool) -> Path:
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc_path(), "-shared", "-Xcompiler", "-fPIC", "-O3", "-std=c++17", *ARCH_FLAGS, "-lineinfo",
           f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}{res.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print(res.stdout + res.stderr)
    return LIB


if __name__ == "__main__":
    print(build_library(force=True, verbose=True))
