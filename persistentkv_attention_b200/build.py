"""Builds the engine's shared library, ``lib/libpkv_b200.so``, with nvcc for sm_100a.

The library is plain C ABI (``include/pkv_b200.h``) with the CUDA runtime linked
statically, so it loads without PyTorch and travels with the source tree.

    python -m persistentkv_attention_b200.build [--force]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libpkv_b200.so"

SOURCES = ["pkv_api.cu", "pkv_sched.cpp", "pkv_engine.cpp"]
HEADERS = ["pkv_device.cuh", "pkv_kernels.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden"]


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [
        REPO_DIR / "include" / "pkv_b200.h",
        Path(__file__),
    ]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _inputs() if p.exists())


def _compile(src: str, verbose: bool) -> Path:
    obj = BUILD_DIR / (src + ".o")
    cmd = [nvcc(), *COMMON_FLAGS, *ARCH_FLAGS, "-I", str(REPO_DIR / "include"),
           "-c", str(CSRC / src), "-o", str(obj)]
    if src.endswith(".cu"):
        cmd[1:1] = ["-Xptxas", "-v"] if verbose else []
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        sys.stdout.write(proc.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles and links the library unless it is newer than every input."""
    if not force and up_to_date():
        return LIB_PATH
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose), SOURCES))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
           *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas register usage")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
