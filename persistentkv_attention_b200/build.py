"""Builds the engine's shared library, ``lib/libpkv_b200.so``, with nvcc for sm_100a.

The library is plain C ABI (``include/pkv_b200.h``) with the CUDA runtime linked
statically, so it loads without PyTorch and travels with the source tree.

A second variant, ``lib/libpkv_b200_stamps.so``, is the same library compiled
with ``PKV_PHASE_STAMPS``: every decode CTA records %globaltimer stamps of its
phases (entry, schedule, first pages, first copy, first data, last stage,
merge, exit), read back with ``pkv_phase_stamps``.  It is a diagnostic build;
``PKV_LIB_VARIANT=stamps`` makes ``_native.load`` pick it.

    python -m persistentkv_attention_b200.build [--force] [--variant all|default|stamps]
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

# the decode-kernel instantiations are split by (dtype, gather) so they build in parallel
SOURCES = ["pkv_api.cu", "pkv_inst_f16_cpasync.cu", "pkv_inst_f16_tma.cu",
           "pkv_inst_bf16_cpasync.cu", "pkv_inst_bf16_tma.cu", "pkv_inst_e4m3.cu",
           "pkv_sched.cpp", "pkv_engine.cpp"]
HEADERS = ["pkv_device.cuh", "pkv_kernels.cuh", "pkv_aux_kernels.cuh", "pkv_launch.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden"]
VARIANTS = {"default": ([], "libpkv_b200.so"),
            "stamps": (["-DPKV_PHASE_STAMPS"], "libpkv_b200_stamps.so")}


def lib_path(variant: str = "default") -> Path:
    return LIB_DIR / VARIANTS[variant][1]


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


def up_to_date(variant: str = "default") -> bool:
    path = lib_path(variant)
    if not path.exists():
        return False
    built = path.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _inputs() if p.exists())


def _compile(src: str, variant: str, verbose: bool) -> Path:
    out_dir = BUILD_DIR / variant
    obj = out_dir / (src + ".o")
    defines = VARIANTS[variant][0]
    cmd = [nvcc(), *COMMON_FLAGS, *defines, *ARCH_FLAGS, "-I", str(REPO_DIR / "include"),
           "-c", str(CSRC / src), "-o", str(obj)]
    if src.endswith(".cu") and verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        sys.stdout.write(proc.stderr)
    return obj


def build_variant(variant: str = "default", force: bool = False, verbose: bool = False) -> Path:
    """Compiles and links one variant unless it is newer than every input."""
    path = lib_path(variant)
    if not force and up_to_date(variant):
        return path
    (BUILD_DIR / variant).mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    workers = max(1, min(len(SOURCES), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        objs = list(pool.map(lambda s: _compile(s, variant, verbose), SOURCES))
    tmp = path.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
           *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, path)
    return path


def build(force: bool = False, verbose: bool = False, variants=("default", "stamps")) -> Path:
    """Builds every requested variant; returns the path of the regular library."""
    for v in variants:
        build_variant(v, force, verbose)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas register usage")
    parser.add_argument("--variant", choices=["all", *VARIANTS], default="all")
    args = parser.parse_args()
    variants = tuple(VARIANTS) if args.variant == "all" else (args.variant,)
    for v in variants:
        print(build_variant(v, force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
