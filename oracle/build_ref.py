"""Builds the reference's own code from its sources, in place, into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY: the artefacts are checkers (and the timed CPU
baseline), never part of the engine.  Nothing is copied from the reference
into this repository; only the compiled outputs land in ``oracle/_ref/``,
which git ignores but which travels with the tree to the GPU box.

Artefacts (all built from the reference checkout: the directory named by
``PKV_REFERENCE_DIR``, else the ``reference_path`` that ``BASELINE.json``
records; nothing is built when neither names an existing checkout):

* ``libref_smoke.so`` -- ``tests/smoke_test.cu`` (with ``kernels/
  persistentkv_attention.cuh``) compiled as a shared library with its ``main``
  renamed; exports the reference's CPU oracle ``cpu_gqa_attention``
  (smoke_test.cu:35-74), callable on any host.
* ``smoke_test`` -- the reference smoke test as an sm_100a executable.
* ``torch_ext/persistentkv_torch_ext*.so`` -- the reference's PyTorch extension
  (``tests/persistentkv_torch_extension.cu``) for sm_100a with the flags of its
  harness (benchmark_serving_trace.py:140-155), the GPU parity target.

    python -m oracle.build_ref [--skip-torch-ext]
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
REF_OUT = ORACLE_DIR / "_ref"


def _reference_dir() -> Path | None:
    env = os.environ.get("PKV_REFERENCE_DIR")
    if env:
        return Path(env)
    baseline = ORACLE_DIR.parent / "BASELINE.json"
    try:
        recorded = json.loads(baseline.read_text()).get("reference_path")
    except (OSError, ValueError):
        recorded = None
    return Path(recorded) if recorded else None


REFERENCE_DIR = _reference_dir()
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")


def reference_present() -> bool:
    return REFERENCE_DIR is not None and (
        REFERENCE_DIR / "kernels" / "persistentkv_attention.cuh").exists()


def _newer(target: Path, *sources: Path) -> bool:
    return target.exists() and all(target.stat().st_mtime >= s.stat().st_mtime for s in sources)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def build_smoke(force: bool = False) -> None:
    src = REFERENCE_DIR / "tests" / "smoke_test.cu"
    hdr = REFERENCE_DIR / "kernels" / "persistentkv_attention.cuh"
    REF_OUT.mkdir(parents=True, exist_ok=True)
    lib = REF_OUT / "libref_smoke.so"
    if force or not _newer(lib, src, hdr):
        # flags of the reference's build script (build_and_run.sh:11) for sm_100a
        _run([NVCC, "-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC", "-shared",
              "-Dmain=pkv_reference_smoke_main", str(src), "-o", str(lib)])
    exe = REF_OUT / "smoke_test"
    if force or not _newer(exe, src, hdr):
        _run([NVCC, "-O3", "-std=c++17", "-lineinfo", *ARCH, str(src), "-o", str(exe)])


def build_torch_ext(force: bool = False) -> Path:
    from torch.utils.cpp_extension import load

    out = REF_OUT / "torch_ext"
    out.mkdir(parents=True, exist_ok=True)
    src = REFERENCE_DIR / "tests" / "persistentkv_torch_extension.cu"
    existing = sorted(out.glob("persistentkv_torch_ext*.so"))
    if existing and not force and _newer(existing[0], src,
                                         REFERENCE_DIR / "kernels" / "persistentkv_attention.cuh"):
        return existing[0]
    load(
        name="persistentkv_torch_ext",
        sources=[str(src)],
        extra_include_paths=[str(REFERENCE_DIR)],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=[
            "-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
            "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
            "-U__CUDA_NO_HALF2_OPERATORS__", "-gencode=arch=compute_100a,code=sm_100a",
        ],
        build_directory=str(out),
        verbose=False,
    )
    return sorted(out.glob("persistentkv_torch_ext*.so"))[0]


def build(force: bool = False, torch_ext: bool = True) -> bool:
    """Builds every artefact; returns False (and builds nothing) without the reference."""
    if not reference_present():
        return False
    build_smoke(force)
    if torch_ext:
        build_torch_ext(force)
    return True


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--skip-torch-ext", action="store_true")
    args = parser.parse_args()
    if not build(args.force, not args.skip_torch_ext):
        print("reference sources not found; nothing built", file=sys.stderr)
        sys.exit(1)
    print(REF_OUT)


if __name__ == "__main__":
    main()
