"""Loaders for the reference artefacts built by ``oracle/build_ref.py``.

TEST INFRASTRUCTURE ONLY (checkers and the timed CPU baseline).  Everything
here reads ``oracle/_ref/``, which travels with the tree; nothing reads the
reference checkout at run time.
"""

from __future__ import annotations

import ctypes
import importlib.util
from pathlib import Path

import numpy as np

REF_OUT = Path(__file__).resolve().parent / "_ref"

_cpu_lib = None


def ref_cpu_available() -> bool:
    return (REF_OUT / "libref_smoke.so").exists()


def _cpu():
    global _cpu_lib
    if _cpu_lib is None:
        lib = ctypes.CDLL(str(REF_OUT / "libref_smoke.so"))
        # void cpu_gqa_attention(const float*, const float*, const float*, float*,
        #                        int B, int Hq, int Hkv, int N, int d)   smoke_test.cu:35
        fn = getattr(lib, "_Z17cpu_gqa_attentionPKfS0_S0_Pfiiiii")
        fp = ctypes.POINTER(ctypes.c_float)
        fn.argtypes = [fp, fp, fp, fp] + [ctypes.c_int] * 5
        fn.restype = None
        _cpu_lib = fn
    return _cpu_lib


def cpu_gqa_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Runs the reference's own fp32 CPU oracle: q [B,Hq,D], k/v [B,Hkv,N,D] -> [B,Hq,D].

    The call releases the GIL, so independent calls can run on several threads.
    """
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    b, hq, d = q.shape
    hkv, n = k.shape[1], k.shape[2]
    out = np.zeros((b, hq, d), dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    _cpu()(q.ctypes.data_as(fp), k.ctypes.data_as(fp), v.ctypes.data_as(fp),
           out.ctypes.data_as(fp), b, hq, hkv, n, d)
    return out


def torch_ext_path() -> Path | None:
    found = sorted((REF_OUT / "torch_ext").glob("persistentkv_torch_ext*.so"))
    return found[0] if found else None


def load_torch_ext():
    """Imports the reference's PyTorch extension built for sm_100a, or None."""
    path = torch_ext_path()
    if path is None:
        return None
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location("persistentkv_torch_ext", str(path))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module
