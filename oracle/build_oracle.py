"""Builds the C oracle port (``oracle/pkv_oracle.c``) into ``oracle/_build/``.

TEST INFRASTRUCTURE ONLY.  ``port_decode`` runs it on numpy arrays.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "pkv_oracle.c"
LIB = ORACLE_DIR / "_build" / "libpkv_oracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", str(SRC),
           "-o", str(LIB), "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stderr}")
    return LIB


_fn = None


def _load():
    global _fn
    if _fn is None:
        lib = ctypes.CDLL(str(build()))
        fn = lib.pkv_oracle_paged_decode
        p = ctypes.c_void_p
        fn.argtypes = [p] * 8 + [ctypes.c_int] * 10
        fn.restype = ctypes.c_int
        _fn = fn
    return _fn


def port_decode(q_source: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray,
                block_table: np.ndarray, seq_lens: np.ndarray, q_indices=None, out_indices=None,
                out_rows=None, is_bf16=False, threads: int | None = None) -> np.ndarray:
    """q_source/k_pages/v_pages as uint16 bit patterns (fp16 or bf16)."""
    q_source = np.ascontiguousarray(q_source.view(np.uint16))
    k_pages = np.ascontiguousarray(k_pages.view(np.uint16))
    v_pages = np.ascontiguousarray(v_pages.view(np.uint16))
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    b = bt.shape[0]
    qi = None if q_indices is None else np.ascontiguousarray(q_indices, dtype=np.int32)
    oi = None if out_indices is None else np.ascontiguousarray(out_indices, dtype=np.int32)
    rows = out_rows if out_rows is not None else b
    out = np.zeros((rows, q_source.shape[1], 128), np.float32)
    threads = threads or len(os.sched_getaffinity(0))
    rc = _load()(q_source.ctypes.data, k_pages.ctypes.data, v_pages.ctypes.data, bt.ctypes.data,
                 sl.ctypes.data, None if qi is None else qi.ctypes.data,
                 None if oi is None else oi.ctypes.data, out.ctypes.data, b, q_source.shape[0],
                 rows, q_source.shape[1], k_pages.shape[1], k_pages.shape[0], k_pages.shape[2],
                 bt.shape[1], 1 if is_bf16 else 0, threads)
    if rc != 0:
        raise ValueError("oracle: out-of-range page id, length or index")
    return out
