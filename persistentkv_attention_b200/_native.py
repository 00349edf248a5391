"""ctypes binding of ``libpkv_b200.so`` (the C ABI of ``include/pkv_b200.h``).

No torch types cross this boundary: tensors are passed as device pointers plus
sizes, streams as raw ``cudaStream_t`` handles.  The library must exist; there
is no fallback path (build it with ``python -m persistentkv_attention_b200.build``).

``PKV_LIB_VARIANT=stamps`` in the environment loads the diagnostic build
``libpkv_b200_stamps.so`` instead (same ABI; decode CTAs record phase stamps).
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int32, c_size_t, c_uint32, c_void_p
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"
LIB_NAMES = {"default": "libpkv_b200.so", "stamps": "libpkv_b200_stamps.so"}
LIB_PATH = LIB_DIR / LIB_NAMES["default"]

PKV_OK = 0
PKV_ERR_INVALID_ARGUMENT = 1
PKV_ERR_UNSUPPORTED = 2
PKV_ERR_MISALIGNED = 3
PKV_ERR_WORKSPACE = 4
PKV_ERR_CUDA = 5
PKV_ERR_NO_DEVICE = 6
PKV_ERR_CAPACITY = 7

PKV_DTYPE_F16 = 0
PKV_DTYPE_BF16 = 1

PKV_SPLITS_REFERENCE = 0
PKV_SPLITS_BALANCED = 1
PKV_SPLITS_FIXED = 2

PKV_GATHER_TMA = 0
PKV_GATHER_CP_ASYNC = 1
GATHER_MODES = {"tma": PKV_GATHER_TMA, "cpasync": PKV_GATHER_CP_ASYNC}
STAMPS_PER_CTA = 32

PKV_ROUTE_SINGLE_PASS = 0
PKV_ROUTE_BUCKET = 1
PKV_ROUTE_WORKQUEUE = 2

DEVERR_BITS = {
    0x1: "page id outside the pool",
    0x2: "token beyond max_pages * page_size",
    0x4: "work item out of range",
    0x8: "partial slot out of range",
    0x10: "q/out index out of range",
    0x20: "pipeline wait timed out",
    0x40: "a peer's sharded state did not arrive in time",
    0x80: "KV append: free-page list exhausted",
}

EXCHANGE_HANDLE_BYTES = 64
MAX_WORLD = 8


class RouterParams(ctypes.Structure):
    """Mirror of ``pkv_router_params``."""

    _fields_ = [
        ("hq", c_int),
        ("hkv", c_int),
        ("head_dim", c_int),
        ("elem_bytes", c_int),
        ("sm_count", c_int),
        ("read_gbps", c_double),
        ("launch_us", c_double),
        ("min_ctas_per_sm", c_double),
        ("supported_g", c_int),
        ("min_split_len", c_int),
        ("ctas_per_sm", c_int),
        ("tasks_per_cta", c_int),
        ("max_splits", c_int),
        ("min_tiles_per_task", c_int),
        ("dev_fixed_us", c_double),
        ("dev_cta_gbps", c_double),
        ("dev_merge_us", c_double),
        ("dev_merge_piece_us", c_double),
    ]


_P = c_void_p
_I32P = POINTER(c_int32)

# name -> (restype, argtypes); every function declared in include/pkv_b200.h
SIGNATURES = {
    "pkv_status_string": (c_char_p, [c_int]),
    "pkv_abi_version": (c_int, []),
    "pkv_last_error_message": (c_char_p, []),
    "pkv_set_gather_mode": (c_int, [c_int]),
    "pkv_get_gather_mode": (c_int, []),
    "pkv_set_math_mode": (c_int, [c_int]),
    "pkv_get_math_mode": (c_int, []),
    "pkv_set_dependent_launch": (c_int, [c_int]),
    "pkv_get_dependent_launch": (c_int, []),
    "pkv_phase_stamps": (c_int, [POINTER(ctypes.c_uint64), c_int, POINTER(c_int)]),
    "pkv_paged_attention": (
        c_int,
        [_P, _P, _P, _P, _P, _P, c_size_t, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_masked": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, c_size_t, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_indexed": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, c_int, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_workqueue": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_auto": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_auto_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "pkv_auto_groups": (c_int, [c_int, c_int]),
    "pkv_auto_plan_bytes": (c_size_t, [c_int, c_int]),
    "pkv_build_auto_plan": (
        c_int, [_I32P, _I32P, c_int, c_int, _I32P, _I32P, c_int, c_int, c_int, c_int, c_int,
                _I32P, c_size_t]),
    "pkv_paged_attention_auto_planned": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, _P, c_size_t, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_auto_state": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_auto_fp8": (
        c_int,
        [_P, _P, _P, c_float, c_float, _P, _P, _P, _P, _P, _P, c_size_t, _P, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_kv_append": (
        c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int,
                c_int, _P]),
    "pkv_engine_create": (
        c_int, [_P, _P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                POINTER(c_void_p)]),
    "pkv_engine_step_host": (
        c_int, [_P, _P, _P, c_int, c_int, _P, _P, _P, POINTER(c_size_t), POINTER(c_size_t)]),
    "pkv_engine_destroy": (c_int, [_P]),
    "pkv_exchange_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "pkv_exchange_create": (
        c_int, [c_int, c_int, c_int, c_int, c_int, POINTER(c_void_p), c_void_p]),
    "pkv_exchange_connect": (c_int, [c_void_p, c_void_p]),
    "pkv_exchange_destroy": (c_int, [c_void_p]),
    "pkv_paged_attention_sharded": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, _P, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_sharded_planned": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _P, _P, _P, c_size_t, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_workqueue_noalloc": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_paged_attention_workqueue_state": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, c_int, c_int, c_int, c_int,
         c_int, c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "pkv_combine_states": (
        c_int, [_P, c_int, _P, _P, c_int, c_int, c_int, c_int, c_int, _P]),
    "pkv_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "pkv_workqueue_workspace_bytes": (c_size_t, [c_int, c_int]),
    "pkv_device_error": (c_int, [POINTER(c_uint32), c_int]),
    "pkv_router_params_reference": (None, [POINTER(RouterParams)]),
    "pkv_router_params_b200": (None, [POINTER(RouterParams)]),
    "pkv_choose_workqueue_row_splits": (c_int, [POINTER(RouterParams), c_int, c_int, c_int, c_int]),
    "pkv_choose_splits": (c_int, [POINTER(RouterParams), _I32P, c_int, c_int, c_int, c_int]),
    "pkv_model_bucket_splits": (c_int, [POINTER(RouterParams), _I32P, c_int]),
    "pkv_model_workqueue_splits": (c_int, [POINTER(RouterParams), _I32P, c_int]),
    "pkv_estimate_route_ms": (c_double, [POINTER(RouterParams), _I32P, c_int, c_int, c_int]),
    "pkv_choose_route": (
        c_int, [POINTER(RouterParams), _I32P, c_int, POINTER(c_int), POINTER(c_double)]),
    "pkv_choose_groups": (c_int, [POINTER(RouterParams), _I32P, c_int, POINTER(c_double)]),
    "pkv_build_workqueue": (
        c_int,
        [POINTER(RouterParams), _I32P, c_int, c_int, c_int, c_int, _I32P, c_int, _I32P,
         POINTER(c_int), POINTER(c_int)],
    ),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library once and declares every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    variant = os.environ.get("PKV_LIB_VARIANT", "default") or "default"
    if variant not in LIB_NAMES:
        raise ImportError(f"PKV_LIB_VARIANT={variant!r}: expected one of {sorted(LIB_NAMES)}")
    path = LIB_DIR / LIB_NAMES[variant]
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m persistentkv_attention_b200.build`"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.pkv_abi_version() != 1:
        raise ImportError("libpkv_b200.so has an unexpected ABI version")
    _lib = lib
    return lib


class PkvError(RuntimeError):
    """Raised for a non-OK status; carries the status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int) -> None:
    if status != PKV_OK:
        lib = load()
        msg = lib.pkv_last_error_message().decode() or lib.pkv_status_string(status).decode()
        raise PkvError(status, msg)


def device_error(clear: bool = True) -> int:
    """Returns (and by default clears) the device error word of the current device."""
    lib = load()
    code = c_uint32(0)
    check(lib.pkv_device_error(ctypes.byref(code), 1 if clear else 0))
    return int(code.value)


def describe_device_error(code: int) -> str:
    return ", ".join(text for bit, text in DEVERR_BITS.items() if code & bit) or "none"


def set_gather_mode(mode: str) -> None:
    """Selects the decode gather of later 16-bit launches: "tma" or "cpasync"."""
    check(load().pkv_set_gather_mode(GATHER_MODES[mode]))


def gather_mode() -> str:
    value = load().pkv_get_gather_mode()
    return {v: k for k, v in GATHER_MODES.items()}[value]


MATH_MODES = {"mma": 0, "fma": 1}


def set_math_mode(mode: str) -> None:
    """Consumer math of later decode launches: "mma" (tensor cores, the
    default) or "fma" (CUDA cores; lean fp16 cp.async route at G = 4)."""
    check(load().pkv_set_math_mode(MATH_MODES[mode]))


def math_mode() -> str:
    value = load().pkv_get_math_mode()
    return {v: k for k, v in MATH_MODES.items()}[value]


def set_dependent_launch(enable: bool) -> None:
    """Programmatic dependent launch for later device-scheduled decode
    launches (``pkv_set_dependent_launch``)."""
    check(load().pkv_set_dependent_launch(1 if enable else 0))


def dependent_launch() -> bool:
    return bool(load().pkv_get_dependent_launch())


def phase_stamps(max_ctas: int = 4096):
    """Per-CTA phase stamps of the last decode launch (diagnostic build only):
    a list of ``STAMPS_PER_CTA``-tuples of %globaltimer nanoseconds."""
    lib = load()
    buf = (ctypes.c_uint64 * (max_ctas * STAMPS_PER_CTA))()
    n = c_int(0)
    check(lib.pkv_phase_stamps(buf, max_ctas, ctypes.byref(n)))
    return [tuple(buf[i * STAMPS_PER_CTA:(i + 1) * STAMPS_PER_CTA]) for i in range(n.value)]
