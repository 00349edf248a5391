"""Split-count router, route cost model and work-queue builder (host side).

Thin Python view of the C++ scheduler in ``csrc/pkv_sched.cpp`` (exported
through the C ABI).  ``Router.reference()`` carries the constants of the
reference's serving harness (tests/benchmark_serving_trace.py:33-43) and
reproduces its integer decisions exactly; ``Router.b200()`` is calibrated for
one B200.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native

ROUTE_NAMES = {
    _native.PKV_ROUTE_SINGLE_PASS: "single_pass",
    _native.PKV_ROUTE_BUCKET: "bucket",
    _native.PKV_ROUTE_WORKQUEUE: "workqueue",
}
ROUTES = {v: k for k, v in ROUTE_NAMES.items()}
POLICIES = {
    "reference": _native.PKV_SPLITS_REFERENCE,
    "balanced": _native.PKV_SPLITS_BALANCED,
    "fixed": _native.PKV_SPLITS_FIXED,
}


def _i32(values) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(values, dtype=np.int32).reshape(-1))


def _ptr(arr: np.ndarray):
    return arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


@dataclass
class WorkQueue:
    """One decode step's compact work queue (reference [T, 5] int32 format)."""

    work_items: np.ndarray      # [T, 5] int32 {row, kvh, split, tile_begin, tile_end}
    split_offsets: np.ndarray   # [B + 1] int32
    total_slots: int

    @property
    def num_items(self) -> int:
        return int(self.work_items.shape[0])


class Router:
    def __init__(self, params: _native.RouterParams):
        self.params = params
        self._lib = _native.load()

    @classmethod
    def reference(cls, hq: int = 32, hkv: int = 8) -> "Router":
        p = _native.RouterParams()
        _native.load().pkv_router_params_reference(ctypes.byref(p))
        p.hq, p.hkv = hq, hkv
        return cls(p)

    @classmethod
    def b200(cls, hq: int = 32, hkv: int = 8, sm_count: int | None = None, **overrides) -> "Router":
        p = _native.RouterParams()
        _native.load().pkv_router_params_b200(ctypes.byref(p))
        p.hq, p.hkv = hq, hkv
        if sm_count is not None:
            p.sm_count = sm_count
        for key, value in overrides.items():
            setattr(p, key, value)
        return cls(p)

    # ---- reference split heuristics (benchmark_serving_trace.py:328-415)
    def choose_workqueue_row_splits(self, length: int, active_count: int,
                                    requested_splits: int, auto_splits: bool) -> int:
        return self._lib.pkv_choose_workqueue_row_splits(
            ctypes.byref(self.params), int(length), int(active_count), int(requested_splits),
            1 if auto_splits else 0)

    def choose_splits(self, lengths, requested_splits: int, auto_splits: bool,
                      single_bucket: bool) -> int:
        arr = _i32(lengths)
        return self._lib.pkv_choose_splits(ctypes.byref(self.params), _ptr(arr), arr.size,
                                           int(requested_splits), 1 if auto_splits else 0,
                                           1 if single_bucket else 0)

    def model_bucket_splits(self, lengths) -> int:
        arr = _i32(lengths)
        return self._lib.pkv_model_bucket_splits(ctypes.byref(self.params), _ptr(arr), arr.size)

    def model_workqueue_splits(self, lengths) -> int:
        arr = _i32(lengths)
        return self._lib.pkv_model_workqueue_splits(ctypes.byref(self.params), _ptr(arr),
                                                    arr.size)

    # ---- cost model (benchmark_serving_trace.py:418-488)
    def estimate_route_ms(self, lengths, route: str, splits: int) -> float:
        arr = _i32(lengths)
        return self._lib.pkv_estimate_route_ms(ctypes.byref(self.params), _ptr(arr), arr.size,
                                               ROUTES[route], int(splits))

    def choose_route(self, lengths) -> tuple[str, int, float]:
        arr = _i32(lengths)
        splits = ctypes.c_int(0)
        ms = ctypes.c_double(0.0)
        route = self._lib.pkv_choose_route(ctypes.byref(self.params), _ptr(arr), arr.size,
                                           ctypes.byref(splits), ctypes.byref(ms))
        return ROUTE_NAMES[route], int(splits.value), float(ms.value)

    def choose_groups(self, lengths) -> tuple[int, float]:
        """Group count of the device-side schedule for one step and its modelled
        microseconds (``pkv_choose_groups``)."""
        arr = _i32(lengths)
        us = ctypes.c_double(0.0)
        ng = self._lib.pkv_choose_groups(ctypes.byref(self.params), _ptr(arr), arr.size,
                                         ctypes.byref(us))
        return int(ng), float(us.value)

    # ---- work-queue builder (benchmark_serving_trace.py:686-703, clamped)
    def build_workqueue(self, seq_lens, active_count: int | None = None,
                        policy: str = "balanced", requested_splits: int = 0,
                        out_items: np.ndarray | None = None) -> WorkQueue:
        lens = _i32(seq_lens)
        b = lens.size
        active = b if active_count is None else int(active_count)
        offsets = np.zeros(b + 1, dtype=np.int32)
        n_items = ctypes.c_int(0)
        n_slots = ctypes.c_int(0)
        capacity = 0 if out_items is None else out_items.shape[0]
        items = out_items
        for _ in range(2):
            status = self._lib.pkv_build_workqueue(
                ctypes.byref(self.params), _ptr(lens), b, active, POLICIES[policy],
                int(requested_splits), None if items is None else _ptr(items), capacity,
                _ptr(offsets), ctypes.byref(n_items), ctypes.byref(n_slots))
            if status == _native.PKV_ERR_CAPACITY:
                capacity = n_items.value
                items = np.zeros((capacity, 5), dtype=np.int32)
                continue
            _native.check(status)
            break
        return WorkQueue(items[: n_items.value], offsets, int(n_slots.value))


def auto_groups(hkv: int, sm_count: int) -> int:
    """NG, the group count of the device-side schedule (``pkv_auto_groups``)."""
    return int(_native.load().pkv_auto_groups(int(hkv), int(sm_count)))


def plan_words(hkv: int, sm_count: int) -> int:
    """int32 words of a host plan (``pkv_auto_plan_bytes`` / 4)."""
    return int(_native.load().pkv_auto_plan_bytes(int(hkv), int(sm_count))) // 4


def build_auto_plan(seq_lens, block_rows, max_pages: int, page_size: int, hkv: int,
                    sm_count: int, q_indices=None, out_indices=None,
                    out: np.ndarray | None = None, groups: int = 0) -> np.ndarray:
    """Host plan of the device-side schedule for one step (``pkv_build_auto_plan``):
    the group entries ``pkv_paged_attention_auto_planned`` starts from.  ``block_rows``
    is the host block table [B, width]; ``max_pages`` the launch's row count;
    ``groups`` the schedule's group count (0: the maximum)."""
    lens = _i32(seq_lens)
    rows = np.ascontiguousarray(block_rows, dtype=np.int32)
    b = lens.size
    words = plan_words(hkv, sm_count)
    plan = out if out is not None else np.empty(words, dtype=np.int32)
    if plan.dtype != np.int32 or plan.size < words or not plan.flags.c_contiguous:
        raise RuntimeError("plan buffer must be contiguous int32 with room for the plan")
    qi = None if q_indices is None else _i32(q_indices)
    oi = None if out_indices is None else _i32(out_indices)
    _native.check(_native.load().pkv_build_auto_plan(
        _ptr(lens), _ptr(rows), b, rows.shape[1], None if qi is None else _ptr(qi),
        None if oi is None else _ptr(oi), int(max_pages), int(page_size), int(hkv),
        int(sm_count), int(groups), _ptr(plan), plan.size * 4))
    return plan
