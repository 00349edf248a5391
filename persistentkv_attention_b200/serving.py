"""Decode-step runtime around the kernels: step plans, CUDA graphs, host I/O.

The reference's serving harness compiles per-step metadata in Python
(``compile_persistentkv_metadata``, tests/benchmark_serving_trace.py:655-729),
copies it to the GPU with ``torch.tensor(..., device="cuda")`` and optionally
captures each step in a CUDA graph (:1439-1452).  ``DecodeEngine`` does the
same jobs for this engine:

* ``plan_step``  -- host metadata of one step (block table padded like the
  reference, seq_lens, request-id q indices, dense out indices, and the
  C++-built work queue) in one pinned int32 staging buffer;
* ``upload``     -- one host-to-device copy of that buffer into a
  device-resident ``StepPlan``;
* ``run``        -- one work-queue decode call (fused merge by default);
* ``capture``    -- a CUDA graph of ``run`` for replay;
* ``step_host``  -- the end-to-end call a server makes: one native call
  (``pkv_engine_step_host``) from host metadata and pinned q rows to pinned
  output rows.

``StepGraph`` goes one step further for a serving loop whose q / output
buffers stay put: one CUDA graph, captured once, holds the metadata upload
and the device-scheduled decode, and is replayed for every step whatever
the lengths (the device schedule needs no host work queue).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .ops import _stream
from .scheduler import Router, build_auto_plan, plan_words

HEAD_DIM = 128


@dataclass
class HostPlan:
    buf: torch.Tensor          # pinned int32 staging buffer
    batch: int
    max_pages: int
    num_items: int
    total_slots: int
    bucket: int
    tokens: int                # sum of seq_lens
    plan_words: int = 0        # host plan of the device-side schedule (0: none)
    groups: int = 0            # the plan's group count (0: the maximum)

    def views(self, t: torch.Tensor):
        """Splits a (host or device) copy of the buffer into its fields."""
        b, mp, n = self.batch, self.max_pages, self.num_items
        o = 0
        out = {}
        for name, size in (("block_table", b * mp), ("seq_lens", b), ("q_indices", b),
                           ("out_indices", b), ("split_offsets", b + 1), ("work_items", 5 * n)):
            out[name] = t[o:o + size]
            o += size
        out["block_table"] = out["block_table"].view(b, mp)
        out["work_items"] = out["work_items"].view(n, 5)
        if self.plan_words:
            o = -(-o // 4) * 4                 # the plan starts 16-byte aligned
            out["plan"] = t[o:o + self.plan_words]
        return out

    @property
    def nbytes(self) -> int:
        return int(self.buf.numel() * 4)


@dataclass
class StepPlan:
    """Device-resident metadata of one decode step."""

    host: HostPlan
    dev: torch.Tensor
    fields: dict

    @property
    def batch(self) -> int:
        return self.host.batch


def _staging_size(batch: int, max_pages: int, items: int, plan_words: int = 0) -> int:
    words = batch * max_pages + 4 * batch + 1 + 5 * items
    return (-(-words // 4) * 4 + plan_words) if plan_words else words


class DecodeEngine:
    """Work-queue decode over one paged K/V pool on the current device."""

    def __init__(self, k_pages: torch.Tensor, v_pages: torch.Tensor, hq: int,
                 router: Router | None = None, policy: str = "device", fused: bool = True,
                 requested_splits: int = 0, kv_scales: tuple[float, float] | None = None,
                 use_plan: bool = True, groups: int | str = "router"):
        """``kv_scales`` = (k_scale, v_scale) for ``torch.float8_e4m3fn`` pools
        (q and output are then fp16; device schedule only).  ``use_plan``: with
        the device schedule, each step carries a host plan of the schedule
        (``scheduler.build_auto_plan``) uploaded with its other metadata.
        ``groups``: the device schedule's group count -- "router" (default) the
        router's choice per step (``Router.choose_groups``), 0 the maximum (two
        CTAs per SM), an int a fixed count; without a plan it is the maximum."""
        self.k_pages = k_pages
        self.v_pages = v_pages
        self.hq = hq
        self.hkv = k_pages.shape[1]
        self.page_size = k_pages.shape[2]
        self.kv8 = k_pages.dtype == torch.float8_e4m3fn
        self.dtype = torch.float16 if self.kv8 else k_pages.dtype
        if self.kv8 and (kv_scales is None or policy != "device"):
            raise RuntimeError("an e4m3 K/V cache needs kv_scales and the device schedule")
        self.kv_scales = kv_scales
        self.device = k_pages.device
        if router is None:
            sms = torch.cuda.get_device_properties(self.device).multi_processor_count
            router = Router.b200(hq=hq, hkv=self.hkv, sm_count=sms)
        self.router = router
        self.policy = policy
        self.fused = fused
        self.requested_splits = requested_splits
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.use_plan = use_plan and policy == "device" and not self.kv8
        if not self.use_plan:
            if groups not in (0, "router"):
                raise RuntimeError("a group count other than the maximum needs the host plan")
            groups = 0
        self.groups = groups
        self._workspace = torch.empty(0, device=self.device, dtype=torch.float32)
        self._counters = torch.zeros(0, device=self.device, dtype=torch.int32)
        # buffers replaced by a larger one stay alive: captured graphs may
        # still reference them
        self._retired: list[torch.Tensor] = []

    # ---------------------------------------------------------------- planning
    def plan_step(self, seq_lens, block_rows: np.ndarray, q_indices=None,
                  out: torch.Tensor | None = None) -> HostPlan:
        """Host metadata of one step into a pinned buffer (``out`` reuses one).

        With ``policy="device"`` the step carries no work queue: the kernel
        schedules itself from seq_lens."""
        seq = np.asarray(seq_lens, dtype=np.int32)
        b = seq.size
        if self.policy == "device":
            items, offsets, n_items = None, np.zeros(b + 1, np.int32), 0
            total_slots = b + self._auto_groups()
        else:
            queue = self.router.build_workqueue(seq, b, self.policy, self.requested_splits)
            items, offsets, n_items = queue.work_items, queue.split_offsets, queue.num_items
            total_slots = queue.total_slots
        mp = block_rows.shape[1]
        pw = plan_words(self.hkv, self.sm_count) if self.use_plan else 0
        size = _staging_size(b, mp, n_items, pw)
        if out is None or out.numel() < size:
            out = torch.empty(size, dtype=torch.int32, pin_memory=True)
        buf = out[:size]
        groups = 0
        if pw and self.groups == "router":
            groups = self.router.choose_groups(seq)[0]
        elif pw:
            groups = int(self.groups)
        plan = HostPlan(buf, b, mp, n_items, total_slots, int(seq.max(initial=1)),
                        int(seq.sum()), pw, groups)
        v = plan.views(buf)
        v["block_table"].numpy()[:] = block_rows
        v["seq_lens"].numpy()[:] = seq
        v["q_indices"].numpy()[:] = np.arange(b) if q_indices is None else q_indices
        v["out_indices"].numpy()[:] = np.arange(b)
        v["split_offsets"].numpy()[:] = offsets
        if items is not None:
            v["work_items"].numpy()[:] = items
        if pw:
            build_auto_plan(seq, block_rows, mp, self.page_size, self.hkv, self.sm_count,
                            q_indices=v["q_indices"].numpy(), out_indices=v["out_indices"].numpy(),
                            out=v["plan"].numpy(), groups=groups)
        return plan

    def _auto_groups(self) -> int:
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        return max(1, (2 * sms) // self.hkv)

    def plan_from_trace(self, requests, state) -> HostPlan:
        """Plan of one reference-style trace step (q rows indexed by request id)."""
        by_id = {r.request_id: r for r in requests}
        page_count = math.ceil(max(state.lengths) / self.page_size)
        rows = np.empty((len(state.active_ids), page_count), dtype=np.int32)
        for i, rid in enumerate(state.active_ids):
            pages = by_id[rid].physical_pages[:page_count]
            if len(pages) < page_count:
                pages = pages + (by_id[rid].physical_pages[-1],) * (page_count - len(pages))
            rows[i] = pages
        return self.plan_step(state.lengths, rows, q_indices=np.asarray(state.active_ids))

    def upload(self, plan: HostPlan, dev_buf: torch.Tensor | None = None,
               non_blocking: bool = False) -> StepPlan:
        if dev_buf is None or dev_buf.numel() < plan.buf.numel():
            dev_buf = torch.empty(plan.buf.numel(), dtype=torch.int32, device=self.device)
        dev = dev_buf[: plan.buf.numel()]
        dev.copy_(plan.buf, non_blocking=non_blocking)
        self.reserve(plan.batch, plan.total_slots)
        return StepPlan(plan, dev, plan.views(dev))

    def reserve(self, batch: int, total_slots: int) -> None:
        """Grows the shared workspace / merge counters (never inside a capture)."""
        need = ops.workqueue_workspace_bytes(total_slots, self.hq) // 4
        if self._workspace.numel() < need:
            self._retired.append(self._workspace)
            self._workspace = torch.empty(need, device=self.device, dtype=torch.float32)
        if self._counters.numel() < batch * self.hkv:
            self._retired.append(self._counters)
            self._counters = torch.zeros(batch * self.hkv, device=self.device, dtype=torch.int32)

    # ---------------------------------------------------------------- execution
    def run(self, plan: StepPlan, q_source: torch.Tensor, out: torch.Tensor) -> None:
        f = plan.fields
        counters = self._counters[: plan.batch * self.hkv].view(plan.batch, self.hkv)
        if self.kv8:
            ops.paged_attention_auto_fp8(
                q_source, self.k_pages, self.v_pages, self.kv_scales[0], self.kv_scales[1],
                f["block_table"], f["seq_lens"], out, self._workspace, f["q_indices"],
                f["out_indices"], counters if self.fused else None)
            return
        if self.policy == "device":
            ops.paged_attention_auto(
                q_source, self.k_pages, self.v_pages, f["block_table"], f["seq_lens"], out,
                self._workspace, f["q_indices"], f["out_indices"],
                counters if self.fused else None, plan=f.get("plan"), groups=plan.host.groups)
            return
        ops.paged_attention_workqueue(
            q_source, self.k_pages, self.v_pages, f["block_table"], f["seq_lens"],
            f["work_items"], f["split_offsets"], counters, f["q_indices"], f["out_indices"], out,
            self._workspace, plan.host.bucket, self.page_size, plan.host.total_slots, self.fused)

    def run_state(self, plan: StepPlan, q_source: torch.Tensor, state_out: torch.Tensor) -> None:
        """One decode of this GPU's pages into the (m, l, acc) state [B, Hq, 130]."""
        f = plan.fields
        counters = self._counters[: plan.batch * self.hkv].view(plan.batch, self.hkv)
        ops.paged_attention_auto_state(
            q_source, self.k_pages, self.v_pages, f["block_table"], f["seq_lens"], state_out,
            self._workspace, f["q_indices"], counters if self.fused else None)

    def run_sharded(self, plan: StepPlan, q_source: torch.Tensor, out: torch.Tensor,
                    exchange) -> None:
        """One sequence-sharded step: this GPU's pages, exchange and merge fused
        into one launch (``ops.paged_attention_sharded``)."""
        f = plan.fields
        counters = self._counters[: plan.batch * self.hkv].view(plan.batch, self.hkv)
        ops.paged_attention_sharded(
            q_source, self.k_pages, self.v_pages, f["block_table"], f["seq_lens"], out,
            self._workspace, counters, exchange, f["q_indices"], f["out_indices"],
            plan=f.get("plan"), groups=plan.host.groups)

    def _step_host_native(self, seq_lens, block_rows, q_host, out_host, scratch):
        seq = np.ascontiguousarray(seq_lens, dtype=np.int32)
        rows = np.ascontiguousarray(block_rows, dtype=np.int32)
        b, width = rows.shape
        if seq.shape != (b,):
            raise RuntimeError("seq_lens batch mismatch")
        # tensor checks once per (q_host, out_host) pair: a serving loop reuses them
        key = (id(q_host), id(out_host), q_host.data_ptr(), out_host.data_ptr())
        if scratch.get("checked") != key:
            if not (q_host.is_contiguous() and out_host.is_contiguous()):
                raise RuntimeError("q_host and out_host must be contiguous")
            if q_host.dtype != self.dtype or out_host.dtype != self.dtype:
                raise RuntimeError("q_host / out_host dtype must match the K/V pool")
            if (q_host.shape[1:] != (self.hq, HEAD_DIM)
                    or out_host.shape[1:] != (self.hq, HEAD_DIM)):
                raise RuntimeError("q_host / out_host shape mismatch")
            scratch["checked"] = key
            scratch["rows_cap"] = min(q_host.shape[0], out_host.shape[0])
        if b > scratch["rows_cap"]:
            raise RuntimeError("q_host / out_host shape mismatch")
        native = scratch.get("native")
        if native is None or native.max_batch < b or native.max_pages < width:
            # grow geometrically: re-creating the engine synchronises the device
            mb = max(b, 2 * native.max_batch if native else b)
            mp = max(width, 2 * native.max_pages if native else width)
            native = self.reserve_host(scratch, mb, mp)
        return native.step(seq, rows, q_host, out_host)

    def reserve_host(self, scratch: dict, max_batch: int, max_pages: int) -> "NativeEngine":
        """Sizes the native host-step engine kept in ``scratch`` for batches of
        up to ``max_batch`` rows of ``max_pages`` pages (call before timing)."""
        native = scratch.get("native")
        if native is not None and native.max_batch >= max_batch and native.max_pages >= max_pages:
            return native
        if native is not None:
            native.close()
        native = scratch["native"] = NativeEngine(self, max_batch, max_pages)
        return native

    def capture(self, plan: StepPlan, q_source: torch.Tensor, out: torch.Tensor,
                stream: torch.cuda.Stream | None = None) -> torch.cuda.CUDAGraph:
        self.run(plan, q_source, out)          # first call outside capture (attributes, maps)
        graph = torch.cuda.CUDAGraph()
        stream = stream or torch.cuda.Stream(self.device)
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                self.run(plan, q_source, out)
        return graph

    def step_host(self, seq_lens, block_rows: np.ndarray, q_host: torch.Tensor,
                  out_host: torch.Tensor, scratch: dict) -> tuple[int, int]:
        """End-to-end step from pinned host buffers; returns (h2d_bytes, d2h_bytes).

        ``q_host`` [B, Hq, 128] and ``out_host`` are pinned host tensors;
        ``scratch`` keeps the pinned staging and device buffers between calls.
        With the device-side schedule the whole step is one native call
        (``pkv_engine_step_host``); a host-built work queue takes the Python
        path below.
        """
        if self.kv8:
            raise RuntimeError("the native host step serves 16-bit K/V caches")
        if self.policy == "device":
            return self._step_host_native(seq_lens, block_rows, q_host, out_host, scratch)
        plan = self.plan_step(seq_lens, block_rows, out=scratch.get("stage"))
        scratch["stage"] = plan.buf if scratch.get("stage") is None or \
            scratch["stage"].numel() < plan.buf.numel() else scratch["stage"]
        step = self.upload(plan, scratch.get("meta"), non_blocking=True)
        scratch["meta"] = step.dev if scratch.get("meta") is None or \
            scratch["meta"].numel() < step.dev.numel() else scratch["meta"]
        b = plan.batch
        q_dev = scratch.get("q")
        if q_dev is None or q_dev.shape[0] < b:
            q_dev = scratch["q"] = torch.empty(max(b, q_host.shape[0]), self.hq, HEAD_DIM,
                                               dtype=self.dtype, device=self.device)
            scratch["o"] = torch.empty_like(q_dev)
        q_dev[:b].copy_(q_host[:b], non_blocking=True)
        self.run(step, q_dev[:b], scratch["o"][:b])
        out_host[:b].copy_(scratch["o"][:b], non_blocking=True)
        h2d = plan.nbytes + b * self.hq * HEAD_DIM * q_host.element_size()
        d2h = b * self.hq * HEAD_DIM * out_host.element_size()
        return h2d, d2h


class NativeEngine:
    """``pkv_engine``: the C ABI's host-to-host decode step over an engine's pool."""

    def __init__(self, engine: DecodeEngine, max_batch: int, max_pages: int):
        import ctypes

        from . import _native

        self._ct = ctypes
        self._lib = _native.load()
        self._check = _native.check
        self.max_batch, self.max_pages = max_batch, max_pages
        self._ptr = ctypes.c_void_p()
        dt = {torch.float16: _native.PKV_DTYPE_F16, torch.bfloat16: _native.PKV_DTYPE_BF16}
        self._check(self._lib.pkv_engine_create(
            engine.k_pages.data_ptr(), engine.v_pages.data_ptr(), engine.k_pages.shape[0],
            engine.hq, engine.hkv, HEAD_DIM, engine.page_size, dt[engine.dtype], max_batch,
            max_pages, ctypes.byref(self._ptr)))
        self._h2d = ctypes.c_size_t()
        self._d2h = ctypes.c_size_t()
        self._h2d_ref = ctypes.byref(self._h2d)
        self._d2h_ref = ctypes.byref(self._d2h)
        self._step = self._lib.pkv_engine_step_host
        self._keep = engine  # the pools must outlive the native engine

    def step(self, seq: np.ndarray, rows: np.ndarray, q_host: torch.Tensor,
             out_host: torch.Tensor) -> tuple[int, int]:
        # the arrays' addresses through the array interface: ``ndarray.ctypes``
        # builds a helper object per access, a measurable share of a step
        st = self._step(
            self._ptr, seq.__array_interface__["data"][0], rows.__array_interface__["data"][0],
            rows.shape[0], rows.shape[1], q_host.data_ptr(), out_host.data_ptr(), _stream(),
            self._h2d_ref, self._d2h_ref)
        if st != 0:
            self._check(st)
        return self._h2d.value, self._d2h.value

    def close(self) -> None:
        if self._ptr:
            self._check(self._lib.pkv_engine_destroy(self._ptr))
            self._ptr = self._ct.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StepGraph:
    """One captured CUDA graph per engine for every decode step of up to
    ``max_batch`` rows of up to ``max_pages`` pages.

    The graph copies one step's metadata from a pinned staging buffer into
    fixed device buffers and runs ``paged_attention_auto`` (fused merge) on
    them, reading ``self.q`` and writing ``self.out``.  ``step`` writes the
    staging buffer and replays: no capture, no host work queue and one launch
    call per step.  Rows beyond the step's batch get length 0, read q row 0
    and write a spare output row, so the captured batch size never changes.
    Two staging buffers and two graphs alternate; a buffer is rewritten only
    after the replay that read it has finished.
    """

    def __init__(self, engine: DecodeEngine, max_batch: int, max_pages: int, q_rows: int,
                 out_rows: int, stream: torch.cuda.Stream | None = None):
        self.engine = engine
        self.max_batch, self.max_pages = max_batch, max_pages
        self.q_rows, self.out_rows = q_rows, out_rows
        dev, hq = engine.device, engine.hq
        self.q = torch.zeros(q_rows, hq, HEAD_DIM, dtype=engine.dtype, device=dev)
        self._out = torch.zeros(out_rows + 1, hq, HEAD_DIM, dtype=engine.dtype, device=dev)
        self.out = self._out[:out_rows]
        b, mp = max_batch, max_pages
        # [block table | seq_lens | q_indices | out_indices | host plan (16-byte aligned)]
        self._plan_off = -(-(b * mp + 3 * b) // 4) * 4
        self._plan_words = plan_words(engine.hkv, engine.sm_count)
        self._words = self._plan_off + self._plan_words
        self._dev = torch.zeros(self._words, dtype=torch.int32, device=dev)
        self._ws = torch.empty(ops.auto_workspace_bytes(b, hq, engine.hkv) // 4,
                               dtype=torch.float32, device=dev)
        self._counters = torch.zeros(b, engine.hkv, dtype=torch.int32, device=dev)
        bt = self._dev[: b * mp].view(b, mp)
        sl = self._dev[b * mp: b * mp + b]
        qi = self._dev[b * mp + b: b * mp + 2 * b]
        oi = self._dev[b * mp + 2 * b: b * mp + 3 * b]
        plan = self._dev[self._plan_off:]
        self._stage = [torch.zeros(self._words, dtype=torch.int32).pin_memory() for _ in range(2)]
        self._done = [torch.cuda.Event() for _ in range(2)]
        self._graphs = []
        self._stream = stream or torch.cuda.Stream(dev)
        for i in range(2):
            self._fill(i, np.zeros(0, np.int32), np.zeros((0, 1), np.int32), None, None)

            def run(i=i):
                self._dev.copy_(self._stage[i], non_blocking=True)
                ops.paged_attention_auto(self.q, engine.k_pages, engine.v_pages, bt, sl,
                                         self._out, self._ws, qi, oi, self._counters, plan=plan)

            with torch.cuda.stream(self._stream):
                run()  # first call outside capture (kernel attributes, maps)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=self._stream):
                    run()
            self._graphs.append(graph)
        self._stream.synchronize()
        self._next = 0

    def _fill(self, i, seq_lens, block_rows, q_indices, out_indices) -> None:
        b, mp = self.max_batch, self.max_pages
        n, width = block_rows.shape
        if n > b or width > mp:
            raise RuntimeError(f"step of {n} rows x {width} pages exceeds the graph's "
                               f"{b} x {mp}")
        v = self._stage[i].numpy()
        bt = v[: b * mp].reshape(b, mp)
        bt[:n, :width] = block_rows
        bt[:n, width:] = block_rows[:, -1:] if width else 0
        bt[n:] = 0
        v[b * mp: b * mp + b] = 0
        v[b * mp: b * mp + n] = seq_lens
        qi = v[b * mp + b: b * mp + 2 * b]
        qi[:] = 0
        qi[:n] = np.arange(n) if q_indices is None else q_indices
        oi = v[b * mp + 2 * b: b * mp + 3 * b]
        oi[:] = self.out_rows            # the spare row
        oi[:n] = np.arange(n) if out_indices is None else out_indices
        build_auto_plan(v[b * mp: b * mp + b], bt, mp, self.engine.page_size, self.engine.hkv,
                        self.engine.sm_count, q_indices=qi, out_indices=oi,
                        out=v[self._plan_off:])

    def step(self, seq_lens, block_rows: np.ndarray, q_indices=None, out_indices=None) -> None:
        """Queues one decode step on the graph's stream (``self.q`` -> ``self.out``),
        ordered after the work already queued on the caller's current stream.

        ``block_rows`` [B, width] and ``seq_lens`` [B] are host int32; q_indices /
        out_indices (host, default identity) select rows of ``self.q`` / ``self.out``.
        Synchronise the stream (or wait on it) before reading ``self.out``."""
        rows = np.ascontiguousarray(block_rows, dtype=np.int32)
        seq = np.ascontiguousarray(seq_lens, dtype=np.int32)
        if rows.ndim != 2 or seq.shape != (rows.shape[0],):
            raise RuntimeError("block_rows must be [B, width] and seq_lens [B]")
        if int(seq.max(initial=0)) > rows.shape[1] * self.engine.page_size:
            raise RuntimeError("a row is longer than its block-table row")
        for name, idx, limit in (("q_indices", q_indices, self.q_rows),
                                 ("out_indices", out_indices, self.out_rows)):
            if idx is not None:
                idx = np.asarray(idx)
                if idx.shape != seq.shape or (idx.size and (idx.min() < 0 or idx.max() >= limit)):
                    raise RuntimeError(f"{name} out of range")
        i = self._next
        self._next ^= 1
        self._done[i].synchronize()      # the replay that last read staging i is over
        self._fill(i, seq, rows, q_indices, out_indices)
        # after whatever the caller queued on its stream (q rows written, ...)
        self._stream.wait_stream(torch.cuda.current_stream(self.engine.device))
        with torch.cuda.stream(self._stream):
            self._graphs[i].replay()
            self._done[i].record(self._stream)

    @property
    def stream(self) -> torch.cuda.Stream:
        return self._stream

