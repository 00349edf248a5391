#!/usr/bin/env python3
"""Decode-step benchmark of the B200 paged decode-attention engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl engine|reference] [--trace-file FILE]
                    [--hkv 32|8|4] [--dtype f16|bf16] [--kv-fp8]
                    [--gather cpasync|tma] [--math mma|fma] [--no-per-config]
                    [--phase-stamps]
                    [--seq-shard [--exchange fused|nccl]]

A step is one continuous-batching decode step of a seeded synthetic trace
(default: BASELINE config 2, B8 uniform [512, 8192] tokens, Hq 32 / Hkv 8,
head_dim 128, page 16, fp16).  With N GPUs every rank decodes its own
independent batch (batch partitioning, weak scaling); the job throughput is
the tokens of all ranks over the slowest rank's device time.

Reported (one JSON line on rank 0):
  value       tokens/s with all inputs resident in HBM, per-step CUDA-event
              intervals around graph-replayed decode steps; before every step,
              outside the intervals, L2 is flushed by a 256 MiB write and a
              256 MiB read (so no dirty lines are left for the timed step);
  e2e         tokens/s through the public API from host buffers
              (DecodeEngine.step_host -> pkv_engine_step_host): per step,
              staging of lengths + block rows, a stage-in kernel copying
              metadata and pinned q rows to the device, the decode (launched
              behind it), output rows written into pinned host memory; with
              the split of one step into host call, interval and decode;
  roofline    algorithmic K/V bytes per step / step interval vs the measured
              HBM copy bandwidth;
  per_config  configs 1 and 3-5, the default config with the other gather,
              the default config and config 5 with CUDA-core math (fp32 FMA
              instead of mma.sync), and 8 model layers back to back, measured
              in the same run, same timing method, each with its correctness
              gate on every row of one step;
  cpu_baseline the reference's torch CPU repack + SDPA path
              (tests/benchmark_torch_paged_sdpa.py:90-109) on the host cores,
              bounded sample, with the reference's own cpu_gqa_attention
              (built from its sources) beside it;
  seq_shard   (N > 1) config 4 sequence-sharded across the N GPUs, states
              exchanged over NVLink inside the decode kernel (strong scaling).

``--impl reference`` times the reference CPU implementation alone on the
same workload (rank 0 only).  ``--phase-stamps`` loads the diagnostic build
and prints per-phase timings of the decode CTAs instead of the bench line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from persistentkv_attention_b200 import trace as tr  # noqa: E402

WORKLOADS = {
    "single_b1": dict(trace=None, requests=1, max_active=1, hole=0.0, hkv=8,
                      desc="config 1: B1, 4096 tokens, 256 pages drawn as a seeded permutation "
                           "of a 1024-page pool"),
    "uniform_8k": dict(trace="uniform_8k", requests=24, max_active=8, hole=0.0, hkv=8,
                       desc="config 2: B8 uniform context [512, 8192], 24 requests, 8 active"),
    "bimodal_32k": dict(trace="bimodal_32k", requests=24, max_active=8, hole=0.0, hkv=8,
                        desc="config 3: B8 bimodal 75% [512, 2048] / 25% [16384, 32768]"),
    "long_b1": dict(trace="long_b1", requests=16, max_active=1, hole=0.0, hkv=8,
                    desc="config 4: B1 long context [24576, 32768], 16 sequential requests"),
    "zipf_b64": dict(trace="zipf_b64", requests=128, max_active=64, hole=0.1, hkv=8,
                     desc="config 5: B64 Zipf(1.1) context [256, 32768], 10% holes"),
}
PER_CONFIG = ["single_b1", "uniform_8k", "bimodal_32k", "long_b1", "zipf_b64"]
HQ = 32
PAGE = 16
DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16}
D = 128
SEED = 20260622
FLUSH_BYTES = 256 << 20
LAYERS = 8            # model layers of the back-to-back measurement
# tolerance of the reference (benchmark_serving_trace.py:37-38); bf16 outputs
# add one bf16 rounding of the value (2^-8 relative), since they are stored in bf16
MAX_ERR = 2e-3


def measured_peak_gbs() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event reasons sampled during the timed regions.

    Polls NVML from a background thread (a timed region lasts milliseconds,
    far shorter than nvidia-smi's sampling period); only samples taken
    between ``__enter__`` and ``__exit__`` count, over every region."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: int):
        self.device = device
        self.samples: list[tuple[float, int]] = []
        self.error = None
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml

            self.nvml = pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device)
            bus = (f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:"
                   f"{props.pci_device_id:02X}.0")
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: the line reports why
            self.error = f"{type(exc).__name__}: {exc}"

    def _poll(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                try:
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                except AttributeError:
                    reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                self.samples.append((float(mhz), int(reasons)))
            except Exception as exc:
                self.error = f"{type(exc).__name__}: {exc}"
                return
            self._stop.wait(0.0005)

    def __enter__(self):
        import threading

        self._stop = threading.Event()
        self._thread = None
        if self.handle is not None:
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"error": self.error or "no samples"}
        mask = 0
        for _, r in self.samples:
            mask |= r
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": [name for bit, name in self.REASONS.items() if mask & bit],
                "source": "NVML, polled during the timed regions"}


class L2Flush:
    """Evicts L2 between timed steps without leaving dirty lines behind.

    Writing a buffer larger than L2 evicts everything but leaves up to a full
    L2 of dirty lines, whose write-back would then be charged to the next
    timed kernel; reading a second buffer larger than L2 afterwards forces
    those write-backs here and leaves L2 holding clean, unrelated lines."""

    def __init__(self, dev):
        self.wbuf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.rbuf = torch.ones(FLUSH_BYTES // 8, dtype=torch.int64, device=dev)
        self.acc = torch.empty((), dtype=torch.int64, device=dev)

    def __call__(self, i: int) -> None:
        self.wbuf.fill_(i & 0xFF)
        torch.sum(self.rbuf, dim=0, out=self.acc)


# ------------------------------------------------------------------ workload
TRACE_FILE = None  # --trace-file: request specs of an external trace replace the synthetic lengths


def build_workload(name: str, rank: int, steps_needed: int):
    """(workload dict, requests, physical pages, steps) of a named config."""
    w = dict(WORKLOADS[name])
    if name == "single_b1":
        # config 1: one request of 4096 tokens whose 256 pages are a seeded
        # permutation drawn from a 1024-page pool; the step repeats
        gen = torch.Generator().manual_seed(SEED + 4096 + rank)
        pages = torch.randperm(1024, generator=gen)[:256].tolist()
        req = tr.Request(0, 0, 4096, 1, tuple(pages))
        return w, [req], 1024, [tr.StepState(0, (0,), (4096,))]
    specs = None
    if TRACE_FILE is not None:
        specs = tr.load_trace_specs(TRACE_FILE, w["requests"], PAGE)
        w["requests"] = len(specs)
        w["desc"] = f"trace file {Path(TRACE_FILE).name} ({len(specs)} requests), " \
                    f"{w['max_active']} active, holes {w['hole']}"
    reqs, physical = tr.build_requests(w["trace"], w["requests"], w["max_active"], SEED + rank,
                                       w["hole"], 0, PAGE, specs=specs)
    steps = tr.build_steps(reqs, w["max_active"])
    steps = steps[: max(1, min(len(steps), max(steps_needed, 48)))]
    return w, reqs, physical, steps


def make_inputs(w, physical: int, hkv: int, dtype, dev, rank: int):
    """Seeded N(0,1) K/V pools [physical, hkv, 16, 128] and q pool [requests, 32, 128],
    generated on the device directly in the compute dtype."""
    gen = torch.Generator(device=dev).manual_seed(SEED + 7 + rank)
    k_pages = torch.randn(physical, hkv, PAGE, D, generator=gen, device=dev, dtype=dtype)
    v_pages = torch.randn(physical, hkv, PAGE, D, generator=gen, device=dev, dtype=dtype)
    q_pool = torch.randn(w["requests"], HQ, D, generator=gen, device=dev, dtype=dtype)
    return k_pages, v_pages, q_pool


def kv_bytes(state, hkv: int, elem: int = 2) -> int:
    return int(sum(state.lengths)) * hkv * D * 2 * elem


# ------------------------------------------------------------------ CPU baselines
def cpu_reference_steps(reqs, steps, k_host, v_host, q_host, budget_s: float, hkv: int):
    """Reference cpu_gqa_attention (oracle/_ref) over trace steps, rows in parallel.

    Returns (tokens/s, steps run, threads, kind, seconds)."""
    from oracle import ref as ref_artefacts

    threads = len(os.sched_getaffinity(0))
    by_id = {r.request_id: r for r in reqs}
    use_ref = ref_artefacts.ref_cpu_available()
    if not use_ref:
        from oracle import build_oracle

    g = HQ // hkv

    def row_job(args):
        # one (row, KV head) group: the reference oracle with Hq = G, Hkv = 1
        rid, n, h = args
        pages = np.asarray(by_id[rid].physical_pages[: (n + PAGE - 1) // PAGE], dtype=np.int64)
        k = np.ascontiguousarray(k_host[pages, h].reshape(-1, D)[:n], dtype=np.float32)
        v = np.ascontiguousarray(v_host[pages, h].reshape(-1, D)[:n], dtype=np.float32)
        q = q_host[rid, h * g:(h + 1) * g][None].astype(np.float32)
        return ref_artefacts.cpu_gqa_attention(q, k[None, None], v[None, None])

    tokens = 0
    done = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as pool:
        for state in steps:
            if use_ref:
                list(pool.map(row_job, [(r, n, h) for r, n in zip(state.active_ids, state.lengths)
                                        for h in range(hkv)]))
            else:
                rows = [list(by_id[r].physical_pages) for r in state.active_ids]
                width = max(len(r) for r in rows)
                bt = np.array([r + [r[-1]] * (width - len(r)) for r in rows], np.int32)
                build_oracle.port_decode(q_host.astype(np.float16), k_host.astype(np.float16),
                                         v_host.astype(np.float16), bt, np.array(state.lengths),
                                         q_indices=np.array(state.active_ids),
                                         threads=threads)
            tokens += len(state.active_ids)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
    secs = time.perf_counter() - t0
    return tokens / secs, done, threads, "reference" if use_ref else "port", secs


def cpu_sdpa_steps(reqs, steps, k_host, v_host, q_host, budget_s: float):
    """The reference's torch CPU repack + SDPA path (benchmark_torch_paged_sdpa.py:90-109,
    restated in oracle.pkv_oracle.sdpa_repack_row) on fp32 host tensors, row
    by row, torch's intra-op threads over the host cores.

    Returns (tokens/s, steps run, torch threads, affinity cores, seconds)."""
    from oracle import pkv_oracle as po

    by_id = {r.request_id: r for r in reqs}
    tokens = done = 0
    t0 = time.perf_counter()
    with torch.inference_mode():
        for state in steps:
            for rid, n in zip(state.active_ids, state.lengths):
                pages = torch.tensor(by_id[rid].physical_pages[: (n + PAGE - 1) // PAGE],
                                     dtype=torch.int64)
                po.sdpa_repack_row(q_host[rid], k_host, v_host, pages, n)
            tokens += len(state.active_ids)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
    secs = time.perf_counter() - t0
    return tokens / secs, done, torch.get_num_threads(), len(os.sched_getaffinity(0)), secs


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w, reqs, physical, steps = build_workload(args.workload, 0, args.steps + args.warmup)
    hkv = w["hkv"]
    gen = torch.Generator().manual_seed(SEED + 7)
    k_host = torch.randn(physical, hkv, PAGE, D, generator=gen).half().float().numpy()
    v_host = torch.randn(physical, hkv, PAGE, D, generator=gen).half().float().numpy()
    q_host = torch.randn(w["requests"], HQ, D, generator=gen).half().float().numpy()
    warm = steps[: args.warmup]
    cpu_reference_steps(reqs, warm, k_host, v_host, q_host, 1e9, hkv)
    timed = [steps[(args.warmup + i) % len(steps)] for i in range(args.steps)]
    per_step = max(0.5, 120.0 / max(1, args.steps))
    value, done, threads, kind, secs = cpu_reference_steps(reqs, timed, k_host, v_host, q_host,
                                                           per_step * args.steps, hkv)
    line = {
        "impl": "reference", "metric": "decode-step tokens/s", "value": value,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": done, "warmup": args.warmup,
        "ms_per_step": 1000.0 * secs / max(1, done), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp16-quantised inputs)",
        "data": "synthetic", "config": {"workload": f"{args.workload}: {w['desc']}",
                                        "hq": HQ, "hkv": hkv, "gqa_group": HQ // hkv,
                                        "head_dim": D, "page_size": PAGE,
                                        "active_per_gpu": w["max_active"],
                                        "parallelism": "host cores: the reference's "
                                                       "cpu_gqa_attention over (row, KV head) "
                                                       "groups"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"{done} decode steps of the trace, (row, KV head) groups "
                                    f"in parallel"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ engine arm
class Config:
    """One workload on this GPU: pools, plans, one captured graph per
    distinct step, and its timed run."""

    def __init__(self, name, args, dev, stream, rank, hkv=None, dtype="f16", kv_fp8=False,
                 steps=None, groups="router", layers=1):
        from persistentkv_attention_b200.serving import DecodeEngine

        self.name = name
        self.steps_timed = steps if steps is not None else args.steps
        self.warmup = args.warmup
        w, reqs, physical, trace_steps = build_workload(name, rank,
                                                        self.steps_timed + self.warmup)
        self.w, self.reqs, self.trace_steps = w, reqs, trace_steps
        self.hkv = hkv or w["hkv"]
        self.dtype = dtype
        self.kv_fp8 = kv_fp8
        tdt = DTYPES[dtype]
        k_pages, v_pages, q_pool = make_inputs(w, physical, self.hkv, tdt, dev, rank)
        self.layers = layers
        # layers > 1: that many distinct K/V pools (one per model layer), each
        # step decodes every layer back to back in one graph
        extra = [make_inputs(w, physical, self.hkv, tdt, dev, rank + 1000 * (i + 1))[:2]
                 for i in range(layers - 1)]
        self.kv_elem = 2
        if kv_fp8:
            # e4m3 cache with per-tensor scales; the pools kept here hold the
            # dequantised values for the correctness gate and the CPU baseline
            scales = (float(k_pages.abs().max()) / 448.0, float(v_pages.abs().max()) / 448.0)
            k8 = (k_pages.float() / scales[0]).to(torch.float8_e4m3fn)
            v8 = (v_pages.float() / scales[1]).to(torch.float8_e4m3fn)
            k_pages = (k8.float() * scales[0]).to(tdt)
            v_pages = (v8.float() * scales[1]).to(tdt)
            self.kv_elem = 1
            self.engine = DecodeEngine(k8, v8, HQ, fused=not args.no_fused, kv_scales=scales)
        else:
            self.engine = DecodeEngine(k_pages, v_pages, HQ, fused=not args.no_fused,
                                       groups=groups)
        self.layer_engines = [DecodeEngine(k, v, HQ, fused=not args.no_fused, groups=groups)
                              for k, v in extra]
        self.k_pages, self.v_pages, self.q_pool = k_pages, v_pages, q_pool
        self.stream = stream
        self.plans, self.graphs, self.outs = [], [], []
        n_distinct = min(len(trace_steps), self.steps_timed + self.warmup)
        for state in trace_steps[:n_distinct]:
            self.plans.append(self.engine.upload(self.engine.plan_from_trace(reqs, state)))
        for p in self.plans:
            o = torch.empty(p.batch, HQ, D, dtype=tdt, device=dev)
            self.outs.append(o)
            if layers == 1:
                self.graphs.append(self.engine.capture(p, q_pool, o, stream))
                continue
            # one graph per step holding every layer's decode (same metadata,
            # each layer its own pool, workspace and output)
            outs_l = [torch.empty_like(o) for _ in self.layer_engines]
            for e, ol in zip(self.layer_engines, outs_l):
                e.reserve(p.batch, p.host.total_slots)
                e.run(p, q_pool, ol)
            self.engine.run(p, q_pool, o)
            # the layers' launches chain with programmatic dependent launch, as
            # in a model step: each starts behind the previous layer's tail
            from persistentkv_attention_b200 import _native

            g = torch.cuda.CUDAGraph()
            _native.set_dependent_launch(True)
            try:
                with torch.cuda.stream(stream):
                    with torch.cuda.graph(g, stream=stream):
                        self.engine.run(p, q_pool, o)
                        for e, ol in zip(self.layer_engines, outs_l):
                            e.run(p, q_pool, ol)
            finally:
                _native.set_dependent_launch(False)
            self.graphs.append(g)
        torch.cuda.synchronize()
        self.sched = [i % n_distinct for i in range(self.warmup + self.steps_timed)]

    def timed(self, flush, barrier, clocks):
        """Warm-up, then one CUDA-event interval per step (L2 flushed before
        each, outside the interval).  Returns the per-step milliseconds."""
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(self.steps_timed)]
        with torch.cuda.stream(self.stream):
            for j in self.sched[: self.warmup]:
                flush(j)
                self.graphs[j].replay()
        barrier()
        with clocks:
            with torch.cuda.stream(self.stream):
                torch.cuda._sleep(20_000_000)         # lets the host queue run ahead (~10 ms)
                for i, j in enumerate(self.sched[self.warmup:]):
                    flush(i)
                    ev[i][0].record(self.stream)
                    self.graphs[j].replay()
                    ev[i][1].record(self.stream)
            barrier()
        # per layer: one layer's decode is one step of the metric
        self.times_ms = [a.elapsed_time(b) / self.layers for a, b in ev]
        self.tokens = sum(self.plans[j].batch for j in self.sched[self.warmup:])
        self.bytes_alg = sum(kv_bytes(self.trace_steps[j], self.hkv, self.kv_elem)
                             for j in self.sched[self.warmup:])
        return self.times_ms

    def gate(self):
        """Every row of one mid-trace step against the float64 checker (after
        timing).  Returns the max abs error; raises past the tolerance."""
        from oracle import pkv_oracle as po  # checker only

        j = len(self.plans) // 2
        with torch.cuda.stream(self.stream):
            self.graphs[j].replay()
        torch.cuda.synchronize()
        st = self.trace_steps[j]
        f = self.plans[j].fields
        want = po.torch_paged_decode(self.q_pool, self.k_pages, self.v_pages, f["block_table"],
                                     st.lengths, q_indices=st.active_ids)
        got = self.outs[j].double()
        excess = (got - want).abs() - (MAX_ERR + (2.0 ** -8 * want.abs()
                                                  if self.dtype == "bf16" else 0.0))
        err = float((got - want).abs().max())
        if bool((excess >= 0).any()):
            raise SystemExit(f"correctness gate failed on {self.name}: max abs error {err:.3e}")
        return err

    def groups_used(self):
        """Group counts of the device schedule over the timed steps."""
        used = sorted({self.plans[j].host.groups for j in self.sched[self.warmup:]})
        return ",".join(str(g) for g in used)

    def summary(self, peak):
        total_ms = sum(self.times_ms)
        per_step_bytes = self.bytes_alg / self.steps_timed
        achieved = per_step_bytes / (total_ms / self.steps_timed / 1000.0) / 1e9
        return {"workload": f"{self.name}: {self.w['desc']}", "hkv": self.hkv,
                "dtype": self.dtype + ("; K/V e4m3" if self.kv_fp8 else ""),
                "steps": self.steps_timed, "value": self.tokens / (total_ms / 1000.0),
                "unit": "tokens/s", "ms_per_step": total_ms / self.steps_timed,
                "us_per_step_median": 1000.0 * statistics.median(self.times_ms),
                "groups": self.groups_used(),
                "kv_bytes_per_step": per_step_bytes, "hbm_gbs": achieved,
                "frac_of_measured_peak": achieved / peak, "frac_of_8tbs": achieved / 8000.0}

    def release(self):
        self.layer_engines = []
        self.graphs.clear()
        self.plans.clear()
        self.outs.clear()
        self.engine = None
        self.k_pages = self.v_pages = self.q_pool = None


def e2e_measure(cfg, flush, barrier, args):
    """Each step through the public API from pinned host buffers.  Returns
    (total ms, h2d bytes, d2h bytes, split dict)."""
    engine, stream = cfg.engine, cfg.stream
    q_host = cfg.q_pool.cpu().pin_memory()
    out_host = torch.empty(max(p.batch for p in cfg.plans), HQ, D,
                           dtype=cfg.q_pool.dtype).pin_memory()
    scratch: dict = {}
    host_rows = []
    for p, state in zip(cfg.plans, cfg.trace_steps):
        v = p.host.views(p.host.buf)
        host_rows.append((np.asarray(state.lengths, np.int32), v["block_table"].numpy().copy(),
                          torch.stack([q_host[r] for r in state.active_ids]).pin_memory()))
    engine.reserve_host(scratch, max(len(r[0]) for r in host_rows),
                        max(r[1].shape[1] for r in host_rows))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(cfg.steps_timed)]
    host_us = []
    bi = bo = 0
    with torch.cuda.stream(stream):
        for j in cfg.sched[: cfg.warmup]:
            lens, rows, qh = host_rows[j]
            engine.step_host(lens, rows, qh, out_host, scratch)
            stream.synchronize()
        barrier()
        for i, j in enumerate(cfg.sched[cfg.warmup:]):
            lens, rows, qh = host_rows[j]
            flush(i)
            stream.synchronize()
            ev[i][0].record(stream)
            t0 = time.perf_counter()
            h, d = engine.step_host(lens, rows, qh, out_host, scratch)
            host_us.append(1e6 * (time.perf_counter() - t0))
            ev[i][1].record(stream)
            stream.synchronize()
            bi += h
            bo += d
        barrier()
    # the last step's output rows, read from host memory, against the device run
    lens, rows, qh = host_rows[cfg.sched[-1]]
    ref = cfg.outs[cfg.sched[-1]].cpu()
    err = float((out_host[: len(lens)].float() - ref.float()).abs().max())
    if err > MAX_ERR:
        raise SystemExit(f"e2e output differs from the device-resident run: {err:.3e}")
    scratch["native"].close()
    times = [a.elapsed_time(b) for a, b in ev]
    split = {"host_call_us_median": statistics.median(host_us),
             "interval_us_median": 1000.0 * statistics.median(times),
             "decode_device_us_median": 1000.0 * statistics.median(cfg.times_ms),
             "note": "interval = host call (staging, graph launch) + launch latency + stage-in "
                     "kernel (metadata and q rows read from pinned host memory) + decode + "
                     "output rows written to pinned host memory"}
    return sum(times), bi, bo, split


def run_engine_arm(args) -> None:
    from persistentkv_attention_b200 import _native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    _native.set_gather_mode(args.gather)
    _native.set_math_mode(args.math)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(dev)
    clocks = ClockSampler(local)
    peak, peak_kind = measured_peak_gbs()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    main = Config(args.workload, args, dev, stream, rank, hkv=args.hkv or None, dtype=args.dtype,
                  kv_fp8=args.kv_fp8)
    main.timed(flush, barrier, clocks)
    code = _native.device_error(clear=True)
    if code:
        raise RuntimeError(f"device error: {_native.describe_device_error(code)}")
    max_err = main.gate()
    total_ms = sum(main.times_ms)
    launches = args.steps * (1 if not args.no_fused else 2)

    # ---- end to end through the public API from pinned host buffers
    e2e_ms, bi, bo, e2e_split = (0.0, 0, 0, None)
    if not main.kv_fp8:
        e2e_ms, bi, bo, e2e_split = e2e_measure(main, flush, barrier, args)

    # ---- aggregate over ranks (max time, summed tokens)
    stats = torch.tensor([total_ms, e2e_ms, float(main.tokens), float(main.bytes_alg)],
                         dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist

        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        total_ms, e2e_ms = float(mx[0]), float(mx[1])
        tokens, bytes_alg = float(sm[2]), float(sm[3])
    else:
        tokens, bytes_alg = float(main.tokens), float(main.bytes_alg)

    # ---- the other configs, same run, same timing method (one GPU)
    per_config = {}
    if world == 1 and not args.no_per_config and TRACE_FILE is None:
        main_summary = main.summary(peak)
        for name in PER_CONFIG:
            if name == args.workload:
                continue
            cfg = Config(name, args, dev, stream, rank, dtype=args.dtype,
                         steps=min(args.steps, 20))
            cfg.timed(flush, barrier, clocks)
            err = cfg.gate()
            per_config[name] = dict(cfg.summary(peak), correctness_max_abs_err=err,
                                    gate="every row of one mid-trace step vs float64 checker")
            cfg.release()
            torch.cuda.empty_cache()
        # the default config under the other gather, for the gather comparison
        other = "tma" if args.gather == "cpasync" else "cpasync"
        _native.set_gather_mode(other)
        cfg = Config(args.workload, args, dev, stream, rank, hkv=args.hkv or None,
                     dtype=args.dtype, steps=args.steps)
        cfg.timed(flush, barrier, clocks)
        err = cfg.gate()
        per_config[f"{args.workload}@gather={other}"] = dict(cfg.summary(peak),
                                                              correctness_max_abs_err=err)
        cfg.release()
        _native.set_gather_mode(args.gather)
        per_config[f"{args.workload}@gather={args.gather}"] = main_summary
        # tensor cores (mma.sync) against CUDA cores (fp32 FMA) for the
        # consumer math at G = 4, on the latency-bound default config and the
        # streaming-bound config 5
        if args.math == "mma" and args.dtype == "f16" and not args.kv_fp8 and \
                (args.hkv or 8) == 8:
            _native.set_math_mode("fma")
            for name in (args.workload, "zipf_b64"):
                cfg = Config(name, args, dev, stream, rank, dtype=args.dtype,
                             steps=min(args.steps, 20))
                cfg.timed(flush, barrier, clocks)
                err = cfg.gate()
                per_config[f"{name}@math=fma"] = dict(cfg.summary(peak),
                                                      correctness_max_abs_err=err)
                cfg.release()
                torch.cuda.empty_cache()
            _native.set_math_mode("mma")
        # back to back: one interval covers a step of LAYERS model layers, each
        # with its own K/V pool (inputs far larger than L2, no flush between
        # the layers), reported per layer
        for name in (args.workload, "long_b1"):
            cfg = Config(name, args, dev, stream, rank, hkv=args.hkv or None, dtype=args.dtype,
                         steps=min(args.steps, 10), layers=LAYERS)
            cfg.timed(flush, barrier, clocks)
            err = cfg.gate()
            per_config[f"{name}@{LAYERS} layers back to back"] = dict(
                cfg.summary(peak), correctness_max_abs_err=err,
                timing=f"one CUDA-event interval per step of {LAYERS} layers (distinct pools, "
                       f"{LAYERS} decode launches back to back, chained with programmatic "
                       f"dependent launch), divided by {LAYERS}; L2 flushed before each step")
            cfg.release()
            torch.cuda.empty_cache()
        code = _native.device_error(clear=True)
        if code:
            raise RuntimeError(f"device error: {_native.describe_device_error(code)}")

    # ---- config 4 sequence-sharded across the ranks (strong scaling)
    seq_shard = None
    if world > 1 and not args.no_per_config:
        seq_shard = measure_seq_shard(args, "fused", dev, stream, flush, clocks, world, rank)

    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    value = tokens / (total_ms / 1000.0)
    per_step_bytes = bytes_alg / args.steps / world
    achieved = per_step_bytes / (total_ms / args.steps / 1000.0) / 1e9
    # DRAM traffic per launch: the ratio dram bytes / algorithmic bytes of a
    # committed ncu capture of this workload, applied to this run's launches.
    traffic = None
    tpath = REPO / "profiles" / f"traffic_{args.workload}.json"
    if (tpath.exists() and main.hkv == 8 and args.dtype == "f16" and TRACE_FILE is None
            and not args.kv_fp8):
        ratio = json.loads(tpath.read_text()).get("traffic_over_algorithmic")
        if ratio:
            traffic = {"bytes_per_launch": ratio * per_step_bytes, "over_algorithmic": ratio,
                       "source": f"profiles/traffic_{args.workload}.json (ncu capture)"}
    line = {
        "metric": "decode-step tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": args.dtype + ("; K/V e4m3" if args.kv_fp8 else ""),
        "data": "synthetic (seeded trace, K/V/q ~ N(0,1))",
        "config": {
            "workload": f"{args.workload}: {main.w['desc']}", "hq": HQ, "hkv": main.hkv,
            "gqa_group": HQ // main.hkv, "head_dim": D,
            "page_size": PAGE, "active_per_gpu": main.w["max_active"],
            "parallelism": f"batch-partitioned x{world} (independent batch per GPU)",
            "l2": "flushed before every step outside the timed intervals: 256 MiB write, "
                  "then 256 MiB read (no dirty lines left for the timed step)",
            "merge": "fused last-task merge" if not args.no_fused else "PDL merge kernel",
            "schedule": "device-side equal-token groups from a host plan uploaded with the "
                        "step's metadata; group count per step from the calibrated router "
                        f"(used: {main.groups_used()})",
            "gather": args.gather,
            "math": args.math,
        },
        "hbm_gbs": achieved, "hbm_frac_of_8tbs": achieved / 8000.0,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "kernel": "pkv_decode_kernel (fused merge), 1 launch per step"},
        "e2e": ({"value": tokens / (e2e_ms / 1000.0), "unit": "tokens/s",
                 "h2d_bytes_per_step": bi // args.steps, "d2h_bytes_per_step": bo // args.steps,
                 "split": e2e_split}
                if not args.kv_fp8 else
                {"value": None, "unit": "tokens/s",
                 "note": "the native host step serves 16-bit caches only"}),
        "gpu_launches": launches,
        "correctness_max_abs_err": max_err,
        "correctness_gate": "every row of one mid-trace step vs a float64 checker, "
                            "max 2e-3 (bf16: + 2^-8 |ref|)",
    }
    if per_config:
        line["per_config"] = per_config
    if seq_shard is not None:
        line["seq_shard"] = seq_shard
    line["clocks"] = clocks.summary()
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baselines(main, args)
    if world > 1:
        torch.distributed.destroy_process_group()
    print(json.dumps(line), flush=True)


def cpu_baselines(cfg, args):
    """The torch CPU repack + SDPA path (the north star's CPU baseline) and,
    beside it, the reference's own cpu_gqa_attention, each a bounded sample
    of the same workload's steps on this host's cores."""
    k_t = cfg.k_pages.float().cpu()
    v_t = cfg.v_pages.float().cpu()
    q_t = cfg.q_pool.float().cpu()
    cycle = [cfg.trace_steps[i % len(cfg.trace_steps)] for i in range(50 * max(1, args.steps))]
    val, done, threads, cores, secs = cpu_sdpa_steps(cfg.reqs, cycle, k_t, v_t, q_t, 10.0)
    out = {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port",
           "affinity_cores": cores, "torch_num_threads": threads,
           "path": "torch CPU repack + scaled_dot_product_attention(enable_gqa=True) in fp32, "
                   "tests/benchmark_torch_paged_sdpa.py:90-109",
           "sample": f"{done} decode steps of the trace, cycled ({secs:.1f} s), rows in turn, "
                     f"torch intra-op threads"}
    rval, rdone, rthreads, rkind, rsecs = cpu_reference_steps(
        cfg.reqs, cycle, k_t.numpy(), v_t.numpy(), q_t.numpy(), 10.0, cfg.hkv)
    out["reference_cpu_gqa_attention"] = {
        "value": rval, "unit": "tokens/s", "cores": rthreads, "kind": rkind,
        "sample": f"{rdone} decode steps ({rsecs:.1f} s), (row, KV head) groups in parallel"}
    return out


# ------------------------------------------------------------------ sequence sharding
def measure_seq_shard(args, exchange, dev, stream, flush, clocks, world, rank,
                      workload="long_b1", steps=None):
    """Config 4 across GPUs: every rank decodes its contiguous page range of the
    active request, and the per-rank (m, l, acc) states are merged exactly on
    every rank (strong scaling).  ``exchange="fused"``: one kernel per step
    pushes the states to the peers over NVLink and merges them; ``"nccl"``:
    state kernel, NCCL all-gather, combine kernel.  Returns a summary dict."""
    import torch.distributed as dist

    from persistentkv_attention_b200 import _native, ops
    from persistentkv_attention_b200 import dist as pdist
    from persistentkv_attention_b200.serving import DecodeEngine

    steps_timed = steps or args.steps
    w, reqs, physical, trace_steps = build_workload(workload, 0, steps_timed + args.warmup)
    hkv = w["hkv"]
    k_pages, v_pages, q_pool = make_inputs(w, physical, hkv, torch.float16, dev, 0)
    engine = DecodeEngine(k_pages, v_pages, HQ, fused=True)
    n = min(len(trace_steps), steps_timed + args.warmup)
    fused = exchange == "fused"
    plans, states, outs, graphs = [], [], [], []
    for state in trace_steps[:n]:
        full = engine.plan_from_trace(reqs, state)
        rows = full.views(full.buf)["block_table"].numpy()
        bt, sl = pdist.shard_rows(rows, state.lengths, PAGE, world, rank)
        plans.append(engine.upload(engine.plan_step(sl, bt,
                                                    q_indices=np.asarray(state.active_ids))))
    xg = pdist.make_exchange(HQ, hkv, max(p.batch for p in plans)) if fused else None
    for p in plans:
        st = torch.empty(p.batch, HQ, 130, dtype=torch.float32, device=dev)
        o = torch.empty(p.batch, HQ, D, dtype=torch.float16, device=dev)
        run = (lambda p=p, o=o: engine.run_sharded(p, q_pool, o, xg)) if fused else \
            (lambda p=p, st=st: engine.run_state(p, q_pool, st))
        run()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                run()
        states.append(st)
        outs.append(o)
        graphs.append(g)
    gathered = [torch.empty((world,) + tuple(st.shape), dtype=torch.float32, device=dev)
                for st in states]
    torch.cuda.synchronize()

    def step(j):
        graphs[j].replay()
        if fused:
            return
        if world > 1:
            dist.all_gather_into_tensor(gathered[j], states[j])
        else:
            gathered[j][0].copy_(states[j])
        ops.combine_states(gathered[j], outs[j])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    sched = [i % n for i in range(args.warmup + steps_timed)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps_timed)]
    with torch.cuda.stream(stream):
        for j in sched[: args.warmup]:
            flush(j)
            step(j)
    barrier()
    with clocks:
        with torch.cuda.stream(stream):
            torch.cuda._sleep(20_000_000)     # host runs ahead: a host hiccup on one rank
                                              # must not stall the coupled peer kernels
            for i, j in enumerate(sched[args.warmup:]):
                flush(i)
                ev[i][0].record(stream)
                step(j)
                ev[i][1].record(stream)
        barrier()
    total_ms = sum(a.elapsed_time(b) for a, b in ev)
    code = _native.device_error(clear=True)
    if code:
        raise RuntimeError(f"device error: {_native.describe_device_error(code)}")
    # correctness: the merged output of one step against the float64 checker
    from oracle import pkv_oracle as po  # checker only

    j = n // 2
    with torch.cuda.stream(stream):
        step(j)
    torch.cuda.synchronize()
    st = trace_steps[j]
    full = engine.plan_from_trace(reqs, st)
    table = full.views(full.buf)["block_table"].numpy()
    want = po.torch_paged_decode(q_pool, k_pages, v_pages, table, st.lengths,
                                 q_indices=st.active_ids)
    max_err = float((outs[j].double() - want).abs().max())
    if max_err >= MAX_ERR:
        raise SystemExit(f"correctness gate failed: max abs error {max_err:.3e}")
    tokens = float(sum(plans[j].batch for j in sched[args.warmup:]))
    full_bytes = float(sum(kv_bytes(trace_steps[j], hkv) for j in sched[args.warmup:]))
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t[0])
    peak, _ = measured_peak_gbs()
    achieved = full_bytes / steps_timed / world / (total_ms / steps_timed / 1000.0) / 1e9
    summary = {
        "workload": f"{workload}: {w['desc']}", "scaling": "strong", "n_gpus": world,
        "steps": steps_timed, "value": tokens / (total_ms / 1000.0), "unit": "tokens/s",
        "ms_per_step": total_ms / steps_timed, "hbm_gbs_per_gpu": achieved,
        "frac_of_measured_peak": achieved / peak,
        "exchange": ("(m, l, acc) pushed to peers over NVLink and merged inside the decode "
                     "kernel" if fused else "(m, l, acc) all-gather over NCCL, LSE combine"),
        "gpu_launches_per_step": 1 if fused else 2, "correctness_max_abs_err": max_err,
    }
    graphs.clear()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()      # no peer kernel still stores into this rank's buffer
    if xg is not None:
        xg.close()
    if world > 1:
        dist.barrier()
    return summary


def run_seq_shard_arm(args) -> None:
    import datetime

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(dev)
    clocks = ClockSampler(local)
    s = measure_seq_shard(args, args.exchange, dev, stream, flush, clocks, world, rank,
                          workload=args.workload)
    if rank == 0:
        peak, peak_kind = measured_peak_gbs()
        line = {
            "metric": "decode-step tokens/s", "value": s["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": s["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded trace, K/V/q ~ N(0,1))",
            "config": {"workload": s["workload"], "hq": HQ, "hkv": 8, "head_dim": D,
                       "page_size": PAGE,
                       "parallelism": f"sequence-sharded x{world}: page ranges per GPU, "
                                      + s["exchange"],
                       "l2": "flushed before every step outside the timed intervals"},
            "hbm_gbs_per_gpu": s["hbm_gbs_per_gpu"],
            "roofline": {"bound": "hbm", "achieved": s["hbm_gbs_per_gpu"], "peak": peak,
                         "unit": "GB/s", "frac": s["frac_of_measured_peak"], "traffic": None,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "pkv_decode_kernel (fused exchange)"
                                   if args.exchange == "fused" else
                                   "pkv_decode_kernel (state) + all-gather + combine"},
            "gpu_launches": args.steps * s["gpu_launches_per_step"],
            "correctness_max_abs_err": s["correctness_max_abs_err"],
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------------------------ group sweep
SWEEP_GROUPS = (37, 32, 28, 24, 18, 14, 9, 6)


def run_group_sweep(args) -> None:
    """Step time of each config under each group count of the device schedule
    (host plans), one B200: the measurements the router's B200 constants are
    fitted to (persistentkv_attention_b200.calibrate)."""
    from persistentkv_attention_b200 import _native
    from persistentkv_attention_b200.scheduler import auto_groups

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _native.set_gather_mode(args.gather)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(dev)
    clocks = ClockSampler(0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    out = {"sm_count": sms, "hkv": 8, "hq": HQ, "steps": args.steps, "configs": {}}
    for name in ("single_b1", "uniform_8k", "bimodal_32k", "long_b1", "zipf_b64"):
        res = {}
        lens = None
        for g in SWEEP_GROUPS:
            if g > auto_groups(8, sms):
                continue
            cfg = Config(name, args, dev, stream, 0, steps=args.steps, groups=g)
            cfg.timed(flush, barrier=torch.cuda.synchronize, clocks=clocks)
            if lens is None:
                lens = [list(cfg.trace_steps[j].lengths) for j in cfg.sched[cfg.warmup:]]
            res[str(g)] = [1000.0 * t for t in cfg.times_ms]
            cfg.release()
            torch.cuda.empty_cache()
        out["configs"][name] = {"lengths": lens, "us": res}
    out["clocks"] = clocks.summary()
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------ phase stamps
PHASES = [("launch_spread", 0, None), ("schedule", 0, 1), ("first_pages", 1, 2),
          ("first_issue", 2, 3), ("first_data", 3, 4), ("stream", 4, 5),
          ("merge", 6, 7)]


def stamp_summary(stamps, event_us):
    """Phases of one launch from the per-CTA stamps (nanoseconds)."""
    s = np.asarray([x for x in stamps if x[0] > 0 and x[7] > 0], dtype=np.float64)
    t0 = s[:, 0].min()
    out = {"ctas": int(s.shape[0]), "event_interval_us": event_us,
           "kernel_span_us": (s[:, 7].max() - t0) / 1e3}
    for name, a, b in PHASES:
        if b is None:
            d = (s[:, a] - t0) / 1e3
        else:
            m = (s[:, a] > 0) & (s[:, b] > 0)
            d = (s[m, b] - s[m, a]) / 1e3
        if d.size:
            out[name + "_us"] = {"median": float(np.median(d)), "max": float(d.max()),
                                 "n": int(d.size)}
    first_data = (s[:, 4][s[:, 4] > 0] - t0) / 1e3
    last_stage = (s[:, 5][s[:, 5] > 0] - t0) / 1e3
    out["first_data_at_us"] = {"min": float(first_data.min()), "median": float(np.median(first_data)),
                               "max": float(first_data.max())}
    out["last_stage_at_us"] = {"min": float(last_stage.min()), "median": float(np.median(last_stage)),
                               "max": float(last_stage.max())}
    out["exit_at_us"] = {"median": float(np.median((s[:, 7] - t0) / 1e3)),
                         "max": float((s[:, 7].max() - t0) / 1e3)}
    return out


def run_phase_stamps(args) -> None:
    """Per-phase timings of the decode CTAs (diagnostic build), per workload:
    each step flushed and replayed like the timed bench, then its stamps read."""
    from persistentkv_attention_b200 import _native

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _native.load()
    _native.set_gather_mode(args.gather)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(dev)
    names = [args.workload] if args.no_per_config else ["uniform_8k", "long_b1", "bimodal_32k"]
    report = {"build": "libpkv_b200_stamps.so (PKV_PHASE_STAMPS)", "gather": args.gather,
              "workloads": {}}
    for name in names:
        cfg = Config(name, args, dev, stream, 0, steps=args.steps)
        runs = []
        with torch.cuda.stream(stream):
            for j in cfg.sched[: cfg.warmup]:
                flush(j)
                cfg.graphs[j].replay()
            torch.cuda.synchronize()
            _native.phase_stamps()
            for i, j in enumerate(cfg.sched[cfg.warmup:]):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                flush(i)
                a.record(stream)
                cfg.graphs[j].replay()
                b.record(stream)
                torch.cuda.synchronize()
                runs.append(stamp_summary(_native.phase_stamps(), 1000.0 * a.elapsed_time(b)))

        def med(path):
            vals = []
            for r in runs:
                v = r
                for k in path:
                    v = v.get(k) if isinstance(v, dict) else None
                if v is not None:
                    vals.append(v)
            return float(np.median(vals)) if vals else None

        keys = [("event_interval_us",), ("kernel_span_us",)] + \
               [(n + "_us", "median") for n, _, _ in PHASES] + \
               [(n + "_us", "max") for n, _, _ in PHASES] + \
               [("first_data_at_us", "min"), ("first_data_at_us", "median"),
                ("first_data_at_us", "max"), ("last_stage_at_us", "median"),
                ("last_stage_at_us", "max"), ("exit_at_us", "median"), ("exit_at_us", "max")]
        report["workloads"][name] = {
            "steps": len(runs), "ctas": runs[0]["ctas"] if runs else 0,
            "median_over_steps": {".".join(k): med(k) for k in keys}}
        cfg.release()
        torch.cuda.empty_cache()
    # the floor under any step: the event interval of a (nearly) empty one-CTA
    # kernel launched after the same flush
    floor = []
    with torch.cuda.stream(stream):
        for i in range(20):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            flush(i)
            a.record(stream)
            torch.cuda._sleep(0)
            b.record(stream)
            floor.append((a, b))
    torch.cuda.synchronize()
    report["empty_launch_floor_us"] = float(np.median([1000.0 * a.elapsed_time(b)
                                                       for a, b in floor]))
    print(json.dumps(report, indent=1), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=48)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="uniform_8k")
    ap.add_argument("--trace-file", default=None,
                    help="CSV / JSON request specs (prompt_len, decode_len, arrival) replacing "
                         "the workload's synthetic lengths; its batch shape and holes stay")
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--hkv", type=int, choices=[32, 8, 4], default=0,
                    help="KV heads (G = 32 / hkv); default: the workload's (8)")
    ap.add_argument("--dtype", choices=sorted(DTYPES), default="f16")
    ap.add_argument("--kv-fp8", action="store_true",
                    help="e4m3 K/V cache with per-tensor scales (q / output fp16)")
    ap.add_argument("--gather", choices=["cpasync", "tma"], default="cpasync",
                    help="decode gather of 16-bit pools (pkv_set_gather_mode)")
    ap.add_argument("--no-fused", action="store_true", help="separate PDL merge kernel")
    ap.add_argument("--math", choices=["mma", "fma"], default="mma",
                    help="consumer math: tensor cores (mma.sync) or CUDA cores (fp32 FMA; lean "
                         "fp16 route at G = 4)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="time only --workload (no per_config / seq_shard sub-objects)")
    ap.add_argument("--sweep-groups", action="store_true",
                    help="time every config under several group counts (router calibration)")
    ap.add_argument("--phase-stamps", action="store_true",
                    help="diagnostic build: print per-phase CTA timings instead of the bench line")
    ap.add_argument("--seq-shard", action="store_true",
                    help="shard each request's pages across the GPUs (config 4 strong scaling)")
    ap.add_argument("--exchange", choices=["fused", "nccl"], default="fused",
                    help="--seq-shard state exchange: inside the decode kernel, or NCCL")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.kv_fp8 and args.dtype != "f16":
        ap.error("--kv-fp8 computes with fp16 q / output (--dtype f16)")
    global TRACE_FILE
    TRACE_FILE = args.trace_file
    if args.phase_stamps:
        os.environ["PKV_LIB_VARIANT"] = "stamps"
        run_phase_stamps(args)
    elif args.sweep_groups:
        run_group_sweep(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    elif args.seq_shard:
        run_seq_shard_arm(args)
    else:
        run_engine_arm(args)


if __name__ == "__main__":
    main()
