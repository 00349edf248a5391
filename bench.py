#!/usr/bin/env python3
"""Decode-step benchmark of the B200 paged decode-attention engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl engine|reference] [--trace-file FILE]
                    [--hkv 32|8|4] [--dtype f16|bf16] [--kv-fp8]
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
              behind it), output rows written into pinned host memory;
  roofline    algorithmic K/V bytes per step / step interval vs the measured
              HBM copy bandwidth;
  cpu_baseline the reference's own fp32 CPU decode (cpu_gqa_attention built
              from its sources) on the host cores, bounded sample.

``--impl reference`` times that reference CPU implementation alone on the
same workload (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
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
    "uniform_8k": dict(trace="uniform_8k", requests=24, max_active=8, hole=0.0, hkv=8,
                       desc="config 2: B8 uniform context [512, 8192], 24 requests, 8 active"),
    "bimodal_32k": dict(trace="bimodal_32k", requests=24, max_active=8, hole=0.0, hkv=8,
                        desc="config 3: B8 bimodal 75% [512, 2048] / 25% [16384, 32768]"),
    "long_b1": dict(trace="long_b1", requests=16, max_active=1, hole=0.0, hkv=8,
                    desc="config 4: B1 long context [24576, 32768], 16 sequential requests"),
    "zipf_b64": dict(trace="zipf_b64", requests=128, max_active=64, hole=0.1, hkv=8,
                     desc="config 5: B64 Zipf(1.1) context [256, 32768], 10% holes"),
}
HQ = 32
PAGE = 16
DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16}
D = 128
SEED = 20260622
FLUSH_BYTES = 256 << 20


def measured_peak_gbs() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event reasons sampled during the timed region.

    Polls NVML from a background thread (the timed region lasts milliseconds,
    far shorter than nvidia-smi's sampling period); only samples taken
    between ``__enter__`` and ``__exit__`` count."""

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
                "source": "NVML, polled during the timed region"}


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
    w = dict(WORKLOADS[name])
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


def kv_bytes(state, hkv: int, elem: int = 2) -> int:
    return int(sum(state.lengths)) * hkv * D * 2 * elem


# ------------------------------------------------------------------ CPU reference
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
                                        "hq": HQ, "hkv": hkv, "head_dim": D, "page_size": PAGE},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"{done} decode steps of the trace, (row, KV head) groups "
                                    f"in parallel"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ engine arm
def run_engine_arm(args) -> None:
    from persistentkv_attention_b200 import _native
    from persistentkv_attention_b200.serving import DecodeEngine

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

    w, reqs, physical, steps = build_workload(args.workload, rank, args.steps + args.warmup)
    hkv = args.hkv or w["hkv"]
    tdt = DTYPES[args.dtype]
    gen = torch.Generator(device=dev).manual_seed(SEED + 7 + rank)
    k_pages = torch.randn(physical, hkv, PAGE, D, generator=gen, device=dev).to(tdt)
    v_pages = torch.randn(physical, hkv, PAGE, D, generator=gen, device=dev).to(tdt)
    q_pool = torch.randn(w["requests"], HQ, D, generator=gen, device=dev).to(tdt)
    kv_elem = 2
    kv_scales = None
    if args.kv_fp8:
        # e4m3 cache with per-tensor scales; the pools below hold the
        # dequantised values for the correctness gate and the CPU baseline
        kv_scales = (float(k_pages.abs().max()) / 448.0, float(v_pages.abs().max()) / 448.0)
        k8 = (k_pages.float() / kv_scales[0]).to(torch.float8_e4m3fn)
        v8 = (v_pages.float() / kv_scales[1]).to(torch.float8_e4m3fn)
        k_pages = (k8.float() * kv_scales[0]).to(tdt)
        v_pages = (v8.float() * kv_scales[1]).to(tdt)
        kv_elem = 1
        engine = DecodeEngine(k8, v8, HQ, fused=not args.no_fused, kv_scales=kv_scales)
    else:
        engine = DecodeEngine(k_pages, v_pages, HQ, fused=not args.no_fused)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(dev)

    # device-resident plans + one CUDA graph per distinct step
    plans, graphs, outs = [], [], []
    n_distinct = min(len(steps), args.steps + args.warmup)
    for state in steps[:n_distinct]:
        p = engine.upload(engine.plan_from_trace(reqs, state))
        plans.append(p)
    for p in plans:
        o = torch.empty(p.batch, HQ, D, dtype=tdt, device=dev)
        outs.append(o)
        graphs.append(engine.capture(p, q_pool, o, stream))
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    sched = [i % n_distinct for i in range(args.warmup + args.steps)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for j in sched[: args.warmup]:
            flush(j)
            graphs[j].replay()
    barrier()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            torch.cuda._sleep(20_000_000)         # lets the host queue run ahead (~10 ms)
            for i, j in enumerate(sched[args.warmup:]):
                flush(i)
                ev[i][0].record(stream)
                graphs[j].replay()
                ev[i][1].record(stream)
        barrier()
    times_ms = [a.elapsed_time(b) for a, b in ev]
    tokens = sum(plans[j].batch for j in sched[args.warmup:])
    bytes_alg = sum(kv_bytes(steps[j], hkv, kv_elem) for j in sched[args.warmup:])
    total_ms = sum(times_ms)
    launches = args.steps * (1 if not args.no_fused else 2)
    code = _native.device_error(clear=True)
    if code:
        raise RuntimeError(f"device error: {_native.describe_device_error(code)}")
    # correctness gate on one step (reference: one mid-trace check, :1082-1088)
    check_step = len(plans) // 2
    graphs[check_step].replay()
    torch.cuda.synchronize()
    from oracle import pkv_oracle as po  # checker only

    st = steps[check_step]
    row = 0
    rid = st.active_ids[row]
    k_row = k_pages[torch.tensor(reqs[rid].physical_pages[: (st.lengths[row] + PAGE - 1) // PAGE],
                                 device=dev)]
    v_row = v_pages[torch.tensor(reqs[rid].physical_pages[: (st.lengths[row] + PAGE - 1) // PAGE],
                                 device=dev)]
    kk = k_row.permute(1, 0, 2, 3).reshape(hkv, -1, D)[:, : st.lengths[row]].double().cpu().numpy()
    vv = v_row.permute(1, 0, 2, 3).reshape(hkv, -1, D)[:, : st.lengths[row]].double().cpu().numpy()
    want = po.attend_row(q_pool[rid].double().cpu().numpy(), kk, vv)
    got = outs[check_step][row].double().cpu().numpy()
    max_err = float(np.abs(got - want).max())
    # fp16 tolerance of the reference; bf16 output adds one bf16 rounding (2^-8 relative)
    excess = np.abs(got - want) - (2e-3 + (2.0 ** -8 * np.abs(want) if args.dtype == "bf16" else 0))
    if (excess >= 0).any():
        raise SystemExit(f"correctness gate failed: max abs error {max_err:.3e}")

    # ---- end to end through the public API from pinned host buffers
    q_host = q_pool.cpu().pin_memory()
    out_host = torch.empty(max(p.batch for p in plans), HQ, D, dtype=tdt).pin_memory()
    scratch: dict = {}
    bi = bo = 0
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    host_rows = []
    for state in steps[:n_distinct]:
        plan = engine.plan_from_trace(reqs, state)
        v = plan.views(plan.buf)
        host_rows.append((list(state.lengths), v["block_table"].numpy().copy(),
                          torch.stack([q_host[r] for r in state.active_ids]).pin_memory()))
    if not engine.kv8:
        engine.reserve_host(scratch, max(len(r[0]) for r in host_rows),
                            max(r[1].shape[1] for r in host_rows))
    with torch.cuda.stream(stream):
        for j in (sched[: args.warmup] if not engine.kv8 else []):
            lens, rows, qh = host_rows[j]
            engine.step_host(lens, rows, qh, out_host, scratch)
            stream.synchronize()
        barrier()
        for i, j in enumerate(sched[args.warmup:] if not engine.kv8 else []):
            lens, rows, qh = host_rows[j]
            flush(i)
            stream.synchronize()
            e2e_ev[i][0].record(stream)
            h, d = engine.step_host(lens, rows, qh, out_host, scratch)
            e2e_ev[i][1].record(stream)
            stream.synchronize()
            bi += h
            bo += d
        barrier()
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_ev) if not engine.kv8 else 0.0

    # ---- aggregate over ranks (max time, summed tokens)
    stats = torch.tensor([total_ms, e2e_ms, float(tokens), float(bytes_alg)], dtype=torch.float64,
                         device=dev)
    if world > 1:
        import torch.distributed as dist

        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        total_ms, e2e_ms = float(mx[0]), float(mx[1])
        tokens, bytes_alg = float(sm[2]), float(sm[3])
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    peak, peak_kind = measured_peak_gbs()
    value = tokens / (total_ms / 1000.0)
    per_step_bytes = bytes_alg / args.steps / world
    achieved = per_step_bytes / (total_ms / args.steps / 1000.0) / 1e9
    # DRAM traffic per launch: the ratio dram bytes / algorithmic bytes of a
    # committed ncu capture of this workload, applied to this run's launches.
    traffic = None
    tpath = REPO / "profiles" / f"traffic_{args.workload}.json"
    if (tpath.exists() and hkv == 8 and args.dtype == "f16" and TRACE_FILE is None
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
            "workload": f"{args.workload}: {w['desc']}", "hq": HQ, "hkv": hkv, "gqa_group": HQ // hkv,
            "head_dim": D,
            "page_size": PAGE, "active_per_gpu": w["max_active"],
            "parallelism": f"batch-partitioned x{world} (independent batch per GPU)",
            "l2": "flushed before every step outside the timed intervals: 256 MiB write, "
                  "then 256 MiB read (no dirty lines left for the timed step)",
            "merge": "fused last-task merge" if not args.no_fused else "PDL merge kernel",
            "schedule": "device-side equal-token groups (no host work queue)",
        },
        "hbm_gbs": achieved, "hbm_frac_of_8tbs": achieved / 8000.0,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "kernel": "pkv_decode_kernel (fused merge), 1 launch per step"},
        "e2e": ({"value": tokens / (e2e_ms / 1000.0), "unit": "tokens/s",
                 "h2d_bytes_per_step": bi // args.steps, "d2h_bytes_per_step": bo // args.steps}
                if not args.kv_fp8 else
                {"value": None, "unit": "tokens/s",
                 "note": "the native host step serves 16-bit caches only"}),
        "gpu_launches": launches,
        "correctness_max_abs_err": max_err,
    }
    c = clocks.summary()
    line["clocks"] = c
    if world == 1 and not args.no_cpu_baseline:
        k_host = k_pages.float().cpu().numpy()
        v_host = v_pages.float().cpu().numpy()
        qn = q_pool.float().cpu().numpy()
        # the trace's steps, cycled, for a bounded ~12 s sample of CPU work
        cycle = [steps[i % len(steps)] for i in range(50 * max(1, args.steps))]
        val, done, threads, kind, secs = cpu_reference_steps(reqs, cycle, k_host, v_host, qn,
                                                             12.0, hkv)
        line["cpu_baseline"] = {"value": val, "unit": "tokens/s", "cores": threads, "kind": kind,
                                "sample": f"{done} decode steps of the trace, cycled "
                                          f"({secs:.1f} s), (row, KV head) groups in parallel"}
    if world > 1:
        torch.distributed.destroy_process_group()
    print(json.dumps(line), flush=True)


def run_seq_shard_arm(args) -> None:
    """Config 4 across GPUs: every rank decodes its contiguous page range of the
    active request, and the per-rank (m, l, acc) states are merged exactly on
    every rank (strong scaling).  ``--exchange fused`` (default): one kernel
    per step pushes the states to the peers over NVLink and merges them;
    ``--exchange nccl``: state kernel, NCCL all-gather, combine kernel."""
    import datetime

    import torch.distributed as dist

    from persistentkv_attention_b200 import _native, ops
    from persistentkv_attention_b200 import dist as pdist
    from persistentkv_attention_b200.serving import DecodeEngine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    w, reqs, physical, steps = build_workload(args.workload, 0, args.steps + args.warmup)
    hkv = w["hkv"]
    gen = torch.Generator(device=dev).manual_seed(SEED + 7)   # same pool on every rank
    k_pages = torch.randn(physical, hkv, PAGE, D, generator=gen, device=dev).half()
    v_pages = torch.randn(physical, hkv, PAGE, D, generator=gen, device=dev).half()
    q_pool = torch.randn(w["requests"], HQ, D, generator=gen, device=dev).half()
    engine = DecodeEngine(k_pages, v_pages, HQ, fused=True)
    flush = L2Flush(dev)
    stream = torch.cuda.Stream(dev)
    n = min(len(steps), args.steps + args.warmup)
    fused = args.exchange == "fused"
    plans, states, outs, graphs = [], [], [], []
    for state in steps[:n]:
        full = engine.plan_from_trace(reqs, state)
        rows = full.views(full.buf)["block_table"].numpy()
        bt, sl = pdist.shard_rows(rows, state.lengths, PAGE, world, rank)
        plans.append(engine.upload(engine.plan_step(sl, bt, q_indices=np.asarray(state.active_ids))))
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

    sched = [i % n for i in range(args.warmup + args.steps)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for j in sched[: args.warmup]:
            flush(j)
            step(j)
    barrier()
    with ClockSampler(local) as clocks:
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
    # correctness: the merged output of one step against the oracle
    from oracle import pkv_oracle as po  # checker only

    j = n // 2
    with torch.cuda.stream(stream):
        step(j)
    torch.cuda.synchronize()
    st = steps[j]
    rid, length = st.active_ids[0], st.lengths[0]
    pages = torch.tensor(reqs[rid].physical_pages[: (length + PAGE - 1) // PAGE], device=dev)
    kk = k_pages[pages].permute(1, 0, 2, 3).reshape(hkv, -1, D)[:, :length].double().cpu().numpy()
    vv = v_pages[pages].permute(1, 0, 2, 3).reshape(hkv, -1, D)[:, :length].double().cpu().numpy()
    want = po.attend_row(q_pool[rid].double().cpu().numpy(), kk, vv)
    max_err = float(np.abs(outs[j][0].double().cpu().numpy() - want).max())
    if max_err >= 2e-3:
        raise SystemExit(f"correctness gate failed: max abs error {max_err:.3e}")
    tokens = float(sum(plans[j].batch for j in sched[args.warmup:]))
    full_bytes = float(sum(kv_bytes(steps[j], hkv) for j in sched[args.warmup:]))
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t[0])
    if rank == 0:
        peak, peak_kind = measured_peak_gbs()
        achieved = full_bytes / args.steps / world / (total_ms / args.steps / 1000.0) / 1e9
        line = {
            "metric": "decode-step tokens/s", "value": tokens / (total_ms / 1000.0),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded trace, K/V/q ~ N(0,1))",
            "config": {"workload": f"{args.workload}: {w['desc']}", "hq": HQ, "hkv": hkv,
                       "head_dim": D, "page_size": PAGE,
                       "parallelism": f"sequence-sharded x{world}: page ranges per GPU, "
                                      + ("(m, l, acc) pushed to peers over NVLink and merged "
                                         "inside the decode kernel" if fused else
                                         "(m, l, acc) all-gather over NCCL, LSE combine"),
                       "l2": "flushed before every step outside the timed intervals"},
            "hbm_gbs_per_gpu": achieved,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "pkv_decode_kernel (fused exchange)" if fused else
                                   "pkv_decode_kernel (state) + all-gather + combine"},
            "gpu_launches": args.steps * (1 if fused else 2), "correctness_max_abs_err": max_err,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    graphs.clear()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()      # no peer kernel still stores into this rank's buffer
    if xg is not None:
        xg.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    ap.add_argument("--no-fused", action="store_true", help="separate PDL merge kernel")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.seq_shard:
        run_seq_shard_arm(args)
    else:
        run_engine_arm(args)


if __name__ == "__main__":
    main()
