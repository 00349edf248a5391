"""Generates the golden fixtures of ``tests/golden`` from the reference itself.

Run where the reference checkout (``PKV_REFERENCE_DIR``) and the artefacts of
``oracle/build_ref.py`` exist:

    python -m oracle.build_ref --skip-torch-ext
    python tests/golden/make_golden.py

Fixtures written (all small):

* ``smoke_kat.npz`` -- the eight correctness cases of the reference smoke test
  (tests/smoke_test.cu:486-493): shapes, splits, page sizes and the output of
  the reference's own ``cpu_gqa_attention`` (compiled from its sources) on the
  ``srand(42)`` input stream, quantised to fp16 exactly as the smoke test does.
  The inputs themselves are not stored: the tests replay them with the
  oracle's glibc ``rand()`` restatement.
* ``scheduler.json`` -- decisions of the reference's Python scheduler
  (tests/benchmark_serving_trace.py): ``choose_workqueue_row_splits``,
  ``choose_splits``, ``model_bucket_splits``, ``model_workqueue_splits``,
  ``estimate_route_ms``, ``choose_adaptive_route_cost_model`` and the work
  queues of ``compile_persistentkv_metadata``.
* ``traces.json`` -- ``make_lengths`` / ``build_requests`` / ``build_steps``
  outputs for each reference trace.
* ``trace_files.json`` -- ``load_trace_specs`` and the requests / steps built
  from the committed ``trace_specs.csv`` / ``trace_specs.json``.
* ``harness_calls.json.gz`` -- the operator calls the reference's serving-trace
  harness makes per decode step: ``compile_persistentkv_metadata`` +
  ``run_persistentkv_step_compiled`` (tests/benchmark_serving_trace.py:655-781,
  :949-1001) run here with a recording module in place of the extension,
  for four of its routes (work queue with auto splits and fused merge, work
  queue with 20 requested splits, length buckets through the indexed entry
  point, one bucket with auto splits).  Each call keeps the entry-point name
  and every argument (metadata tensors as int lists, the q / K / V /
  workspace / output operands by role), so a GPU test can replay the
  harness's exact call sequence through this engine's ``ops`` and through the
  reference's extension.
"""

from __future__ import annotations

import gzip
import json
import random
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import pkv_oracle as po  # noqa: E402
from oracle import ref  # noqa: E402

from oracle.build_ref import REFERENCE_DIR  # noqa: E402  (PKV_REFERENCE_DIR or BASELINE.json)

# (kind, B, Hq, Hkv, N, splits, page_size) in smoke_test.cu order (:486-493)
SMOKE_CASES = [
    ("contiguous", 1, 4, 1, 257, 1, 0),
    ("contiguous", 1, 8, 2, 257, 4, 0),
    ("contiguous", 1, 32, 8, 512, 4, 0),
    ("contiguous", 2, 32, 8, 259, 3, 0),
    ("contiguous", 1, 32, 4, 511, 4, 0),
    ("contiguous", 1, 8, 8, 256, 2, 0),
    ("paged", 1, 8, 2, 257, 4, 16),
    ("paged", 2, 8, 2, 259, 3, 32),
]


def smoke_inputs():
    """Yields (case, q, k, v) with the smoke test's srand(42) stream, fp16-quantised."""
    rng = po.GlibcRand(42)
    for case in SMOKE_CASES:
        _, b, hq, hkv, n, _, _ = case
        q = rng.smoke_uniform(b * hq * 128).reshape(b, hq, 128)
        k = rng.smoke_uniform(b * hkv * n * 128).reshape(b, hkv, n, 128)
        v = rng.smoke_uniform(b * hkv * n * 128).reshape(b, hkv, n, 128)
        yield case, po.quantize(q), po.quantize(k), po.quantize(v)


def make_smoke() -> None:
    arrays = {}
    meta = []
    for i, (case, q, k, v) in enumerate(smoke_inputs()):
        out = ref.cpu_gqa_attention(q, k, v)
        arrays[f"out_{i}"] = out
        arrays[f"q_head_{i}"] = q.reshape(-1)[:8]       # first values, pins the replay
        meta.append(case)
    np.savez_compressed(HERE / "smoke_kat.npz", cases=np.array(meta, dtype=object), **arrays)


class _CpuTorch:
    """Stand-in for the harness's ``torch`` that keeps tensors on the CPU."""

    def __getattr__(self, name):
        return getattr(torch, name)

    @staticmethod
    def tensor(*args, device=None, **kwargs):
        return torch.tensor(*args, **kwargs)

    @staticmethod
    def empty(*args, device=None, **kwargs):
        return torch.empty(*args, **kwargs)

    @staticmethod
    def zeros(*args, device=None, **kwargs):
        return torch.zeros(*args, **kwargs)


def load_harness():
    if REFERENCE_DIR is None or not (REFERENCE_DIR / "tests").is_dir():
        raise SystemExit("set PKV_REFERENCE_DIR to the reference checkout")
    sys.path.insert(0, str(REFERENCE_DIR / "tests"))
    import benchmark_serving_trace as harness  # noqa: PLC0415

    harness.torch = _CpuTorch()
    return harness


def make_scheduler(h) -> None:
    out = {"row_splits": [], "choose_splits": [], "bucket_splits": [], "workqueue_splits": [],
           "route_ms": [], "routes": [], "workqueues": []}
    lengths = [1, 16, 31, 32, 33, 96, 97, 128, 500, 512, 640, 700, 1024, 2048, 4095, 4096,
               8192, 12288, 16384, 20000, 24576, 32768, 40000, 65536, 100000]
    for hkv in (8, 4, 32):
        h.HKV = hkv
        for length in lengths:
            for active in (1, 2, 3, 4, 5, 8, 16):
                for requested in (1, 16, 24):
                    for auto in (False, True):
                        out["row_splits"].append(
                            [hkv, length, active, requested, int(auto),
                             h.choose_workqueue_row_splits(length, active, requested, auto)])
    rnd = random.Random(20260622)
    for hkv in (8, 4):
        h.HKV = hkv
        for trial in range(120):
            n = rnd.choice([1, 2, 3, 4, 5, 6, 8, 12])
            lens = [rnd.choice([rnd.randint(1, 2048), rnd.randint(2048, 40000),
                                rnd.randint(30000, 70000)]) for _ in range(n)]
            requested = rnd.choice([8, 16, 24])
            for auto in (False, True):
                for single in (False, True):
                    out["choose_splits"].append(
                        [hkv, lens, requested, int(auto), int(single),
                         h.choose_splits(lens, requested, auto, single)])
            state = h.StepState(trial, tuple(range(n)), tuple(lens))
            out["bucket_splits"].append([hkv, lens, h.model_bucket_splits(state)])
            out["workqueue_splits"].append([hkv, lens, h.model_workqueue_splits(state)])
            for route, splits in (("flashinfer", 1), ("persistentkv_bucket", 16),
                                  ("persistentkv_workqueue", 24)):
                out["route_ms"].append([hkv, lens, route, splits,
                                        h.estimate_route_ms(state, route, splits)])
            est = h.choose_adaptive_route_cost_model(state)
            out["routes"].append([hkv, lens, est.route, est.splits, est.estimated_ms])
    h.HKV = 8
    for trace, seed, max_active, splits, auto in (("bimodal", 20260623, 8, 20, False),
                                                 ("uniform", 20260624, 8, 24, True),
                                                 ("zipf", 20260625, 4, 24, True)):
        reqs, _ = h.build_requests(trace, 24, max_active, seed, 0.0, 0, None)
        steps = h.build_steps(reqs, max_active)[:3]
        metas = h.compile_persistentkv_metadata(reqs, steps, splits, 0, False, auto, False, True)
        for state, meta in zip(steps, metas):
            out["workqueues"].append({
                "lengths": list(state.lengths), "active": len(state.active_ids),
                "requested": splits, "auto": int(auto),
                "items": meta.work_items.tolist(), "split_offsets": meta.split_offsets.tolist(),
                "total_slots": meta.total_partial_slots,
            })
    (HERE / "scheduler.json").write_text(json.dumps(out))


def make_traces(h) -> None:
    out = []
    for trace in ("uniform", "bimodal", "zipf", "bucketed", "homogeneous"):
        for seed, hole in ((20260622, 0.5), (20260627, 0.0)):
            reqs, physical = h.build_requests(trace, 12, 4, seed, hole, 0, None)
            steps = h.build_steps(reqs, 4)
            out.append({
                "trace": trace, "seed": seed, "hole": hole, "requests": 12, "max_active": 4,
                "lengths": h.make_lengths(trace, 12, seed),
                "physical_pages": physical,
                "pages_head": [list(r.physical_pages[:5]) for r in reqs],
                "pages_len": [len(r.physical_pages) for r in reqs],
                "arrivals": [r.arrival for r in reqs],
                "steps": [[s.step, list(s.active_ids), list(s.lengths)] for s in steps[::7]],
                "n_steps": len(steps),
            })
    (HERE / "traces.json").write_text(json.dumps(out))


def make_trace_files(h) -> None:
    """The reference's ``load_trace_specs`` + ``build_requests(trace_file=...)``
    + ``build_steps`` on the two committed trace files."""
    out = []
    for name, limit, max_active, seed, hole in (("trace_specs.csv", 100, 3, 20260624, 0.1),
                                                ("trace_specs.json", 4, 2, 20260625, 0.0)):
        path = HERE / name
        specs = h.load_trace_specs(path, limit)
        reqs, physical = h.build_requests("uniform", limit, max_active, seed, hole, 0, path)
        steps = h.build_steps(reqs, max_active)
        out.append({
            "file": name, "limit": limit, "max_active": max_active, "seed": seed, "hole": hole,
            "specs": [[s.arrival, s.prompt_len, s.decode_len] for s in specs],
            "physical_pages": physical,
            "pages": [list(r.physical_pages) for r in reqs],
            "steps": [[s.step, list(s.active_ids), list(s.lengths)] for s in steps],
        })
    (HERE / "trace_files.json").write_text(json.dumps(out))


class _Role:
    """Stands for a large operand the replay supplies itself."""

    def __init__(self, role):
        self.role = role

    def __getitem__(self, index):          # q_pool[state_index] -> q source of that step
        return _Role(f"{self.role}[{int(index)}]")


class _Recorder:
    """Records the harness's calls of the extension's four entry points."""

    def __init__(self, outputs):
        self.calls = []
        self.outputs = outputs

    def __getattr__(self, name):
        if not name.startswith("paged_attention"):
            raise AttributeError(name)

        def record(*args):
            enc = []
            for a in args:
                if isinstance(a, _Role):
                    enc.append({"role": a.role})
                elif isinstance(a, torch.Tensor):
                    if id(a) in self.outputs:
                        enc.append({"role": "output", "shape": list(a.shape)})
                    else:
                        enc.append({"dtype": str(a.dtype).replace("torch.", ""),
                                    "shape": list(a.shape), "values": a.reshape(-1).tolist()})
                else:
                    enc.append(a)
            self.calls.append({"fn": name, "args": enc})

        return record


def make_harness_calls(h) -> None:
    h.HKV = 8
    out = []
    routes = [
        # (trace, requested splits, bucket tokens, single bucket, auto, workqueue, fused)
        ("uniform", 16, 0, False, True, True, True),
        ("bimodal", 20, 0, False, False, True, False),
        ("bimodal", 16, 2048, False, False, False, False),
        ("uniform", 16, 0, True, True, False, False),
    ]
    for trace, splits, bucket, single, auto, wq, fused in routes:
        reqs, physical = h.build_requests(trace, 24, 8, 20260622, 0.0, 0, None)
        steps = h.build_steps(reqs, 8)
        metas = h.compile_persistentkv_metadata(reqs, steps, splits, bucket, single, auto, False,
                                                wq)
        for idx in (0, len(steps) // 2, len(steps) - 1):
            meta = metas[idx]
            rec = _Recorder({id(meta.output)})
            h.run_persistentkv_step_compiled(rec, _Role("q_pool"), _Role("k_pages"),
                                             _Role("v_pages"), idx, _Role("workspace"), metas,
                                             fused)
            state = steps[idx]
            out.append({
                "route": {"trace": trace, "splits": splits, "bucket_tokens": bucket,
                          "single_bucket": single, "auto_splits": auto, "workqueue": wq,
                          "fused_merge": fused},
                "step": idx, "requests": 24, "physical_pages": physical,
                "active_ids": list(state.active_ids), "lengths": list(state.lengths),
                "output_shape": list(meta.output.shape), "calls": rec.calls,
            })
    with gzip.open(HERE / "harness_calls.json.gz", "wt") as f:
        f.write(json.dumps(out))


def main() -> None:
    if not ref.ref_cpu_available():
        raise SystemExit("build oracle/_ref first: python -m oracle.build_ref --skip-torch-ext")
    make_smoke()
    h = load_harness()
    make_scheduler(h)
    make_traces(h)
    make_trace_files(h)
    make_harness_calls(h)
    for p in sorted(HERE.glob("*.*")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
