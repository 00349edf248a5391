"""Synthetic continuous-batching decode traces.

Restates the trace mechanics of the reference's serving harness
(tests/benchmark_serving_trace.py): ``rounded_length`` (:159-160),
``make_lengths`` (:163-195), ``build_requests`` (:232-282) and ``build_steps``
(:285-298) and ``load_trace_specs`` (:198-229, external trace files) -- same
seeded torch CPU generators, same page-universe permutation with holes, same
admission rule -- and adds the length distributions of the benchmark
configurations of this engine:

* ``uniform_8k``  -- prompt U[512, 8192], decode U[16, 96]        (config 2)
* ``bimodal_32k`` -- 75% U[512, 2048] / 25% U[16384, 32768]       (config 3)
* ``long_b1``     -- prompt U[24576, 32768], 64 decode steps,
                     requests arriving back to back                (config 4)
* ``zipf_b64``    -- prompt 256 * k, k ~ Zipf(s = 1.1), clipped to
                     [256, 32768], decode U[16, 96]                (config 5)
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

REFERENCE_TRACES = ("uniform", "bimodal", "zipf", "bucketed", "homogeneous")
ENGINE_TRACES = ("uniform_8k", "bimodal_32k", "long_b1", "zipf_b64")


@dataclass(frozen=True)
class Request:
    request_id: int
    arrival: int
    prompt_len: int
    decode_len: int
    physical_pages: tuple


@dataclass(frozen=True)
class StepState:
    step: int
    active_ids: tuple
    lengths: tuple


def rounded_length(value: int, page_size: int = 16) -> int:
    return max(page_size, ((value + page_size - 1) // page_size) * page_size)


def _zipf_tail(s: float, n: int) -> float:
    # sum_{k >= n} k^-s by Euler-Maclaurin (error ~ n^(-s-3))
    return n ** (1 - s) / (s - 1) + 0.5 * n ** (-s) + s * n ** (-s - 1) / 12.0


def _zipf_weights(s: float, k_max: int) -> torch.Tensor:
    k = torch.arange(1, k_max, dtype=torch.float64)
    w = k.pow(-s)
    return torch.cat([w, torch.tensor([_zipf_tail(s, k_max)], dtype=torch.float64)])


def make_lengths(trace: str, requests: int, seed: int, page_size: int = 16):
    """(prompt, decode) per request; reference traces draw exactly like the reference."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)

    def randint(lo: int, hi: int) -> int:
        return int(torch.randint(lo, hi, (1,), generator=gen).item())

    zipf_w = _zipf_weights(1.1, 128) if trace == "zipf_b64" else None
    result = []
    for index in range(requests):
        if trace == "uniform":
            prompt = randint(4096, 32769)
            decode = randint(16, 97)
        elif trace == "bimodal":
            if index % 4 == 0:
                prompt = randint(24576, 65537)
                decode = randint(32, 129)
            else:
                prompt = randint(2048, 12289)
                decode = randint(8, 65)
        elif trace == "zipf":
            rank = randint(1, 33)
            prompt = int(2048 + 65536 / math.sqrt(rank))
            jitter = randint(-512, 513)
            prompt = max(1024, prompt + jitter)
            decode = randint(8, 129)
        elif trace == "bucketed":
            prompt = [8192, 16384, 32768, 65536][index % 4]
            decode = randint(32, 97)
        elif trace == "homogeneous":
            prompt = 32768
            decode = randint(32, 97)
        elif trace == "uniform_8k":
            prompt = randint(512, 8193)
            decode = randint(16, 97)
        elif trace == "bimodal_32k":
            if index % 4 == 0:
                prompt = randint(16384, 32769)
                decode = randint(32, 129)
            else:
                prompt = randint(512, 2049)
                decode = randint(8, 65)
        elif trace == "long_b1":
            prompt = randint(24576, 32769)
            decode = 64
        elif trace == "zipf_b64":
            k = int(torch.multinomial(zipf_w, 1, generator=gen).item()) + 1
            prompt = min(32768, max(256, 256 * k))
            decode = randint(16, 97)
        else:
            raise ValueError(f"unknown trace: {trace}")
        result.append((rounded_length(prompt, page_size), decode))
    return result


def load_trace_specs(path, limit: int, page_size: int = 16):
    """Request specs of an external trace file, like the reference's
    ``load_trace_specs`` (tests/benchmark_serving_trace.py:198-229).

    A ``.json`` file holds a list of objects; anything else is read as CSV
    with a header.  Each row gives ``prompt_len`` (or ``prompt``) and
    ``decode_len`` (or ``decode``), optionally ``arrival`` (or
    ``arrival_step``; default: the row index).  At most ``limit`` rows are
    read; prompts are rounded up to whole pages.  Returns a list of
    (arrival, prompt_len, decode_len) for ``build_requests(specs=...)``.
    """
    import csv
    import json
    from pathlib import Path

    path = Path(path)
    if path.suffix.lower() == ".json":
        raw = json.loads(path.read_text())
        if not isinstance(raw, list):
            raise ValueError("--trace-file JSON must contain a list of request objects")
        rows = raw
    else:
        with path.open(newline="") as handle:
            rows = list(csv.DictReader(handle))
    specs = []
    for index, row in enumerate(rows[:limit]):
        try:
            prompt = int(row.get("prompt_len", row.get("prompt", "")))
            decode = int(row.get("decode_len", row.get("decode", "")))
        except ValueError as error:
            raise ValueError("trace-file rows must define integer prompt_len/prompt and "
                             "decode_len/decode fields") from error
        arrival = int(row.get("arrival", row.get("arrival_step", index)))
        specs.append((arrival, rounded_length(prompt, page_size), decode))
    if not specs:
        raise ValueError(f"trace file produced no requests: {path}")
    return specs


def build_requests(trace: str, requests: int, max_active: int, seed: int, hole_fraction: float,
                   bucket_tokens: int = 0, page_size: int = 16, specs=None):
    """Requests with physical pages drawn from a seeded permutation of the pool.

    Returns (requests, physical_pages).  ``specs`` (a list of
    (arrival, prompt, decode)) replaces the synthetic lengths, like the
    reference's ``--trace-file``.
    """
    if specs is None:
        lengths = make_lengths(trace, requests, seed, page_size)
        if trace == "long_b1":
            specs = [(i * d, p, d) for i, (p, d) in enumerate(lengths)]
        else:
            specs = [(i // max_active, p, d) for i, (p, d) in enumerate(lengths)]
    logical_pages = []
    for _, prompt, decode in specs:
        exact = prompt + decode
        if bucket_tokens > 0:
            reserved = rounded_length(((exact + bucket_tokens - 1) // bucket_tokens) * bucket_tokens,
                                      page_size)
        else:
            reserved = rounded_length(exact, page_size)
        logical_pages.append(math.ceil(reserved / page_size))
    total = sum(logical_pages)
    physical_pages = math.ceil(total / max(1e-6, 1.0 - hole_fraction))
    ids = torch.randperm(physical_pages, generator=torch.Generator().manual_seed(seed + 99))
    ids = ids.numpy()
    built = []
    cursor = 0
    for rid, ((arrival, prompt, decode), pages) in enumerate(zip(specs, logical_pages)):
        built.append(Request(rid, arrival, prompt, decode,
                             tuple(int(x) for x in ids[cursor:cursor + pages])))
        cursor += pages
    return built, physical_pages


def build_steps(requests, max_active: int):
    """Active set per step: the first max_active requests with 0 <= step - arrival < decode_len."""
    steps = []
    max_step = max(r.arrival + r.decode_len for r in requests)
    for step in range(max_step):
        cand = []
        for r in requests:
            generated = step - r.arrival
            if 0 <= generated < r.decode_len:
                cand.append((r.request_id, r.prompt_len + generated))
        cand = cand[:max_active]
        if cand:
            ids, lens = zip(*cand)
            steps.append(StepState(step, tuple(ids), tuple(lens)))
    return steps


def block_table_rows(requests, state: StepState, page_size: int = 16) -> np.ndarray:
    """Block table of one step: each active row padded to the step's longest
    row by repeating its last page (reference :677-684)."""
    by_id = {r.request_id: r for r in requests}
    page_count = math.ceil(max(state.lengths) / page_size)
    rows = np.empty((len(state.active_ids), page_count), dtype=np.int32)
    for i, rid in enumerate(state.active_ids):
        pages = by_id[rid].physical_pages[:page_count]
        if len(pages) < page_count:
            pages = pages + (by_id[rid].physical_pages[-1],) * (page_count - len(pages))
        rows[i] = pages
    return rows
