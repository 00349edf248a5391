"""Fits the router's step-time model of the device-side schedule to measured
step times on this GPU.

    python bench.py --sweep-groups --steps 10 --warmup 3 > sweep.json
    python -m persistentkv_attention_b200.calibrate sweep.json

The model (``pkv_choose_groups``, ``pkv_router_params.dev_*``) prices a step
with NG groups of the schedule as

    fixed_us + KV bytes / min(read_gbps, NG * Hkv * cta_gbps)
             + (merge_us + merge_piece_us * n)   if the most split row has n >= 2 pieces

the launch and prologue, the stream (HBM-bound, or bound by what the NG * Hkv
CTAs stream on their own), and the end-of-CTA merge of the most split row.
The fit is a least-squares fit of fixed_us / merge_us / merge_piece_us
(non-negative) for each (read_gbps, cta_gbps) on a grid, keeping the best.
The reference fits its own constants to its GPU the same way in spirit
(tests/benchmark_serving_trace.py:39-43, :418-442).
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass

import numpy as np


@dataclass
class Sample:
    config: str
    groups: int
    us: float
    bytes: float
    pieces: int


def max_pieces(lengths, groups: int) -> int:
    """Most pieces of one row when the rows' 32-token tiles, concatenated, are
    cut into `groups` equal ranges (the kernel's schedule)."""
    tiles = [(max(0, int(n)) + 31) // 32 for n in lengths]
    total = sum(tiles)
    best = 1
    prefix = 0
    for t in tiles:
        if t > 0 and total > 0:
            first = ((prefix + 1) * groups - 1) // total
            last = ((prefix + t) * groups - 1) // total
            best = max(best, last - first + 1)
        prefix += t
    return best


def samples(sweep: dict) -> list[Sample]:
    hkv, d, eb = sweep["hkv"], sweep.get("head_dim", 128), sweep.get("elem_bytes", 2)
    out = []
    for name, c in sweep["configs"].items():
        steps = c["lengths"]
        byts = float(np.mean([sum(s) for s in steps])) * hkv * d * 2 * eb
        for g, us in c["us_median"].items():
            pieces = int(round(np.mean([max_pieces(s, int(g)) for s in steps])))
            out.append(Sample(name, int(g), float(us), byts, pieces))
    return out


def predict(params: dict, s: Sample, hkv: int) -> float:
    gbps = min(params["read_gbps"], s.groups * hkv * params["dev_cta_gbps"])
    us = params["dev_fixed_us"] + s.bytes / (gbps * 1e3)
    if s.pieces >= 2:
        us += params["dev_merge_us"] + params["dev_merge_piece_us"] * s.pieces
    return us


def fit(sweep: dict) -> tuple[dict, float]:
    hkv = sweep["hkv"]
    data = samples(sweep)
    y = np.array([s.us for s in data])
    best, best_err = None, np.inf
    for read in np.arange(5000.0, 7001.0, 50.0):
        for cta in np.arange(10.0, 80.01, 0.5):
            stream = np.array([s.bytes / (min(read, s.groups * hkv * cta) * 1e3) for s in data])
            split = np.array([1.0 if s.pieces >= 2 else 0.0 for s in data])
            a = np.stack([np.ones_like(y), split, split * np.array([s.pieces for s in data])], 1)
            coef, *_ = np.linalg.lstsq(a, y - stream, rcond=None)
            coef = np.maximum(coef, 0.0)
            err = float(np.mean(((a @ coef + stream) - y) ** 2 / y ** 2))
            if err < best_err:
                best_err = err
                best = {"read_gbps": float(read), "dev_cta_gbps": float(cta),
                        "dev_fixed_us": float(coef[0]), "dev_merge_us": float(coef[1]),
                        "dev_merge_piece_us": float(coef[2])}
    return best, best_err


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("sweep", help="JSON of bench.py --sweep-groups (or its profiles/ summary)")
    args = ap.parse_args()
    text = open(args.sweep).read().strip().splitlines()
    sweep = json.loads(text[-1]) if len(text) == 1 or text[-1].startswith("{") else \
        json.loads("\n".join(text))
    if "us_median" not in next(iter(sweep["configs"].values())):
        for c in sweep["configs"].values():
            c["us_median"] = {g: float(np.median(v)) for g, v in c["us"].items()}
    params, err = fit(sweep)
    print(json.dumps({"fitted": params, "rms_relative_error": err ** 0.5}, indent=1))
    hkv = sweep["hkv"]
    for s in samples(sweep):
        print(f"{s.config:12s} NG={s.groups:3d} measured {s.us:8.2f} us  model "
              f"{predict(params, s, hkv):8.2f} us")


if __name__ == "__main__":
    main()
