"""Seeded paged-decode cases shared by the GPU parity tests."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from oracle import pkv_oracle as po

DT = {"f16": torch.float16, "bf16": torch.bfloat16}

# tolerances of the reference (benchmark_serving_trace.py:37-38, smoke_test.cu:104-106)
MAX_ERR = 2e-3
MEAN_ERR = 3e-4


@dataclass
class Case:
    q_source: torch.Tensor     # [R, Hq, D] (CPU)
    k_pages: torch.Tensor      # [P, Hkv, page, D]
    v_pages: torch.Tensor
    block_table: np.ndarray    # [B, max_pages] int32
    seq_lens: np.ndarray       # [B] int32
    q_indices: np.ndarray      # [B] int32
    out_indices: np.ndarray    # [B] int32
    out_rows: int
    page_size: int
    dtype: str

    @property
    def hq(self):
        return self.q_source.shape[1]

    @property
    def hkv(self):
        return self.k_pages.shape[1]

    def oracle(self, seq_lens=True, context=None):
        f = lambda t: t.float().numpy()  # noqa: E731
        return po.paged_decode(f(self.q_source), f(self.k_pages), f(self.v_pages),
                               self.block_table,
                               seq_lens=self.seq_lens if seq_lens else None, context=context,
                               q_indices=self.q_indices, out_indices=self.out_indices,
                               out_rows=self.out_rows)

    def cuda(self):
        d = torch.device("cuda")
        return dict(
            q_source=self.q_source.to(d), k_pages=self.k_pages.to(d), v_pages=self.v_pages.to(d),
            block_table=torch.from_numpy(self.block_table).to(d),
            seq_lens=torch.from_numpy(self.seq_lens).to(d),
            q_indices=torch.from_numpy(self.q_indices).to(d),
            out_indices=torch.from_numpy(self.out_indices).to(d),
        )


def make_case(lens, hq=32, hkv=8, page_size=16, dtype="f16", seed=0, holes=0.25,
              indexed=False, extra_pages=0, scale=1.0) -> Case:
    """Rows of the given lengths over a shuffled, partly unused page pool."""
    gen = torch.Generator().manual_seed(seed)
    lens = [int(x) for x in lens]
    b = len(lens)
    pages_per_row = [max(1, (n + page_size - 1) // page_size) for n in lens]
    max_pages = max(pages_per_row) + extra_pages
    used = sum(pages_per_row)
    pool = int(np.ceil(used / (1.0 - holes))) + 1
    perm = torch.randperm(pool, generator=gen).numpy().astype(np.int32)
    table = np.zeros((b, max_pages), np.int32)
    cur = 0
    for i, n in enumerate(pages_per_row):
        table[i, :n] = perm[cur:cur + n]
        table[i, n:] = perm[cur + n - 1]          # pad with the row's last page
        cur += n
    k = (torch.randn(pool, hkv, page_size, 128, generator=gen) * scale).to(DT[dtype])
    v = torch.randn(pool, hkv, page_size, 128, generator=gen).to(DT[dtype])
    if indexed:
        rows = b + 3
        q = torch.randn(rows, hq, 128, generator=gen).to(DT[dtype])
        q_idx = torch.randperm(rows, generator=gen)[:b].numpy().astype(np.int32)
        o_idx = torch.randperm(rows, generator=gen)[:b].numpy().astype(np.int32)
        out_rows = rows
    else:
        q = torch.randn(b, hq, 128, generator=gen).to(DT[dtype])
        q_idx = np.arange(b, dtype=np.int32)
        o_idx = np.arange(b, dtype=np.int32)
        out_rows = b
    return Case(q, k, v, table, np.asarray(lens, np.int32), q_idx, o_idx, out_rows, page_size,
                dtype)


def assert_close(got: torch.Tensor, ref: np.ndarray, dtype: str, what=""):
    """fp16: max 2e-3 / mean 3e-4 (reference).  bf16: the same plus one bf16
    rounding of the output value (2^-8 relative), since the result is stored
    in bf16."""
    g = got.float().cpu().numpy().astype(np.float64)
    mask = ~np.isnan(ref)
    diff = np.abs(g[mask] - ref[mask])
    assert np.isfinite(g[mask]).all(), f"non-finite output {what}"
    if dtype == "bf16":
        bound = MAX_ERR + np.abs(ref[mask]) * 2.0 ** -8
        assert (diff <= bound).all(), f"{what}: max excess {np.max(diff - bound):.3e}"
        assert diff.mean() < MEAN_ERR + np.abs(ref[mask]).mean() * 2.0 ** -9, what
    else:
        assert diff.max() < MAX_ERR, f"{what}: max err {diff.max():.3e}"
        assert diff.mean() < MEAN_ERR, f"{what}: mean err {diff.mean():.3e}"
    return float(diff.max()), float(diff.mean())


def config1_case(seed: int = 20260615 + 4096) -> Case:
    """BASELINE config 1 exactly: B=1, 4096 tokens, Hq 32 / Hkv 8, head_dim 128,
    page 16, so 256 logical pages, drawn as a seeded random permutation from a
    pool of 1024 pages; q / K / V fp16 N(0,1) (every pool page filled).  The
    seed follows the reference's per-context seeding of its single-request
    baselines (20260615 + context, benchmark_native_paged_baselines.py:49-51)."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(1, 32, 128, generator=gen).half()
    k = torch.randn(1024, 8, 16, 128, generator=gen).half()
    v = torch.randn(1024, 8, 16, 128, generator=gen).half()
    table = torch.randperm(1024, generator=gen)[:256].numpy().astype(np.int32)[None]
    zero = np.zeros(1, np.int32)
    return Case(q, k, v, table, np.array([4096], np.int32), zero, zero, 1, 16, "f16")
