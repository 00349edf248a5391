"""CPU oracle of the paged GQA decode path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker (or the timed CPU
baseline), never as the engine: the product path is the CUDA library and
fails loudly without it.

It restates, in numpy, the reference's CPU algorithm for the path:

* ``cpu_gqa_attention`` -- ``tests/smoke_test.cu:35-74`` of the reference:
  exact softmax(q k^T / sqrt(d)) v per query head, KV head = qh // G, with the
  reference's ``/(l + 1e-8)`` normalisation (:70), on fp16-quantised inputs
  (:125-138);
* ``paged_decode`` -- the same computation on the paged cache layout
  ``[P, Hkv, page, D]`` with block tables, row-local ``seq_lens`` masking and
  ``q_indices`` / ``out_indices`` row indirection, i.e. the semantics of the
  reference's four extension entry points
  (``tests/persistentkv_torch_extension.cu:35-317``) and of its repack + SDPA
  oracle (``tests/benchmark_torch_paged_sdpa.py:90-109``);
* ``sdpa_repack_row`` / ``torch_paged_decode`` -- the reference's repack +
  SDPA oracle in torch (``tests/benchmark_torch_paged_sdpa.py:90-109``:
  index_select of the row's pages, permute to [Hkv, tokens, D], slice to the
  row's length, ``scaled_dot_product_attention(enable_gqa=True)``): the
  first in fp32 through torch's own SDPA (the timed CPU baseline of
  ``bench.py``), the second in float64 on any device (the checker of
  full-size steps whose K/V are too large to copy to the host);
* ``GlibcRand`` -- glibc's ``rand()`` (the TYPE_3 additive-feedback generator
  with its LCG seeding, as published), so the smoke test's ``srand(42)`` input
  stream (``tests/smoke_test.cu:77-81, :438``) can be replayed here and on a
  machine without the reference.

Parity is pinned by ``tests/golden`` (outputs of the reference's own
``cpu_gqa_attention`` compiled from its sources, and of its Python scheduler
functions) and, on a GPU, by the reference's CUDA extension built for sm_100a.
"""

from __future__ import annotations

import numpy as np

HEAD_DIM = 128


class GlibcRand:
    """glibc ``srand``/``rand``: the TYPE_3 additive-feedback generator
    x[i] = x[i-3] + x[i-31] (mod 2^32), seeded by the Park-Miller LCG
    x[i] = 16807 x[i-1] mod (2^31 - 1), first 310 outputs discarded,
    rand() = x >> 1."""

    RAND_MAX = 2147483647

    def __init__(self, seed: int = 1):
        self.seed(seed)

    def seed(self, seed: int) -> None:
        seed &= 0xFFFFFFFF
        if seed == 0:
            seed = 1
        word = seed - (1 << 32) if seed >= (1 << 31) else seed
        r = [word]
        for _ in range(1, 31):
            # Schrage's method with C (truncating) division, as in glibc
            hi = int(word / 127773)
            lo = word - hi * 127773
            word = 16807 * lo - 2836 * hi
            if word < 0:
                word += 2147483647
            r.append(word)
        r = [x & 0xFFFFFFFF for x in r]
        r += r[:3]                      # x[31..33] = x[0..2]
        for _ in range(310):
            r.append((r[-31] + r[-3]) & 0xFFFFFFFF)
        self._hist = r[-31:]

    def rand_array(self, n: int) -> np.ndarray:
        """The next ``n`` values of ``rand()`` as int64."""
        buf = self._hist + [0] * n
        for i in range(31, 31 + n):
            buf[i] = (buf[i - 31] + buf[i - 3]) & 0xFFFFFFFF
        self._hist = buf[-31:]
        return np.asarray(buf[31:], dtype=np.int64) >> 1

    def smoke_uniform(self, n: int) -> np.ndarray:
        """``(float)rand() / RAND_MAX * 2.0f - 1.0f`` in float32 (smoke_test.cu:77)."""
        r = self.rand_array(n).astype(np.float32)
        return r / np.float32(self.RAND_MAX) * np.float32(2.0) - np.float32(1.0)


def quantize(x: np.ndarray, dtype: str = "f16") -> np.ndarray:
    """Round to fp16 / bf16 and return float32 (what the GPU sees)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        bits = x.view(np.uint32).astype(np.uint64)
        rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
        return rounded.astype(np.uint32).view(np.float32)
    raise ValueError(dtype)


def cpu_gqa_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Reference cpu_gqa_attention (tests/smoke_test.cu:35-74) in float64.

    q [B, Hq, D], k/v [B, Hkv, N, D] -> O [B, Hq, D].
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    b, hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    scale = 1.0 / np.sqrt(np.float32(d))
    out = np.empty((b, hq, d), dtype=np.float64)
    for bi in range(b):
        for kvh in range(hkv):
            qs = q[bi, kvh * g:(kvh + 1) * g]                  # [G, D]
            s = (qs @ k[bi, kvh].T) * scale                    # [G, N]
            m = s.max(axis=1, keepdims=True)
            w = np.exp(s - m)
            l = w.sum(axis=1, keepdims=True)
            out[bi, kvh * g:(kvh + 1) * g] = (w @ v[bi, kvh]) / (l + 1e-8)
    return out


def attend_row(q_row: np.ndarray, k_tok: np.ndarray, v_tok: np.ndarray) -> np.ndarray:
    """One row: q [Hq, D], k/v [Hkv, N, D] (float64) -> [Hq, D]; N may be 0."""
    hq = q_row.shape[0]
    hkv = k_tok.shape[0]
    g = hq // hkv
    n = k_tok.shape[1]
    if n == 0:
        return np.zeros((hq, HEAD_DIM), dtype=np.float64)
    scale = 1.0 / np.sqrt(np.float32(HEAD_DIM))
    qg = q_row.reshape(hkv, g, HEAD_DIM)
    s = np.einsum("hgd,hnd->hgn", qg, k_tok) * scale
    m = s.max(axis=2, keepdims=True)
    w = np.exp(s - m)
    l = w.sum(axis=2, keepdims=True)
    o = np.einsum("hgn,hnd->hgd", w, v_tok) / l
    return o.reshape(hq, HEAD_DIM)


def gather_row(k_pages: np.ndarray, v_pages: np.ndarray, table_row: np.ndarray, n: int):
    """Repack one row's first n tokens to [Hkv, n, D] (float64), following the
    reference's index_select + permute repack (benchmark_torch_paged_sdpa.py:90-103)."""
    page = k_pages.shape[2]
    pages = (n + page - 1) // page
    ids = np.asarray(table_row[:pages], dtype=np.int64)
    k = k_pages[ids].astype(np.float64)                    # [pages, Hkv, page, D]
    v = v_pages[ids].astype(np.float64)
    hkv = k.shape[1]
    k = k.transpose(1, 0, 2, 3).reshape(hkv, pages * page, HEAD_DIM)[:, :n]
    v = v.transpose(1, 0, 2, 3).reshape(hkv, pages * page, HEAD_DIM)[:, :n]
    return k, v


def paged_decode(q_source, k_pages, v_pages, block_table, seq_lens=None, context=None,
                 q_indices=None, out_indices=None, out_rows=None) -> np.ndarray:
    """Paged decode of every row b of ``block_table`` (float64 result).

    Row b attends to the first ``seq_lens[b]`` tokens (or ``context`` when
    ``seq_lens`` is None) of its block-table row, reads ``q_source[q_indices[b]]``
    and writes ``out[out_indices[b]]``.  Rows never written stay NaN.
    """
    q_source = np.asarray(q_source, dtype=np.float64)
    bt = np.asarray(block_table)
    b = bt.shape[0]
    hq = q_source.shape[1]
    rows = out_rows if out_rows is not None else (b if out_indices is None else q_source.shape[0])
    out = np.full((rows, hq, HEAD_DIM), np.nan, dtype=np.float64)
    for bi in range(b):
        n = int(seq_lens[bi]) if seq_lens is not None else int(context)
        qi = int(q_indices[bi]) if q_indices is not None else bi
        oi = int(out_indices[bi]) if out_indices is not None else bi
        k, v = gather_row(k_pages, v_pages, bt[bi], n)
        out[oi] = attend_row(q_source[qi], k, v)
    return out


def row_state(q_row, k_tok, v_tok):
    """Unnormalised log-sum-exp state of one row: (m [Hq], l [Hq], acc [Hq, D]),
    m in natural units of the scaled scores (layout of the engine's state_out)."""
    hq = q_row.shape[0]
    hkv = k_tok.shape[0]
    g = hq // hkv
    if k_tok.shape[1] == 0:
        return (np.full(hq, -np.finfo(np.float32).max), np.zeros(hq),
                np.zeros((hq, HEAD_DIM)))
    scale = 1.0 / np.sqrt(np.float32(HEAD_DIM))
    s = np.einsum("hgd,hnd->hgn", q_row.reshape(hkv, g, HEAD_DIM), k_tok) * scale
    m = s.max(axis=2)
    w = np.exp(s - m[..., None])
    return m.reshape(hq), w.sum(axis=2).reshape(hq), np.einsum(
        "hgn,hnd->hgd", w, v_tok).reshape(hq, HEAD_DIM)


def combine_states(ms, ls, accs):
    """LSE merge of n partial states (reference merge, kernels/...cuh:719-751)."""
    ms = np.asarray(ms, dtype=np.float64)
    mx = ms.max(axis=0)
    w = np.exp(ms - mx)
    l = (w * np.asarray(ls)).sum(axis=0)
    acc = (w[..., None] * np.asarray(accs)).sum(axis=0)
    return np.where(l[..., None] > 0, acc / np.where(l > 0, l, 1)[..., None], 0.0)


def error_stats(got, ref) -> tuple[float, float]:
    """Max and mean absolute error over the rows the reference defines."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    mask = ~np.isnan(ref)
    diff = np.abs(got[mask] - ref[mask])
    return float(diff.max(initial=0.0)), float(diff.mean() if diff.size else 0.0)


def kv_append(k_new, v_new, k_pages, v_pages, block_table, positions, free_pages=None,
              free_count=None):
    """CPU restatement of ``pkv_kv_append`` (in place on numpy arrays).

    Row b writes k_new[b] / v_new[b] at token positions[b] of its block-table
    row.  With a free list, the rows whose token opens a page (position %
    page_size == 0), in row order, take free_pages[free_count - 1],
    free_pages[free_count - 2], ...; the page id goes into the block table.
    Rows with an invalid position, an out-of-pool page or no free page left
    write nothing.  Returns (new free_count, error bits) with the bits of
    ``pkv_device_error`` (0x1 page id, 0x2 position, 0x80 list exhausted).
    The reference has no append: its pool is pre-filled
    (tests/benchmark_serving_trace.py:253-263); this follows the C ABI's
    documented semantics.
    """
    page = k_pages.shape[2]
    num_pages = k_pages.shape[0]
    max_pages = block_table.shape[1]
    errors = 0
    taken = 0
    avail = int(free_count) if free_pages is not None else 0
    for b, pos in enumerate(np.asarray(positions)):
        pos = int(pos)
        if pos < 0 or pos >= max_pages * page:
            errors |= 0x2
            continue
        slot = pos // page
        if free_pages is not None and pos % page == 0:
            k = avail - 1 - taken
            taken += 1
            if k < 0:
                errors |= 0x80
                continue
            pid = int(free_pages[k])
            if pid < 0 or pid >= num_pages:
                errors |= 0x1
                continue
            block_table[b, slot] = pid
        else:
            pid = int(block_table[b, slot])
            if pid < 0 or pid >= num_pages:
                errors |= 0x1
                continue
        k_pages[pid, :, pos % page, :] = k_new[b]
        v_pages[pid, :, pos % page, :] = v_new[b]
    new_count = avail - min(taken, avail) if free_pages is not None else free_count
    return new_count, errors



def sdpa_repack_row(q_row, k_pages, v_pages, pages, n):
    """One row through the reference's torch repack + SDPA path
    (tests/benchmark_torch_paged_sdpa.py:90-109) in fp32 on torch tensors:
    q_row [Hq, D], pools [P, Hkv, page, D], pages = the row's physical page
    ids (int64 tensor) -> [Hq, D]."""
    import torch
    import torch.nn.functional as F

    hkv, page = k_pages.shape[1], k_pages.shape[2]
    n_pages = pages.numel()
    k = (torch.index_select(k_pages, 0, pages).permute(1, 0, 2, 3).contiguous()
         .view(1, hkv, n_pages * page, HEAD_DIM))[:, :, :n]
    v = (torch.index_select(v_pages, 0, pages).permute(1, 0, 2, 3).contiguous()
         .view(1, hkv, n_pages * page, HEAD_DIM))[:, :, :n]
    out = F.scaled_dot_product_attention(q_row[None, :, None, :], k, v, is_causal=False,
                                         enable_gqa=True)
    return out[0, :, 0, :]


def torch_paged_decode(q_source, k_pages, v_pages, block_table, seq_lens, q_indices=None,
                       out_indices=None, out_rows=None):
    """``paged_decode`` in float64 with torch on the tensors' own device: per
    row, the repack of benchmark_torch_paged_sdpa.py:90-103 and exact
    softmax(q k^T / sqrt(128)) v.  Rows never written stay NaN."""
    import torch

    dev = k_pages.device
    bt = torch.as_tensor(block_table, device=dev).long()
    sl = [int(x) for x in (seq_lens.tolist() if hasattr(seq_lens, "tolist") else seq_lens)]
    b = bt.shape[0]
    hq = q_source.shape[1]
    hkv, page = k_pages.shape[1], k_pages.shape[2]
    g = hq // hkv
    qi = list(range(b)) if q_indices is None else [int(x) for x in q_indices]
    oi = list(range(b)) if out_indices is None else [int(x) for x in out_indices]
    rows = out_rows if out_rows is not None else b
    out = torch.full((rows, hq, HEAD_DIM), float("nan"), dtype=torch.float64, device=dev)
    # the fp32 scale 1.0f / sqrtf(128) of the reference (smoke_test.cu:35-74)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(HEAD_DIM)))
    for r in range(b):
        n = sl[r]
        if n <= 0:
            out[oi[r]] = 0.0
            continue
        pages = bt[r, : (n + page - 1) // page]
        k = k_pages.index_select(0, pages).permute(1, 0, 2, 3).reshape(hkv, -1, HEAD_DIM)[:, :n]
        v = v_pages.index_select(0, pages).permute(1, 0, 2, 3).reshape(hkv, -1, HEAD_DIM)[:, :n]
        q = q_source[qi[r]].double().view(hkv, g, HEAD_DIM)
        s = torch.einsum("hgd,hnd->hgn", q, k.double()) * scale
        w = torch.exp(s - s.amax(dim=2, keepdim=True))
        o = torch.einsum("hgn,hnd->hgd", w, v.double()) / w.sum(dim=2, keepdim=True)
        out[oi[r]] = o.reshape(hq, HEAD_DIM)
    return out
