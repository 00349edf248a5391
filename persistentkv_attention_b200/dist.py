"""Multi-GPU decode: batch partitioning and sequence sharding.

The reference never crosses a GPU.  Two forms are provided here:

* batch partitioning -- each rank owns a disjoint set of active requests and
  their pages (in its own pool) and runs the single-GPU engine on them; no
  data-path collective (``partition_rows``);
* sequence sharding of a long request -- rank r owns the contiguous logical
  page range ``shard_pages(...)[r]`` of every row, decodes it into a log-sum-
  exp state ``[B, Hq, 130]`` (``ops.paged_attention_workqueue_state``), the
  states are all-gathered, and each rank merges them exactly
  (``ops.combine_states``): LSE merging is associative, so the result equals
  the single-GPU decode.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

STATE_WIDTH = 130


def shard_pages(num_pages: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, balanced logical page ranges [lo, hi) for each rank."""
    base, extra = divmod(num_pages, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def shard_rows(block_table: np.ndarray, seq_lens, page_size: int, world: int, rank: int):
    """Block table and lengths of this rank's page range of every row.

    Rows whose range is empty keep one (padding) page and length 0.
    """
    seq = np.asarray(seq_lens, dtype=np.int64)
    rows, lens = [], []
    for b, n in enumerate(seq):
        pages = (int(n) + page_size - 1) // page_size
        lo, hi = shard_pages(pages, world)[rank]
        toks = max(0, min(int(n), hi * page_size) - lo * page_size) if hi > lo else 0
        row = block_table[b, lo:hi] if hi > lo else block_table[b, :1]
        rows.append(np.asarray(row, dtype=np.int32))
        lens.append(toks)
    width = max(1, max(len(r) for r in rows))
    table = np.stack([np.pad(r, (0, width - len(r)), mode="edge") for r in rows]).astype(np.int32)
    return table, np.asarray(lens, dtype=np.int32)


def partition_rows(kv_bytes, world: int) -> list[list[int]]:
    """Greedy longest-processing-time assignment of rows to ranks by KV bytes."""
    order = sorted(range(len(kv_bytes)), key=lambda i: -kv_bytes[i])
    load = [0] * world
    out = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: load[k])
        out[r].append(i)
        load[r] += kv_bytes[i]
    return [sorted(x) for x in out]


def gather_states(state: torch.Tensor, group=None) -> torch.Tensor:
    """All-gathers ``[B, Hq, 130]`` float32 states into ``[world, B, Hq, 130]``."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(state.shape), dtype=state.dtype, device=state.device)
    if state.is_cuda:
        dist.all_gather_into_tensor(out, state.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), state.contiguous(), group=group)
    return out


class SequenceShardedDecoder:
    """One rank of a sequence-sharded work-queue decode (NCCL exchange).

    Each step: decode this rank's pages into a state, all-gather the states of
    all ranks, merge them into ``out`` on every rank.
    """

    def __init__(self, engine, group=None):
        self.engine = engine
        self.group = group
        self.state = None

    def step(self, plan, q_source: torch.Tensor, out: torch.Tensor) -> None:
        from . import ops

        e = self.engine
        b = plan.batch
        if self.state is None or self.state.shape[0] < b:
            self.state = torch.empty(b, e.hq, STATE_WIDTH, device=e.device, dtype=torch.float32)
        st = self.state[:b]
        f = plan.fields
        counters = e._counters[: b * e.hkv].view(b, e.hkv)
        ops.paged_attention_workqueue_state(
            q_source, e.k_pages, e.v_pages, f["block_table"], f["seq_lens"], f["work_items"],
            f["split_offsets"], counters, f["q_indices"], st, e._workspace, e.page_size,
            plan.host.total_slots, True)
        states = gather_states(st, self.group)
        ops.combine_states(states, out)


def make_exchange(hq: int, hkv: int, max_batch: int, group=None):
    """Creates this rank's ``ops.Exchange`` and maps every peer's buffer.

    The IPC handles travel over the process group (``all_gather_object``);
    a barrier makes sure every rank is connected before any kernel uses it."""
    from . import ops

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    x = ops.Exchange(world, rank, max_batch, hq, hkv)
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, x.handle, group=group)
        x.connect(handles)
        dist.barrier(group=group)
    return x


class FusedShardedDecoder:
    """One rank of a sequence-sharded decode whose state exchange runs inside
    the decode kernel (peer stores over NVLink, no NCCL call per step)."""

    def __init__(self, engine, max_batch: int, group=None):
        self.engine = engine
        self.exchange = make_exchange(engine.hq, engine.hkv, max_batch, group)

    def step(self, plan, q_source: torch.Tensor, out: torch.Tensor) -> None:
        self.engine.run_sharded(plan, q_source, out, self.exchange)

    def close(self, group=None) -> None:
        """Frees the exchange once no rank's kernel can still store into it."""
        torch.cuda.synchronize()
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.barrier(group=group)
        self.exchange.close()

