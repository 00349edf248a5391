"""The entry point that allocates nothing (pkv_paged_attention_workqueue_noalloc).

Some callers cannot allocate device memory on the decode path: an FFI host
(Go, Java, C) that only receives device pointers from an inference server
owning every allocation through its own pool, or code that must not call
cudaMalloc there.  They cannot supply the workspace the other entry points
need, so this variant keeps its split partial states in a static device
array inside the library.  This test calls it through the C ABI several
times in a row (the array keeps the previous call's contents): twice with the
same row lengths, hence the same slot layout, on different data -- so a call
whose partial writes went missing would merge the previous call's partials
and fail -- then once with another shape.  Each result is checked against
the ordinary work-queue entry point and against the CPU oracle.  It lives in
its own file so pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from persistentkv_attention_b200 import _native, ops
from persistentkv_attention_b200.scheduler import Router
from tests.helpers import MAX_ERR, assert_close, make_case

pytestmark = pytest.mark.gpu


def _noalloc(lib, c, d, queue, out):
    items = torch.from_numpy(queue.work_items).cuda()
    offsets = torch.from_numpy(queue.split_offsets).cuda()
    status = lib.pkv_paged_attention_workqueue_noalloc(
        d["q_source"].data_ptr(), d["k_pages"].data_ptr(), d["v_pages"].data_ptr(),
        d["block_table"].data_ptr(), d["seq_lens"].data_ptr(), items.data_ptr(),
        offsets.data_ptr(), d["q_indices"].data_ptr(), d["out_indices"].data_ptr(),
        out.data_ptr(), len(c.seq_lens), c.q_source.shape[0], out.shape[0], c.hq, c.hkv, 128,
        c.k_pages.shape[0], c.page_size, c.block_table.shape[1], int(c.seq_lens.max()),
        queue.num_items, queue.total_slots, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return status, (items, offsets)


def _with_workspace(c, d, queue):
    out = torch.full((c.out_rows, c.hq, 128), float("nan"), device="cuda", dtype=torch.float16)
    ws = torch.empty(ops.workqueue_workspace_bytes(queue.total_slots, c.hq) // 4, device="cuda")
    counters = torch.zeros(len(c.seq_lens), c.hkv, device="cuda", dtype=torch.int32)
    ops.paged_attention_workqueue(
        d["q_source"], d["k_pages"], d["v_pages"], d["block_table"], d["seq_lens"],
        torch.from_numpy(queue.work_items).cuda(), torch.from_numpy(queue.split_offsets).cuda(),
        counters, d["q_indices"], d["out_indices"], out, ws, int(c.seq_lens.max()), c.page_size,
        queue.total_slots, False)
    torch.cuda.synchronize()
    return out


def test_noalloc_matches_workspace_entry_twice_in_a_row():
    lib = _native.load()
    same = [4096, 700, 9000, 33, 2048]
    cases = [make_case(same, seed=101, indexed=True),
             make_case(same, seed=202, indexed=True),      # same slots, other data
             make_case([12000, 1, 517, 6000], seed=303, indexed=True)]
    for c in cases:  # calls in a row: each sees the previous call's scratch contents
        d = c.cuda()
        queue = Router.b200(32, c.hkv).build_workqueue(c.seq_lens)
        assert queue.total_slots > len(c.seq_lens)  # real splits: the scratch is used
        want = _with_workspace(c, d, queue)
        got = torch.full_like(want, float("nan"))
        status, _ = _noalloc(lib, c, d, queue, got)
        assert status == _native.PKV_OK, lib.pkv_last_error_message()
        rows = torch.from_numpy(c.out_indices).long().cuda()
        diff = (got[rows].float() - want[rows].float()).abs().max().item()
        assert diff < MAX_ERR, diff
        assert torch.isfinite(got[rows].float()).all()
        want_cpu = c.oracle()
        assert_close(got[rows], want_cpu[c.out_indices], "f16", "no-alloc vs oracle")
    assert _native.device_error(clear=True) == 0


def test_noalloc_rejects_more_slots_than_its_scratch_holds():
    lib = _native.load()
    c = make_case([64], seed=7)
    d = c.cuda()
    queue = Router.b200(32, c.hkv).build_workqueue(c.seq_lens)
    out = torch.empty(1, 32, 128, device="cuda", dtype=torch.float16)
    limit_slots = (8 << 20) // (32 * 130 * 4)
    items = torch.from_numpy(queue.work_items).cuda()
    offsets = torch.from_numpy(queue.split_offsets).cuda()
    status = lib.pkv_paged_attention_workqueue_noalloc(
        d["q_source"].data_ptr(), d["k_pages"].data_ptr(), d["v_pages"].data_ptr(),
        d["block_table"].data_ptr(), d["seq_lens"].data_ptr(), items.data_ptr(),
        offsets.data_ptr(), d["q_indices"].data_ptr(), d["out_indices"].data_ptr(),
        out.data_ptr(), 1, 1, 1, 32, c.hkv, 128, c.k_pages.shape[0], 16,
        c.block_table.shape[1], 64, queue.num_items, limit_slots + 1, 0,
        torch.cuda.current_stream().cuda_stream)
    assert status == _native.PKV_ERR_CAPACITY
    assert b"holds at most" in lib.pkv_last_error_message()
