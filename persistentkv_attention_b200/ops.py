"""PyTorch-facing operator surface of the B200 decode engine.

The four functions below keep the names, argument order, argument meaning and
error behaviour (``RuntimeError`` with the same messages) of the reference's
extension module, ``tests/persistentkv_torch_extension.cu:319-336``, so the
reference's serving harness can load this module in place of its own:

    paged_attention(q, k_pages, v_pages, block_table, output, workspace,
                    context, page_size, num_splits)
    paged_attention_masked(q, k_pages, v_pages, block_table, seq_lens, output,
                           workspace, bucket_context, page_size, num_splits)
    paged_attention_indexed(q_source, k_pages, v_pages, block_table, seq_lens,
                            q_indices, out_indices, output, workspace,
                            bucket_context, page_size, num_splits)
    paged_attention_workqueue(q_source, k_pages, v_pages, block_table, seq_lens,
                              work_items, split_offsets, merge_counters,
                              q_indices, out_indices, output, workspace,
                              bucket_context, page_size, total_partial_slots,
                              fused_merge)

Each call only validates tensors and forwards raw pointers to the C ABI of
``libpkv_b200.so`` on the current CUDA stream; PyTorch supplies device memory
and streams, never the computation.  Beyond the reference, q/K/V/output may be
bfloat16 (all of them), and two calls serve sequence sharding across GPUs
(``paged_attention_workqueue_state`` and ``combine_states``).
"""

from __future__ import annotations

import torch

from . import _native

HEAD_DIM = 128
STATE_STRIDE = HEAD_DIM + 2

_DTYPES = {torch.float16: _native.PKV_DTYPE_F16, torch.bfloat16: _native.PKV_DTYPE_BF16}


def _check_tensor(tensor: torch.Tensor, name: str, dtype, dims: int) -> None:
    # reference check_tensor (tests/persistentkv_torch_extension.cu:9-19)
    if not tensor.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if (tensor.dtype not in dtype) if isinstance(dtype, tuple) else tensor.dtype != dtype:
        raise RuntimeError(f"{name} has wrong dtype")
    if tensor.dim() != dims:
        raise RuntimeError(f"{name} has wrong rank")
    if not tensor.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_supported_gqa(hq: int, hkv: int) -> None:
    # reference check_supported_gqa (tests/persistentkv_torch_extension.cu:21-31)
    if hkv <= 0:
        raise RuntimeError("Hkv must be positive")
    if hq % hkv != 0:
        raise RuntimeError("Hq must be divisible by Hkv")
    g = hq // hkv
    if g not in (1, 2, 4, 8):
        raise RuntimeError(
            f"PersistentKV supports G=Hq/Hkv in {{1,2,4,8}}; got G={g} from Hq={hq} Hkv={hkv}"
        )


def _check_kv(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, page_size: int):
    dt = q.dtype
    _check_tensor(k_pages, "k_pages", dt, 4)
    _check_tensor(v_pages, "v_pages", dt, 4)
    d = q.size(2)
    hkv = k_pages.size(1)
    physical_pages = k_pages.size(0)
    if d != HEAD_DIM:
        raise RuntimeError("PersistentKV extension currently requires d=128")
    if not (v_pages.size(0) == physical_pages and v_pages.size(1) == hkv
            and v_pages.size(2) == page_size and v_pages.size(3) == d):
        raise RuntimeError("v_pages shape mismatch")
    if not (k_pages.size(2) == page_size and k_pages.size(3) == d):
        raise RuntimeError("k_pages shape mismatch")
    return hkv, physical_pages


def _workspace(workspace: torch.Tensor):
    if not workspace.is_cuda:
        raise RuntimeError("workspace must be a CUDA tensor")
    if not workspace.is_contiguous():
        raise RuntimeError("workspace must be contiguous")
    if workspace.numel() == 0:
        return None, 0
    return workspace.data_ptr(), workspace.numel() * workspace.element_size()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream() -> int:
    """Raw ``cudaStream_t`` of the current stream on the current device (the
    raw getter avoids building a ``torch.cuda.Stream`` object per call)."""
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return torch.cuda.current_stream().cuda_stream


def _positive(value: int, name: str) -> None:
    if value <= 0:
        raise RuntimeError(f"{name} must be positive")


def paged_attention(q, k_pages, v_pages, block_table, output, workspace, context: int,
                    page_size: int, num_splits: int) -> None:
    """Reference ``persistentkv_paged_attention`` (extension :35-93)."""
    _check_tensor(q, "q", tuple(_DTYPES), 3)
    hkv, physical_pages = _check_kv(q, k_pages, v_pages, page_size)
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(output, "output", q.dtype, 3)
    ws_ptr, ws_bytes = _workspace(workspace)
    b, hq, d = q.shape
    if not (output.size(0) == b and output.size(1) == hq and output.size(2) == d):
        raise RuntimeError("output shape must match q")
    if block_table.size(0) != b:
        raise RuntimeError("block_table batch mismatch")
    _check_supported_gqa(hq, hkv)
    _positive(context, "context")
    _positive(page_size, "page_size")
    _positive(num_splits, "num_splits")
    lib = _native.load()
    _native.check(lib.pkv_paged_attention(
        q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        output.data_ptr(), ws_ptr, ws_bytes, b, hq, hkv, d, physical_pages, page_size,
        block_table.size(1), int(context), int(num_splits), _DTYPES[q.dtype], _stream()))


def paged_attention_masked(q, k_pages, v_pages, block_table, seq_lens, output, workspace,
                           bucket_context: int, page_size: int, num_splits: int) -> None:
    """Reference ``persistentkv_paged_attention_masked`` (extension :95-157)."""
    _check_tensor(q, "q", tuple(_DTYPES), 3)
    hkv, physical_pages = _check_kv(q, k_pages, v_pages, page_size)
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(seq_lens, "seq_lens", torch.int32, 1)
    _check_tensor(output, "output", q.dtype, 3)
    ws_ptr, ws_bytes = _workspace(workspace)
    b, hq, d = q.shape
    if not (output.size(0) == b and output.size(1) == hq and output.size(2) == d):
        raise RuntimeError("output shape must match q")
    if seq_lens.size(0) != b:
        raise RuntimeError("seq_lens batch mismatch")
    if block_table.size(0) != b:
        raise RuntimeError("block_table batch mismatch")
    _check_supported_gqa(hq, hkv)
    _positive(bucket_context, "bucket_context")
    _positive(page_size, "page_size")
    _positive(num_splits, "num_splits")
    lib = _native.load()
    _native.check(lib.pkv_paged_attention_masked(
        q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), output.data_ptr(), ws_ptr, ws_bytes, b, hq, hkv, d,
        physical_pages, page_size, block_table.size(1), int(bucket_context), int(num_splits),
        _DTYPES[q.dtype], _stream()))


def paged_attention_indexed(q_source, k_pages, v_pages, block_table, seq_lens, q_indices,
                            out_indices, output, workspace, bucket_context: int,
                            page_size: int, num_splits: int) -> None:
    """Reference ``persistentkv_paged_attention_indexed`` (extension :159-228)."""
    _check_tensor(q_source, "q_source", tuple(_DTYPES), 3)
    hkv, physical_pages = _check_kv(q_source, k_pages, v_pages, page_size)
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(seq_lens, "seq_lens", torch.int32, 1)
    _check_tensor(q_indices, "q_indices", torch.int32, 1)
    _check_tensor(out_indices, "out_indices", torch.int32, 1)
    _check_tensor(output, "output", q_source.dtype, 3)
    ws_ptr, ws_bytes = _workspace(workspace)
    b = block_table.size(0)
    hq, d = q_source.size(1), q_source.size(2)
    if not (output.size(1) == hq and output.size(2) == d):
        raise RuntimeError("output shape must match q head dimensions")
    if seq_lens.size(0) != b:
        raise RuntimeError("seq_lens batch mismatch")
    if q_indices.size(0) != b:
        raise RuntimeError("q_indices batch mismatch")
    if out_indices.size(0) != b:
        raise RuntimeError("out_indices batch mismatch")
    _check_supported_gqa(hq, hkv)
    _positive(bucket_context, "bucket_context")
    _positive(page_size, "page_size")
    _positive(num_splits, "num_splits")
    lib = _native.load()
    _native.check(lib.pkv_paged_attention_indexed(
        q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), q_indices.data_ptr(), out_indices.data_ptr(), output.data_ptr(),
        ws_ptr, ws_bytes, b, q_source.size(0), output.size(0), hq, hkv, d, physical_pages,
        page_size, block_table.size(1), int(bucket_context), int(num_splits),
        _DTYPES[q_source.dtype], _stream()))


def _check_workqueue(q_source, k_pages, v_pages, block_table, seq_lens, work_items,
                     split_offsets, merge_counters, q_indices, page_size):
    _check_tensor(q_source, "q_source", tuple(_DTYPES), 3)
    hkv, physical_pages = _check_kv(q_source, k_pages, v_pages, page_size)
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(seq_lens, "seq_lens", torch.int32, 1)
    _check_tensor(work_items, "work_items", torch.int32, 2)
    _check_tensor(split_offsets, "split_offsets", torch.int32, 1)
    _check_tensor(merge_counters, "merge_counters", torch.int32, 2)
    _check_tensor(q_indices, "q_indices", torch.int32, 1)
    b = block_table.size(0)
    if work_items.size(1) != 5:
        raise RuntimeError("work_items must have shape [T, 5]")
    if split_offsets.size(0) != b + 1:
        raise RuntimeError("split_offsets batch mismatch")
    if not (merge_counters.size(0) == b and merge_counters.size(1) == hkv):
        raise RuntimeError("merge_counters shape mismatch")
    if seq_lens.size(0) != b:
        raise RuntimeError("seq_lens batch mismatch")
    if q_indices.size(0) != b:
        raise RuntimeError("q_indices batch mismatch")
    return hkv, physical_pages, b


def paged_attention_workqueue(q_source, k_pages, v_pages, block_table, seq_lens, work_items,
                              split_offsets, merge_counters, q_indices, out_indices, output,
                              workspace, bucket_context: int, page_size: int,
                              total_partial_slots: int, fused_merge: bool) -> None:
    """Reference ``persistentkv_paged_attention_workqueue`` (extension :230-317)."""
    hkv, physical_pages, b = _check_workqueue(q_source, k_pages, v_pages, block_table, seq_lens,
                                              work_items, split_offsets, merge_counters,
                                              q_indices, page_size)
    _check_tensor(out_indices, "out_indices", torch.int32, 1)
    _check_tensor(output, "output", q_source.dtype, 3)
    ws_ptr, ws_bytes = _workspace(workspace)
    hq, d = q_source.size(1), q_source.size(2)
    if not (output.size(1) == hq and output.size(2) == d):
        raise RuntimeError("output shape must match q head dimensions")
    if out_indices.size(0) != b:
        raise RuntimeError("out_indices batch mismatch")
    _check_supported_gqa(hq, hkv)
    _positive(bucket_context, "bucket_context")
    _positive(page_size, "page_size")
    if work_items.size(0) <= 0:
        raise RuntimeError("work_items must not be empty")
    if total_partial_slots <= 0:
        raise RuntimeError("total_partial_slots must be positive")
    lib = _native.load()
    _native.check(lib.pkv_paged_attention_workqueue(
        q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), work_items.data_ptr(), split_offsets.data_ptr(),
        merge_counters.data_ptr(), q_indices.data_ptr(), out_indices.data_ptr(),
        output.data_ptr(), ws_ptr, ws_bytes, b, q_source.size(0), output.size(0), hq, hkv, d,
        physical_pages, page_size, block_table.size(1), int(bucket_context),
        work_items.size(0), int(total_partial_slots), 1 if fused_merge else 0,
        _DTYPES[q_source.dtype], _stream()))


def paged_attention_workqueue_state(q_source, k_pages, v_pages, block_table, seq_lens,
                                    work_items, split_offsets, merge_counters, q_indices,
                                    state_out, workspace, page_size: int,
                                    total_partial_slots: int, fused_merge: bool) -> None:
    """Work-queue decode that writes each row's combined (m, l, acc) state.

    ``state_out`` is float32 ``[B, Hq, 130]``; no counterpart in the reference.
    """
    hkv, physical_pages, b = _check_workqueue(q_source, k_pages, v_pages, block_table, seq_lens,
                                              work_items, split_offsets, merge_counters,
                                              q_indices, page_size)
    _check_tensor(state_out, "state_out", torch.float32, 3)
    hq, d = q_source.size(1), q_source.size(2)
    if tuple(state_out.shape) != (b, hq, STATE_STRIDE):
        raise RuntimeError("state_out must have shape [B, Hq, 130]")
    _check_supported_gqa(hq, hkv)
    ws_ptr, ws_bytes = _workspace(workspace)
    lib = _native.load()
    _native.check(lib.pkv_paged_attention_workqueue_state(
        q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), work_items.data_ptr(), split_offsets.data_ptr(),
        merge_counters.data_ptr() if fused_merge else None, q_indices.data_ptr(),
        state_out.data_ptr(), ws_ptr, ws_bytes, b, q_source.size(0), hq, hkv, d,
        physical_pages, page_size, block_table.size(1), work_items.size(0),
        int(total_partial_slots), _DTYPES[q_source.dtype], _stream()))


def paged_attention_auto(q_source, k_pages, v_pages, block_table, seq_lens, output, workspace,
                         q_indices=None, out_indices=None, merge_counters=None,
                         plan=None, groups: int = 0) -> None:
    """Paged decode with the device-side schedule (no work queue, no host builder).

    Row b attends to ``seq_lens[b]`` tokens of ``block_table[b]``, reads
    ``q_source[q_indices[b]]`` and writes ``output[out_indices[b]]`` (identity
    when an index tensor is None).  ``merge_counters`` (zeroed int32
    ``[B, Hkv]``) selects the fused merge.  ``workspace`` needs
    ``auto_workspace_bytes(B, Hq, Hkv)`` bytes.  ``plan`` (optional) is a
    device int32 copy of ``scheduler.build_auto_plan`` for exactly this step's
    metadata: the kernel then starts from it instead of deriving the schedule;
    ``groups`` is the group count the plan was built for (0: the maximum).
    No counterpart in the reference.
    """
    _check_tensor(q_source, "q_source", tuple(_DTYPES), 3)
    hkv, physical_pages = _check_kv(q_source, k_pages, v_pages, k_pages.size(2))
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(seq_lens, "seq_lens", torch.int32, 1)
    _check_tensor(output, "output", q_source.dtype, 3)
    b = block_table.size(0)
    hq, d = q_source.size(1), q_source.size(2)
    if seq_lens.size(0) != b:
        raise RuntimeError("seq_lens batch mismatch")
    if not (output.size(1) == hq and output.size(2) == d):
        raise RuntimeError("output shape must match q head dimensions")
    ptrs = []
    for name, t in (("q_indices", q_indices), ("out_indices", out_indices)):
        if t is None:
            ptrs.append(None)
        else:
            _check_tensor(t, name, torch.int32, 1)
            if t.size(0) != b:
                raise RuntimeError(f"{name} batch mismatch")
            ptrs.append(t.data_ptr())
    ctr = None
    if merge_counters is not None:
        _check_tensor(merge_counters, "merge_counters", torch.int32, 2)
        if not (merge_counters.size(0) == b and merge_counters.size(1) == hkv):
            raise RuntimeError("merge_counters shape mismatch")
        ctr = merge_counters.data_ptr()
    _check_supported_gqa(hq, hkv)
    ws_ptr, ws_bytes = _workspace(workspace)
    lib = _native.load()
    if plan is not None:
        _check_tensor(plan, "plan", torch.int32, 1)
        _native.check(lib.pkv_paged_attention_auto_planned(
            q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
            seq_lens.data_ptr(), ptrs[0], ptrs[1], output.data_ptr(), ws_ptr, ws_bytes, ctr,
            plan.data_ptr(), plan.numel() * 4, int(groups), b, q_source.size(0), output.size(0),
            hq, hkv, d,
            physical_pages,
            k_pages.size(2), block_table.size(1), _DTYPES[q_source.dtype], _stream()))
        return
    _native.check(lib.pkv_paged_attention_auto(
        q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), ptrs[0], ptrs[1], output.data_ptr(), ws_ptr, ws_bytes, ctr, b,
        q_source.size(0), output.size(0), hq, hkv, d, physical_pages, k_pages.size(2),
        block_table.size(1), _DTYPES[q_source.dtype], _stream()))


def paged_attention_auto_state(q_source, k_pages, v_pages, block_table, seq_lens, state_out,
                               workspace, q_indices=None, merge_counters=None) -> None:
    """``paged_attention_auto`` writing each row's (m, l, acc) state to the float32
    ``state_out[B, Hq, 130]`` (one GPU's part of a sequence-sharded decode)."""
    _check_tensor(q_source, "q_source", tuple(_DTYPES), 3)
    hkv, physical_pages = _check_kv(q_source, k_pages, v_pages, k_pages.size(2))
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(seq_lens, "seq_lens", torch.int32, 1)
    _check_tensor(state_out, "state_out", torch.float32, 3)
    b = block_table.size(0)
    hq, d = q_source.size(1), q_source.size(2)
    if tuple(state_out.shape) != (b, hq, STATE_STRIDE):
        raise RuntimeError("state_out must have shape [B, Hq, 130]")
    qi = None
    if q_indices is not None:
        _check_tensor(q_indices, "q_indices", torch.int32, 1)
        qi = q_indices.data_ptr()
    ctr = None
    if merge_counters is not None:
        _check_tensor(merge_counters, "merge_counters", torch.int32, 2)
        ctr = merge_counters.data_ptr()
    _check_supported_gqa(hq, hkv)
    ws_ptr, ws_bytes = _workspace(workspace)
    _native.check(_native.load().pkv_paged_attention_auto_state(
        q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), qi, state_out.data_ptr(), ws_ptr, ws_bytes, ctr, b,
        q_source.size(0), hq, hkv, d, physical_pages, k_pages.size(2), block_table.size(1),
        _DTYPES[q_source.dtype], _stream()))


class Exchange:
    """This rank's end of the fused sharded-decode exchange (``pkv_exchange``).

    Create one per rank on its own device, gather every rank's ``handle`` (in
    rank order) and pass them to :meth:`connect`; ``world == 1`` needs no
    connect.  ``close`` synchronises the device and frees the buffer: call it
    only after every rank has synchronised its device (a barrier), since a
    peer's kernel stores into this rank's buffer.
    """

    def __init__(self, world: int, rank: int, max_batch: int, hq: int, hkv: int):
        import ctypes

        lib = _native.load()
        self._ptr = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(_native.EXCHANGE_HANDLE_BYTES)
        _native.check(lib.pkv_exchange_create(world, rank, max_batch, hq, hkv,
                                              ctypes.byref(self._ptr), buf))
        self.handle = bytes(buf.raw)
        self.world, self.rank, self.max_batch, self.hq, self.hkv = world, rank, max_batch, hq, hkv
        self.device = torch.cuda.current_device()

    def connect(self, handles) -> None:
        """``handles``: every rank's ``handle`` bytes, in rank order."""
        if len(handles) != self.world:
            raise RuntimeError("one handle per rank is required")
        blob = b"".join(bytes(h) for h in handles)
        _native.check(_native.load().pkv_exchange_connect(self._ptr, blob))

    @property
    def ptr(self):
        if not self._ptr:
            raise RuntimeError("exchange is closed")
        return self._ptr

    def close(self) -> None:
        if self._ptr:
            _native.check(_native.load().pkv_exchange_destroy(self._ptr))
            self._ptr = type(self._ptr)()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exchange_bytes(world: int, max_batch: int, hq: int, hkv: int) -> int:
    return int(_native.load().pkv_exchange_bytes(world, max_batch, hq, hkv))


def paged_attention_sharded(q_source, k_pages, v_pages, block_table, seq_lens, output, workspace,
                            merge_counters, exchange: Exchange, q_indices=None,
                            out_indices=None, plan=None, groups: int = 0) -> None:
    """One step of sequence-sharded decode with the state exchange fused into
    the kernel: ``block_table`` / ``seq_lens`` hold this rank's page range of
    every row; every rank gets the merged ``output``.  All ranks must call it
    with the same batch, in the same order.  ``plan``: a device int32 copy of
    this rank's host plan (``scheduler.build_auto_plan`` over the same rows,
    indices and ``groups``).  No counterpart in the reference."""
    _check_tensor(q_source, "q_source", tuple(_DTYPES), 3)
    hkv, physical_pages = _check_kv(q_source, k_pages, v_pages, k_pages.size(2))
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(seq_lens, "seq_lens", torch.int32, 1)
    _check_tensor(output, "output", q_source.dtype, 3)
    _check_tensor(merge_counters, "merge_counters", torch.int32, 2)
    b = block_table.size(0)
    hq, d = q_source.size(1), q_source.size(2)
    if seq_lens.size(0) != b:
        raise RuntimeError("seq_lens batch mismatch")
    if not (output.size(1) == hq and output.size(2) == d):
        raise RuntimeError("output shape must match q head dimensions")
    if not (merge_counters.size(0) == b and merge_counters.size(1) == hkv):
        raise RuntimeError("merge_counters shape mismatch")
    ptrs = []
    for name, t in (("q_indices", q_indices), ("out_indices", out_indices)):
        if t is None:
            ptrs.append(None)
        else:
            _check_tensor(t, name, torch.int32, 1)
            if t.size(0) != b:
                raise RuntimeError(f"{name} batch mismatch")
            ptrs.append(t.data_ptr())
    _check_supported_gqa(hq, hkv)
    ws_ptr, ws_bytes = _workspace(workspace)
    if plan is not None:
        _check_tensor(plan, "plan", torch.int32, 1)
        _native.check(_native.load().pkv_paged_attention_sharded_planned(
            q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
            seq_lens.data_ptr(), ptrs[0], ptrs[1], output.data_ptr(), ws_ptr, ws_bytes,
            merge_counters.data_ptr(), exchange.ptr, plan.data_ptr(), plan.numel() * 4,
            int(groups), b, q_source.size(0), output.size(0), hq, hkv, d, physical_pages,
            k_pages.size(2), block_table.size(1), _DTYPES[q_source.dtype], _stream()))
        return
    _native.check(_native.load().pkv_paged_attention_sharded(
        q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
        seq_lens.data_ptr(), ptrs[0], ptrs[1], output.data_ptr(), ws_ptr, ws_bytes,
        merge_counters.data_ptr(), exchange.ptr, b, q_source.size(0), output.size(0), hq, hkv, d,
        physical_pages, k_pages.size(2), block_table.size(1), _DTYPES[q_source.dtype],
        _stream()))


def paged_attention_auto_fp8(q_source, k_pages, v_pages, k_scale: float, v_scale: float,
                             block_table, seq_lens, output, workspace, q_indices=None,
                             out_indices=None, merge_counters=None) -> None:
    """``paged_attention_auto`` over an e4m3 (``torch.float8_e4m3fn``) K/V cache
    with per-tensor scales (K = k_scale * k_pages, V = v_scale * v_pages); q and
    output are fp16.  No counterpart in the reference."""
    _check_tensor(q_source, "q_source", torch.float16, 3)
    _check_tensor(k_pages, "k_pages", torch.float8_e4m3fn, 4)
    _check_tensor(v_pages, "v_pages", torch.float8_e4m3fn, 4)
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(seq_lens, "seq_lens", torch.int32, 1)
    _check_tensor(output, "output", torch.float16, 3)
    if tuple(v_pages.shape) != tuple(k_pages.shape) or k_pages.size(3) != HEAD_DIM:
        raise RuntimeError("k_pages / v_pages shape mismatch")
    hkv, physical_pages, page_size = k_pages.size(1), k_pages.size(0), k_pages.size(2)
    b = block_table.size(0)
    hq, d = q_source.size(1), q_source.size(2)
    if d != HEAD_DIM:
        raise RuntimeError("PersistentKV extension currently requires d=128")
    if seq_lens.size(0) != b:
        raise RuntimeError("seq_lens batch mismatch")
    if not (output.size(1) == hq and output.size(2) == d):
        raise RuntimeError("output shape must match q head dimensions")
    ptrs = []
    for name, t in (("q_indices", q_indices), ("out_indices", out_indices)):
        if t is None:
            ptrs.append(None)
        else:
            _check_tensor(t, name, torch.int32, 1)
            if t.size(0) != b:
                raise RuntimeError(f"{name} batch mismatch")
            ptrs.append(t.data_ptr())
    ctr = None
    if merge_counters is not None:
        _check_tensor(merge_counters, "merge_counters", torch.int32, 2)
        if not (merge_counters.size(0) == b and merge_counters.size(1) == hkv):
            raise RuntimeError("merge_counters shape mismatch")
        ctr = merge_counters.data_ptr()
    _check_supported_gqa(hq, hkv)
    ws_ptr, ws_bytes = _workspace(workspace)
    _native.check(_native.load().pkv_paged_attention_auto_fp8(
        q_source.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), float(k_scale),
        float(v_scale), block_table.data_ptr(), seq_lens.data_ptr(), ptrs[0], ptrs[1],
        output.data_ptr(), ws_ptr, ws_bytes, ctr, b, q_source.size(0), output.size(0), hq, hkv,
        d, physical_pages, page_size, block_table.size(1), _stream()))


def kv_append(k_new, v_new, k_pages, v_pages, block_table, positions, free_pages=None,
              free_count=None, counters=None) -> None:
    """Writes one new token per row into the paged pools (``pkv_kv_append``).

    ``k_new`` / ``v_new`` [B, Hkv, 128] (the pools' dtype) land at token
    ``positions[b]`` of row b.  With ``free_pages`` (int32 stack), ``free_count``
    (int32 [1]) and zeroed ``counters`` (int32 [1]), rows whose token opens a
    page take pages from the top of the stack in row order and record them in
    ``block_table``.  No counterpart in the reference."""
    dt = k_pages.dtype
    _check_tensor(k_new, "k_new", dt, 3)
    _check_tensor(v_new, "v_new", dt, 3)
    _check_tensor(k_pages, "k_pages", tuple(_DTYPES), 4)
    _check_tensor(v_pages, "v_pages", dt, 4)
    _check_tensor(block_table, "block_table", torch.int32, 2)
    _check_tensor(positions, "positions", torch.int32, 1)
    b, hkv, d = k_new.shape
    if tuple(v_new.shape) != (b, hkv, d) or k_pages.size(1) != hkv or d != HEAD_DIM:
        raise RuntimeError("k_new / v_new shape must be [B, Hkv, 128] matching the pools")
    if tuple(v_pages.shape) != tuple(k_pages.shape):
        raise RuntimeError("v_pages shape mismatch")
    if block_table.size(0) != b or positions.size(0) != b:
        raise RuntimeError("block_table / positions batch mismatch")
    fp = fc = ctr = None
    if free_pages is not None:
        _check_tensor(free_pages, "free_pages", torch.int32, 1)
        if free_count is None or counters is None:
            raise RuntimeError("a free-page list needs free_count and counters")
        _check_tensor(free_count, "free_count", torch.int32, 1)
        _check_tensor(counters, "counters", torch.int32, 1)
        fp, fc, ctr = free_pages.data_ptr(), free_count.data_ptr(), counters.data_ptr()
    _native.check(_native.load().pkv_kv_append(
        k_new.data_ptr(), v_new.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
        block_table.data_ptr(), positions.data_ptr(), fp, fc, ctr, b, hkv, d, k_pages.size(0),
        k_pages.size(2), block_table.size(1), _DTYPES[dt], _stream()))


def auto_workspace_bytes(batch: int, hq: int, hkv: int, sm_count: int = 0) -> int:
    """Workspace of ``paged_attention_auto`` (sm_count 0: the current device)."""
    return int(_native.load().pkv_auto_workspace_bytes(batch, hq, hkv, sm_count))


def combine_states(states, output, out_indices=None) -> None:
    """Merges ``states[n_parts, B, Hq, 130]`` into ``output`` rows (LSE combine)."""
    _check_tensor(states, "states", torch.float32, 4)
    _check_tensor(output, "output", tuple(_DTYPES), 3)
    n_parts, b, hq, width = states.shape
    if width != STATE_STRIDE:
        raise RuntimeError("states must have 130 values per head")
    if output.size(1) != hq or output.size(2) != HEAD_DIM:
        raise RuntimeError("output shape must match q head dimensions")
    idx_ptr = None
    if out_indices is not None:
        _check_tensor(out_indices, "out_indices", torch.int32, 1)
        if out_indices.size(0) != b:
            raise RuntimeError("out_indices batch mismatch")
        idx_ptr = out_indices.data_ptr()
    lib = _native.load()
    _native.check(lib.pkv_combine_states(
        states.data_ptr(), n_parts, idx_ptr, output.data_ptr(), b, output.size(0), hq,
        HEAD_DIM, _DTYPES[output.dtype], _stream()))


def workspace_bytes(batch: int, hq: int, num_splits: int) -> int:
    """Reference ``persistentkv_workspace_bytes`` (kernels/persistentkv_attention.cuh:891)."""
    return int(_native.load().pkv_workspace_bytes(batch, hq, num_splits))


def workqueue_workspace_bytes(total_partial_slots: int, hq: int) -> int:
    return int(_native.load().pkv_workqueue_workspace_bytes(total_partial_slots, hq))
