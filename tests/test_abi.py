"""The C ABI library: exports and host-side validation (no GPU, no kernel launch)."""

import ctypes
import re

import pytest
import torch

from persistentkv_attention_b200 import _native, ops
from tests.conftest import REPO, gpu_available

HEADER = REPO / "include" / "pkv_b200.h"
FAKE = 0x10000  # never dereferenced: every call below fails validation first


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pkv_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_native.SIGNATURES)


def test_status_strings(lib):
    assert lib.pkv_status_string(0) == b"PKV_OK"
    assert lib.pkv_status_string(4) == b"PKV_ERR_WORKSPACE"
    assert lib.pkv_abi_version() == 1


def test_workspace_bytes_formula(lib):
    # reference persistentkv_workspace_bytes (kernels/persistentkv_attention.cuh:891-898)
    assert lib.pkv_workspace_bytes(1, 32, 1) == 0
    assert lib.pkv_workspace_bytes(8, 32, 24) == 8 * 32 * 24 * 130 * 4
    assert lib.pkv_workqueue_workspace_bytes(100, 32) == 100 * 32 * 130 * 4


def call_paged(lib, **kw):
    args = dict(q=FAKE, k=FAKE, v=FAKE, bt=FAKE, out=FAKE, ws=FAKE, ws_bytes=1 << 30, B=1,
                Hq=32, Hkv=8, d=128, P=64, page=16, maxp=32, context=512, splits=4,
                dtype=0, stream=None)
    args.update(kw)
    return lib.pkv_paged_attention(*args.values())


@pytest.mark.parametrize("kw,status,msg", [
    (dict(d=64), 2, "requires d=128"),
    (dict(Hkv=0), 1, "Hkv must be positive"),
    (dict(Hq=30), 1, "divisible"),
    (dict(Hq=24), 2, "G=3"),
    (dict(Hq=128, Hkv=8), 2, "G=16"),
    (dict(page=12), 2, "multiple of 8"),
    (dict(page=0), 1, "page_size must be positive"),
    (dict(context=0), 1, "context must be positive"),
    (dict(splits=0), 1, "num_splits must be positive"),
    (dict(splits=17), 1, "exceeds the 16 tiles"),
    (dict(maxp=31), 1, "block_table has 31 pages"),
    (dict(ws=None), 4, "Split dispatch requires workspace"),
    (dict(ws_bytes=100), 4, "workspace holds 100 bytes"),
    (dict(k=FAKE + 8), 3, "16-byte aligned"),
    (dict(q=None), 1, "q must be a CUDA tensor"),
    (dict(dtype=7), 2, "wrong dtype"),
    (dict(P=1 << 22, Hkv=8, page=128), 2, "2^31 rows"),
])
def test_rectangular_validation(lib, kw, status, msg):
    assert call_paged(lib, **kw) == status
    assert msg in lib.pkv_last_error_message().decode()


def test_workqueue_validation(lib):
    base = [FAKE] * 12 + [1 << 30] + [1, 1, 1, 32, 8, 128, 64, 16, 32, 512, 10, 40, 0, 0, None]
    if not gpu_available():  # a valid call would launch on the fake pointers
        assert lib.pkv_paged_attention_workqueue(*base) == _native.PKV_ERR_NO_DEVICE
    bad = list(base)
    bad[23] = 0  # num_tasks
    assert lib.pkv_paged_attention_workqueue(*bad) == 1
    assert b"work_items must not be empty" in lib.pkv_last_error_message()
    bad = list(base)
    bad[24] = 0  # total_partial_slots
    assert lib.pkv_paged_attention_workqueue(*bad) == 1
    bad = list(base)
    bad[11] = None  # workspace
    assert lib.pkv_paged_attention_workqueue(*bad) == 4
    assert b"Workqueue dispatch requires workspace" in lib.pkv_last_error_message()
    bad = list(base)
    bad[12] = 10  # workspace bytes
    assert lib.pkv_paged_attention_workqueue(*bad) == 4
    bad = list(base)
    bad[7] = None  # merge_counters with fused merge
    bad[25] = 1
    assert lib.pkv_paged_attention_workqueue(*bad) == 1


@pytest.mark.skipif(gpu_available(), reason="would launch on fake pointers")
def test_valid_call_without_gpu_reports_no_device(lib):
    assert call_paged(lib) == _native.PKV_ERR_NO_DEVICE
    code = ctypes.c_uint32(0)
    assert lib.pkv_device_error(ctypes.byref(code), 0) == _native.PKV_ERR_NO_DEVICE


def test_torch_mirror_errors_match_reference_messages():
    q = torch.zeros(1, 32, 128, dtype=torch.float16)
    k = torch.zeros(4, 8, 16, 128, dtype=torch.float16)
    bt = torch.zeros(1, 4, dtype=torch.int32)
    out = torch.zeros_like(q)
    ws = torch.zeros(0)
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        ops.paged_attention(q, k, k, bt, out, ws, 64, 16, 1)
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        ops.paged_attention_masked(q, k, k, bt, bt[0], out, ws, 64, 16, 1)
    with pytest.raises(RuntimeError, match="q_source must be a CUDA tensor"):
        ops.paged_attention_indexed(q, k, k, bt, bt[0], bt[0], bt[0], out, ws, 64, 16, 1)
    with pytest.raises(RuntimeError, match="q_source must be a CUDA tensor"):
        ops.paged_attention_workqueue(q, k, k, bt, bt[0], bt, bt[0], bt, bt[0], bt[0], out, ws,
                                      64, 16, 1, False)


def test_noalloc_capacity_checked_before_any_device_call(lib):
    """The no-alloc entry point refuses a queue whose partial states exceed its
    static scratch (PKV_NOALLOC_SCRATCH_BYTES) before it touches a device."""
    limit_slots = (8 << 20) // (32 * 130 * 4)
    st = lib.pkv_paged_attention_workqueue_noalloc(
        FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 4, 4, 4, 32, 8, 128, 64, 16,
        8, 128, 16, limit_slots + 1, 0, None)
    assert st == _native.PKV_ERR_CAPACITY
    assert b"holds at most" in lib.pkv_last_error_message()


def test_gather_mode_switch(lib):
    """Both gathers are selectable at run time; unknown modes are refused."""
    prev = _native.gather_mode()
    try:
        for mode in ("tma", "cpasync"):
            _native.set_gather_mode(mode)
            assert _native.gather_mode() == mode
        assert lib.pkv_set_gather_mode(7) == _native.PKV_ERR_INVALID_ARGUMENT
    finally:
        _native.set_gather_mode(prev)


def test_math_mode_switch(lib):
    """Tensor-core and CUDA-core consumer math are selectable at run time;
    unknown modes are refused; the default is the tensor-core path."""
    prev = _native.math_mode()
    assert prev == "mma"
    try:
        for mode in ("fma", "mma"):
            _native.set_math_mode(mode)
            assert _native.math_mode() == mode
        assert lib.pkv_set_math_mode(3) == _native.PKV_ERR_INVALID_ARGUMENT
        assert b"math mode" in lib.pkv_last_error_message()
    finally:
        _native.set_math_mode(prev)


def test_dependent_launch_switch(lib):
    """Programmatic dependent launch of the device-scheduled route is off by
    default and can be switched."""
    assert not _native.dependent_launch()
    try:
        _native.set_dependent_launch(True)
        assert _native.dependent_launch()
    finally:
        _native.set_dependent_launch(False)
    assert lib.pkv_get_dependent_launch() == 0


def test_phase_stamps_only_in_the_diagnostic_build(lib):
    import os

    n = ctypes.c_int(5)
    buf = (ctypes.c_uint64 * 8)()
    st = lib.pkv_phase_stamps(buf, 1, ctypes.byref(n))
    if os.environ.get("PKV_LIB_VARIANT") == "stamps":
        assert st in (_native.PKV_OK, _native.PKV_ERR_NO_DEVICE)
    else:
        assert st == _native.PKV_ERR_UNSUPPORTED and n.value == 0


def test_no_cpu_fallback_in_product_path():
    """The engine never imports the oracle."""
    for path in (REPO / "persistentkv_attention_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path


def test_newer_entry_points_validate_before_touching_a_device(lib):
    """The entry points beyond the reference's surface reject bad arguments
    with a status and a message, before any device call."""
    P = ctypes.c_void_p
    # e4m3 cache: scales must be positive and finite
    st = lib.pkv_paged_attention_auto_fp8(FAKE, FAKE, FAKE, 0.0, 1.0, FAKE, FAKE, None, None,
                                          FAKE, FAKE, 1 << 20, None, 1, 1, 1, 32, 8, 128, 64,
                                          16, 4, None)
    assert st == 1 and b"k_scale and v_scale" in lib.pkv_last_error_message()
    st = lib.pkv_paged_attention_auto_fp8(FAKE, FAKE, FAKE, 1.0, float("inf"), FAKE, FAKE, None,
                                          None, FAKE, FAKE, 1 << 20, None, 1, 1, 1, 32, 8, 128,
                                          64, 16, 4, None)
    assert st == 1
    # KV append: missing buffers, a free list without its counters, bad head_dim
    st = lib.pkv_kv_append(None, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, None, 4, 8, 128, 64,
                           16, 8, 0, None)
    assert st == 1 and b"k_new and v_new" in lib.pkv_last_error_message()
    st = lib.pkv_kv_append(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 4, 8, 128, 64,
                           16, 8, 0, None)
    assert st == 1 and b"free_count" in lib.pkv_last_error_message()
    st = lib.pkv_kv_append(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, None, 4, 8, 64, 64,
                           16, 8, 0, None)
    assert st == 2 and b"d=128" in lib.pkv_last_error_message()
    # exchange: world beyond PKV_MAX_WORLD, rank outside the world
    out = P()
    handle = ctypes.create_string_buffer(64)
    assert lib.pkv_exchange_create(9, 0, 4, 32, 8, ctypes.byref(out), handle) == 2
    assert lib.pkv_exchange_create(2, 2, 4, 32, 8, ctypes.byref(out), handle) == 1
    assert lib.pkv_exchange_bytes(0, 4, 32, 8) == 0
    assert lib.pkv_exchange_bytes(2, 4, 32, 8) == 256 + 2 * 2 * 4 * 32 * 130 * 8
    # sharded step without an exchange
    st = lib.pkv_paged_attention_sharded(FAKE, FAKE, FAKE, FAKE, FAKE, None, None, FAKE, FAKE,
                                         1 << 20, FAKE, None, 1, 1, 1, 32, 8, 128, 64, 16, 4, 0,
                                         None)
    assert st == 1 and b"exchange" in lib.pkv_last_error_message()
    # planned sharded step: the plan is checked before anything else
    st = lib.pkv_paged_attention_sharded_planned(
        FAKE, FAKE, FAKE, FAKE, FAKE, None, None, FAKE, FAKE, 1 << 20, FAKE, FAKE, None, 0, 0,
        1, 1, 1, 32, 8, 128, 64, 16, 4, 0, None)
    assert st == 1 and b"plan" in lib.pkv_last_error_message()
    # native engine: head_dim and dtype are checked first
    eng = P()
    assert lib.pkv_engine_create(FAKE, FAKE, 64, 32, 8, 64, 16, 0, 8, 32, ctypes.byref(eng)) == 2
    assert lib.pkv_engine_create(FAKE, FAKE, 64, 32, 8, 128, 16, 7, 8, 32, ctypes.byref(eng)) == 2
    assert lib.pkv_engine_destroy(None) == 0
