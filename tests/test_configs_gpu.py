"""Parity at the benchmark's own configurations, against the CPU / float64
checkers and against the reference's CUDA path built for sm_100a.

* config 1 exactly: B=1, 4096 tokens, Hq 32 / Hkv 8, page 16, 256 logical
  pages drawn as a seeded permutation of a 1024-page pool, fp16 N(0,1), through
  every entry point of this engine and of the reference extension;
* one full mid-trace step of configs 2-5 from ``bench.py``'s own workload
  builder, every row;
* G = 1, 2, 8 in fp16 against the reference kernel (which supports them,
  kernels/persistentkv_attention.cuh:74-76);
* the reference serving harness's own call sequence
  (``run_persistentkv_step_compiled``, tests/benchmark_serving_trace.py:949-1001,
  recorded in ``tests/golden/harness_calls.json.gz``) replayed through this
  engine's ``ops`` and through the reference extension.
"""

import gzip
import json

import numpy as np
import pytest
import torch

import bench
from oracle import pkv_oracle as po
from oracle import ref as ref_artefacts
from persistentkv_attention_b200 import _native, ops
from persistentkv_attention_b200.scheduler import Router
from persistentkv_attention_b200.serving import DecodeEngine
from tests.conftest import GOLDEN
from tests.helpers import MAX_ERR, assert_close, config1_case, make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_error_word():
    _native.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    code = _native.device_error(clear=True)
    assert code == 0, _native.describe_device_error(code)


def _ext():
    ext = ref_artefacts.load_torch_ext()
    if ext is None:
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    return ext


def _agree(ours, theirs, what):
    err = (ours.float() - theirs.float()).abs().max().item()
    assert err < MAX_ERR, f"{what}: engine vs reference kernel max abs {err:.3e}"
    return err


def _ws_floats(slots, hq=32):
    return torch.zeros(max(1, slots * hq * 130), device="cuda")


def test_config1_exact_every_entry_point():
    """BASELINE config 1 as specified, through all four entry points of this
    engine and of the reference extension, each against the fp64 oracle."""
    ext = _ext()
    c = config1_case()
    d = c.cuda()
    want = c.oracle()
    assert c.block_table.shape == (1, 256) and len(set(c.block_table[0].tolist())) == 256
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    results = {}
    for impl_name, impl in (("engine", ops), ("reference", ext)):
        for splits in (1, 8, 32):
            out = torch.full((1, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
            impl.paged_attention(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                 out, _ws_floats(splits), 4096, 16, splits)
            results[(impl_name, "paged", splits)] = out
            out = torch.full_like(out, float("nan"))
            impl.paged_attention_masked(d["q_source"], d["k_pages"], d["v_pages"],
                                        d["block_table"], d["seq_lens"], out, _ws_floats(splits),
                                        4096, 16, splits)
            results[(impl_name, "masked", splits)] = out
            out = torch.full_like(out, float("nan"))
            impl.paged_attention_indexed(d["q_source"], d["k_pages"], d["v_pages"],
                                         d["block_table"], d["seq_lens"], idx, idx, out,
                                         _ws_floats(splits), 4096, 16, splits)
            results[(impl_name, "indexed", splits)] = out
        queue = Router.reference(32, 8).build_workqueue(c.seq_lens, 1, "reference")
        for fused in (False, True):
            out = torch.full((1, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
            counters = torch.zeros(1, 8, dtype=torch.int32, device="cuda")
            impl.paged_attention_workqueue(
                d["q_source"], d["k_pages"], d["v_pages"], d["block_table"], d["seq_lens"],
                torch.from_numpy(queue.work_items).cuda(),
                torch.from_numpy(queue.split_offsets).cuda(), counters, idx, idx, out,
                _ws_floats(queue.total_slots), 4096, 16, queue.total_slots, fused)
            results[(impl_name, "workqueue", fused)] = out
    out = torch.full((1, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
    ops.paged_attention_auto(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                             d["seq_lens"], out,
                             torch.empty(ops.auto_workspace_bytes(1, 32, 8) // 4, device="cuda"),
                             merge_counters=torch.zeros(1, 8, dtype=torch.int32, device="cuda"))
    results[("engine", "auto", 0)] = out
    torch.cuda.synchronize()
    for key, out in results.items():
        assert_close(out, want, "f16", f"config 1 {key}")
        if key[0] == "engine" and key[1] != "auto":
            _agree(out, results[("reference",) + key[1:]], f"config 1 {key[1:]}")


def _full_step(name, hkv, dtype):
    """A mid-trace step of a bench workload: pools, q pool and plan exactly as
    bench.py builds them."""
    w, reqs, physical, steps = bench.build_workload(name, 0, 48)
    dev = torch.device("cuda")
    k_pages, v_pages, q_pool = bench.make_inputs(w, physical, hkv, bench.DTYPES[dtype], dev, 0)
    state = steps[len(steps) // 2]
    return w, reqs, state, k_pages, v_pages, q_pool


def _checker(engine, plan, q_pool, k_pages, v_pages, state):
    f = plan.fields
    return po.torch_paged_decode(q_pool, k_pages, v_pages, f["block_table"], state.lengths,
                                 q_indices=state.active_ids).cpu().numpy()


@pytest.mark.parametrize("name,hkv,dtype", [
    ("uniform_8k", 8, "f16"), ("bimodal_32k", 8, "f16"), ("long_b1", 8, "f16"),
    ("zipf_b64", 8, "f16"), ("zipf_b64", 32, "f16"), ("zipf_b64", 4, "f16"),
    ("zipf_b64", 8, "bf16")])
def test_full_bench_step_every_row(name, hkv, dtype):
    """Every row of one step of the bench's own workload: the engine's default
    route (device schedule, fused merge) and its balanced work queue against a
    float64 checker, and (fp16) against the reference kernel's work-queue route
    with the reference scheduler's queue."""
    w, reqs, state, k_pages, v_pages, q_pool = _full_step(name, hkv, dtype)
    engine = DecodeEngine(k_pages, v_pages, 32)
    plan = engine.upload(engine.plan_from_trace(reqs, state))
    b = plan.batch
    out = torch.full((b, 32, 128), float("nan"), device="cuda", dtype=q_pool.dtype)
    engine.run(plan, q_pool, out)
    torch.cuda.synchronize()
    want = _checker(engine, plan, q_pool, k_pages, v_pages, state)
    assert_close(out, want, dtype, f"{name} hkv={hkv} device schedule")
    bal = DecodeEngine(k_pages, v_pages, 32, policy="balanced")
    bplan = bal.upload(bal.plan_from_trace(reqs, state))
    out_b = torch.full_like(out, float("nan"))
    bal.run(bplan, q_pool, out_b)
    torch.cuda.synchronize()
    assert_close(out_b, want, dtype, f"{name} hkv={hkv} balanced queue")
    if dtype != "f16":
        return
    ext = _ext()
    f = plan.fields
    queue = Router.reference(32, hkv).build_workqueue(np.asarray(state.lengths), b, "reference")
    theirs = torch.full_like(out, float("nan"))
    ext.paged_attention_workqueue(
        q_pool, k_pages, v_pages, f["block_table"], f["seq_lens"],
        torch.from_numpy(queue.work_items).cuda(), torch.from_numpy(queue.split_offsets).cuda(),
        torch.zeros(b, hkv, dtype=torch.int32, device="cuda"), f["q_indices"], f["out_indices"],
        theirs, _ws_floats(queue.total_slots), int(max(state.lengths)), 16, queue.total_slots,
        False)
    torch.cuda.synchronize()
    _agree(out, theirs, f"{name} hkv={hkv}")
    assert_close(theirs, want, "f16", f"{name} hkv={hkv} reference kernel vs checker")


@pytest.mark.parametrize("g", [1, 2, 8])
def test_reference_kernel_other_group_sizes(g):
    """G = 1, 2, 8 (fp16) against the reference's own kernels: rectangular
    masked splits and the work queue, all rows, plus both against the oracle."""
    ext = _ext()
    lens = [4096, 517, 3000, 12000, 33, 1]
    hkv = 32 // g
    c = make_case(lens, hq=32, hkv=hkv, seed=200 + g, indexed=True)
    d = c.cuda()
    want = c.oracle()
    bucket = int(c.seq_lens.max())
    b = len(lens)
    for splits in (1, 8):
        outs = []
        for impl in (ops, ext):
            out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda",
                             dtype=torch.float16)
            impl.paged_attention_indexed(d["q_source"], d["k_pages"], d["v_pages"],
                                         d["block_table"], d["seq_lens"], d["q_indices"],
                                         d["out_indices"], out, _ws_floats(b * splits), bucket,
                                         16, splits)
            outs.append(out)
        torch.cuda.synchronize()
        rows = torch.from_numpy(c.out_indices).long().cuda()
        _agree(outs[0][rows], outs[1][rows], f"G={g} indexed splits={splits}")
        assert_close(outs[0], want, "f16", f"engine G={g} splits={splits}")
        assert_close(outs[1], want, "f16", f"reference G={g} splits={splits}")
    queue = Router.reference(32, hkv).build_workqueue(c.seq_lens, b, "reference")
    outs = []
    for impl in (ops, ext):
        out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
        impl.paged_attention_workqueue(
            d["q_source"], d["k_pages"], d["v_pages"], d["block_table"], d["seq_lens"],
            torch.from_numpy(queue.work_items).cuda(), torch.from_numpy(queue.split_offsets).cuda(),
            torch.zeros(b, hkv, dtype=torch.int32, device="cuda"), d["q_indices"],
            d["out_indices"], out, _ws_floats(queue.total_slots), bucket, 16, queue.total_slots,
            False)
        outs.append(out)
    torch.cuda.synchronize()
    rows = torch.from_numpy(c.out_indices).long().cuda()
    _agree(outs[0][rows], outs[1][rows], f"G={g} workqueue")


def _decode_arg(a, roles, dev):
    if isinstance(a, dict):
        if "role" in a:
            return roles[a["role"]]
        t = torch.tensor(a["values"], dtype=getattr(torch, a["dtype"]))
        return t.view(a["shape"]).to(dev)
    return a


def test_reference_harness_call_sequence():
    """The serving-trace harness's own per-step calls (recorded from
    run_persistentkv_step_compiled on the reference's CPU side) replayed
    through this engine's ops, with the same argument lists, and through the
    reference extension: every output row agrees, and with the oracle."""
    ext = _ext()
    with gzip.open(GOLDEN / "harness_calls.json.gz", "rt") as f:
        cases = json.loads(f.read())
    dev = torch.device("cuda")
    pools = {}
    for case in cases:
        physical = case["physical_pages"]
        if physical not in pools:
            gen = torch.Generator(device=dev).manual_seed(20260622 + 7)
            pools[physical] = (
                torch.randn(physical, 8, 16, 128, generator=gen, device=dev, dtype=torch.float16),
                torch.randn(physical, 8, 16, 128, generator=gen, device=dev, dtype=torch.float16))
        k_pages, v_pages = pools[physical]
        gen = torch.Generator(device=dev).manual_seed(20260622 + 2026 + case["step"])
        q_src = torch.randn(case["requests"], 32, 128, generator=gen, device=dev,
                            dtype=torch.float16)
        outs = []
        for impl in (ops, ext):
            out = torch.full(case["output_shape"], float("nan"), device=dev, dtype=torch.float16)
            # zeroed scratch: the harness's 20-split work queue leaves the slots of
            # splits past a short row's tile count unwritten, and zeros are
            # neutral in the log-sum-exp merge of both implementations
            ws = torch.zeros(64 * 48 * 32 * 130, device=dev)
            roles = {f"q_pool[{case['step']}]": q_src, "k_pages": k_pages, "v_pages": v_pages,
                     "workspace": ws, "output": out}
            for call in case["calls"]:
                args = [_decode_arg(a, roles, dev) for a in call["args"]]
                getattr(impl, call["fn"])(*args)
            outs.append(out)
        torch.cuda.synchronize()
        what = f"{case['route']} step {case['step']}"
        _agree(outs[0], outs[1], what)
        lens = np.asarray(case["lengths"], np.int32)
        table = case["calls"][0]["args"][3]
        # checker on the step's rows (block rows of the request's pages)
        want = po.torch_paged_decode(q_src, k_pages, v_pages,
                                     _full_rows(case, k_pages.shape[0]), lens,
                                     q_indices=case["active_ids"]).cpu().numpy()
        assert table["shape"][0] >= 1
        assert_close(outs[0], want, "f16", what)


def _full_rows(case, physical):
    """Block rows of the step, rebuilt from the recorded calls (each call's
    rows go to its out_indices)."""
    b = len(case["lengths"])
    width = max(c["args"][3]["shape"][1] for c in case["calls"])
    rows = np.zeros((b, width), np.int64)
    for call in case["calls"]:
        a = call["args"]
        bt = np.asarray(a[3]["values"], np.int64).reshape(a[3]["shape"])
        out_idx = a[9 if call["fn"] == "paged_attention_workqueue" else 6]["values"]
        for r, o in enumerate(out_idx):
            rows[o, : bt.shape[1]] = bt[r]
            rows[o, bt.shape[1]:] = bt[r, -1]
    assert rows.max() < physical
    return rows
