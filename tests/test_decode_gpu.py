"""GPU parity of the four operator entry points against the CPU oracle, the
reference's golden outputs and (when built) the reference's own CUDA path."""

import numpy as np
import pytest
import torch

from oracle import pkv_oracle as po
from oracle import ref as ref_artefacts
from persistentkv_attention_b200 import _native, ops
from persistentkv_attention_b200.scheduler import Router
from tests.golden.make_golden import smoke_inputs
from tests.helpers import DT as DT_
from tests.helpers import MAX_ERR, assert_close, make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_error_word():
    _native.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    code = _native.device_error(clear=True)
    assert code == 0, _native.describe_device_error(code)


def _ws(b, hq, splits):
    return torch.empty(max(1, ops.workspace_bytes(b, hq, splits) // 4), device="cuda",
                       dtype=torch.float32) if splits > 1 else torch.empty(0, device="cuda")


def test_smoke_kat(smoke_kat):
    """The reference smoke-test cases (tests/smoke_test.cu:486-493) on the paged
    path, against the reference's own cpu_gqa_attention outputs."""
    for i, (case, q, k, v) in enumerate(smoke_inputs()):
        kind, b, hq, hkv, n, splits, page = case
        page = page or 16
        per = (n + page - 1) // page
        kp = np.zeros((b * per, hkv, page, 128), np.float32)
        vp = np.zeros_like(kp)
        table = np.zeros((b, per), np.int32)
        for bi in range(b):
            for lp in range(per):
                phys = bi * per + (per - 1 - lp)   # reversed, smoke_test.cu:239-258
                table[bi, lp] = phys
                t0, t1 = lp * page, min(n, (lp + 1) * page)
                kp[phys, :, : t1 - t0] = k[bi, :, t0:t1]
                vp[phys, :, : t1 - t0] = v[bi, :, t0:t1]
        dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
        out = torch.zeros(b, hq, 128, device="cuda", dtype=torch.float16)
        ops.paged_attention(dev(q).half(), dev(kp).half(), dev(vp).half(), dev(table), out,
                            _ws(b, hq, splits), n, page, splits)
        torch.cuda.synchronize()
        assert_close(out, smoke_kat[f"out_{i}"].astype(np.float64), "f16", str(case))


EDGE_LENS = [1, 7, 15, 16, 17, 31, 32, 33, 63, 100, 257, 513, 1000]


@pytest.mark.parametrize("g", [1, 2, 4, 8])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("page", [8, 16, 32, 64])
def test_masked_splits(g, dtype, page):
    hq = 32 if g > 1 else 8
    c = make_case(EDGE_LENS, hq=hq, hkv=hq // g, page_size=page, dtype=dtype, seed=g * 7 + page)
    d = c.cuda()
    want = c.oracle()
    bucket = int(c.seq_lens.max())
    for splits in (1, 3, 8):
        out = torch.full((len(EDGE_LENS), hq, 128), float("nan"), device="cuda",
                         dtype=d["q_source"].dtype)
        ops.paged_attention_masked(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                   d["seq_lens"], out, _ws(len(EDGE_LENS), hq, splits), bucket,
                                   page, splits)
        torch.cuda.synchronize()
        assert_close(out, want, dtype, f"splits={splits}")


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_unmasked_context(dtype):
    c = make_case([700, 700, 700], dtype=dtype, seed=5, extra_pages=3)
    d = c.cuda()
    want = c.oracle(seq_lens=False, context=700)
    for splits in (1, 2, 22):
        out = torch.empty(3, 32, 128, device="cuda", dtype=d["q_source"].dtype)
        ops.paged_attention(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"], out,
                            _ws(3, 32, splits), 700, 16, splits)
        torch.cuda.synchronize()
        assert_close(out, want, dtype, f"splits={splits}")


def test_indexed_rows():
    c = make_case([40, 5000, 1, 333, 2048], seed=9, indexed=True)
    d = c.cuda()
    want = c.oracle()
    out = torch.full((c.out_rows, 32, 128), 7.0, device="cuda", dtype=torch.float16)
    ops.paged_attention_indexed(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                d["seq_lens"], d["q_indices"], d["out_indices"], out,
                                _ws(5, 32, 4), 5000, 16, 4)
    torch.cuda.synchronize()
    assert_close(out, want, "f16")
    untouched = sorted(set(range(c.out_rows)) - set(c.out_indices.tolist()))
    assert (out[untouched] == 7.0).all()          # rows nobody writes stay as they were


def _run_workqueue(c, d, queue, fused, dtype):
    items = torch.from_numpy(queue.work_items).cuda()
    offsets = torch.from_numpy(queue.split_offsets).cuda()
    counters = torch.zeros(len(c.seq_lens), c.hkv, device="cuda", dtype=torch.int32)
    ws = torch.empty(ops.workqueue_workspace_bytes(queue.total_slots, c.hq) // 4, device="cuda")
    out = torch.full((c.out_rows, c.hq, 128), float("nan"), device="cuda",
                     dtype=d["q_source"].dtype)
    ops.paged_attention_workqueue(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                  d["seq_lens"], items, offsets, counters, d["q_indices"],
                                  d["out_indices"], out, ws, int(c.seq_lens.max()), c.page_size,
                                  queue.total_slots, fused)
    torch.cuda.synchronize()
    assert (counters == 0).all(), "fused merge must leave the counters at zero"
    return out


@pytest.mark.parametrize("policy", ["reference", "balanced"])
@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("g,dtype", [(4, "f16"), (1, "f16"), (8, "bf16"), (2, "bf16")])
def test_workqueue(policy, fused, g, dtype):
    lens = [4096, 517, 1, 0, 12000, 64, 2500, 8191]
    c = make_case(lens, hq=32, hkv=32 // g, dtype=dtype, seed=3 + g, indexed=True)
    d = c.cuda()
    want = c.oracle()
    router = Router.reference(32, c.hkv) if policy == "reference" else Router.b200(32, c.hkv)
    queue = router.build_workqueue(c.seq_lens, len(lens), policy)
    out = _run_workqueue(c, d, queue, fused, dtype)
    assert_close(out, want, dtype, f"{policy} fused={fused}")


def test_state_shards_combine():
    """Sequence sharding: per-shard (m, l, acc) states merge to the full answer."""
    lens = [9000, 33, 4000]
    c = make_case(lens, seed=21)
    want = c.oracle()
    d = c.cuda()
    router = Router.b200(32, 8)
    states = []
    cut_pages = [int(np.ceil(n / 16) * 0.4) for n in lens]
    for shard in range(2):
        tables, sl = [], []
        for b, n in enumerate(lens):
            cut = cut_pages[b]
            row = c.block_table[b]
            if shard == 0:
                tables.append(row[:cut]), sl.append(min(n, cut * 16))
            else:
                tables.append(row[cut:]), sl.append(max(0, n - cut * 16))
        width = max(len(t) for t in tables) or 1
        bt = np.stack([np.pad(t, (0, width - len(t)), mode="edge") if len(t) else
                       np.zeros(width, np.int32) for t in tables]).astype(np.int32)
        queue = router.build_workqueue(sl)
        st = torch.empty(len(lens), 32, 130, device="cuda")
        ws = torch.empty(ops.workqueue_workspace_bytes(queue.total_slots, 32) // 4, device="cuda")
        counters = torch.zeros(len(lens), 8, device="cuda", dtype=torch.int32)
        ops.paged_attention_workqueue_state(
            d["q_source"], d["k_pages"], d["v_pages"], torch.from_numpy(bt).cuda(),
            torch.tensor(sl, dtype=torch.int32, device="cuda"),
            torch.from_numpy(queue.work_items).cuda(), torch.from_numpy(queue.split_offsets).cuda(),
            counters, d["q_indices"], st, ws, 16, queue.total_slots, shard == 1)
        states.append(st)
    out = torch.empty(len(lens), 32, 128, device="cuda", dtype=torch.float16)
    ops.combine_states(torch.stack(states), out)
    torch.cuda.synchronize()
    assert_close(out, want, "f16")


def test_cuda_graph_replay():
    c = make_case([3000, 800, 5000, 16], seed=31)
    d = c.cuda()
    queue = Router.b200(32, 8).build_workqueue(c.seq_lens)
    items = torch.from_numpy(queue.work_items).cuda()
    offsets = torch.from_numpy(queue.split_offsets).cuda()
    counters = torch.zeros(4, 8, device="cuda", dtype=torch.int32)
    ws = torch.empty(ops.workqueue_workspace_bytes(queue.total_slots, 32) // 4, device="cuda")
    out = torch.zeros(4, 32, 128, device="cuda", dtype=torch.float16)

    def step():
        ops.paged_attention_workqueue(d["q_source"], d["k_pages"], d["v_pages"],
                                      d["block_table"], d["seq_lens"], items, offsets, counters,
                                      d["q_indices"], d["out_indices"], out, ws, 5000, 16,
                                      queue.total_slots, True)

    step()
    torch.cuda.synchronize()
    first = out.clone()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            step()
    out.zero_()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert_close(out, c.oracle(), "f16")


def test_full_size_properties():
    """A BASELINE-size row (config 4: 32k tokens): equal results for every split
    plan, exact invariance under relabelling of physical pages, and agreement
    with the oracle."""
    n = 32768
    c = make_case([n], seed=77, holes=0.1)
    d = c.cuda()
    results = []
    for splits in (1, 37, 128):
        out = torch.empty(1, 32, 128, device="cuda", dtype=torch.float16)
        ops.paged_attention_masked(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                   d["seq_lens"], out, _ws(1, 32, splits), n, 16, splits)
        results.append(out)
    torch.cuda.synchronize()
    for r in results[1:]:
        assert (r.float() - results[0].float()).abs().max().item() < MAX_ERR
    # relabel physical pages: same answer, bit for bit
    perm = torch.randperm(c.k_pages.shape[0], generator=torch.Generator().manual_seed(1))
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel())
    kp2 = d["k_pages"][perm.cuda()].contiguous()
    vp2 = d["v_pages"][perm.cuda()].contiguous()
    bt2 = inv.cuda()[d["block_table"].long()].to(torch.int32)
    out2 = torch.empty(1, 32, 128, device="cuda", dtype=torch.float16)
    ops.paged_attention_masked(d["q_source"], kp2, vp2, bt2, d["seq_lens"], out2,
                               _ws(1, 32, 37), n, 16, 37)
    torch.cuda.synchronize()
    assert torch.equal(out2, results[1])
    assert_close(results[1], c.oracle(), "f16")


def test_device_errors_are_flagged_not_faults():
    """Out-of-range page ids / lengths are skipped in-kernel and reported."""
    c = make_case([300, 200], seed=41)
    d = c.cuda()
    bt = d["block_table"].clone()
    bt[0, 3] = c.k_pages.shape[0] + 5
    bt[1, 0] = -3
    out = torch.empty(2, 32, 128, device="cuda", dtype=torch.float16)
    ops.paged_attention_masked(d["q_source"], d["k_pages"], d["v_pages"], bt, d["seq_lens"], out,
                               _ws(2, 32, 2), 300, 16, 2)
    torch.cuda.synchronize()
    code = _native.device_error(clear=True)
    assert code & 0x1
    sl = d["seq_lens"].clone()
    sl[1] = 10 ** 6
    ops.paged_attention_masked(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"], sl,
                               out, _ws(2, 32, 2), 300, 16, 2)
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) & 0x2


def _ref_ext():
    ext = ref_artefacts.load_torch_ext()
    if ext is None:
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    return ext


def test_reference_cuda_path_rectangular():
    """Same inputs through the reference's own kernels built for sm_100a."""
    ext = _ref_ext()
    c = make_case([4096, 4096], seed=51, indexed=True)
    d = c.cuda()
    for splits in (1, 16):
        ours = torch.zeros(c.out_rows, 32, 128, device="cuda", dtype=torch.float16)
        theirs = torch.zeros_like(ours)
        ws = torch.empty(2 * 32 * 16 * 130, device="cuda")
        ops.paged_attention_indexed(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                    d["seq_lens"], d["q_indices"], d["out_indices"], ours, ws,
                                    4096, 16, splits)
        ext.paged_attention_indexed(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                    d["seq_lens"], d["q_indices"], d["out_indices"], theirs, ws,
                                    4096, 16, splits)
        torch.cuda.synchronize()
        assert (ours.float() - theirs.float()).abs().max().item() < MAX_ERR


def test_reference_cuda_path_workqueue():
    ext = _ref_ext()
    lens = [7000, 650, 3000, 1500, 20000, 800, 4100, 900]
    c = make_case(lens, seed=52, indexed=True)
    d = c.cuda()
    queue = Router.reference(32, 8).build_workqueue(c.seq_lens, len(lens), "reference")
    ours = _run_workqueue(c, d, queue, True, "f16")
    items = torch.from_numpy(queue.work_items).cuda()
    offsets = torch.from_numpy(queue.split_offsets).cuda()
    counters = torch.zeros(len(lens), 8, device="cuda", dtype=torch.int32)
    ws = torch.zeros(queue.total_slots * 32 * 130, device="cuda")
    theirs = torch.full_like(ours, float("nan"))
    ext.paged_attention_workqueue(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                  d["seq_lens"], items, offsets, counters, d["q_indices"],
                                  d["out_indices"], theirs, ws, 20000, 16, queue.total_slots,
                                  False)
    torch.cuda.synchronize()
    rows = torch.from_numpy(c.out_indices).long().cuda()
    assert (ours[rows].float() - theirs[rows].float()).abs().max().item() < MAX_ERR
    assert_close(theirs, c.oracle(), "f16", "reference kernel vs oracle")


def _run_auto(c, d, fused):
    ws = torch.empty(ops.auto_workspace_bytes(len(c.seq_lens), c.hq, c.hkv) // 4, device="cuda")
    out = torch.full((c.out_rows, c.hq, 128), float("nan"), device="cuda",
                     dtype=d["q_source"].dtype)
    counters = torch.zeros(len(c.seq_lens), c.hkv, device="cuda", dtype=torch.int32)
    ops.paged_attention_auto(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                             d["seq_lens"], out, ws, d["q_indices"], d["out_indices"],
                             counters if fused else None)
    torch.cuda.synchronize()
    assert (counters == 0).all()
    return out


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("g,dtype,page", [(4, "f16", 16), (1, "f16", 8), (8, "bf16", 32),
                                          (2, "bf16", 16), (4, "bf16", 64)])
def test_auto_route(fused, g, dtype, page):
    """Device-side schedule: equal-token groups, no work queue."""
    lens = [0] + EDGE_LENS + [9000, 4096]
    c = make_case(lens, hq=32, hkv=32 // g, page_size=page, dtype=dtype, seed=60 + g,
                  indexed=True)
    out = _run_auto(c, c.cuda(), fused)
    assert_close(out, c.oracle(), dtype, f"auto fused={fused}")


@pytest.mark.parametrize("fused", [False, True])
def test_auto_route_many_rows(fused):
    rng = np.random.default_rng(8)
    lens = np.minimum(32768, np.maximum(1, (256 * rng.zipf(1.1, 200)))).tolist()
    lens[5] = 0
    c = make_case(lens, seed=61, holes=0.1)
    out = _run_auto(c, c.cuda(), fused)
    assert_close(out, c.oracle(), "f16", f"200 rows fused={fused}")


def test_auto_route_all_rows_empty_and_graph():
    c = make_case([0, 0, 0], seed=62)
    out = _run_auto(c, c.cuda(), True)
    assert (out.float() == 0).all()
    c = make_case([5000, 100, 3000], seed=63)
    d = c.cuda()
    ws = torch.empty(ops.auto_workspace_bytes(3, 32, 8) // 4, device="cuda")
    out = torch.zeros(3, 32, 128, device="cuda", dtype=torch.float16)
    counters = torch.zeros(3, 8, device="cuda", dtype=torch.int32)

    def step():
        ops.paged_attention_auto(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                 d["seq_lens"], out, ws, None, None, counters)

    step()
    torch.cuda.synchronize()
    first = out.clone()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            step()
    out.zero_()
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert_close(out, c.oracle(), "f16")


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("world", [2, 3, 5])
def test_auto_state_sequence_shards(fused, world):
    """Sequence sharding on the device-side schedule: each shard's (m, l, acc)
    state from paged_attention_auto_state, merged by combine_states.  With 5
    shards the 33-token row (3 pages) leaves two shards empty."""
    from persistentkv_attention_b200 import dist as pdist

    lens = [30000, 33, 4000, 0, 777]
    c = make_case(lens, seed=64 + world, indexed=True)
    d = c.cuda()
    b = len(lens)
    states = []
    for rank in range(world):
        bt, sl = pdist.shard_rows(c.block_table, c.seq_lens, 16, world, rank)
        st = torch.full((b, 32, 130), float("nan"), device="cuda")
        ws = torch.empty(ops.auto_workspace_bytes(b, 32, 8) // 4, device="cuda")
        counters = torch.zeros(b, 8, device="cuda", dtype=torch.int32)
        ops.paged_attention_auto_state(d["q_source"], d["k_pages"], d["v_pages"],
                                       torch.from_numpy(bt).cuda(),
                                       torch.from_numpy(sl).cuda(), st, ws, d["q_indices"],
                                       counters if fused else None)
        torch.cuda.synchronize()
        assert not torch.isnan(st).any()
        assert (counters == 0).all()
        states.append(st)
    out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
    ops.combine_states(torch.stack(states), out, d["out_indices"])
    torch.cuda.synchronize()
    assert_close(out, c.oracle(), "f16", f"auto state x{world} fused={fused}")


def test_sharded_fused_exchange_single_rank():
    """The fused-exchange step with world 1: every CTA flags and merges its
    own part; several launches (eager and graph-replayed) advance the step
    number and alternate the gather-buffer parity."""
    from persistentkv_attention_b200 import dist as pdist

    x = ops.Exchange(1, 0, 8, 32, 8)
    try:
        cases = [make_case(lens, seed=70 + i, indexed=True)
                 for i, lens in enumerate([[30000, 33, 0, 777], [5000], [1, 2, 3, 4, 5, 6, 7, 9000]])]
        for c in cases:
            d = c.cuda()
            b = len(c.seq_lens)
            bt, sl = pdist.shard_rows(c.block_table, c.seq_lens, 16, 1, 0)
            ws = torch.empty(ops.auto_workspace_bytes(b, 32, 8) // 4, device="cuda")
            counters = torch.zeros(b, 8, device="cuda", dtype=torch.int32)
            out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda",
                             dtype=torch.float16)
            bt_d, sl_d = torch.from_numpy(bt).cuda(), torch.from_numpy(sl).cuda()

            def step():
                ops.paged_attention_sharded(d["q_source"], d["k_pages"], d["v_pages"], bt_d, sl_d,
                                            out, ws, counters, x, d["q_indices"],
                                            d["out_indices"])

            for _ in range(3):
                step()
            torch.cuda.synchronize()
            assert (counters == 0).all()
            assert_close(out, c.oracle(), "f16", f"sharded x1 B{b}")
            # with this rank's host plan: the same schedule, the same bits
            from persistentkv_attention_b200.scheduler import build_auto_plan

            sms = torch.cuda.get_device_properties(0).multi_processor_count
            plan = torch.from_numpy(build_auto_plan(sl, bt, bt.shape[1], 16, 8, sms,
                                                    q_indices=c.q_indices,
                                                    out_indices=c.out_indices)).cuda()
            planned = torch.full_like(out, float("nan"))
            ops.paged_attention_sharded(d["q_source"], d["k_pages"], d["v_pages"], bt_d, sl_d,
                                        planned, ws, counters, x, d["q_indices"],
                                        d["out_indices"], plan=plan)
            torch.cuda.synchronize()
            assert (counters == 0).all()
            assert _native.device_error(clear=True) == 0
            rows = torch.from_numpy(c.out_indices).long().cuda()
            assert torch.equal(planned[rows], out[rows])
            graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                with torch.cuda.graph(graph, stream=s):
                    step()
            first = out.clone()
            out.fill_(float("nan"))
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out[torch.from_numpy(c.out_indices).long().cuda()],
                               first[torch.from_numpy(c.out_indices).long().cuda()])
        # a batch beyond the exchange's capacity is refused before launch
        c = make_case([100] * 9, seed=79)
        d = c.cuda()
        with pytest.raises(_native.PkvError) as err:
            ops.paged_attention_sharded(
                d["q_source"], d["k_pages"], d["v_pages"], d["block_table"], d["seq_lens"],
                torch.empty(9, 32, 128, device="cuda", dtype=torch.float16),
                torch.empty(ops.auto_workspace_bytes(9, 32, 8) // 4, device="cuda"),
                torch.zeros(9, 8, device="cuda", dtype=torch.int32), x)
        assert err.value.status == _native.PKV_ERR_CAPACITY
    finally:
        torch.cuda.synchronize()
        x.close()
    # Many short rows: CTAs whose group holds many rows exchange one row
    # after another within the launch.
    x = ops.Exchange(1, 0, 32, 32, 8)
    try:
        lens = [1 + i for i in range(20)] + [3000, 5, 7, 9000]
        c = make_case(lens, seed=81, indexed=True)
        d = c.cuda()
        b = len(lens)
        bt, sl = pdist.shard_rows(c.block_table, c.seq_lens, 16, 1, 0)
        out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
        counters = torch.zeros(b, 8, device="cuda", dtype=torch.int32)
        for _ in range(2):
            ops.paged_attention_sharded(
                d["q_source"], d["k_pages"], d["v_pages"], torch.from_numpy(bt).cuda(),
                torch.from_numpy(sl).cuda(), out,
                torch.empty(ops.auto_workspace_bytes(b, 32, 8) // 4, device="cuda"), counters, x,
                d["q_indices"], d["out_indices"])
        torch.cuda.synchronize()
        assert (counters == 0).all()
        assert _native.device_error(clear=True) == 0
        assert_close(out, c.oracle(), "f16", "sharded x1, many rows")
    finally:
        torch.cuda.synchronize()
        x.close()


def test_native_host_step():
    """pkv_engine_step_host: host lengths / block rows / pinned q in, pinned
    output out, one native call per step; batches grow the engine."""
    from persistentkv_attention_b200.serving import DecodeEngine

    c = make_case([7000, 1, 333, 4096, 0, 12000], seed=81)
    d = c.cuda()
    engine = DecodeEngine(d["k_pages"], d["v_pages"], 32)
    want = c.oracle()
    scratch = {}
    q_host = c.q_source.clone().pin_memory()
    out_host = torch.full((6, 32, 128), float("nan"), dtype=torch.float16).pin_memory()
    for b in (2, 6, 3, 6):
        out_host.fill_(float("nan"))
        h2d, d2h = engine.step_host(c.seq_lens[:b], c.block_table[:b], q_host, out_host, scratch)
        torch.cuda.current_stream().synchronize()
        nat = scratch["native"]
        # staged metadata: lengths (padded to 16 bytes), the host plan of the
        # schedule (padded to 16 bytes), then b rows of the engine's width
        from persistentkv_attention_b200.scheduler import plan_words
        pw = -(-plan_words(8, torch.cuda.get_device_properties(0).multi_processor_count) // 4) * 4
        meta = (-(-nat.max_batch // 4) * 4 + pw + b * nat.max_pages) * 4
        assert h2d == meta + b * 32 * 128 * 2
        assert d2h == b * 32 * 128 * 2
        assert_close(out_host[:b], want[:b], "f16", f"native step B{b}")
    # a side stream: the engine captures its two launches and replays them;
    # alternating q buffers re-point the captured stage-in
    s = torch.cuda.Stream()
    q_other = c.q_source.clone().pin_memory()
    with torch.cuda.stream(s):
        for rep in range(4):
            for b in (6, 3):
                out_host.fill_(float("nan"))
                qh = q_host if rep % 2 == 0 else q_other
                engine.step_host(c.seq_lens[:b], c.block_table[:b], qh, out_host, scratch)
                s.synchronize()
                assert_close(out_host[:b], want[:b], "f16", f"graph-replayed native step B{b}")
    scratch["native"].close()


def test_step_graph_reused_across_steps():
    """StepGraph: one captured graph (metadata upload + device-scheduled decode)
    replayed for steps of different batch sizes and lengths."""
    from persistentkv_attention_b200.serving import DecodeEngine, StepGraph

    c = make_case([9000, 33, 4096, 1, 700, 12000, 0, 2500], seed=91, indexed=True)
    d = c.cuda()
    engine = DecodeEngine(d["k_pages"], d["v_pages"], 32)
    sg = StepGraph(engine, max_batch=8, max_pages=c.block_table.shape[1], q_rows=c.out_rows,
                   out_rows=c.out_rows)
    sg.q.copy_(d["q_source"])
    kf, vf, qf = (t.float().numpy() for t in (c.k_pages, c.v_pages, c.q_source))
    steps = [[0, 1, 2], [3, 4, 5, 6, 7], list(range(8)), [5]]
    for n, rows in enumerate(steps):
        lens = c.seq_lens[rows] // (1 + n % 2)
        width = max(1, int(np.ceil(lens.max(initial=1) / 16)))
        table = c.block_table[rows][:, :width]
        qi, oi = c.q_indices[rows], c.out_indices[rows]
        sg.out.fill_(float("nan"))
        sg.step(lens, table, qi, oi)
        sg.stream.synchronize()
        want = po.paged_decode(qf, kf, vf, table, seq_lens=lens, q_indices=qi, out_indices=oi,
                               out_rows=c.out_rows)
        assert_close(sg.out, want, "f16", f"graph step {n}")
    assert len(sg._graphs) == 2


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_kv_append_matches_oracle(dtype):
    """KV append, bit-exact against the CPU restatement: rows that open a page
    take pages from the free list in row order; the others write into pages
    already mapped; then a decode over the appended tokens matches the oracle."""
    gen = torch.Generator().manual_seed(95)
    P, hkv, page, mp = 64, 8, 16, 8
    k_pages = torch.randn(P, hkv, page, 128, generator=gen).to(DT_[dtype])
    v_pages = torch.randn(P, hkv, page, 128, generator=gen).to(DT_[dtype])
    B = 6
    table = np.full((B, mp), 0, np.int32)
    table[:, 0] = np.arange(B)            # every row owns one page already
    table[:, 1] = np.arange(B) + 10
    positions = np.array([16, 5, 32, 31, 0, 17], np.int32)   # rows 0, 2, 4 open a page
    table[4, 0] = 0                       # row 4 opens page slot 0 (will be overwritten)
    free = np.array([40, 41, 42, 43, 44], np.int32)
    k_new = torch.randn(B, hkv, 128, generator=gen).to(DT_[dtype])
    v_new = torch.randn(B, hkv, 128, generator=gen).to(DT_[dtype])
    # oracle on copies (bit patterns carried through float32 views of 16-bit values)
    kp_o, vp_o = k_pages.clone(), v_pages.clone()
    tab_o = table.copy()
    cnt_o, err_o = po.kv_append(k_new.numpy() if dtype == "f16" else k_new.view(torch.int16).numpy(),
                                v_new.numpy() if dtype == "f16" else v_new.view(torch.int16).numpy(),
                                kp_o.numpy() if dtype == "f16" else kp_o.view(torch.int16).numpy(),
                                vp_o.numpy() if dtype == "f16" else vp_o.view(torch.int16).numpy(),
                                tab_o, positions, free, 4)
    dk, dv = k_pages.cuda(), v_pages.cuda()
    dtab = torch.from_numpy(table).cuda()
    fc = torch.tensor([4], dtype=torch.int32, device="cuda")
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.kv_append(k_new.cuda(), v_new.cuda(), dk, dv, dtab, torch.from_numpy(positions).cuda(),
                  torch.from_numpy(free).cuda(), fc, ctr)
    torch.cuda.synchronize()
    assert err_o == 0 and cnt_o == 1
    assert int(fc.item()) == cnt_o and int(ctr.item()) == 0
    assert np.array_equal(dtab.cpu().numpy(), tab_o)
    assert torch.equal(dk.cpu(), kp_o) and torch.equal(dv.cpu(), vp_o)
    # the appended tokens are attended to by the decode
    lens = positions + 1
    q = torch.randn(B, 32, 128, generator=gen).to(DT_[dtype])
    out = torch.empty(B, 32, 128, dtype=DT_[dtype], device="cuda")
    ws = torch.empty(ops.auto_workspace_bytes(B, 32, hkv) // 4, device="cuda")
    ops.paged_attention_auto(q.cuda(), dk, dv, dtab, torch.from_numpy(lens).cuda(), out, ws,
                             merge_counters=torch.zeros(B, hkv, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    want = po.paged_decode(q.float().numpy(), kp_o.float().numpy(), vp_o.float().numpy(), tab_o,
                           seq_lens=lens)
    assert_close(out, want, dtype, "decode after append")


def test_kv_append_errors_are_flagged():
    """List exhausted, position beyond the table, page outside the pool: the
    rows write nothing and set their device error bits; no fault."""
    P, hkv, page, mp = 8, 2, 16, 2
    dk = torch.zeros(P, hkv, page, 128, dtype=torch.float16, device="cuda")
    dv = torch.zeros_like(dk)
    tab = torch.tensor([[1, 0], [99, 0], [2, 0], [3, 0]], dtype=torch.int32, device="cuda")
    pos = torch.tensor([16, 3, 64, 32], dtype=torch.int32, device="cuda")   # 16 opens, 64 is past
    k_new = torch.ones(4, hkv, 128, dtype=torch.float16, device="cuda")
    free = torch.tensor([5], dtype=torch.int32, device="cuda")
    fc = torch.tensor([0], dtype=torch.int32, device="cuda")               # empty list
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.kv_append(k_new, k_new, dk, dv, tab, pos, free, fc, ctr)
    torch.cuda.synchronize()
    code = _native.device_error(clear=True)
    assert code & 0x80 and code & 0x2 and code & 0x1
    assert float(dk.abs().sum()) == 0.0
    assert int(fc.item()) == 0 and int(ctr.item()) == 0


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("g,page", [(4, 16), (1, 16), (8, 16), (4, 8)])
def test_auto_route_fp8_kv(fused, g, page):
    """e4m3 K/V cache with per-tensor scales against the oracle on the
    dequantized values (every e4m3 value is exact in fp16 and fp64)."""
    lens = [0] + EDGE_LENS + [9000, 4096, 20000]
    c = make_case(lens, hq=32, hkv=32 // g, page_size=page, seed=120 + g + page, indexed=True)
    kf, vf = c.k_pages.float(), c.v_pages.float()
    k_scale = float(kf.abs().max()) / 448.0
    v_scale = float(vf.abs().max()) / 448.0
    k8 = (kf / k_scale).to(torch.float8_e4m3fn)
    v8 = (vf / v_scale).to(torch.float8_e4m3fn)
    kd = k8.float().numpy() * k_scale
    vd = v8.float().numpy() * v_scale
    want = po.paged_decode(c.q_source.float().numpy(), kd, vd, c.block_table,
                           seq_lens=c.seq_lens, q_indices=c.q_indices,
                           out_indices=c.out_indices, out_rows=c.out_rows)
    d = c.cuda()
    b = len(lens)
    out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
    ws = torch.empty(ops.auto_workspace_bytes(b, 32, c.hkv) // 4, device="cuda")
    counters = torch.zeros(b, c.hkv, device="cuda", dtype=torch.int32)
    ops.paged_attention_auto_fp8(d["q_source"], k8.cuda(), v8.cuda(), k_scale, v_scale,
                                 d["block_table"], d["seq_lens"], out, ws, d["q_indices"],
                                 d["out_indices"], counters if fused else None)
    torch.cuda.synchronize()
    assert_close(out, want, "f16", f"fp8 kv G{g} page{page} fused={fused}")


@pytest.mark.parametrize("g,dtype,page", [(4, "f16", 16), (1, "bf16", 8), (8, "f16", 32),
                                          (2, "bf16", 16)])
def test_gather_modes_bit_identical(g, dtype, page):
    """The TMA (cp.async.bulk.tensor) and the 16-byte cp.async gathers feed
    the same math: every route gives bit-identical outputs under both, and
    both match the oracle."""
    lens = [0] + EDGE_LENS + [9000, 4096]
    c = make_case(lens, hq=32, hkv=32 // g, page_size=page, dtype=dtype, seed=300 + g,
                  indexed=True)
    d = c.cuda()
    want = c.oracle()
    prev = _native.gather_mode()
    results = {}
    try:
        for mode in ("cpasync", "tma"):
            _native.set_gather_mode(mode)
            results[(mode, "auto")] = _run_auto(c, d, True)
            queue = Router.b200(32, c.hkv).build_workqueue(c.seq_lens)
            results[(mode, "queue")] = _run_workqueue(c, d, queue, False, dtype)
            out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda",
                             dtype=d["q_source"].dtype)
            ops.paged_attention_indexed(d["q_source"], d["k_pages"], d["v_pages"],
                                        d["block_table"], d["seq_lens"], d["q_indices"],
                                        d["out_indices"], out, _ws(c.out_rows, 32, 3),
                                        int(c.seq_lens.max()), page, 3)
            torch.cuda.synchronize()
            results[(mode, "indexed")] = out
    finally:
        _native.set_gather_mode(prev)
    rows = torch.from_numpy(c.out_indices).long().cuda()
    for route in ("auto", "queue", "indexed"):
        a, b = results[("cpasync", route)][rows], results[("tma", route)][rows]
        assert torch.equal(a, b), f"{route}: gathers differ"
        assert_close(results[("tma", route)], want, dtype, f"tma {route}")


@pytest.mark.parametrize("g,dtype,page", [(4, "f16", 16), (1, "f16", 8), (8, "bf16", 32),
                                          (2, "bf16", 16)])
def test_planned_schedule_bit_identical(g, dtype, page):
    """A host plan of the device schedule (pkv_paged_attention_auto_planned)
    gives the same bits as the schedule the kernel derives itself, and a plan
    of another batch shape is detected, ignored and flagged."""
    from persistentkv_attention_b200.scheduler import build_auto_plan

    lens = [0] + EDGE_LENS + [9000, 4096]
    c = make_case(lens, hq=32, hkv=32 // g, page_size=page, dtype=dtype, seed=400 + g,
                  indexed=True)
    d = c.cuda()
    want = c.oracle()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    plan = torch.from_numpy(build_auto_plan(c.seq_lens, c.block_table, c.block_table.shape[1],
                                            page, c.hkv, sms, q_indices=c.q_indices,
                                            out_indices=c.out_indices)).cuda()
    outs = []
    for pl in (None, plan):
        for fused in (True, False):
            ws = torch.empty(ops.auto_workspace_bytes(len(lens), 32, c.hkv) // 4, device="cuda")
            out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda",
                             dtype=d["q_source"].dtype)
            ctr = torch.zeros(len(lens), c.hkv, device="cuda", dtype=torch.int32)
            ops.paged_attention_auto(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                     d["seq_lens"], out, ws, d["q_indices"], d["out_indices"],
                                     ctr if fused else None, plan=pl)
            torch.cuda.synchronize()
            assert (ctr == 0).all()
            outs.append(out)
    rows = torch.from_numpy(c.out_indices).long().cuda()
    # same merge (fused: 0, 2; separate kernel: 1, 3), planned or derived schedule
    assert torch.equal(outs[2][rows], outs[0][rows]), "planned and derived schedules differ"
    assert torch.equal(outs[3][rows], outs[1][rows]), "planned and derived schedules differ"
    assert_close(outs[2], want, dtype, "planned")
    assert_close(outs[3], want, dtype, "planned, separate merge")
    # a plan built for one row fewer: ignored (the kernel derives its schedule) and flagged
    bad = torch.from_numpy(build_auto_plan(c.seq_lens[:-1], c.block_table[:-1],
                                           c.block_table.shape[1], page, c.hkv, sms)).cuda()
    ws = torch.empty(ops.auto_workspace_bytes(len(lens), 32, c.hkv) // 4, device="cuda")
    out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda", dtype=d["q_source"].dtype)
    ops.paged_attention_auto(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                             d["seq_lens"], out, ws, d["q_indices"], d["out_indices"],
                             torch.zeros(len(lens), c.hkv, device="cuda", dtype=torch.int32),
                             plan=bad)
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) & 0x4
    assert torch.equal(out[rows], outs[0][rows])


@pytest.mark.parametrize("groups", [1, 6, 18, 36])
def test_planned_fewer_groups(groups):
    """A plan for fewer groups than the maximum (a router's choice): a grid of
    groups x Hkv CTAs, same result as the oracle; the engine's router route."""
    from persistentkv_attention_b200.scheduler import build_auto_plan
    from persistentkv_attention_b200.serving import DecodeEngine

    lens = [0, 33, 9000, 4096, 700, 12000, 1]
    c = make_case(lens, seed=500 + groups, indexed=True)
    d = c.cuda()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    plan = torch.from_numpy(build_auto_plan(c.seq_lens, c.block_table, c.block_table.shape[1],
                                            16, 8, sms, q_indices=c.q_indices,
                                            out_indices=c.out_indices, groups=groups)).cuda()
    for fused in (True, False):
        ws = torch.empty(ops.auto_workspace_bytes(len(lens), 32, 8) // 4, device="cuda")
        out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda", dtype=torch.float16)
        ctr = torch.zeros(len(lens), 8, device="cuda", dtype=torch.int32)
        ops.paged_attention_auto(d["q_source"], d["k_pages"], d["v_pages"], d["block_table"],
                                 d["seq_lens"], out, ws, d["q_indices"], d["out_indices"],
                                 ctr if fused else None, plan=plan, groups=groups)
        torch.cuda.synchronize()
        assert (ctr == 0).all()
        assert_close(out, c.oracle(), "f16", f"groups={groups} fused={fused}")
    engine = DecodeEngine(d["k_pages"], d["v_pages"], 32, groups="router")
    step = engine.upload(engine.plan_step(c.seq_lens, c.block_table,
                                          q_indices=np.arange(len(lens))))
    assert 1 <= step.host.groups <= 37
    out = torch.full((len(lens), 32, 128), float("nan"), device="cuda", dtype=torch.float16)
    engine.run(step, d["q_source"], out)
    torch.cuda.synchronize()
    want = po.paged_decode(c.q_source.float().numpy(), c.k_pages.float().numpy(),
                           c.v_pages.float().numpy(), c.block_table, seq_lens=c.seq_lens)
    assert_close(out, want, "f16", "router groups")


@pytest.mark.parametrize("page", [16, 8, 32])
def test_cuda_core_math_matches_oracle(page):
    """The CUDA-core consumer math (pkv_set_math_mode(PKV_MATH_FMA): fp32 FMA
    instead of mma.sync) on the lean route it serves -- host plan, fused merge,
    G = 4, fp16 -- against the float64 oracle, and against the tensor-core
    result of the same launch within the same tolerance; other routes keep
    the tensor-core path under that mode."""
    from persistentkv_attention_b200.scheduler import build_auto_plan

    lens = [0] + EDGE_LENS + [9000, 4096]
    c = make_case(lens, hq=32, hkv=8, page_size=page, seed=800 + page, indexed=True)
    d = c.cuda()
    want = c.oracle()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    plan = torch.from_numpy(build_auto_plan(c.seq_lens, c.block_table, c.block_table.shape[1],
                                            page, 8, sms, q_indices=c.q_indices,
                                            out_indices=c.out_indices)).cuda()
    outs = {}
    prev = _native.math_mode()
    try:
        for mode in ("mma", "fma"):
            _native.set_math_mode(mode)
            for planned in (True, False):
                ws = torch.empty(ops.auto_workspace_bytes(len(lens), 32, 8) // 4, device="cuda")
                out = torch.full((c.out_rows, 32, 128), float("nan"), device="cuda",
                                 dtype=torch.float16)
                ctr = torch.zeros(len(lens), 8, device="cuda", dtype=torch.int32)
                ops.paged_attention_auto(d["q_source"], d["k_pages"], d["v_pages"],
                                         d["block_table"], d["seq_lens"], out, ws,
                                         d["q_indices"], d["out_indices"], ctr,
                                         plan=plan if planned else None)
                torch.cuda.synchronize()
                assert (ctr == 0).all()
                assert _native.device_error(clear=True) == 0
                assert_close(out, want, "f16", f"math={mode} planned={planned}")
                outs[(mode, planned)] = out
    finally:
        _native.set_math_mode(prev)
    rows = torch.from_numpy(c.out_indices).long().cuda()
    diff = (outs[("fma", True)][rows].float() - outs[("mma", True)][rows].float()).abs().max()
    assert diff.item() < MAX_ERR
    # without a plan the launch is not the lean route: the tensor-core path, same bits
    assert torch.equal(outs[("fma", False)][rows], outs[("mma", False)][rows])


def test_dependent_launch_chain_in_a_graph():
    """Decode launches chained with programmatic dependent launch (one per
    model layer, each over its own pool, captured in one CUDA graph): each
    waits for the previous kernel before reading, so every layer's output
    equals its own launch run alone, and the oracle."""
    from persistentkv_attention_b200.serving import DecodeEngine

    lens = [4096, 700, 9000, 33, 2048, 1, 5000, 300]
    cases = [make_case(lens, seed=900 + i, indexed=True) for i in range(3)]
    dev = [c.cuda() for c in cases]
    engines = [DecodeEngine(d["k_pages"], d["v_pages"], 32) for d in dev]
    c0 = cases[0]
    plans = [e.upload(e.plan_step(c0.seq_lens, c.block_table, q_indices=c0.q_indices))
             for e, c in zip(engines, cases)]
    q = dev[0]["q_source"]
    alone = []
    for e, p in zip(engines, plans):
        o = torch.full((len(lens), 32, 128), float("nan"), device="cuda", dtype=torch.float16)
        e.run(p, q, o)
        alone.append(o)
    torch.cuda.synchronize()
    outs = [torch.full_like(a, float("nan")) for a in alone]
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    _native.set_dependent_launch(True)
    try:
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for e, p, o in zip(engines, plans, outs):
                    e.run(p, q, o)
    finally:
        _native.set_dependent_launch(False)
    for _ in range(3):
        for o in outs:
            o.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for a, o in zip(alone, outs):
            assert torch.equal(a, o)
    assert _native.device_error(clear=True) == 0
    for c, o in zip(cases, outs):
        # every layer reads the first case's q rows (the plans carry its q_indices)
        want = po.paged_decode(c0.q_source.float().numpy(), c.k_pages.float().numpy(),
                               c.v_pages.float().numpy(), c.block_table, seq_lens=c0.seq_lens,
                               q_indices=c0.q_indices)
        assert_close(o, want, "f16", "dependent-launch chain")
