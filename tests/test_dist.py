"""Multi-rank host logic on CPU (gloo, world size 2): sequence-shard split,
state exchange and exact LSE combine; a failing rank does not hang its peer."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import pkv_oracle as po
from persistentkv_attention_b200 import dist as pdist


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(seed=5):
    rng = np.random.default_rng(seed)
    lens = [5000, 17, 1, 900]
    page = 16
    pool = 1400
    kp = po.quantize(rng.standard_normal((pool, 8, page, 128)))
    vp = po.quantize(rng.standard_normal((pool, 8, page, 128)))
    table = rng.permutation(pool)[: 4 * 320].reshape(4, 320).astype(np.int32)
    q = po.quantize(rng.standard_normal((4, 32, 128)))
    return lens, page, kp, vp, table, q


def _worker(rank, world, port, result_q, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        lens, page, kp, vp, table, q = _case()
        bt, sl = pdist.shard_rows(table, lens, page, world, rank)
        states = np.zeros((len(lens), 32, 130), np.float32)
        for b in range(len(lens)):
            k, v = po.gather_row(kp, vp, bt[b], int(sl[b]))
            m, l, acc = po.row_state(q[b].astype(np.float64), k, v)
            states[b, :, 0], states[b, :, 1], states[b, :, 2:] = m, l, acc
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the exchange")
        gathered = pdist.gather_states(torch.from_numpy(states))
        g = gathered.double().numpy()
        out = po.combine_states(g[..., 0], g[..., 1], g[..., 2:])
        want = po.paged_decode(q, kp, vp, table, seq_lens=np.asarray(lens))
        result_q.put((rank, "ok", float(np.abs(out - want).max())))
    except Exception as exc:  # reported to the parent, never hangs
        result_q.put((rank, "error", type(exc).__name__ + ": " + str(exc)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results)


def test_shard_pages_cover_exactly():
    for pages in (1, 7, 2048, 2049):
        for world in (1, 2, 3, 8):
            rngs = pdist.shard_pages(pages, world)
            assert rngs[0][0] == 0 and rngs[-1][1] == pages
            assert all(a[1] == b[0] for a, b in zip(rngs, rngs[1:]))
            sizes = [hi - lo for lo, hi in rngs]
            assert max(sizes) - min(sizes) <= 1


def test_shard_rows_token_counts_sum():
    lens, page, _, _, table, _ = _case()
    for world in (2, 3, 8):
        total = np.zeros(len(lens), np.int64)
        for r in range(world):
            _, sl = pdist.shard_rows(table, lens, page, world, r)
            total += sl
        assert total.tolist() == lens


def test_partition_rows_balances_kv_bytes():
    sizes = [8000, 600, 5000, 7000, 512, 3000, 8192, 1000]
    parts = pdist.partition_rows(sizes, 4)
    assert sorted(i for p in parts for i in p) == list(range(8))
    loads = [sum(sizes[i] for i in p) for p in parts]
    assert max(loads) <= 1.35 * (sum(sizes) / 4)


@pytest.mark.timeout(300)
def test_sequence_shard_merge_two_ranks():
    res = _run(2)
    assert [r[1] for r in res] == ["ok", "ok"], res
    assert all(r[2] < 1e-5 for r in res), res  # states travel as float32


@pytest.mark.timeout(300)
def test_rank_failure_surfaces_as_error_not_hang():
    res = _run(2, fail_rank=1)
    status = {r[0]: r for r in res}
    assert status[1][1] == "error" and "injected" in status[1][2]
    # the surviving rank's collective ends with an error within the timeout
    assert status[0][1] == "error", status[0]
