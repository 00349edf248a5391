"""Sequence-sharded decode on 2 GPUs (one process per GPU, NCCL for set-up):
the fused peer exchange and the NCCL all-gather path both reproduce the
single-GPU oracle.  Skipped on a box with fewer than two GPUs."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_q):
    import torch.distributed as dist

    from persistentkv_attention_b200 import dist as pdist
    from persistentkv_attention_b200 import ops
    from tests.helpers import make_case

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    xg = None
    try:
        cases = [make_case(lens, seed=90 + i, indexed=True)
                 for i, lens in enumerate([[32768], [30000, 33, 0, 777], [1, 9000, 4096]])]
        xg = pdist.make_exchange(32, 8, 4)
        errs = []
        for c in cases:
            d = {k: v.to(dev) for k, v in c.cuda().items()}
            b = len(c.seq_lens)
            bt, sl = pdist.shard_rows(c.block_table, c.seq_lens, 16, world, rank)
            bt_d, sl_d = torch.from_numpy(bt).to(dev), torch.from_numpy(sl).to(dev)
            ws = torch.empty(ops.auto_workspace_bytes(b, 32, 8) // 4, device=dev)
            counters = torch.zeros(b, 8, device=dev, dtype=torch.int32)
            want = c.oracle()
            rows = torch.from_numpy(c.out_indices).long()
            # fused exchange, eager then graph-replayed
            out = torch.full((c.out_rows, 32, 128), float("nan"), device=dev,
                             dtype=torch.float16)

            def step():
                ops.paged_attention_sharded(d["q_source"], d["k_pages"], d["v_pages"], bt_d,
                                            sl_d, out, ws, counters, xg, d["q_indices"],
                                            d["out_indices"])

            for _ in range(2):
                step()
            torch.cuda.synchronize()
            got = out.cpu().double().numpy()
            errs.append(float(np.abs(got[rows] - want[rows]).max()))
            graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(dev)
            with torch.cuda.stream(s):
                with torch.cuda.graph(graph, stream=s):
                    step()
            out.fill_(float("nan"))
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            got = out.cpu().double().numpy()
            errs.append(float(np.abs(got[rows] - want[rows]).max()))
            del graph
            # NCCL path: state kernel, all-gather, combine
            st = torch.empty(b, 32, 130, device=dev)
            ops.paged_attention_auto_state(d["q_source"], d["k_pages"], d["v_pages"], bt_d, sl_d,
                                           st, ws, d["q_indices"], counters)
            gathered = pdist.gather_states(st)
            out2 = torch.full_like(out, float("nan"))
            ops.combine_states(gathered, out2, d["out_indices"])
            torch.cuda.synchronize()
            got = out2.cpu().double().numpy()
            errs.append(float(np.abs(got[rows] - want[rows]).max()))
            dist.barrier()
        result_q.put((rank, "ok", max(errs)))
    except Exception as exc:  # reported to the parent
        result_q.put((rank, "error", type(exc).__name__ + ": " + str(exc)[:300]))
    finally:
        torch.cuda.synchronize()
        try:
            dist.barrier()
        except Exception:
            pass
        if xg is not None:
            xg.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs two GPUs")
def test_sequence_sharded_two_gpus():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        rank, status, value = q.get(timeout=600)
        results[rank] = (status, value)
    for p in procs:
        p.join(timeout=120)
    for r in range(WORLD):
        status, value = results[r]
        assert status == "ok", f"rank {r}: {value}"
        assert value < 2e-3, f"rank {r}: max abs error {value}"
