"""CPU, 2 gloo ranks: the row-shard plan of the multi-GPU layer (hgemm_shard_rows /
hgemm_shard_chunk_rows) reassembles the full GEMM when every rank computes its own rows and
the blocks are exchanged; and a rank that leaves before the exchange is detected by the
others through a short process-group timeout instead of a hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, M, N, K, chunks, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    import hopper_gemm_b200 as hg
    from hopper_gemm_b200.sharded import chunk_rows, row_plan
    from oracle import oracle as orc
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    g = orc.MT19937Stream(77)               # every rank draws the same A, B, C
    A = g.uniform_half((M, K))
    B = g.uniform_half((K, N))
    C = g.normal_half((M, N))
    plan = row_plan(M, world)
    b, n = hg.shard_rows(M, world, rank)
    assert plan[rank] == (b, n)
    full = np.zeros((M, N), np.float64)
    # per chunk: this rank computes its chunk rows, then every rank's chunk is exchanged
    for ch in range(chunks):
        cb, cn = chunk_rows(n, chunks, ch)
        mine = orc.gemm_f64(A, B, C, 1.5, 0.5, rows=np.arange(b + cb, b + cb + cn, dtype=np.int32))
        sizes = [chunk_rows(plan[r][1], chunks, ch)[1] for r in range(world)]
        pad = max(sizes + [1])
        send = torch.zeros((pad, N), dtype=torch.float64)
        send[:cn] = torch.from_numpy(mine)
        recv = [torch.zeros_like(send) for _ in range(world)]
        dist.all_gather(recv, send)
        for r in range(world):
            rb = plan[r][0] + chunk_rows(plan[r][1], chunks, ch)[0]
            full[rb:rb + sizes[r]] = recv[r][:sizes[r]].numpy()
    ref = orc.gemm_f64(A, B, C, 1.5, 0.5)
    out[rank] = bool(np.array_equal(full, ref))
    dist.destroy_process_group()


@pytest.mark.parametrize("M,chunks", [(64, 1), (37, 1), (37, 3), (1, 2)])
def test_row_shards_reassemble_full_gemm(M, chunks):
    world, N, K = 2, 19, 23
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, M, N, K, chunks, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(out) == {0: True, 1: True}


def _leaver_worker(rank, world, port, out):
    import time
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, without joining the exchange
    t0 = time.time()
    try:
        dist.all_gather([torch.zeros(4) for _ in range(world)], torch.ones(4))
        out[rank] = "no error"
    except Exception as e:  # noqa: BLE001 -- any error is the detection we want
        out[rank] = f"detected after {time.time() - t0:.1f}s: {type(e).__name__}"


def test_departed_rank_is_detected_not_hung():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert out.get(0, "").startswith("detected"), out.get(0)
