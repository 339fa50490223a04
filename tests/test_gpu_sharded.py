"""GPU: the row-sharded NCCL layer (hgemm_sharded_rank) against the single-GPU GEMM.

With one GPU the communicator has one rank (the NCCL path is still loaded and exercised);
with two or more visible GPUs, two processes shard the rows and every rank must end with
the full C, bit-identical to the single-GPU result (each row block is computed by the same
kernel on the same inputs)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(M, N, K, seed=5):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as orc
    g = orc.MT19937Stream(seed)
    return g.uniform_half((M, K)), g.uniform_half((K, N)), g.normal_half((M, N))


def _worker(rank, world, port, M, N, K, chunks, alpha, beta, out, fused=False):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    import hopper_gemm_b200 as hg
    from hopper_gemm_b200.sharded import RowShardedGemm
    A, B, C = _inputs(M, N, K)
    b, n = hg.shard_rows(M, world, rank)
    dA = torch.from_numpy(np.ascontiguousarray(A[b:b + n])).cuda()
    dB = torch.from_numpy(B).cuda()
    dC = torch.from_numpy(C).cuda()
    sg = RowShardedGemm(M, N, K, rank, world, chunks=chunks)
    if fused:
        # peer-store path: registration maps the other rank's C; two calls in a row
        assert sg.register_output(dC)
        sg(dA, dB, dC, alpha, beta)
        torch.cuda.synchronize()
        dC.copy_(torch.from_numpy(C).cuda())
        dist.barrier()
    sg(dA, dB, dC, alpha, beta)
    torch.cuda.synchronize()
    assert sg.healthy()
    sg.close()
    ref = torch.from_numpy(C).cuda()
    hg.launch(torch.from_numpy(A).cuda(), dB, ref, M, N, K, alpha, beta)
    torch.cuda.synchronize()
    out[rank] = bool(torch.equal(dC.view(torch.int16), ref.view(torch.int16)))
    dist.barrier()
    dist.destroy_process_group()


def test_single_rank_communicator(cuda):
    import ctypes
    from hopper_gemm_b200 import lib
    M, N, K = 1000, 768, 512
    A, B, C = _inputs(M, N, K)
    uid = (ctypes.c_ubyte * 128)()
    assert lib.hgemm_comm_unique_id(uid, 128) == 0
    comm = ctypes.c_void_p()
    assert lib.hgemm_comm_init(ctypes.byref(comm), 1, bytes(uid), 128, 0) == 0
    dA, dB, dC, ref = dev(A), dev(B), dev(C), dev(C)
    s = torch.cuda.current_stream().cuda_stream
    for chunks in (1, 3):
        dC.copy_(dev(C))
        assert lib.hgemm_sharded_rank(comm, dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), M, N, K,
                                      1.25, 0.5, chunks, s) == 0
        torch.cuda.synchronize()
        ref.copy_(dev(C))
        cuda.launch(dA, dB, ref, M, N, K, 1.25, 0.5)
        assert np.array_equal(host(dC).view(np.uint16), host(ref).view(np.uint16)), chunks
    assert lib.hgemm_comm_check(comm) == 0
    assert lib.hgemm_comm_destroy(comm) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
@pytest.mark.parametrize("M,chunks", [(4096, 1), (3001, 1), (4096, 4)])
def test_two_ranks_gather_full_c(cuda, M, chunks):
    world, N, K = 2, 1024, 768
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, chunks, 1.0, 0.5, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(out) == {0: True, 1: True}


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
@pytest.mark.parametrize("M,N", [(4096, 1024), (2048, 1002), (3001, 1024)])
def test_two_ranks_fused_peer_stores(cuda, M, N):
    # (4096, 1024): one kernel per rank stores every tile into both ranks' C;
    # (2048, 1002): N % 8 != 0 has no TMA-store epilogue, rows are pushed with copies;
    # (3001, 1024): unequal row blocks keep the NCCL exchange although C is registered.
    world, K = 2, 768
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, 1, 1.5, 0.5, out, True))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(out) == {0: True, 1: True}


def _steps_worker(rank, world, port, M, N, K, steps, slow_rank, out):
    """Back-to-back fused calls with a different A every step and a reader of the whole C
    after each call, without any host-side barrier in between: the slow rank's reader sleeps
    on the GPU first, so a peer that stored its next step's rows early would show up in the
    slow rank's snapshot of the previous step."""
    import sys
    sys.path.insert(0, ROOT)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    import hopper_gemm_b200 as hg
    from hopper_gemm_b200.sharded import RowShardedGemm
    from tests.gpu_util import hash_fill_
    b, n = hg.shard_rows(M, world, rank)
    dB = hash_fill_(torch.empty((K, N), dtype=torch.float16, device="cuda"), 0x85EBCA6B)
    dC = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    sg = RowShardedGemm(M, N, K, rank, world)
    assert sg.register_output(dC)
    dist.barrier()
    torch.cuda.synchronize()
    snaps = []
    for s in range(steps):
        A = hash_fill_(torch.empty((M, K), dtype=torch.float16, device="cuda"), 0x51ED + s)
        sg(A[b:b + n], dB, dC)
        if rank == slow_rank:
            torch.cuda._sleep(40_000_000)  # a slow reader: ~20 ms on the stream first
        snaps.append(dC.clone())           # reads the whole C on the same stream
    torch.cuda.synchronize()
    st, where = hg.device_status(clear=True)
    ok = st == 0
    for s in range(steps):
        A = hash_fill_(torch.empty((M, K), dtype=torch.float16, device="cuda"), 0x51ED + s)
        ref = torch.empty((M, N), dtype=torch.float16, device="cuda")
        hg.launch(A, dB, ref, M, N, K, 1.0, 0.0)
        torch.cuda.synchronize()
        ok = ok and bool(torch.equal(snaps[s].view(torch.int16), ref.view(torch.int16)))
    out[rank] = (ok, st, where)
    dist.barrier()
    sg.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
@pytest.mark.parametrize("N,slow_rank", [(1024, 1), (1024, 0), (1000, 1)])
def test_two_ranks_fused_back_to_back_steps(cuda, N, slow_rank):
    # N = 1024: the gated peer-store kernel; N = 1000 (N % 8 != 0): local GEMM, entry barrier
    # kernel, then copies to the peer.
    world, M, K, steps = 2, 2048, 512, 4
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_steps_worker, args=(r, world, port, M, N, K, steps, slow_rank,
                                                     out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(out) == {0: (True, 0, 0), 1: (True, 0, 0)}, dict(out)
