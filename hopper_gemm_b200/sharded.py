"""Row-sharded multi-GPU GEMM (one process per GPU) over the library's NCCL layer.

Rank r of P owns rows shard_rows(M, P, r) of A and C; B is replicated on every rank. Each
call computes the local C row block with the single-GPU GEMM and exchanges the blocks so
every rank ends with the whole C (hgemm_sharded_rank in libhgemm_b200.so: one in-place
ncclAllGather for equal blocks, grouped send/recv otherwise or when the local rows are split
into chunks whose exchange overlaps the next chunk's GEMM).

register_output(C) switches a communicator to the fused path for that output buffer: the
peers' C buffers and step-flag arrays are mapped into every process (CUDA IPC) and a single
kernel per rank stores each finished tile into every rank's C over NVLink while it computes,
so the exchange overlaps the math tile by tile. No NCCL call is made per step: the kernel
stores into a peer's C only once that peer's stream has entered the same step (an entry
epoch each rank's kernel announces when it starts), and a one-warp barrier kernel after it
waits until every rank has finished the step (an exit epoch); both are release/acquire flags
at system scope with bounded waits, failures recorded in the device status word. Readers of
C must therefore be ordered on the stream passed to each call (or before it).

torch.distributed (any backend) is used only for the rendezvous: rank 0 creates the NCCL id
and broadcasts it; the library then owns its own NCCL communicator. The reference
(yz-wqf/Hopper_GEMM) is single-GPU; this layer has no counterpart there.
"""
import ctypes

from . import HGEMM_OK, HgemmError, lib, shard_rows

ID_BYTES = 128


def chunk_rows(rows, chunks, chunk):
    b, n = ctypes.c_int(0), ctypes.c_int(0)
    st = lib.hgemm_shard_chunk_rows(int(rows), int(chunks), int(chunk), ctypes.byref(b),
                                    ctypes.byref(n))
    if st != HGEMM_OK:
        raise HgemmError(st, "hgemm_shard_chunk_rows")
    return b.value, n.value


def row_plan(M, world):
    """[(row_begin, row_count)] for every rank."""
    return [shard_rows(M, world, r) for r in range(world)]


class RowShardedGemm:
    def __init__(self, M, N, K, rank, world, chunks=1, device=None, group=None):
        import torch
        import torch.distributed as dist
        self.M, self.N, self.K = int(M), int(N), int(K)
        self.rank, self.world, self.chunks = int(rank), int(world), int(chunks)
        self.row_begin, self.rows = shard_rows(self.M, self.world, self.rank)
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        buf = torch.zeros(ID_BYTES, dtype=torch.uint8,
                          device=dev if dist.get_backend(group) == "nccl" else "cpu")
        if self.rank == 0:
            raw = (ctypes.c_ubyte * ID_BYTES)()
            st = lib.hgemm_comm_unique_id(raw, ID_BYTES)
            if st != HGEMM_OK:
                raise HgemmError(st, "hgemm_comm_unique_id")
            buf.copy_(torch.tensor(list(raw), dtype=torch.uint8))
        dist.broadcast(buf, 0, group=group)
        uid = bytes(buf.cpu().tolist())
        self._comm = ctypes.c_void_p()
        st = lib.hgemm_comm_init(ctypes.byref(self._comm), self.world, uid, ID_BYTES, self.rank)
        if st != HGEMM_OK:
            raise HgemmError(st, "hgemm_comm_init")

    def __call__(self, A_local, B, C, alpha=1.0, beta=0.0, stream=None):
        """A_local: this rank's rows of A; B: all of B; C: all of C (in/out) on this GPU."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream()
        st = lib.hgemm_sharded_rank(self._comm, A_local.data_ptr(), B.data_ptr(), C.data_ptr(),
                                    self.M, self.N, self.K, float(alpha), float(beta),
                                    self.chunks, s.cuda_stream)
        if st != HGEMM_OK:
            raise HgemmError(st, "hgemm_sharded_rank")
        return C

    def register_output(self, C):
        """Collective: use the fused peer-store path whenever C (this rank's full M x N output
        buffer, the same tensor on every later call) is passed. Returns False when some rank
        could not map its buffer (the NCCL path stays in use)."""
        st = lib.hgemm_comm_register_output(self._comm, C.data_ptr(),
                                            C.numel() * C.element_size())
        if st not in (HGEMM_OK,):
            return False
        return True

    def unregister_output(self):
        st = lib.hgemm_comm_register_output(self._comm, None, 0)
        if st != HGEMM_OK:
            raise HgemmError(st, "hgemm_comm_register_output")

    def healthy(self):
        return lib.hgemm_comm_check(self._comm) == HGEMM_OK

    def abort(self):
        if self._comm:
            lib.hgemm_comm_abort(self._comm)
            self._comm = None

    def close(self):
        if self._comm:
            lib.hgemm_comm_destroy(self._comm)
            self._comm = None
