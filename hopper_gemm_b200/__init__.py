"""hopper_gemm_b200 -- B200 (sm_100a) FP16 GEMM, a drop-in for yz-wqf/Hopper_GEMM's `solve`.

    C[M,N] = alpha * (A[M,K] @ B[K,N]) + beta * C[M,N]     row-major, half in/out, fp32 acc

The Python functions mirror the reference's host interface (mma_half.cu):
    solve(A, B, C, M, N, K, alpha, beta)                       <- extern "C" solve, 1636-1640
    launch(A, B, C, M, N, K, alpha, beta, stream, force_bm, force_bn, group_m)
                                                               <- h100_hgemm::launch, 1530
    launch_tuned(A, B, C, M, N, K, alpha, beta, stream)        <- h100_hgemm::launch_tuned, 1624
A, B, C may be integer device addresses or CUDA tensors (their data_ptr() is used). Like the
reference, `solve` returns nothing and synchronizes the device; its outcome is available from
last_status(). `launch*` return immediately (asynchronous) and raise HgemmError on a failed
launch. Everything goes through the C ABI of libhgemm_b200.so; there is no fallback path.
"""
import ctypes

from . import _native
from ._native import (HGEMM_ERR_DEVICE_TIMEOUT, HGEMM_ERR_INVALID_ARG, HGEMM_OK,  # noqa: F401
                      HgemmPlan, lib)

__all__ = ["solve", "launch", "launch_tuned", "launch_host", "gemm", "plan", "last_status",
           "status_string",
           "device_status", "release", "HgemmError", "set_wait_timeout_ns",
           "selftest_wait_timeout", "shard_rows"]


class HgemmError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


def _addr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    raise TypeError(f"expected a device address or a CUDA tensor, got {type(x)!r}")


def _stream(stream):
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream  # torch.cuda.Stream


def status_string(status):
    return lib.hgemm_status_string(int(status)).decode()


def last_status():
    return lib.hgemm_last_status()


def solve(A, B, C, M, N, K, alpha, beta):
    """Reference-compatible entry: launch on the default stream, then synchronize."""
    lib.solve(_addr(A), _addr(B), _addr(C), int(M), int(N), int(K), float(alpha), float(beta))


def launch(A, B, C, M, N, K, alpha=1.0, beta=0.0, stream=None, force_bm=0, force_bn=0,
           group_m=0):
    st = lib.hgemm_launch_ex(_addr(A), _addr(B), _addr(C), int(M), int(N), int(K), float(alpha),
                             float(beta), _stream(stream), int(force_bm), int(force_bn),
                             int(group_m))
    if st != HGEMM_OK:
        raise HgemmError(st, "hgemm_launch_ex")


def launch_tuned(A, B, C, M, N, K, alpha=1.0, beta=0.0, stream=None):
    st = lib.hgemm_launch_tuned(_addr(A), _addr(B), _addr(C), int(M), int(N), int(K),
                                float(alpha), float(beta), _stream(stream))
    if st != HGEMM_OK:
        raise HgemmError(st, "hgemm_launch_tuned")


def launch_host(A_h, B_h, C_h, dA, dB, dC, M, N, K, alpha=1.0, beta=0.0, stream=None):
    """GEMM on host buffers (page-locked for overlap) through caller-owned device buffers:
    the copies in and out run in row blocks overlapped with the GEMM (hgemm_launch_host).
    Asynchronous: C_h holds the result once `stream` has passed the call."""
    st = lib.hgemm_launch_host(_addr(A_h), _addr(B_h), _addr(C_h), _addr(dA), _addr(dB),
                               _addr(dC), int(M), int(N), int(K), float(alpha), float(beta),
                               _stream(stream))
    if st != HGEMM_OK:
        raise HgemmError(st, "hgemm_launch_host")


def gemm(A, B, C=None, alpha=1.0, beta=0.0, stream=None):
    """Convenience for CUDA fp16 tensors: returns C (allocated when None) after launching."""
    import torch
    if A.dtype != torch.float16 or B.dtype != torch.float16:
        raise TypeError("A and B must be float16")
    if not (A.is_cuda and B.is_cuda and A.is_contiguous() and B.is_contiguous()):
        raise ValueError("A and B must be contiguous CUDA tensors")
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    if C is None:
        if beta != 0.0:
            raise ValueError("beta != 0 needs C")
        C = torch.empty((M, N), dtype=torch.float16, device=A.device)
    elif tuple(C.shape) != (M, N) or not C.is_contiguous() or C.dtype != torch.float16:
        raise ValueError("C must be a contiguous float16 M x N tensor")
    if stream is None:
        stream = torch.cuda.current_stream(A.device)
    launch(A, B, C, M, N, K, alpha, beta, stream)
    return C


def plan(M, N, K, beta=0.0, aligned16=True, force_bm=0, force_bn=0, group_m=0, sm_count=0,
         pair_slots=0):
    """What launch() would run for this shape (host-only; needs no GPU)."""
    out = HgemmPlan()
    st = lib.hgemm_plan(int(M), int(N), int(K), float(beta), int(bool(aligned16)), int(force_bm),
                        int(force_bn), int(group_m), int(sm_count), int(pair_slots),
                        ctypes.byref(out))
    if st != HGEMM_OK:
        raise HgemmError(st, "hgemm_plan")
    return out.as_dict()


def device_status(clear=True):
    """(status, where) of the current device's kernel wait-timeout word (synchronizes)."""
    where = ctypes.c_int(0)
    st = lib.hgemm_device_status(int(bool(clear)), ctypes.byref(where))
    return st, where.value


def set_wait_timeout_ns(ns):
    lib.hgemm_set_wait_timeout_ns(int(ns))


def selftest_wait_timeout(timeout_ns=50_000_000):
    return lib.hgemm_selftest_wait_timeout(int(timeout_ns))


def release():
    lib.hgemm_release()


def shard_rows(M, nranks, rank):
    b, c = ctypes.c_int(0), ctypes.c_int(0)
    st = lib.hgemm_shard_rows(int(M), int(nranks), int(rank), ctypes.byref(b), ctypes.byref(c))
    if st != HGEMM_OK:
        raise HgemmError(st, "hgemm_shard_rows")
    return b.value, c.value
