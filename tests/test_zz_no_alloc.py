"""GPU: the no-allocation entry point, hgemm_launch_noalloc.

It exists for callers that may not allocate device memory while they run a GEMM (a host
framework that owns a fixed device-memory pool, or a latency-critical path that must not
take the allocator's lock or its implicit synchronisation). Instead of cudaMalloc'ing the
scratch for the restrided operand copies, it uses a fixed array the library keeps on each
device. These tests call it through the C ABI and compare it with hgemm_launch, two calls in
a row (the second call finds the first call's leftovers in the shared array). This file is
collected last so that a run stopping at the first failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu


def _inputs(oracle, M, N, K, seed):
    g = oracle.MT19937Stream(seed)
    return g.uniform_half((M, K)), g.uniform_half((K, N)), g.normal_half((M, N))


def _call(lib_fn, A, B, C, M, N, K, alpha, beta):
    s = torch.cuda.current_stream().cuda_stream
    st = lib_fn(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, alpha, beta, s)
    torch.cuda.synchronize()
    return st


@pytest.mark.parametrize("M,N,K,alpha,beta", [
    (2048, 2047, 2048, 1.5, 0.5),   # B restrided (N % 8 != 0), beta != 0
    (1000, 999, 1001, 1.0, 0.0),    # A and B restrided
    (777, 1024, 333, -2.0, 0.25),   # A restrided only
    (512, 384, 256, 1.0, 0.0),      # aligned: no scratch needed at all
])
def test_noalloc_matches_launch_two_calls(cuda, oracle, M, N, K, alpha, beta):
    lib = cuda.lib
    assert lib.hgemm_noalloc_scratch_bytes() == 64 << 20
    for call in range(2):
        A, B, C = _inputs(oracle, M, N, K, seed=1000 * call + M + N + K)
        dA, dB = dev(A), dev(B)
        ref_C, out_C = dev(C), dev(C)
        assert _call(lib.hgemm_launch, dA, dB, ref_C, M, N, K, alpha, beta) == 0
        assert _call(lib.hgemm_launch_noalloc, dA, dB, out_C, M, N, K, alpha, beta) == 0
        ref, out = host(ref_C), host(out_C)
        # the same kernels on the same inputs: expected bit-identical; the bar is the
        # tolerance the parity tests use against the fp64 oracle
        fp64 = oracle.gemm_f64(A, B, C, alpha, beta)
        ok, worst, _ = oracle.check(out, fp64, K)
        assert ok, (call, worst)
        assert np.array_equal(out.view(np.uint16), ref.view(np.uint16)), call
    assert cuda.device_status(clear=True)[0] == 0


def test_noalloc_rejects_oversize_without_work(cuda):
    lib = cuda.lib
    # both operands restrided: (4095 + 8191) * 8192 halves = 201 MB, over the 64 MiB array
    M, N, K = 4095, 8191, 8191
    A = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    B = torch.zeros((K, N), dtype=torch.float16, device="cuda")
    C = torch.full((M, N), 7.0, dtype=torch.float16, device="cuda")
    st = _call(lib.hgemm_launch_noalloc, A, B, C, M, N, K, 1.0, 0.0)
    plan = cuda.plan(M, N, K)
    assert plan["scratch_bytes"] > lib.hgemm_noalloc_scratch_bytes()
    assert st == cuda._native.HGEMM_ERR_TOO_LARGE
    assert bool((C == 7.0).all())  # nothing ran


def test_noalloc_padded_c_counts_against_the_array(cuda):
    """The padded C copy (N % 8 != 0 with beta != 0) also comes from the fixed array: here it
    alone is over the limit (A needs no restride, B is 8 rows), so the same shape runs with
    beta == 0 and is rejected, untouched, with beta != 0."""
    lib = cuda.lib
    M, N, K = 8192, 8191, 8
    cap = lib.hgemm_noalloc_scratch_bytes()
    p0, p1 = cuda.plan(M, N, K, beta=0.0), cuda.plan(M, N, K, beta=0.5)
    assert not p1["pad_a"] and p1["pad_c"] and p1["scratch_bytes"] > cap
    assert not p0["pad_c"] and p0["scratch_bytes"] <= cap
    A = torch.ones((M, K), dtype=torch.float16, device="cuda")
    B = torch.ones((K, N), dtype=torch.float16, device="cuda")
    C = torch.full((M, N), 7.0, dtype=torch.float16, device="cuda")
    assert _call(lib.hgemm_launch_noalloc, A, B, C, M, N, K, 1.0, 0.5) == \
        cuda._native.HGEMM_ERR_TOO_LARGE
    assert bool((C == 7.0).all())  # nothing ran
    assert _call(lib.hgemm_launch_noalloc, A, B, C, M, N, K, 1.0, 0.0) == 0
    assert bool((C == float(K)).all())
    assert cuda.device_status(clear=True)[0] == 0


def test_noalloc_misaligned_pointers_run_without_scratch(cuda, oracle):
    """Pointers off a 16-byte boundary would need restride copies in the fixed array (8192^3:
    256 MiB); the no-allocation entry point runs them on the scalar kernel instead, which needs
    no scratch. Within the parity bar of the fp64 oracle and of hgemm_launch (which copies
    them and stays on the tensor cores), two calls in a row."""
    lib = cuda.lib
    M, N, K = 1024, 1024, 1024
    for call, (alpha, beta) in enumerate(((1.0, 0.5), (-1.5, 0.0))):
        A, B, C = _inputs(oracle, M, N, K, seed=77 + call)

        def placed(x):
            buf = torch.zeros(x.size + 1, dtype=torch.float16, device="cuda")
            buf[1:] = dev(x).view(-1)
            return buf
        bA, bB, bRef, bOut = placed(A), placed(B), placed(C), placed(C)
        s = torch.cuda.current_stream().cuda_stream
        args = (M, N, K, alpha, beta, s)
        assert lib.hgemm_launch(bA.data_ptr() + 2, bB.data_ptr() + 2, bRef.data_ptr() + 2,
                                *args) == 0
        assert lib.hgemm_launch_noalloc(bA.data_ptr() + 2, bB.data_ptr() + 2,
                                        bOut.data_ptr() + 2, *args) == 0
        torch.cuda.synchronize()
        ref, out = host(bRef)[1:].reshape(M, N), host(bOut)[1:].reshape(M, N)
        fp64 = oracle.gemm_f64(A, B, C if beta != 0 else None, alpha, beta)
        for got in (out, ref):
            ok, worst, _ = oracle.check(got, fp64, K)
            assert ok, (call, worst)
    assert cuda.device_status(clear=True)[0] == 0
