"""GPU: split-K (a cluster of one-CTA tiles sharing each tile's k-blocks, partial sums
reduced over distributed shared memory in split order) against the fp64 oracle.

Every forced (tile, ksplit) combination, uneven k-block splits, more splits than k-blocks,
partial tiles on the M and N edges, beta != 0, repeat runs bit-identical, and the automatic
choice for the small shapes of the reference's grid."""
import numpy as np
import pytest
import torch

from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu


def _inputs(oracle, M, N, K, seed):
    g = oracle.MT19937Stream(seed)
    return g.uniform_half((M, K)), g.uniform_half((K, N)), g.normal_half((M, N))


def _splitk(cuda, dA, dB, dC, M, N, K, alpha, beta, bn, ks):
    s = torch.cuda.current_stream().cuda_stream
    st = cuda.lib.hgemm_launch_splitk(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), M, N, K,
                                      float(alpha), float(beta), s, bn, ks)
    assert st == 0, cuda.status_string(st)


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("ks", [2, 3, 4, 8])
def test_forced_split(cuda, oracle, bn, ks):
    M, N, K = 300, 2 * bn + 40, 1000  # partial tiles on both edges; 16 k-blocks, uneven splits
    A, B, C = _inputs(oracle, M, N, K, seed=bn + ks)
    dA, dB = dev(A), dev(B)
    dC = dev(C)
    _splitk(cuda, dA, dB, dC, M, N, K, 1.5, 0.5, bn, ks)
    out = host(dC)
    ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, B, C, 1.5, 0.5), K)
    assert ok, worst
    assert cuda.device_status(clear=False)[0] == 0
    # bit-stable: the same call again gives the same bits
    dC2 = dev(C)
    _splitk(cuda, dA, dB, dC2, M, N, K, 1.5, 0.5, bn, ks)
    assert np.array_equal(host(dC2).view(np.uint16), out.view(np.uint16))


def test_more_splits_than_k_blocks(cuda, oracle):
    M, N, K = 128, 128, 130  # 3 k-blocks, 8 splits requested
    A, B, _ = _inputs(oracle, M, N, K, seed=3)
    dC = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    _splitk(cuda, dev(A), dev(B), dC, M, N, K, 1.0, 0.0, 128, 8)
    ok, worst, _ = oracle.check(host(dC), oracle.gemm_f64(A, B), K)
    assert ok, worst


def test_split_matches_unsplit_within_tolerance_and_exact_on_integers(cuda, oracle):
    # Small integers: every partial and total is exact in fp32, so any split order gives
    # the same bits as the unsplit kernel.
    rng = np.random.default_rng(5)
    M, N, K = 256, 256, 1024
    A = rng.integers(-2, 3, size=(M, K)).astype(np.float16)
    B = rng.integers(-2, 3, size=(K, N)).astype(np.float16)
    dA, dB = dev(A), dev(B)
    ref = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    cuda.launch(dA, dB, ref, M, N, K, 1.0, 0.0, force_bm=128, force_bn=128)
    for ks in (2, 4):
        dC = torch.zeros(M, N, dtype=torch.float16, device="cuda")
        _splitk(cuda, dA, dB, dC, M, N, K, 1.0, 0.0, 128, ks)
        assert np.array_equal(host(dC).view(np.uint16), host(ref).view(np.uint16)), ks


def test_ragged_n_runs_unsplit(cuda, oracle):
    M, N, K = 256, 250, 512  # N % 8 != 0: no TMA-store epilogue, split request ignored
    A, B, _ = _inputs(oracle, M, N, K, seed=4)
    dC = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    _splitk(cuda, dev(A), dev(B), dC, M, N, K, 1.0, 0.0, 128, 4)
    ok, worst, _ = oracle.check(host(dC), oracle.gemm_f64(A, B), K)
    assert ok, worst


@pytest.mark.parametrize("M,N,K", [(256, 256, 4096), (128, 128, 8192), (512, 512, 8192)])
def test_automatic_split_shapes(cuda, oracle, M, N, K):
    assert cuda.plan(M, N, K)["ksplit"] > 1
    A, B, _ = _inputs(oracle, M, N, K, seed=M + N)
    dC = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    cuda.launch(dev(A), dev(B), dC, M, N, K, 1.0, 0.0)
    rows = np.arange(0, M, 7)
    ref = oracle.gemm_f64(A, B, rows=rows)
    ok, worst, _ = oracle.check(host(dC)[rows], ref, K)
    assert ok, worst
