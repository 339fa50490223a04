"""GPU: three-way cross-check on the aligned grid shapes: this library, cuBLAS and a CUTLASS
SM100 build of the same contract (the reference's 3-way table, three_way.cu, with its CUTLASS
column mma_half_cutlass.cu re-targeted to B200). Every pair must agree within the reference's
cuBLAS bar (rel_l2 < 3e-3, check_all.cu:72), and sampled rows of all three must meet the fp64
oracle's per-element tolerance."""
import numpy as np
import pytest
import torch

from tests.gpu_util import cublas, hash_fill_, host
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cutlass_lib():
    from hopper_gemm_b200._native import cutlass_ref_lib
    lib = cutlass_ref_lib()
    if lib is None:
        pytest.skip("libhgemm_cutlass_ref.so not built (no CUTLASS headers on the build machine)")
    return lib


def _l2(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-30))


@pytest.mark.parametrize("M,N,K,al,be", [
    (1024, 1024, 1024, 1.0, 0.0), (4096, 8192, 128, 1.0, 0.0), (2048, 2048, 512, 1.0, 0.0),
    (4096, 512, 4096, 1.0, 0.0), (3000, 1000, 2000, 1.5, 0.5), (384, 2048, 2048, 2.5, -1.5),
    (8192, 8192, 8192, 1.0, 0.0)])
def test_three_way(cuda, oracle, cutlass_lib, M, N, K, al, be):
    A = hash_fill_(torch.empty((M, K), dtype=torch.float16, device="cuda"), 0x9E3779B9 ^ M)
    B = hash_fill_(torch.empty((K, N), dtype=torch.float16, device="cuda"), 0x85EBCA6B ^ N)
    C0 = hash_fill_(torch.empty((M, N), dtype=torch.float16, device="cuda"), 0x1234 ^ K)
    ours, ref, cut = C0.clone(), C0.clone(), C0.clone()
    cuda.launch(A, B, ours, M, N, K, al, be)
    cublas(A, B, ref, M, N, K, al, be)
    s = torch.cuda.current_stream().cuda_stream
    st = cutlass_lib.hgemm_cutlass_ref(A.data_ptr(), B.data_ptr(), cut.data_ptr(), M, N, K, al,
                                       be, s)
    assert st == 0, st
    torch.cuda.synchronize()
    assert _l2(ours, ref) < 3e-3
    assert _l2(ours, cut) < 3e-3
    assert _l2(cut, ref) < 3e-3
    hA, hB, hC = host(A), host(B), host(C0)
    rows = np.random.RandomState(M ^ N ^ K).randint(0, M, 8)
    for out in (ours, cut):
        assert_close(oracle, host(out), hA, hB, hC, al, be, rows=rows)
