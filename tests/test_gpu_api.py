"""GPU: semantics of the drop-in entry points (mma_half.cu:1530-1640 behaviour) and the
bounded-wait failure path."""
import numpy as np
import pytest
import torch

from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu


def _inputs(oracle, M, N, K, seed=1):
    g = oracle.MT19937Stream(seed)
    return g.uniform_half((M, K)), g.uniform_half((K, N)), g.uniform_half((M, N))


def test_beta_zero_never_reads_c(cuda, oracle):
    A, B, _ = _inputs(oracle, 200, 136, 72)
    for N in (136, 135):  # TMA-store epilogue and the SIMT epilogue
        Bn = np.ascontiguousarray(B[:, :N])
        dA, dB = dev(A), dev(Bn)
        dC = torch.full((200, N), float("nan"), dtype=torch.float16, device="cuda")
        cuda.solve(dA, dB, dC, 200, N, 72, 1.0, 0.0)
        out = host(dC)
        assert np.isfinite(out).all()
        ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, Bn), 72)
        assert ok, worst


def test_k_zero_scales_c(cuda, oracle):
    _, _, C = _inputs(oracle, 64, 48, 8)
    dC = dev(C)
    dummy = torch.zeros(16, dtype=torch.float16, device="cuda")
    cuda.solve(dummy, dummy, dC, 64, 48, 0, 2.0, -0.5)
    assert cuda.last_status() == 0
    want = oracle.f32_to_f16((-0.5 * C.astype(np.float32)).astype(np.float32))
    assert np.array_equal(host(dC).view(np.uint16), want.view(np.uint16))


def test_empty_m_or_n_is_noop(cuda):
    C = torch.full((4, 4), 3.0, dtype=torch.float16, device="cuda")
    a = torch.zeros(16, dtype=torch.float16, device="cuda")
    cuda.solve(a, a, C, 0, 4, 4, 1.0, 0.0)
    cuda.solve(a, a, C, 4, 0, 4, 1.0, 0.0)
    assert cuda.last_status() == 0
    assert bool((C == 3.0).all())


def test_misaligned_pointers(cuda, oracle):
    M, N, K = 70, 90, 50
    A, B, C = _inputs(oracle, M, N, K, seed=4)
    bufA = torch.zeros(M * K + 1, dtype=torch.float16, device="cuda")
    bufB = torch.zeros(K * N + 1, dtype=torch.float16, device="cuda")
    bufC = torch.zeros(M * N + 1, dtype=torch.float16, device="cuda")
    bufA[1:] = dev(A).view(-1)
    bufB[1:] = dev(B).view(-1)
    bufC[1:] = dev(C).view(-1)
    esz = 2
    cuda.solve(bufA.data_ptr() + esz, bufB.data_ptr() + esz, bufC.data_ptr() + esz, M, N, K,
               1.25, 0.75)
    assert cuda.last_status() == 0
    out = host(bufC)[1:].reshape(M, N)
    ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, B, C, 1.25, 0.75), K)
    assert ok, worst


@pytest.mark.parametrize("M,N,K", [(70, 90, 50), (1000, 1024, 520), (777, 1001, 129)])
@pytest.mark.parametrize("which", ["A", "B", "C", "ABC"])
@pytest.mark.parametrize("off", [1, 3])
def test_misaligned_operands_each(cuda, oracle, M, N, K, which, off):
    """Operands that start `off` halves past a 16-byte boundary, one at a time and all three:
    A and B go through the restride copy, C is read and written in place by the SIMT-store
    epilogue. Every element vs fp64 at beta != 0 and at beta == 0 with NaN in C (never read),
    and the halves just before and after C untouched."""
    A, B, C = _inputs(oracle, M, N, K, seed=M + N + K + off)
    for alpha, beta in ((1.25, 0.75), (1.0, 0.0)):
        def place(x, shift):
            buf = torch.full((x.size + shift + 8,), 7.0, dtype=torch.float16, device="cuda")
            buf[shift:shift + x.size] = dev(x).view(-1)
            return buf
        sa, sb, sc = (off if w in which else 0 for w in "ABC")
        Cin = C if beta != 0 else np.full_like(C, np.nan)
        bA, bB, bC = place(A, sa), place(B, sb), place(Cin, sc)
        cuda.launch(bA.data_ptr() + 2 * sa, bB.data_ptr() + 2 * sb, bC.data_ptr() + 2 * sc,
                    M, N, K, alpha, beta)
        torch.cuda.synchronize()
        hb = host(bC)
        out = hb[sc:sc + M * N].reshape(M, N)
        ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, B, C if beta != 0 else None,
                                                        alpha, beta), K)
        assert ok, (which, alpha, beta, worst)
        assert np.all(hb[:sc] == 7.0) and np.all(hb[sc + M * N:] == 7.0)
    assert cuda.device_status(clear=True)[0] == 0


def test_side_stream_launch(cuda, oracle):
    M, N, K = 512, 512, 512
    A, B, _ = _inputs(oracle, M, N, K, seed=5)
    dA, dB = dev(A), dev(B)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        dC = cuda.gemm(dA, dB, stream=s)
    s.synchronize()
    ok, worst, _ = oracle.check(host(dC), oracle.gemm_f64(A, B), K)
    assert ok, worst


def test_deterministic_bits(cuda, oracle):
    A, B, _ = _inputs(oracle, 1536, 1280, 2000, seed=6)
    dA, dB = dev(A), dev(B)
    r1 = host(cuda.gemm(dA, dB))
    r2 = host(cuda.gemm(dA, dB))
    assert np.array_equal(r1.view(np.uint16), r2.view(np.uint16))


@pytest.mark.parametrize("M,N,K,alpha,beta", [
    (2304, 512, 256, 1.0, 0.0),   # two row blocks (1280 + 1024 rows)
    (3000, 1000, 136, 1.5, 0.5),  # beta != 0: the C blocks are copied in too
    (1100, 999, 72, 1.0, 0.25),   # N % 8 != 0: one block (B restrided once)
    (8192, 256, 64, 1.0, 0.0),    # eight row blocks
    (8192, 256, 1024, 1.0, 0.0),  # a 1024-row block alone would be split along K
    (3072, 64, 4096, 1.0, 0.5),   # the whole GEMM is split along K (6 ways): one block
])
def test_launch_host_pipelined_copies(cuda, oracle, M, N, K, alpha, beta):
    """hgemm_launch_host: host (page-locked) A, B, C in and C out through caller-owned device
    buffers, row blocks copied and computed in overlap; the result is the GEMM's, within the
    parity bar against the fp64 oracle, the device buffers hold the same C, and that C is
    bit-identical to one hgemm_launch of the whole GEMM on the same inputs."""
    A, B, C = _inputs(oracle, M, N, K, seed=M + N + K)
    hA = torch.from_numpy(np.ascontiguousarray(A)).pin_memory()
    hB = torch.from_numpy(np.ascontiguousarray(B)).pin_memory()
    hC = torch.from_numpy(np.ascontiguousarray(C).copy()).pin_memory()
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    dC = torch.empty((M, N), dtype=torch.float16, device="cuda")
    s = torch.cuda.Stream()
    cuda.launch_host(hA, hB, hC, dA, dB, dC, M, N, K, alpha, beta, s)
    s.synchronize()
    out = hC.numpy()
    ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, B, C, alpha, beta), K)
    assert ok, worst
    assert np.array_equal(out.view(np.uint16), host(dC).view(np.uint16))
    one = dev(C)
    cuda.launch(dev(A), dev(B), one, M, N, K, alpha, beta)
    torch.cuda.synchronize()
    assert np.array_equal(out.view(np.uint16), host(one).view(np.uint16))
    assert cuda.device_status(clear=True)[0] == 0


def test_tuned_launch_matches_default(cuda, oracle):
    M, N, K = 768, 640, 384
    A, B, C = _inputs(oracle, M, N, K, seed=8)
    dA, dB = dev(A), dev(B)
    dC = dev(C)
    cuda.launch_tuned(dA, dB, dC, M, N, K, 1.0, 0.5)
    torch.cuda.synchronize()
    ok, worst, _ = oracle.check(host(dC), oracle.gemm_f64(A, B, C, 1.0, 0.5), K)
    assert ok, worst  # C was not clobbered by the search (beta != 0 still correct)
    dC2 = dev(C)
    cuda.launch_tuned(dA, dB, dC2, M, N, K, 1.0, 0.5)  # cached plan
    assert np.array_equal(host(dC).view(np.uint16), host(dC2).view(np.uint16))


def test_bounded_wait_gives_up_and_context_survives(cuda, oracle):
    """A kernel waiting on an mbarrier nothing arrives on must return an error status after
    its bound, with the context still usable."""
    st = cuda.selftest_wait_timeout(20_000_000)  # 20 ms
    assert st == cuda.HGEMM_ERR_DEVICE_TIMEOUT
    assert cuda.device_status(clear=True)[0] == 0
    A, B, _ = _inputs(oracle, 256, 256, 256, seed=9)
    out = host(cuda.gemm(dev(A), dev(B)))
    ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, B), 256)
    assert ok, worst


def test_peer_barrier_wait_gives_up(cuda, oracle):
    """The multi-GPU step barrier waits on a flag that only a peer GPU writes; with a partner
    that never announces, its bounded wait must give up, record its site and leave the
    context usable (one GPU, local memory only)."""
    st = cuda.lib.hgemm_selftest_peer_barrier(5_000_000)  # 5 ms
    assert st == cuda.HGEMM_ERR_DEVICE_TIMEOUT
    assert cuda.device_status(clear=True)[0] == 0
    A, B, _ = _inputs(oracle, 128, 64, 64, seed=10)
    out = host(cuda.gemm(dev(A), dev(B)))
    ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, B), 64)
    assert ok, worst


def test_peer_entry_gate(cuda, oracle):
    """The fused multi-GPU path stores into a peer's C only after that peer has entered the
    same step. One GPU, local memory only: with the peer's entry flag already set the peer
    copy is written and equals C; with a flag nobody sets, the gate's bounded wait gives up,
    records its site, leaves the peer copy untouched, and the local C is still written."""
    assert cuda.lib.hgemm_selftest_peer_entry(1, 2_000_000_000) == cuda.HGEMM_OK
    assert cuda.lib.hgemm_selftest_peer_entry(0, 20_000_000) == cuda.HGEMM_ERR_DEVICE_TIMEOUT
    assert cuda.device_status(clear=True)[0] == 0
    A, B, _ = _inputs(oracle, 256, 256, 128, seed=11)
    out = host(cuda.gemm(dev(A), dev(B)))
    ok, worst, _ = oracle.check(out, oracle.gemm_f64(A, B), 128)
    assert ok, worst


def test_device_status_clean(cuda):
    assert cuda.device_status(clear=False)[0] == 0
