"""GPU: seeded random shapes (small, mid, ragged N and K, four alpha/beta pairs) through
hgemm_launch against a PyTorch fp32 reference of the same op, with the per-element tolerance
|C - C_ref| <= 1e-2 |C_ref| + 2e-3 sqrt(K), and a clean device status after every call."""
import random

import pytest
import torch

pytestmark = pytest.mark.gpu


def _shapes(n, seed=1234):
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        kind = rng.random()
        if kind < 0.3:
            M, N, K = rng.randint(1, 300), rng.randint(1, 300), rng.randint(1, 300)
        elif kind < 0.7:
            M, N, K = rng.randint(1, 3000), rng.randint(1, 3000), rng.randint(1, 3000)
        else:
            M = rng.choice([128, 256, 512, 1024, 2048, 4096])
            N = rng.choice([64, 128, 256, 512, 1024, 2048, 4096])
            K = rng.choice([8, 64, 128, 192, 256, 512, 1024, 4096, 8192])
        if rng.random() < 0.3:
            N = max(1, N + rng.choice([-1, 1, 3, 7]))
        if rng.random() < 0.3:
            K = max(1, K + rng.choice([-1, 1, 5]))
        al, be = rng.choice([(1.0, 0.0), (1.5, 0.5), (-0.5, 1.0), (2.0, -1.0)])
        out.append((M, N, K, al, be))
    return out


@pytest.mark.parametrize("M,N,K,al,be", _shapes(120))
def test_random_shape(cuda, M, N, K, al, be):
    g = torch.Generator(device="cuda").manual_seed(M * 7919 + N * 104729 + K)
    A = (torch.rand(M, K, device="cuda", generator=g) * 2 - 1).half()
    B = (torch.rand(K, N, device="cuda", generator=g) * 2 - 1).half()
    C0 = torch.randn(M, N, device="cuda", generator=g).half()
    C = C0.clone()
    cuda.launch(A, B, C, M, N, K, al, be)
    torch.cuda.synchronize()
    st, where = cuda.device_status(clear=True)
    assert st == 0, f"device wait gave up at site {where}"
    ref = al * (A.float() @ B.float()) + be * C0.float()
    err = (C.float() - ref).abs()
    tol = 1e-2 * ref.abs() + 2e-3 * K ** 0.5
    assert bool(torch.isfinite(C.float()).all())
    assert bool((err <= tol).all()), float((err / tol).max())
