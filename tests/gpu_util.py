"""Helpers for the GPU tests: device copies, on-device seeded fills, cuBLAS comparator."""
import numpy as np
import torch


def dev(a):
    """numpy float16 (or its uint16 bits) -> contiguous CUDA half tensor."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.float16)
    return torch.from_numpy(a).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def hash_fill_(t, seed):
    """three_way.cu:22-33 counter-hash fill of a CUDA half tensor, in place, on the device:
    h = (i * 2654435761) ^ seed, xorshift-multiply mixing, value (h & 0xffff)/32768 - 1."""
    flat = t.view(-1)
    n = flat.numel()
    step = 1 << 25
    M32 = 0xFFFFFFFF
    for b in range(0, n, step):
        e = min(n, b + step)
        i = torch.arange(b, e, device=t.device, dtype=torch.int64)
        h = ((i * 2654435761) & M32) ^ (seed & M32)
        h ^= h >> 15
        h = (h * 2246822519) & M32
        h ^= h >> 13
        h = (h * 3266489917) & M32
        h ^= h >> 16
        flat[b:e] = ((h & 0xFFFF).to(torch.float32) / 32768.0 - 1.0).to(torch.float16)
    return t


def cublas(A, B, C, M, N, K, alpha, beta, stream=None):
    """The reference harness's cublasGemmEx call (row-major via column-major swap)."""
    from hopper_gemm_b200._native import cublas_ref_lib
    s = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
    st = cublas_ref_lib().hgemm_cublas_ref(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K,
                                           float(alpha), float(beta), s)
    assert st == 0, st


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(np.sum((a - b) ** 2) / (np.sum(b * b) + 1e-30)))
