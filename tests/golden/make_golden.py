"""Generate the golden vectors that pin the CPU oracle (run from the repo root:
`python tests/golden/make_golden.py`). Independent of oracle/: it uses numpy and the C
library only, so the oracle is checked against values it did not produce.

1. Known-answer tests of the reference's descriptor probes. The inputs are the probes' own
   integer-valued matrices, drawn from the C library's rand() exactly as the probes draw them:
     probe_kmajor.cu:117-125   srand(0); A[64x64] = rand()%7-3; Bt[64x64] (N x K) = rand()%5-2;
                               C[m][n] = sum_k A[m][k] * Bt[n][k]
     probe_mnmajor.cu:63-68    srand(1); A[64x64] = rand()%7-3; B[64x128] (K x N) = rand()%5-2
     (probe_mnmajor_kadv.cu:65-68 draws the same matrices and sums all 64 k.)
   The GEMM row-major B operand is Bt transposed for the first case. Expected C is exact
   integer arithmetic.
2. The harnesses' generator: std::mt19937(seed) + uniform_real_distribution<float>(lo, hi)
   (check_all.cu:14, check_fp64.cu:16), restated here from the published algorithms (MT19937
   via numpy's legacy seeding, then libstdc++'s generate_canonical<float, 24>: one 32-bit
   draw u, float(u) / 2^32 in float, clamped below 1, then x * (hi - lo) + lo in float).
3. The check_fp64.cu suite (check_fp64.cu:20-23): inputs from one mt19937(3) stream over all
   shapes in order (A, B, C per shape, U(-2,2), rounded to half), and for the small shapes
   the fp64 result accumulated in the reference's k order (check_fp64.cu:39-44). Inputs and
   results are stored as SHA-256 digests of their bytes, which keeps the fixture small and
   still pins the oracle bit for bit.
"""
import ctypes
import ctypes.util
import hashlib
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

CHECK_FP64_SHAPES = [(128, 256, 64, 1, 0), (256, 512, 128, 1, 0), (1024, 1024, 1024, 1, 0),
                     (129, 260, 72, 1, 0), (100, 300, 64, 1, 0), (512, 512, 512, 2.5, -1.5),
                     (1024, 1024, 256, 0.5, 1.0), (17, 33, 16, 1, 0), (1, 1, 8, 1, 0),
                     (2048, 2048, 512, 1, 0), (4096, 512, 4096, 1, 0), (255, 257, 264, 1.0, 0.25),
                     (1, 4096, 4096, 1, 0), (4096, 4096, 8, 1, 0), (2047, 1023, 512, 1, 0)]
# Shapes whose fp64 result is pinned (small enough to recompute in a CPU test).
PINNED_RESULTS = [0, 3, 4, 5, 7, 8, 11]


def libc_rand_matrix(seed, shapes_and_mods):
    libc = ctypes.CDLL(ctypes.util.find_library("c"))
    libc.srand(seed)
    out = []
    for (rows, cols), mod, off in shapes_and_mods:
        vals = np.array([libc.rand() % mod - off for _ in range(rows * cols)], np.int64)
        out.append(vals.reshape(rows, cols))
    return out


class MT19937Float:
    """mt19937 + uniform_real_distribution<float>, restated (see module docstring)."""

    def __init__(self, seed):
        self.bg = np.random.MT19937()
        self.bg._legacy_seeding(seed)

    def uniform(self, n, lo, hi):
        u = self.bg.random_raw(n).astype(np.uint64)
        f = u.astype(np.float32)  # uint -> float, round to nearest even
        canon = f / np.float32(4294967296.0)
        canon = np.where(canon >= np.float32(1.0), np.nextafter(np.float32(1), np.float32(0)),
                         canon).astype(np.float32)
        return (canon * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)


def fp64_reference_k_order(A, B, C, alpha, beta):
    """check_fp64.cu:39-44, vectorised over (i, j) but summing k in increasing order."""
    Ad = A.astype(np.float64)
    Bd = B.astype(np.float64)
    acc = np.zeros((A.shape[0], B.shape[1]), np.float64)
    for k in range(A.shape[1]):
        acc += Ad[:, k:k + 1] * Bd[k:k + 1, :]
    r = np.float64(np.float32(alpha)) * acc
    if beta != 0:
        r = r + np.float64(np.float32(beta)) * C.astype(np.float64)
    return r


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    arrays = {}
    # 1. probe KATs
    a0, bt0 = libc_rand_matrix(0, [((64, 64), 7, 3), ((64, 64), 5, 2)])
    arrays["kat_kmajor_A"] = a0.astype(np.float16)
    arrays["kat_kmajor_B"] = np.ascontiguousarray(bt0.T).astype(np.float16)
    arrays["kat_kmajor_C"] = (a0 @ bt0.T).astype(np.int64)
    a1, b1 = libc_rand_matrix(1, [((64, 64), 7, 3), ((64, 128), 5, 2)])
    arrays["kat_mnmajor_A"] = a1.astype(np.float16)
    arrays["kat_mnmajor_B"] = b1.astype(np.float16)
    arrays["kat_mnmajor_C"] = (a1 @ b1).astype(np.int64)
    arrays["kat_mnmajor_C_k16"] = (a1[:, :16] @ b1[:16, :]).astype(np.int64)

    # 2. generator draws
    arrays["mt2024_u11_first4096"] = MT19937Float(2024).uniform(4096, -1.0, 1.0)
    arrays["mt3_u22_first4096"] = MT19937Float(3).uniform(4096, -2.0, 2.0)
    arrays["mt11_u11_first4096"] = MT19937Float(11).uniform(4096, -1.0, 1.0)
    np.savez_compressed(os.path.join(HERE, "reference_kats.npz"), **arrays)

    # 3. check_fp64 suite digests
    g = MT19937Float(3)
    suite = []
    for idx, (M, N, K, al, be) in enumerate(CHECK_FP64_SHAPES):
        A = g.uniform(M * K, -2.0, 2.0).astype(np.float16).reshape(M, K)
        B = g.uniform(K * N, -2.0, 2.0).astype(np.float16).reshape(K, N)
        C = g.uniform(M * N, -2.0, 2.0).astype(np.float16).reshape(M, N)
        entry = {"index": idx, "M": M, "N": N, "K": K, "alpha": al, "beta": be,
                 "A_sha256": sha(A.view(np.uint16)), "B_sha256": sha(B.view(np.uint16)),
                 "C_sha256": sha(C.view(np.uint16))}
        if idx in PINNED_RESULTS:
            entry["ref_f64_sha256"] = sha(fp64_reference_k_order(A, B, C, al, be))
        suite.append(entry)
    with open(os.path.join(HERE, "check_fp64_suite.json"), "w") as f:
        json.dump({"seed": 3, "lo": -2.0, "hi": 2.0, "source": "check_fp64.cu:16-44",
                   "shapes": suite}, f, indent=1)
    print("wrote reference_kats.npz and check_fp64_suite.json")


if __name__ == "__main__":
    main()
