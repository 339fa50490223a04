"""CPU: the oracle pinned against the reference's own known answers and generators."""
import hashlib
import json
import os

import numpy as np
import pytest


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def kats(golden_dir):
    return np.load(os.path.join(golden_dir, "reference_kats.npz"))


def test_probe_kmajor_kat_exact(oracle, kats):
    # probe_kmajor.cu:117-125 -- integer inputs, exact answer.
    r = oracle.gemm_f64(kats["kat_kmajor_A"], kats["kat_kmajor_B"])
    assert np.array_equal(r, kats["kat_kmajor_C"].astype(np.float64))


def test_probe_mnmajor_kat_exact(oracle, kats):
    # probe_mnmajor.cu:63-68 (all 64 k, as probe_mnmajor_kadv.cu:65-68 sums them).
    r = oracle.gemm_f64(kats["kat_mnmajor_A"], kats["kat_mnmajor_B"])
    assert np.array_equal(r, kats["kat_mnmajor_C"].astype(np.float64))
    # and the single-k16 slice the first probe checks
    r16 = oracle.gemm_f64(np.ascontiguousarray(kats["kat_mnmajor_A"][:, :16]),
                          np.ascontiguousarray(kats["kat_mnmajor_B"][:16, :]))
    assert np.array_equal(r16, kats["kat_mnmajor_C_k16"].astype(np.float64))


@pytest.mark.parametrize("seed,lo,hi,key", [(2024, -1.0, 1.0, "mt2024_u11_first4096"),
                                            (3, -2.0, 2.0, "mt3_u22_first4096"),
                                            (11, -1.0, 1.0, "mt11_u11_first4096")])
def test_generator_matches_restatement(oracle, kats, seed, lo, hi, key):
    g = oracle.MT19937Stream(seed)
    got = g.uniform_f32(4096, lo, hi)
    assert np.array_equal(got.view(np.uint32), kats[key].view(np.uint32))


def test_check_fp64_suite_pinned(oracle, golden_dir):
    """Replays check_fp64.cu's single mt19937(3) stream over its 15 shapes; inputs and the
    fp64 results of the pinned shapes must match the golden digests bit for bit."""
    with open(os.path.join(golden_dir, "check_fp64_suite.json")) as f:
        suite = json.load(f)
    g = oracle.MT19937Stream(suite["seed"])
    for e in suite["shapes"]:
        M, N, K = e["M"], e["N"], e["K"]
        A = g.uniform_half((M, K), suite["lo"], suite["hi"])
        B = g.uniform_half((K, N), suite["lo"], suite["hi"])
        C = g.uniform_half((M, N), suite["lo"], suite["hi"])
        assert _sha(A.view(np.uint16)) == e["A_sha256"], e["index"]
        assert _sha(B.view(np.uint16)) == e["B_sha256"], e["index"]
        assert _sha(C.view(np.uint16)) == e["C_sha256"], e["index"]
        if "ref_f64_sha256" in e:
            r = oracle.gemm_f64(A, B, C, e["alpha"], e["beta"])
            assert _sha(r) == e["ref_f64_sha256"], e["index"]


def test_half_rounding_matches_numpy(oracle):
    rs = np.random.RandomState(0)
    for scale in (1e-7, 1e-5, 1e-2, 1.0, 1e3, 6e4, 7e4):
        x = (rs.randn(50000) * scale).astype(np.float32)
        assert np.array_equal(oracle.f32_to_f16(x).view(np.uint16),
                              x.astype(np.float16).view(np.uint16)), scale


def test_reference_loop_order_bit_identical(oracle):
    rs = np.random.RandomState(5)
    A = rs.uniform(-1, 1, (33, 70)).astype(np.float16)
    B = rs.uniform(-1, 1, (70, 41)).astype(np.float16)
    C = rs.uniform(-1, 1, (33, 41)).astype(np.float16)
    fast = oracle.gemm_f64(A, B, C, 1.5, 0.5)
    lit = oracle.gemm_f64_ref_order(A, B, C, 1.5, 0.5)
    cols = oracle.gemm_f64_cols(A, B, np.arange(41), C, 1.5, 0.5)
    assert np.array_equal(fast, lit)
    assert np.array_equal(fast, cols)


def test_hash_fill_matches_three_way_formula(oracle):
    seed = 0x9E3779B9
    got = oracle.hash_fill_half((1000,), seed, offset=123).astype(np.float32)
    i = np.arange(123, 1123, dtype=np.uint64)
    h = ((i * np.uint64(2654435761)) & np.uint64(0xFFFFFFFF)) ^ np.uint64(seed)
    h ^= h >> np.uint64(15)
    h = (h * np.uint64(2246822519)) & np.uint64(0xFFFFFFFF)
    h ^= h >> np.uint64(13)
    h = (h * np.uint64(3266489917)) & np.uint64(0xFFFFFFFF)
    h ^= h >> np.uint64(16)
    want = ((h & np.uint64(0xFFFF)).astype(np.float32) / np.float32(32768.0) - np.float32(1.0))
    assert np.array_equal(got, want.astype(np.float16).astype(np.float32))


def test_tolerance_rejects_planted_error(oracle):
    """A mistake planted in a copy of the oracle's answer must be caught by the checker."""
    rs = np.random.RandomState(9)
    A = rs.uniform(-1, 1, (16, 256)).astype(np.float16)
    B = rs.uniform(-1, 1, (256, 24)).astype(np.float16)
    ref = oracle.gemm_f64(A, B)
    good = ref.astype(np.float16)
    assert oracle.check(good, ref, 256)[0]
    bad = good.copy()
    bad[3, 7] = np.float16(float(bad[3, 7]) + 0.5)
    assert not oracle.check(bad, ref, 256)[0]
