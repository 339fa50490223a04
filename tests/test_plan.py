"""CPU: the per-shape dispatcher (the B200 counterpart of launch_mainloop / launch,
mma_half.cu:1441-1563), exercised through the host-only hgemm_plan()."""
import pytest

import hopper_gemm_b200 as hg

B200 = dict(sm_count=148, pair_slots=74)


def test_noop_and_fallback_paths():
    assert hg.plan(0, 128, 64, **B200)["path"] == 0
    assert hg.plan(128, 0, 64, **B200)["path"] == 0
    # K == 0 takes the scalar kernel (C = beta * C)
    assert hg.plan(128, 128, 0, **B200)["path"] == 2
    # pointers off a 16-byte boundary: A and B are restrided like ragged operands and C is
    # written in place by the SIMT-store epilogue (beta != 0 too: no padded copy of C)
    for beta in (0.0, 0.5):
        for N in (128, 127):
            p = hg.plan(128, N, 64, beta=beta, aligned16=False, **B200)
            assert p["path"] == 1
            assert (p["pad_a"], p["pad_b"], p["pad_c"], p["tma_store"]) == (1, 1, 0, 0)
            assert p["ldc"] == N
            assert p["scratch_bytes"] == 2 * (128 * p["lda"] + 64 * p["ldb"])


@pytest.mark.parametrize("M,N,K,beta,pad_a,pad_b,pad_c,tma", [
    (4095, 4095, 4095, 0.0, 1, 1, 0, 0),   # both operands restrided, SIMT stores (N odd)
    (4095, 4095, 4095, 0.5, 1, 1, 1, 1),   # beta != 0: C computed in a padded copy
    (4096, 4095, 4096, 0.0, 0, 1, 0, 0),
    (4096, 4095, 4096, 0.5, 0, 1, 1, 1),
    (2048, 2047, 2048, 0.5, 0, 1, 1, 1),
    (3000, 1000, 2000, 0.5, 0, 0, 0, 1),   # aligned strides, ragged tiles only
    (1023, 1, 1025, 0.0, 1, 1, 0, 0),
    (8192, 8192, 8192, 0.0, 0, 0, 0, 1),
])
def test_restride_and_padded_c(M, N, K, beta, pad_a, pad_b, pad_c, tma):
    p = hg.plan(M, N, K, beta=beta, **B200)
    assert p["path"] == 1
    assert (p["pad_a"], p["pad_b"], p["pad_c"], p["tma_store"]) == (pad_a, pad_b, pad_c, tma)
    assert p["lda"] % 8 == 0 and p["ldb"] % 8 == 0
    assert p["lda"] >= K and p["ldb"] >= N and p["ldc"] >= N
    assert p["ldc"] == (p["ldb"] if pad_c else N)
    want = 2 * ((M * p["lda"] if pad_a else 0) + (K * p["ldb"] if pad_b else 0) +
                (M * p["ldc"] if pad_c else 0))
    assert p["scratch_bytes"] == want


def test_large_square_uses_widest_pair_tile():
    # enough tiles to fill the machine several times: the 256x512 pair tile (fewest operand
    # bytes per flop) is chosen
    p = hg.plan(8192, 8192, 8192, **B200)
    assert (p["tile_m"], p["tile_n"], p["pair"]) == (256, 512, 2)
    assert p["grid_ctas"] == 2 * 32 * 16 and p["stages"] >= 3
    assert 1 <= p["group_m"] <= p["tiles_m"]


def test_small_problem_spreads_over_sms():
    p = hg.plan(1024, 1024, 1024, **B200)
    assert p["grid_ctas"] >= 64  # uses at least 64 SMs
    # a handful of tiles would leave most SMs idle: split-K clusters of one-CTA tiles
    p = hg.plan(256, 256, 4096, **B200)
    assert p["ksplit"] > 1 and p["pair"] == 1
    assert p["grid_ctas"] == p["tiles_m"] * p["tiles_n"] * p["ksplit"] <= 148


@pytest.mark.parametrize("bm,bn", [(256, 512), (256, 256), (256, 128), (128, 256), (128, 128),
                                   (128, 64)])
def test_forced_tiles(bm, bn):
    p = hg.plan(2048, 2048, 512, force_bm=bm, force_bn=bn, **B200)
    assert (p["tile_m"], p["tile_n"]) == (bm, bn)
    assert p["pair"] == bm // 128
    assert p["grid_ctas"] % p["pair"] == 0


def test_invalid_forced_tile_rejected():
    with pytest.raises(hg.HgemmError):
        hg.plan(256, 256, 256, force_bm=64, force_bn=64, **B200)
    with pytest.raises(hg.HgemmError):
        hg.plan(256, 256, 256, force_bm=256, force_bn=64, **B200)


def test_grid_is_one_cluster_per_tile():
    for M, N, K in [(16384, 16384, 16384), (384, 2048, 2048), (1, 4096, 4096), (8192, 8, 8192)]:
        p = hg.plan(M, N, K, **B200)
        assert p["grid_ctas"] == p["tiles_m"] * p["tiles_n"] * p["pair"] * p["ksplit"]


def test_schedule_choice():
    # long tiles: one cluster per tile, the running clusters take over the rest
    p = hg.plan(8192, 8192, 8192, **B200)
    assert p["sched_static"] == 0
    # short tiles (K = 128): persistent clusters, one per slot, static tile order
    p = hg.plan(4096, 8192, 128, **B200)
    assert p["sched_static"] == 1
    slots = B200["pair_slots"] if p["pair"] == 2 else B200["sm_count"]
    assert p["grid_ctas"] == min(p["tiles_m"] * p["tiles_n"], slots) * p["pair"]
    # every tile co-resident: static, one cluster per tile
    p = hg.plan(2048, 2048, 2048, **B200)
    assert p["sched_static"] == 1 and p["ksplit"] == 1
    assert p["grid_ctas"] == p["tiles_m"] * p["tiles_n"] * p["pair"]


def test_split_k_choice():
    # big enough to fill the machine: never split
    for shape in [(8192, 8192, 8192), (4096, 8192, 128), (2048, 2048, 512), (1024, 1024, 1024),
                  (384, 2048, 2048)]:
        assert hg.plan(*shape, **B200)["ksplit"] == 1
    # a handful of tiles: split, at most 8 per cluster, at least 4 k-blocks per split
    for M, N, K in [(256, 256, 4096), (128, 128, 8192), (512, 512, 8192)]:
        p = hg.plan(M, N, K, **B200)
        assert 2 <= p["ksplit"] <= 8 and p["pair"] == 1
        assert (K + 63) // 64 >= 4 * p["ksplit"]
        assert p["grid_ctas"] <= 148
    # ragged N has no TMA-store epilogue: no split
    assert hg.plan(384, 2046, 2048, **B200)["ksplit"] == 1
