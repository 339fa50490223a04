"""CPU: the C-ABI library loads, exports exactly what include/hgemm_b200.h declares, and its
host-only logic (planner, shard ranges, argument checks) behaves; no GPU calls here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hgemm_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_ ]*?\**\s*\b([a-z_][a-z0-9_]*)\s*\(",
                       text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "sizeof")))


def test_header_declares_reference_entry_point():
    names = declared_functions()
    assert "solve" in names
    assert "hgemm_launch" in names and "hgemm_launch_ex" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    import hopper_gemm_b200._native as nat
    lib = ctypes.CDLL(nat.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python bindings cover exactly the declared set
    assert sorted(nat.SIGNATURES) == declared_functions()


def test_status_strings():
    import hopper_gemm_b200 as hg
    assert hg.status_string(0) == "ok"
    assert "wait" in hg.status_string(hg.HGEMM_ERR_DEVICE_TIMEOUT)
    assert hg.status_string(12345) == "unknown status"


def test_invalid_and_empty_sizes_need_no_device():
    import hopper_gemm_b200 as hg
    from hopper_gemm_b200 import lib
    assert lib.hgemm_launch(None, None, None, -1, 4, 4, 1.0, 0.0, None) == hg.HGEMM_ERR_INVALID_ARG
    # M == 0 or N == 0: a no-op that touches nothing (reference: zero-sized grid)
    assert lib.hgemm_launch(None, None, None, 0, 4, 4, 1.0, 0.0, None) == hg.HGEMM_OK
    assert lib.hgemm_launch(None, None, None, 4, 0, 4, 1.0, 0.0, None) == hg.HGEMM_OK
    lib.solve(None, None, None, 0, 0, 0, 1.0, 0.0)
    # null pointers with real work are rejected before any CUDA call
    assert lib.hgemm_launch(None, None, None, 4, 4, 4, 1.0, 0.0, None) == hg.HGEMM_ERR_INVALID_ARG
    assert hg.last_status() == hg.HGEMM_ERR_INVALID_ARG
    # the host-buffer entry point checks the same before any CUDA call
    assert lib.hgemm_launch_host(None, None, None, None, None, None, -1, 4, 4, 1.0, 0.0,
                                 None) == hg.HGEMM_ERR_INVALID_ARG
    assert lib.hgemm_launch_host(None, None, None, None, None, None, 0, 4, 4, 1.0, 0.0,
                                 None) == hg.HGEMM_OK
    assert lib.hgemm_launch_host(None, None, None, None, None, None, 4, 4, 4, 1.0, 0.0,
                                 None) == hg.HGEMM_ERR_INVALID_ARG


@pytest.mark.parametrize("M,nr", [(32768, 8), (4095, 8), (7, 3), (0, 2), (1, 4)])
def test_shard_rows_partition(M, nr):
    import hopper_gemm_b200 as hg
    covered = []
    for r in range(nr):
        b, c = hg.shard_rows(M, nr, r)
        assert c >= 0
        covered.extend(range(b, b + c))
        assert c in (M // nr, M // nr + 1)
    assert covered == list(range(M))


def test_comparators_load_and_export_their_entry_points():
    """bench.py and the GPU tests' comparators: cuBLAS always, CUTLASS SM100 when it was built
    (the build skips it only where no CUTLASS headers are installed)."""
    import hopper_gemm_b200._native as nat
    assert hasattr(ctypes.CDLL(nat.CUBLAS_REF_PATH), "hgemm_cublas_ref")
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "_hgemm_build", os.path.join(ROOT, "hopper_gemm_b200", "build.py"))
    hb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(hb)
    if hb._cutlass_include() is None:
        pytest.skip("no CUTLASS headers on this machine")
    lib = nat.cutlass_ref_lib()
    assert lib is not None and hasattr(lib, "hgemm_cutlass_ref")
