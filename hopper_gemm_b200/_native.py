"""ctypes bindings for libhgemm_b200.so (the C ABI declared in include/hgemm_b200.h).

The library is built in-tree by hopper_gemm_b200/build.py. There is no CPU or PyTorch
fallback: if the library is missing, importing this module raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhgemm_b200.so")
CUBLAS_REF_PATH = os.path.join(HERE, "libhgemm_cublas_ref.so")
CUTLASS_REF_PATH = os.path.join(HERE, "libhgemm_cutlass_ref.so")

HGEMM_OK = 0
HGEMM_ERR_INVALID_ARG = 1
HGEMM_ERR_CUDA = 2
HGEMM_ERR_TENSOR_MAP = 3
HGEMM_ERR_ALLOC = 4
HGEMM_ERR_LAUNCH = 5
HGEMM_ERR_DEVICE_TIMEOUT = 6
HGEMM_ERR_UNSUPPORTED_DEVICE = 7
HGEMM_ERR_NCCL = 8
HGEMM_ERR_TOO_LARGE = 9
HGEMM_ERR_NOT_FUSABLE = 10


class HgemmPlan(ctypes.Structure):
    _fields_ = [("path", ctypes.c_int), ("tile_m", ctypes.c_int), ("tile_n", ctypes.c_int),
                ("pair", ctypes.c_int), ("group_m", ctypes.c_int), ("stages", ctypes.c_int),
                ("tiles_m", ctypes.c_int), ("tiles_n", ctypes.c_int),
                ("grid_ctas", ctypes.c_int), ("pad_a", ctypes.c_int), ("pad_b", ctypes.c_int),
                ("lda", ctypes.c_int), ("ldb", ctypes.c_int), ("tma_store", ctypes.c_int),
                ("scratch_bytes", ctypes.c_size_t), ("sched_static", ctypes.c_int), ("ksplit", ctypes.c_int),
                ("epi_warps", ctypes.c_int), ("pad_c", ctypes.c_int), ("ldc", ctypes.c_int)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_GEMM = [_vp, _vp, _vp, _i, _i, _i, _f, _f]

# name -> (restype, argtypes); exactly the functions include/hgemm_b200.h declares.
SIGNATURES = {
    "solve": (None, _GEMM),
    "hgemm_launch": (_i, _GEMM + [_vp]),
    "hgemm_launch_ex": (_i, _GEMM + [_vp, _i, _i, _i]),
    "hgemm_launch_tuned": (_i, _GEMM + [_vp]),
    "hgemm_launch_sm_limit": (_i, _GEMM + [_vp, _i]),
    "hgemm_launch_splitk": (_i, _GEMM + [_vp, _i, _i]),
    "hgemm_launch_peers": (_i, _GEMM + [_vp, _vp, _i, _i]),
    "hgemm_launch_noalloc": (_i, _GEMM + [_vp]),
    "hgemm_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "hgemm_launch_host": (_i, [_vp] * 6 + [_i, _i, _i, _f, _f, _vp]),
    "hgemm_last_status": (_i, []),
    "hgemm_status_string": (ctypes.c_char_p, [_i]),
    "hgemm_device_status": (_i, [_i, ctypes.POINTER(_i)]),
    "hgemm_set_wait_timeout_ns": (None, [ctypes.c_ulonglong]),
    "hgemm_selftest_wait_timeout": (_i, [ctypes.c_ulonglong]),
    "hgemm_selftest_peer_barrier": (_i, [ctypes.c_ulonglong]),
    "hgemm_selftest_peer_entry": (_i, [_i, ctypes.c_ulonglong]),
    "hgemm_release": (None, []),
    "hgemm_plan": (_i, [_i, _i, _i, _f, _i, _i, _i, _i, _i, _i, ctypes.POINTER(HgemmPlan)]),
    "hgemm_comm_unique_id": (_i, [_vp, ctypes.c_size_t]),
    "hgemm_comm_init": (_i, [ctypes.POINTER(_vp), _i, _vp, ctypes.c_size_t, _i]),
    "hgemm_comm_destroy": (_i, [_vp]),
    "hgemm_comm_set_reserved_sms": (_i, [_vp, _i]),
    "hgemm_comm_register_output": (_i, [_vp, _vp, ctypes.c_size_t]),
    "hgemm_comm_output_ptr": (_i, [_vp, _i, ctypes.POINTER(_vp)]),
    "hgemm_sharded_rank": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _f, _f, _i, _vp]),
    "hgemm_shard_rows": (_i, [_i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "hgemm_shard_chunk_rows": (_i, [_i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "hgemm_comm_check": (_i, [_vp]),
    "hgemm_comm_abort": (_i, [_vp]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is not built: run `python -c 'import __graft_entry__ as g; g.build()'` "
            "(nvcc, sm_100a). The GEMM has no CPU fallback.")
    # RTLD_LOCAL: the library's exported names stay out of the global symbol scope, so
    # they cannot interpose on another library that exports the same names.
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

_cublas = None


def cublas_ref_lib():
    """The cuBLAS comparator (bench/test infrastructure, not the product)."""
    global _cublas
    if _cublas is None:
        if not os.path.exists(CUBLAS_REF_PATH):
            raise ImportError(f"{CUBLAS_REF_PATH} is not built")
        L = ctypes.CDLL(CUBLAS_REF_PATH)
        L.hgemm_cublas_ref.restype = _i
        L.hgemm_cublas_ref.argtypes = _GEMM + [_vp]
        _cublas = L
    return _cublas


_cutlass = None


def cutlass_ref_lib():
    """The CUTLASS SM100 comparator (bench/test infrastructure, not the product), or None
    when it was not built (no CUTLASS headers on the build machine)."""
    global _cutlass
    if _cutlass is None:
        if not os.path.exists(CUTLASS_REF_PATH):
            return None
        L = ctypes.CDLL(CUTLASS_REF_PATH, mode=ctypes.RTLD_LOCAL)
        L.hgemm_cutlass_ref.restype = _i
        L.hgemm_cutlass_ref.argtypes = _GEMM + [_vp]
        _cutlass = L
    return _cutlass
