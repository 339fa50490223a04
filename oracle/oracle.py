"""TEST INFRASTRUCTURE ONLY: ctypes front end of the CPU oracle (oracle/liboracle.so).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg -- never by the
GEMM product. It restates the reference's host fp64 GEMM (check_fp64.cu:39-44) and the
seeded input generators of the reference's harnesses (check_*.cu, three_way.cu:22-33); see
hgemm_oracle.cpp for the line-by-line correspondence.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f64p = ctypes.POINTER(ctypes.c_double)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)


def build(force=False):
    src = os.path.join(HERE, "hgemm_oracle.cpp")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(LIB_PATH):
        subprocess.run(["make", "-C", HERE, "-B", "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return LIB_PATH


def build_ref():
    """Builds the reference's own correctness harnesses against this repository's GEMM library
    (oracle/_ref/, see oracle/Makefile `ref`). Needs the reference checkout; where it is absent
    (e.g. on a GPU box that only runs the prebuilt binaries) this reports False and leaves any
    binaries already there untouched."""
    r = subprocess.run(["make", "-C", HERE, "ref"], stdout=subprocess.PIPE,
                       stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        print("note: reference harnesses not rebuilt: " + r.stdout.strip().splitlines()[-1]
              if r.stdout.strip() else "note: reference harnesses not rebuilt", flush=True)
    return r.returncode == 0


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_gemm_f64_rows.argtypes = [_u16p, _u16p, _u16p, _f64p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_double, ctypes.c_double, _i32p,
                                           ctypes.c_int, ctypes.c_int]
        L.oracle_gemm_f64_cols.argtypes = L.oracle_gemm_f64_rows.argtypes
        L.oracle_gemm_f64_ref_order.argtypes = [_u16p, _u16p, _u16p, _f64p, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                                ctypes.c_double, ctypes.c_int, ctypes.c_int]
        L.oracle_mt_new.restype = ctypes.c_void_p
        L.oracle_mt_new.argtypes = [ctypes.c_uint32]
        L.oracle_mt_free.argtypes = [ctypes.c_void_p]
        L.oracle_mt_uniform_half.argtypes = [ctypes.c_void_p, _u16p, ctypes.c_size_t,
                                             ctypes.c_float, ctypes.c_float]
        L.oracle_mt_uniform_f32.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_size_t,
                                            ctypes.c_float, ctypes.c_float]
        L.oracle_mt_normal_half.argtypes = L.oracle_mt_uniform_half.argtypes
        L.oracle_hash_fill_half.argtypes = [_u16p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_size_t]
        L.oracle_f32_to_f16_array.argtypes = [_f32p, _u16p, ctypes.c_size_t]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _halfbits(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    assert a.dtype == np.uint16
    return a


def gemm_f64(A, B, C=None, alpha=1.0, beta=0.0, rows=None, threads=0):
    """fp64 reference: alpha * A @ B + beta * C for the listed rows (all rows by default).

    A (M x K), B (K x N), C (M x N) are float16 (or their uint16 bit patterns)."""
    A, B = _halfbits(A), _halfbits(B)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    if beta != 0.0:
        assert C is not None
        Cb = _halfbits(C)
    else:
        Cb = np.zeros((1, 1), np.uint16)
    rows = np.arange(M, dtype=np.int32) if rows is None else np.ascontiguousarray(rows, np.int32)
    out = np.empty((len(rows), N), np.float64)
    lib().oracle_gemm_f64_rows(_p(A, _u16p), _p(B, _u16p), _p(Cb, _u16p), _p(out, _f64p), M, N, K,
                               float(alpha), float(beta), _p(rows, _i32p), len(rows), int(threads))
    return out


def gemm_f64_cols(A, B, cols, C=None, alpha=1.0, beta=0.0, threads=0):
    """fp64 reference for the listed columns of C, all rows: result is M x len(cols)."""
    A, B = _halfbits(A), _halfbits(B)
    M, K = A.shape
    N = B.shape[1]
    Cb = _halfbits(C) if beta != 0.0 else np.zeros((1, 1), np.uint16)
    cols = np.ascontiguousarray(cols, np.int32)
    if len(cols) >= 64:
        # Many columns: the row kernel on B's (and C's) selected columns gives the same sums
        # in the same k order, blocked and vectorised.
        Bs = np.ascontiguousarray(B[:, cols])
        Cs = np.ascontiguousarray(Cb[:, cols]) if beta != 0.0 else None
        return gemm_f64(A, Bs, Cs, alpha, beta, threads=threads)
    out = np.empty((M, len(cols)), np.float64)
    lib().oracle_gemm_f64_cols(_p(A, _u16p), _p(B, _u16p), _p(Cb, _u16p), _p(out, _f64p), M, N, K,
                               float(alpha), float(beta), _p(cols, _i32p), len(cols), int(threads))
    return out


def gemm_f64_ref_order(A, B, C=None, alpha=1.0, beta=0.0, row_begin=0, row_end=None):
    """The reference's literal i-j-k loop, single thread (for timing the CPU baseline)."""
    A, B = _halfbits(A), _halfbits(B)
    M, K = A.shape
    N = B.shape[1]
    row_end = M if row_end is None else row_end
    Cb = _halfbits(C) if beta != 0.0 else np.zeros((1, 1), np.uint16)
    out = np.empty((row_end - row_begin, N), np.float64)
    lib().oracle_gemm_f64_ref_order(_p(A, _u16p), _p(B, _u16p), _p(Cb, _u16p), _p(out, _f64p),
                                    M, N, K, float(alpha), float(beta), row_begin, row_end)
    return out


class MT19937Stream:
    """std::mt19937(seed) shared across draws, as the reference harnesses use one engine for
    every matrix of every shape in order (check_all.cu:14, check_fp64.cu:16)."""

    def __init__(self, seed):
        self._g = lib().oracle_mt_new(seed)

    def __del__(self):
        if getattr(self, "_g", None):
            lib().oracle_mt_free(self._g)
            self._g = None

    def uniform_half(self, shape, lo=-1.0, hi=1.0):
        out = np.empty(shape, np.uint16)
        lib().oracle_mt_uniform_half(self._g, _p(out, _u16p), out.size, lo, hi)
        return out.view(np.float16)

    def uniform_f32(self, n, lo=-1.0, hi=1.0):
        out = np.empty(n, np.float32)
        lib().oracle_mt_uniform_f32(self._g, _p(out, _f32p), n, lo, hi)
        return out

    def normal_half(self, shape, mean=0.0, std=1.0):
        out = np.empty(shape, np.uint16)
        lib().oracle_mt_normal_half(self._g, _p(out, _u16p), out.size, mean, std)
        return out.view(np.float16)


def hash_fill_half(shape, seed, offset=0):
    """three_way.cu:22-33 counter-hash fill (values k/32768 - 1 rounded to half)."""
    out = np.empty(shape, np.uint16)
    lib().oracle_hash_fill_half(_p(out, _u16p), out.size, seed & 0xFFFFFFFF, offset)
    return out.view(np.float16)


def f32_to_f16(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_f32_to_f16_array(_p(x, _f32p), _p(out, _u16p), x.size)
    return out.view(np.float16)


def max_threads():
    return lib().oracle_max_threads()


def tolerance(ref, K):
    """north_star's per-element bound: |C - C_ref| <= 1e-2 |C_ref| + 2e-3 sqrt(K)."""
    return 1e-2 * np.abs(ref) + 2e-3 * np.sqrt(max(K, 1))


def check(out_half, ref, K):
    """(ok, worst_ratio, rel_l2) of a half result against the fp64 reference."""
    o = np.asarray(out_half, np.float64)
    err = np.abs(o - ref)
    tol = tolerance(ref, K)
    worst = float(np.max(err / tol)) if err.size else 0.0
    den = float(np.sum(ref * ref))
    rel_l2 = float(np.sqrt(np.sum(err * err) / (den + 1e-30)))
    return bool(np.all(err <= tol)), worst, rel_l2
