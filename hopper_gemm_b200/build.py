"""Build recipe for the in-tree CUDA libraries (sm_100a only).

Produces, next to this file:
  libhgemm_b200.so       the GEMM product: tcgen05 kernel, dispatcher, C ABI, NCCL row shards,
                         host-buffer pipeline
  libhgemm_cublas_ref.so the cuBLAS comparator used by bench.py and the GPU tests
  libhgemm_cutlass_ref.so the CUTLASS SM100 comparator (third grid column, cross-check tests),
                         built when CUTLASS's headers are found (the copies vendored in the
                         flashinfer or tilelang wheels); skipped with a notice otherwise
Both are compiled with `-gencode arch=compute_100a,code=sm_100a`; nvcc cross-compiles them on
a machine without a GPU.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB = os.path.join(HERE, "libhgemm_b200.so")
CUBLAS_LIB = os.path.join(HERE, "libhgemm_cublas_ref.so")
CUTLASS_LIB = os.path.join(HERE, "libhgemm_cutlass_ref.so")


def _cutlass_include():
    """CUTLASS include dirs (include/ and tools/util/include/) from an installed wheel that
    vendors them, located without importing the package; None if there is none."""
    import importlib.util
    for pkg, sub in (("flashinfer", ("data", "cutlass")), ("tilelang", ("3rdparty", "cutlass"))):
        try:
            spec = importlib.util.find_spec(pkg)
        except (ImportError, ValueError):
            spec = None
        if not spec or not spec.submodule_search_locations:
            continue
        root = os.path.join(list(spec.submodule_search_locations)[0], *sub)
        inc, util = os.path.join(root, "include"), os.path.join(root, "tools", "util", "include")
        if os.path.exists(os.path.join(inc, "cutlass", "gemm", "collective",
                                       "collective_builder.hpp")) and os.path.isdir(util):
            return [inc, util]
    return None


def _nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force=False, verbose=True, extra_flags=()):
    nvcc = _nvcc()
    common = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE,
                     "-I" + CSRC] + list(extra_flags)
    srcs = [os.path.join(CSRC, f) for f in ("hgemm_sm100.cu", "hgemm_sharded.cpp", "hgemm_host.cpp")]
    deps = srcs + [os.path.join(CSRC, "ptx_sm100.cuh"), os.path.join(INCLUDE, "hgemm_b200.h")]
    if force or _stale(LIB, deps):
        _run([nvcc] + common + ["-shared", "-o", LIB] + srcs + ["-ldl"], verbose)
    csrc = [os.path.join(CSRC, "cublas_ref.cu")]
    if force or _stale(CUBLAS_LIB, csrc):
        _run([nvcc] + common + ["-shared", "-o", CUBLAS_LIB] + csrc + ["-lcublas"], verbose)
    tsrc = [os.path.join(CSRC, "cutlass_ref.cu")]
    if force or _stale(CUTLASS_LIB, tsrc):
        inc = _cutlass_include()
        if inc is None:
            print("note: CUTLASS headers not found; libhgemm_cutlass_ref.so (comparator) skipped",
                  flush=True)
        else:
            _run([nvcc] + common + ["--expt-relaxed-constexpr"] + ["-I" + d for d in inc] +
                 ["-shared", "-o", CUTLASS_LIB] + tsrc, verbose)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
