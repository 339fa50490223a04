"""GPU: the reference's own correctness harnesses, compiled unchanged against this library.

oracle/Makefile (`make ref`, run by build()) compiles yz-wqf/Hopper_GEMM's check_fp64.cu,
check_all.cu and check_large.cu for sm_100a with their `#include "mma_half.cu"` resolved to
oracle/ref_shim/mma_half.cu, so their calls of `solve` and `h100_hgemm::launch` reach
libhgemm_b200.so. Each binary generates its own mt19937 inputs, runs this library's GEMM on
the GPU and judges the result with its own code and its own bars:
  * check_fp64: 15 shapes against its host fp64 loop, rel_l2 < 5e-3 (check_fp64.cu:39-47);
  * check_all: 57 shapes against cuBLAS, rel_l2 < 3e-3, exit status 1 on any failure
    (check_all.cu:66-78);
  * check_large: 12 large and odd-N shapes against cuBLAS, rel_l2 < 3e-3 (check_large.cu:18-63).
The check_fp64 rows also pin this repository's CPU oracle to the reference's own fp64 code:
for the same inputs (the oracle's mt19937 restatement) and the same GEMM output (the kernel
is deterministic), the oracle must reproduce the max_abs and rel_l2 the reference printed,
digit for digit."""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")

ROW = re.compile(r"^(\d+),(\d+),(\d+)\s+(-?[\d.]+)\s+(-?[\d.]+)\s+(\S+)\s+(\S+)\s+(.*)$")


def _run(name, *args, timeout=900):
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        pytest.fail(f"{path} is not built: run `make -C oracle ref` (build() does)")
    p = subprocess.run([path, *args], capture_output=True, text=True, timeout=timeout)
    return p.returncode, p.stdout, p.stderr


def _rows(out):
    rows = []
    for line in out.splitlines():
        m = ROW.match(line.strip())
        if m:
            M, N, K = (int(m.group(i)) for i in (1, 2, 3))
            rows.append((M, N, K, float(m.group(4)), float(m.group(5)), m.group(6), m.group(7),
                         m.group(8)))
    return rows


def test_reference_check_all(cuda):
    rc, out, err = _run("check_all")
    rows = _rows(out)
    assert len(rows) == 57, out[-2000:] + err[-2000:]
    # each row ends with its source tag and the harness's verdict ("OK" or "*** FAIL ***")
    bad = [r for r in rows if r[7].split()[-1] != "OK" or "FAIL" in r[7]]
    assert not bad, bad
    assert "57 shapes, 0 failures" in out
    assert rc == 0


def test_reference_check_large(cuda):
    rc, out, err = _run("check_large")
    rows = _rows(out)
    assert len(rows) == 12, out[-2000:] + err[-2000:]
    # each row's verdict ("OK" or "*** FAIL ***") comes before the row's note
    bad = [r for r in rows if r[7].split()[0] != "OK" or "FAIL" in r[7]]
    assert not bad, bad
    assert rc == 0


def test_reference_check_fp64_and_oracle_pin(cuda, oracle):
    rc, out, err = _run("check_fp64", "3")
    assert rc == 0, err[-2000:]
    corr = out.split("== performance")[0]
    rows = []
    for line in corr.splitlines():
        p = line.split()
        if len(p) == 6 and p[0].count(",") == 2:
            rows.append(p)
    assert len(rows) == 15, corr
    assert all(r[5] == "OK" for r in rows), rows
    # The oracle against the reference's own fp64 loop, on the reference's own inputs.
    g = oracle.MT19937Stream(3)
    for r in rows:
        M, N, K = (int(v) for v in r[0].split(","))
        al, be = float(r[1]), float(r[2])
        A = g.uniform_half((M, K), -2.0, 2.0)
        B = g.uniform_half((K, N), -2.0, 2.0)
        C = g.uniform_half((M, N), -2.0, 2.0)
        import torch
        dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C))
        cuda.solve(dA, dB, dC, M, N, K, al, be)
        assert cuda.last_status() == 0
        out_k = dC.cpu().numpy().astype(np.float64)
        ref = oracle.gemm_f64(A, B, C, al, be)
        e = np.abs(out_k - ref)
        ma = float(e.max())
        l2 = float(np.sqrt(np.sum(e * e) / (np.sum(ref * ref) + 1e-30)))
        assert f"{ma:.3e}" == r[3] and f"{l2:.3e}" == r[4], (r, f"{ma:.3e}", f"{l2:.3e}")
    # the harness's own performance section ran through h100_hgemm::launch
    perf = out.split("== performance")[1]
    assert len([l for l in perf.splitlines() if re.match(r"^\d+x\d+x\d+\s", l)]) == 5, perf
