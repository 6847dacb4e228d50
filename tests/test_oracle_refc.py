"""The numpy row-ops restatement (oracle/spec.py) against the reference's own
C++ row-ops oracle (rowops_ref.h, compiled by oracle/Makefile into
oracle/_ref/) on the fixture jobs and on seeded random jobs; and the compiled
oracle against the reference's chain fixtures.  Skipped when the reference
build is absent (it is made by __graft_entry__.build() where the reference
checkout exists)."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import spec
from tests import fixtures as fx

SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "librowops_ref.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(SO):
        pytest.skip("oracle/_ref/librowops_ref.so not built")
    L = C.CDLL(SO)
    L.ro_ref_run.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_int]
    L.ro_ref_run.restype = C.c_int
    return L


def run_ref(L, mem, jobs):
    regs = np.array([[int(v) for v in j] + [0] * (20 - len(j)) for j in jobs], np.uint64)
    assert L.ro_ref_run(mem.ctypes.data, mem.size, regs.ctypes.data, len(jobs)) == 0


def test_fixtures_ref_c(ref, golden):
    z = golden("hw_rowops.npz")
    for label, r, a, b, p, cexp in fx.rowops_cases(z):
        mem, off = fx.rowops_memory(a, b, p, len(cexp))
        run_ref(ref, mem, [[r["op"], r["n"], r["c1"], r["c2"], off["a"], r["a_s1"], r["a_s2"], off["b"], r["b_s1"],
                            r["b_s2"], off["c"], r["c_s1"], r["c_s2"], off["p"], r["eps"], r["aux"], r["bq_sh"],
                            r["win_lo"], r["win_hi"]]])
        assert np.array_equal(mem[off["c"]:off["c"] + len(cexp)], cexp), label


def test_chain_fixtures_ref_c(ref, golden):
    z = golden("hw_rowops.npz")
    cp = z["chain_params"]
    for ci in sorted(set(int(v) for v in cp[:, 0])):
        mem = z[f"chain{ci}_mem"].copy()
        jobs = [list(row[2:21]) for row in cp if int(row[0]) == ci]
        run_ref(ref, mem, jobs)
        assert np.array_equal(mem, z[f"chain{ci}_out"]), ci


@pytest.mark.parametrize("seed", range(12))
def test_random_jobs_numpy_vs_ref_c(ref, seed):
    rng = np.random.default_rng(seed)
    code = [1, 2, 3, 4, 5, 6, 10][seed % 7]
    ak = int(rng.integers(0, 2)) if code in (1, 2, 3, 5) else 0
    ck = (2 if code == 3 else int(rng.integers(0, 2))) if code in (1, 2, 3) else 0
    op = code | (ak << 4) | (ck << 8) | (spec.F_B_EN if code in (1, 2, 4, 10) else 0)
    if code == 5 and rng.integers(0, 2):
        op |= spec.F_NORM_LN
    if code in (1, 2) and rng.integers(0, 2):
        op |= spec.F_RELU
    n = 64 if code == 6 else int(rng.integers(1, 300))
    rows = int(rng.integers(1, 5))
    row_b = (n * 4 + 15) // 16 * 16
    mem = rng.integers(0, 256, size=4 * rows * row_b + 32 * n + 4096).astype(np.uint8)
    oa, ob, op_ = 0, rows * row_b, 2 * rows * row_b
    oc = op_ + ((16 * n + 255) // 256) * 256
    pb = mem[op_:op_ + 16 * n].reshape(n, 16)
    pb[:, 8] = rng.integers(0, 6, size=n)
    pb[:, 9] = rng.integers(0, 6, size=n)
    pb[:, 10] = rng.integers(8, 40, size=n)
    mem[op_:op_ + 16 * n] = pb.reshape(-1)
    job = [op, n, rows, 1, oa, row_b, 0, ob, 0 if code == 6 else row_b, 0, oc, row_b, 0, op_,
           int(rng.integers(0, 1 << 20)), 64 if code == 6 else 0, int(rng.integers(0, 8)), 0, 0xFFFFFFFF]
    m1 = mem.copy()
    run_ref(ref, m1, [job])
    m2 = spec.RowOpsMem(mem.copy())
    spec.rowops_job(m2, *job)
    assert np.array_equal(m1, m2.buf)
