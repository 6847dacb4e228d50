"""The Xilinx-style drivers a generated inference.c calls
(include/cormorant_b200_xdrv.h: X*_Set_* / Start / IsDone over the C ABI) on
the reference's register-level fixtures: a C program (tests/xdrv/xdrv_run.c,
compiled here with gcc against libcorm_b200.so and the CUDA runtime) programs
every VectorOP, MatMul, Conv, Pool and RowOps case and the row-ops descriptor
chains (a device-memory descriptor list) through the drivers; the outputs
must equal the fixtures'."""
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

from tests import fixtures as fx

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = "/usr/local/cuda"


@pytest.fixture(scope="module")
def runner(tmp_path_factory):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not shutil.which("gcc"):
        pytest.skip("no gcc")
    from cormorant_b200 import _lib
    _lib.lib()  # built in-tree
    d = tmp_path_factory.mktemp("xdrv")
    exe = str(d / "xdrv_run")
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-I",
                    f"{CUDA}/include", os.path.join(ROOT, "tests", "xdrv", "xdrv_run.c"), "-o", exe, "-L", lib_dir,
                    "-lcorm_b200", "-L", f"{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{lib_dir}",
                    f"-Wl,-rpath,{CUDA}/lib64"], check=True)
    return exe, d


class Jobs:
    def __init__(self):
        self.bufs, self.jobs = [], []

    def buf(self, data=None, nbytes=None):
        b = bytes(np.ascontiguousarray(data).view(np.uint8)) if data is not None else None
        self.bufs.append((len(b) if b is not None else int(nbytes), b))
        return len(self.bufs)  # address of buffer i: (i + 1) << 40

    @staticmethod
    def at(b, off=0):
        return (b << 40) | off if b else 0

    def job(self, kind, regs):
        self.jobs.append((kind, [int(v) & 0xFFFFFFFFFFFFFFFF for v in regs]))

    def run(self, runner):
        exe, d = runner
        inp, out = str(d / "jobs.bin"), str(d / "out.bin")
        with open(inp, "wb") as f:
            f.write(struct.pack("<III", 0x56524458, len(self.bufs), len(self.jobs)))
            for n, b in self.bufs:
                f.write(struct.pack("<QB", n, b is not None))
                if b is not None:
                    f.write(b)
            for kind, regs in self.jobs:
                f.write(struct.pack("<II", kind, len(regs)) + struct.pack(f"<{len(regs)}Q", *regs))
        r = subprocess.run([exe, inp, out], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        raw = open(out, "rb").read()
        res, pos = [], 0
        for n, _b in self.bufs:
            res.append(raw[pos:pos + n])
            pos += n
        return res


POISON = -8531


def test_xdrv_vectorop_matmul_pool(runner, golden):
    J, checks = Jobs(), []
    for label, regs, a, b, c_len, check in fx.vecop_cases(golden("hw_vecop.npz")):
        ba, bb = J.buf(a), J.buf(b)
        bc = J.buf(np.full(max(c_len, 1) + 8, POISON, np.int16))
        J.job(0, [J.at(ba), J.at(bb), J.at(bc)] + [regs[k] for k in ("size", "op", "outer", "a_inc", "b_inc", "act",
                                                                       "alpha", "smx_cm", "smx_cfg", "smx_mask")])
        checks.append(("vop", label, bc, check))
    for label, regs, a, b, cv in fx.matmul_cases(golden("hw_matmul.npz")):
        ba = J.buf(np.concatenate([a, np.zeros(8, np.int16)]))
        bb = J.buf(np.concatenate([b, np.zeros(8, np.int16)]))
        bc = J.buf(np.full(max(1, regs["batch"] * regs["c_batch_stride"]), POISON, np.int16))
        J.job(1, [J.at(ba), J.at(bb), J.at(bc)] + [regs[k] for k in ("n", "k", "m", "batch", "a_batch_stride",
                                                                       "b_batch_stride", "c_batch_stride", "b_packed",
                                                                       "gemv_kw")])
        checks.append(("mm", label, bc, cv))
    for label, r, x, y in fx.pool_cases(golden("hw_pool.npz")):
        bx, by = J.buf(x), J.buf(np.full(len(y), POISON, np.int16))
        J.job(3, [J.at(bx), J.at(by)] + list(r.values()))
        checks.append(("pool", label, by, y))
    out = J.run(runner)
    fails = []
    for kind, label, bi, exp in checks:
        got = np.frombuffer(out[bi - 1], np.int16)
        ok = (not exp(got)) if kind == "vop" else np.array_equal(got[:len(exp)], exp)
        if not ok:
            fails.append((kind, label))
    assert not fails, fails[:8]


def test_xdrv_conv_rowops_chains(runner, golden):
    J, checks = Jobs(), []
    for label, r, x, w, b, y in fx.conv_cases(golden("hw_conv.npz")):
        P = r["out_h"] * r["out_w"]
        CS = r["y_cs"] or P
        offs = [((m % r["y_cn"]) * CS + (m // r["y_cn"]) * r["y_gs"] if r["y_cn"] else m * CS)
                for m in range(r["out_ch"])]
        span = r["batch"] * r["out_ch"] * P if not (r["y_cn"] or r["y_cs"]) else max(offs) + P
        bx, bw = J.buf(x), J.buf(w)
        bb = J.buf(b) if r["has_bias"] else 0
        by = J.buf(np.full(span, POISON, np.int16))
        J.job(2, [J.at(bx), J.at(bw), J.at(bb), J.at(by)] + list(r.values()))
        checks.append(("conv", label, by, (r, y, offs, P)))
    zr = golden("hw_rowops.npz")
    for label, r, a, b, p, cexp in fx.rowops_cases(zr):
        mem, off = fx.rowops_memory(a, b, p, len(cexp))
        bm = J.buf(mem)
        J.job(4, [J.at(bm, off["a"]), J.at(bm, off["b"]), J.at(bm, off["c"]), J.at(bm, off["p"]), 0, r["eps"], r["op"],
                  r["n"], r["c1"], r["c2"], r["a_s1"], r["a_s2"], r["b_s1"], r["b_s2"], r["c_s1"], r["c_s2"], r["aux"],
                  r["bq_sh"], r["win_lo"], r["win_hi"], 0])
        checks.append(("ro", label, bm, (off["c"], cexp)))
    cp = zr["chain_params"]
    for ci in sorted(set(int(v) for v in cp[:, 0])):
        bm = J.buf(zr[f"chain{ci}_mem"])
        words = []
        for row in cp[cp[:, 0] == ci]:
            (op, n, c1, c2, a, a1, a2, b, b1, b2, c, c1s, c2s, p, eps, aux, bq, wl, wh) = (int(v) for v in row[2:21])
            w = [op, n, c1, c2, a, 0, a1, a2, b, 0, b1, b2, c, 0, c1s, c2s, p, 0, eps & 0xFFFFFFFF, eps >> 32, aux, bq,
                 wl, wh] + [0] * 8
            for lo in (4, 8, 12, 16):  # offsets into the chain's memory, as buffer addresses
                v = J.at(bm, w[lo])
                w[lo], w[lo + 1] = v & 0xFFFFFFFF, v >> 32
            words.append(w)
        bd = J.buf(np.array(words, np.uint32).reshape(-1))
        J.job(5, [J.at(bd), len(words)])            # the list in device memory, device addresses
        J.job(4, [0, 0, 0, 0, J.at(bd)] + [0] * 15 + [len(words)])
        checks.append(("chain", ci, bm, zr[f"chain{ci}_out"]))
    out = J.run(runner)
    fails = []
    for kind, label, bi, exp in checks:
        got = np.frombuffer(out[bi - 1], np.uint8 if kind in ("ro", "chain") else np.int16)
        if kind == "conv":
            r, y, offs, P = exp
            ok = (all(np.array_equal(got[o:o + P], y[m * P:(m + 1) * P]) for m, o in enumerate(offs))
                  if (r["y_cn"] or r["y_cs"]) else np.array_equal(got, y))
        elif kind == "ro":
            c0, cexp = exp
            ok = np.array_equal(got[c0:c0 + len(cexp)], cexp)
        else:
            ok = np.array_equal(got, exp)
        if not ok:
            fails.append((kind, label))
    assert not fails, fails[:8]
