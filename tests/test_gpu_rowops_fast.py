"""The row-ops fast paths against the oracle's job model (rowops_job, the
restatement of rowops_ref.h): ro_stream16 (COPY / ADDX, int16, one broadcast
parameter entry, rows of whole words), ro_xpose8 (TRANSPOSE of 8-row tiles
with 16-byte aligned granules) and ro_norm16 (NORM on int16 rows, warp per
row) — each over rows x blocks with strides, and the geometry BERT uses."""
import numpy as np
import pytest

from oracle import spec

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from cormorant_b200 import ops as o
    return o


def _dev(arr):
    import torch
    return torch.from_numpy(arr.copy()).cuda()


def _pentry(g=0, bq=0, sa=0, sb=0, sc=0):
    e = np.zeros(16, np.uint8)
    e[0:4] = np.array([g & 0xFFFFFFFF], "<u4").view(np.uint8)
    e[4:8] = np.array([bq & 0xFFFFFFFF], "<u4").view(np.uint8)
    e[8], e[9], e[10] = sa, sb, sc
    return e


def _run(ops, mem, offs, regs):
    buf = _dev(mem)
    ops.rowops(buf, buf, buf, buf, a_off=offs["a"], b_off=offs["b"], c_off=offs["c"], p_off=offs["p"], **regs)
    m = spec.RowOpsMem(mem.copy())
    spec.rowops_job(m, regs["op"], regs["n"], regs["rows"], regs["blocks"], offs["a"], regs["a_s1"], regs["a_s2"],
                    offs["b"], regs.get("b_s1", 0), regs.get("b_s2", 0), offs["c"], regs["c_s1"], regs["c_s2"],
                    offs["p"], regs.get("eps", 0), regs.get("aux", 0), regs.get("bq_sh", 0), regs.get("win_lo", 0),
                    regs.get("win_hi", 0xFFFFFFFF))
    return buf.cpu().numpy(), m.buf


def _image(rng, a_len, b_len, p, c_len):
    from tests.fixtures import rowops_memory
    a = rng.integers(0, 256, size=a_len).astype(np.uint8)
    b = rng.integers(0, 256, size=b_len).astype(np.uint8)
    return rowops_memory(a, b, p, c_len)


STREAM = [  # name, op, param entry, bq_sh, window
    ("copy_ident", 1 | spec.F_P_BCAST, dict(), 0, None),
    ("addx_ident_relu", 2 | spec.F_P_BCAST | spec.F_B_EN | spec.F_RELU, dict(), 0, None),
    ("addx_shifts", 2 | spec.F_P_BCAST | spec.F_B_EN, dict(bq=-12345, sa=3, sb=1, sc=4), 2, None),
    ("copy_scale", 1 | spec.F_P_BCAST | spec.F_SCALE, dict(g=3 << 20, sa=2, sc=22), 0, None),
    ("copy_window", 1 | spec.F_P_BCAST | spec.F_B_EN, dict(sb=1, sc=1), 0, (2, 5)),
]


@pytest.mark.parametrize("case", STREAM, ids=[c[0] for c in STREAM])
@pytest.mark.parametrize("n,rows,blocks", [(64, 7, 3), (8, 1, 1), (768, 4, 2)])
def test_stream16(ops, case, n, rows, blocks):
    name, op, pe, bq_sh, win = case
    rng = np.random.default_rng(n * 7 + rows)
    a_s1, a_s2 = 2 * n + 32, (2 * n + 32) * rows + 64
    b_s1, b_s2 = 2 * n + 16, (2 * n + 16) * rows
    c_s1, c_s2 = 2 * n + 48, (2 * n + 48) * rows + 16
    mem, offs = _image(rng, a_s2 * blocks, b_s2 * blocks, _pentry(**pe), c_s2 * blocks)
    regs = dict(op=op, n=n, rows=rows, blocks=blocks, a_s1=a_s1, a_s2=a_s2, b_s1=b_s1, b_s2=b_s2, c_s1=c_s1,
                c_s2=c_s2, bq_sh=bq_sh, win_lo=win[0] if win else 0, win_hi=win[1] if win else 0xFFFFFFFF)
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("L,M,B,c_gap", [(64, 384, 3, 0), (72, 24, 2, 0), (8, 136, 1, 0), (200, 40, 2, 32),
                                         (64, 64, 5, 0)])
def test_xpose8(ops, L, M, B, c_gap):
    """K^T-style jobs: B blocks of an [M][L] int16 matrix (row stride sM) to
    [L][M]: tiles of 8 source rows, granules at the output row stride."""
    rng = np.random.default_rng(L * 3 + M)
    sM = L + 8 * (1 if c_gap else 0)            # source row stride (elements)
    sB = sM * M + 8                               # block stride (elements)
    out_row = M * 2 + c_gap                       # output row stride (bytes)
    regs = dict(op=7, n=L, rows=M // 8, blocks=B, a_s1=8 * sM * 2, a_s2=sB * 2, b_s1=sM * 2, b_s2=out_row,
                c_s1=16, c_s2=L * out_row + 64, aux=8)
    mem, offs = _image(rng, sB * 2 * B, 16, _pentry(), (L * out_row + 64) * B)
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)


def test_xpose8_contiguous_granules(ops):
    """b_s2 = 16: a tile's granules contiguous (the packed image)."""
    rng = np.random.default_rng(9)
    L, M = 96, 48
    regs = dict(op=7, n=L, rows=M // 8, blocks=2, a_s1=8 * L * 2, a_s2=M * L * 2, b_s1=L * 2, b_s2=16,
                c_s1=L * 16, c_s2=M * L * 2, aux=8)
    mem, offs = _image(rng, M * L * 2 * 2, 16, _pentry(), M * L * 2 * 2)
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n", [8, 768, 1000, 2048, 4096])
@pytest.mark.parametrize("ln,bcast", [(True, False), (True, True), (False, False)])
def test_norm16(ops, n, ln, bcast):
    rng = np.random.default_rng(n + 3 * ln + bcast)
    rows, blocks = 5, 2
    a_s1 = 2 * n + 16
    a_s2 = a_s1 * rows
    c_s1, c_s2 = 2 * n, 2 * n * rows + 32
    npar = 1 if bcast else n
    p = np.concatenate([_pentry(int(rng.integers(1, 1 << 30)), int(rng.integers(-(1 << 21), 1 << 21)), 0, 0,
                                int(rng.integers(24, 40))) for _ in range(npar)])
    mem, offs = _image(rng, a_s2 * blocks, 16, p, c_s2 * blocks)
    # one constant row (V = 0) and a full-scale row
    mem[offs["a"]:offs["a"] + 2 * n] = np.full(n, 77, "<i2").view(np.uint8)
    op = 5 | (spec.F_NORM_LN if ln else 0) | (spec.F_P_BCAST if bcast else 0)
    regs = dict(op=op, n=n, rows=rows, blocks=blocks, a_s1=a_s1, a_s2=a_s2, c_s1=c_s1, c_s2=c_s2,
                eps=int(rng.integers(0, 1 << 20)), bq_sh=int(rng.integers(0, 30)))
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)
