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


def _params(rng, n, bcast, **ranges):
    """n (or one) random entries; ranges: field -> (lo, hi)."""
    out = []
    for _ in range(1 if bcast else n):
        f = {k: int(rng.integers(lo, hi)) for k, (lo, hi) in ranges.items()}
        out.append(_pentry(**f))
    return np.concatenate(out)


@pytest.mark.parametrize("n", [8, 960, 2048])
@pytest.mark.parametrize("bcast", [False, True])
@pytest.mark.parametrize("small", [False, True])
def test_norm32_rms(ops, n, bcast, small):
    """NORM (RMS) on int32 rows (the LLM residual): ro_norm16<., 1>."""
    rng = np.random.default_rng(n + 2 * bcast + small)
    rows, blocks = 4, 2
    a_s1 = 4 * n + 16
    a_s2 = a_s1 * rows
    c_s1, c_s2 = 2 * n, 2 * n * rows + 32
    p = _params(rng, n, bcast, g=(1, 1 << 30), bq=(-(1 << 21), 1 << 21), sc=(24, 50))
    mem, offs = _image(rng, a_s2 * blocks, 16, p, c_s2 * blocks)
    if small:  # residual-like values
        vals = rng.integers(-(1 << 20), 1 << 20, a_s2 * blocks // 4).astype("<i4")
        mem[offs["a"]:offs["a"] + a_s2 * blocks] = vals.view(np.uint8)
    op = 5 | (1 << 4) | (spec.F_P_BCAST if bcast else 0)
    regs = dict(op=op, n=n, rows=rows, blocks=blocks, a_s1=a_s1, a_s2=a_s2, c_s1=c_s1, c_s2=c_s2,
                eps=int(rng.integers(0, 1 << 40)), bq_sh=int(rng.integers(0, 30)))
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("ak,ln,n", [(0, True, 768), (0, False, 1000), (1, False, 960)])
def test_norm_many_rows(ops, ak, ln, n):
    """NORM over 1200 rows (600 x 2 blocks): the warp-per-row form (the tests
    above, with a handful of rows, take the form that spreads a row over the
    8 warps of a block)."""
    rng = np.random.default_rng(ak + 2 * ln + n)
    rows, blocks = 600, 2
    eb = 4 if ak else 2
    a_s1 = eb * n + 16
    a_s2 = a_s1 * rows
    c_s1, c_s2 = 2 * n, 2 * n * rows + 32
    p = _params(rng, n, False, g=(1, 1 << 30), bq=(-(1 << 21), 1 << 21), sc=(24, 46))
    mem, offs = _image(rng, a_s2 * blocks, 16, p, c_s2 * blocks)
    if ak:  # residual-like values on every other row
        vals = rng.integers(-(1 << 20), 1 << 20, a_s1 // 4).astype("<i4").view(np.uint8)
        for r in range(0, rows * blocks, 2):
            mem[offs["a"] + r * a_s1:offs["a"] + (r + 1) * a_s1] = vals
    op = 5 | (ak << 4) | (spec.F_NORM_LN if ln else 0)
    regs = dict(op=op, n=n, rows=rows, blocks=blocks, a_s1=a_s1, a_s2=a_s2, c_s1=c_s1, c_s2=c_s2,
                eps=int(rng.integers(0, 1 << 20)), bq_sh=int(rng.integers(0, 30)))
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)


KINDS = [(ak, bk, ck) for ak in (0, 1) for bk in (0, 1) for ck in (0, 1)]


@pytest.mark.parametrize("kinds", KINDS)
@pytest.mark.parametrize("variant", ["small", "wide", "relu_window", "scale"])
def test_stream_any(ops, kinds, variant):
    """COPY / ADDX on int16 / int32 rows with per-column entries
    (ro_stream_any): int64 shifts, the 128-bit fallback (wide shifts,
    SCALE), RELU and the row window."""
    ak, bk, ck = kinds
    rng = np.random.default_rng(sum(k << i for i, k in enumerate(kinds)) + 17 * len(variant))
    n, rows, blocks = 96, 5, 2
    nb = lambda k: 2 if k == 0 else 4  # noqa: E731
    a_s1, b_s1, c_s1 = nb(ak) * n + 16, nb(bk) * n + 32, nb(ck) * n
    a_s2, b_s2, c_s2 = a_s1 * rows, b_s1 * rows + 16, c_s1 * rows + 48
    sh = dict(small=(0, 12), wide=(20, 40), relu_window=(0, 6), scale=(0, 4))[variant]
    p = _params(rng, n, False, g=(-(1 << 20), 1 << 20), bq=(-(1 << 21), 1 << 21), sa=sh, sb=sh, sc=(0, 30))
    mem, offs = _image(rng, a_s2 * blocks, b_s2 * blocks, p, c_s2 * blocks)
    op = 2 | (ak << 4) | (bk << 6) | (ck << 8) | spec.F_B_EN
    if variant == "relu_window":
        op |= spec.F_RELU
    if variant == "scale":
        op |= spec.F_SCALE
    win = (1, 4) if variant == "relu_window" else (0, 0xFFFFFFFF)
    regs = dict(op=op, n=n, rows=rows, blocks=blocks, a_s1=a_s1, a_s2=a_s2, b_s1=b_s1, b_s2=b_s2, c_s1=c_s1,
                c_s2=c_s2, bq_sh=int(rng.integers(0, 20)), win_lo=win[0], win_hi=win[1])
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("bcast", [False, True])
@pytest.mark.parametrize("sa_hi", [9, 30])
def test_mulact_fast(ops, bcast, sa_hi):
    """MULACT (SiLU(g) u) on int16 rows: int64 path (sa <= 23) and the
    128-bit fallback."""
    rng = np.random.default_rng(5 + bcast + sa_hi)
    n, rows, blocks = 2560 // 4, 3, 2
    s1 = 2 * n + 16
    p = _params(rng, n, bcast, sa=(0, sa_hi), sc=(10, 30))
    mem, offs = _image(rng, s1 * rows * blocks, s1 * rows * blocks, p, 2 * n * rows * blocks)
    op = 4 | spec.F_B_EN | (spec.F_P_BCAST if bcast else 0)
    regs = dict(op=op, n=n, rows=rows, blocks=blocks, a_s1=s1, a_s2=s1 * rows, b_s1=s1, b_s2=s1 * rows,
                c_s1=2 * n, c_s2=2 * n * rows)
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("HD,heads", [(64, 15), (128, 2), (16, 3)])
@pytest.mark.parametrize("bcast,sh_hi", [(False, 4), (True, 3), (False, 40)])
def test_rope_fast(ops, HD, heads, bcast, sh_hi):
    """ROPE on int16 rows (ro_rope_fast): cos / sin rows of 2 HD int24 words,
    per-column or broadcast shifts, the 128-bit fallback for shifts > 23."""
    rng = np.random.default_rng(HD + heads + sh_hi)
    n, rows, blocks = HD * heads, 6, 2
    a_s1 = 2 * n + 16
    b_s1 = 8 * HD
    p = _params(rng, n, bcast, sa=(0, sh_hi), sb=(0, sh_hi), sc=(20, 50))
    cs = rng.integers(-(1 << 23), (1 << 23) + 1, (rows, 2 * HD)).astype("<i4").view(np.uint8).reshape(-1)
    mem, offs = _image(rng, a_s1 * rows * blocks, b_s1 * rows, p, 2 * n * rows * blocks)
    mem[offs["b"]:offs["b"] + cs.size] = cs
    op = 6 | (1 << 6) | spec.F_B_EN | (spec.F_P_BCAST if bcast else 0)
    regs = dict(op=op, n=n, rows=rows, blocks=blocks, a_s1=a_s1, a_s2=a_s1 * rows, b_s1=b_s1, b_s2=0,
                c_s1=2 * n, c_s2=2 * n * rows, aux=HD)
    got, want = _run(ops, mem, offs, regs)
    assert np.array_equal(got, want)
