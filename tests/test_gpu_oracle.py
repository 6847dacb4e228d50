"""GPU parity against the CPU oracle (oracle/spec.py) on seeded inputs: the
tensor-core GEMM path of MatMul and Conv, saturation and int32 wrap, the
softmax unit in both modes with causal masks, the activation unit, pooling
and row-ops — bit-exact."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import spec  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import ops as o
    return o


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rnd16(rng, shape, lo=-32768, hi=32768):
    return rng.integers(lo, hi, size=shape).astype(np.int16)


MM_CASES = [  # n, k, m, batch, a_bs0, b_bs0, lo, hi
    (17, 33, 5, 1, False, False, -256, 256),
    (128, 64, 32, 1, False, False, -256, 256),
    (129, 129, 129, 1, False, False, -32768, 32768),
    (200, 300, 130, 3, False, False, -300, 300),
    (64, 512, 256, 4, True, False, -256, 256),
    (96, 1000, 40, 3, False, True, -256, 256),
    (300, 4096, 300, 1, False, False, -256, 256),
    (256, 256, 256, 2, False, False, -32768, 32768),
    (1, 4096, 1000, 1, False, False, -256, 256),
    (8, 1024, 4096, 2, False, False, -256, 256),
    (16, 4096, 32, 16, False, False, -256, 256),
    (3, 7, 5, 2, True, False, -32768, 32768),
]


@pytest.mark.parametrize("case", MM_CASES)
@pytest.mark.parametrize("wrap", [False, True])
def test_matmul_vs_oracle(ops, case, wrap):
    n, k, m, batch, a_bc, b_bc, lo, hi = case
    rng = np.random.default_rng(n * 7 + k * 13 + m + batch)
    A = rnd16(rng, (1 if a_bc else batch, n, k), lo, hi)
    B = rnd16(rng, (1 if b_bc else batch, k, m), lo, hi)
    c = torch.full((batch * n * m,), -8531, dtype=torch.int16, device="cuda")
    ops.matmul(dev(A.reshape(-1)), dev(B.reshape(-1)), c, n=n, k=k, m=m, batch=batch,
               a_batch_stride=0 if a_bc else n * k, b_batch_stride=0 if b_bc else k * m, c_batch_stride=n * m,
               flags=1 if wrap else 0)
    exp = spec.matmul_raw(np.broadcast_to(A, (batch, n, k)), np.broadcast_to(B, (batch, k, m)), wrap=wrap)
    assert np.array_equal(c.cpu().numpy().reshape(batch, n, m), exp)


@pytest.mark.parametrize("packed,kw", [(1, 0), (0, 2), (0, 4), (0, 8)])
def test_matmul_layouts_tensor_path(ops, packed, kw):
    """Packed-B and GEMV images on the split / tensor-core path (n > 16)."""
    rng = np.random.default_rng(3 + kw)
    n, k, m = 40, 256, 72
    A = rnd16(rng, (n, k), -300, 300)
    Bl = rnd16(rng, (k, m), -300, 300)
    idx = spec.b_index(k, m, packed, kw)
    img = np.zeros(int(idx.max()) + 1 + 64, np.int16)
    img[idx] = Bl
    c = torch.zeros(n * m, dtype=torch.int16, device="cuda")
    ops.matmul(dev(A.reshape(-1)), dev(img), c, n=n, k=k, m=m, batch=1, b_packed=packed, gemv_kw=kw)
    assert np.array_equal(c.cpu().numpy().reshape(n, m), spec.matmul_raw(A, Bl))


CONV_CASES = [  # N, C, H, W, M, kh, kw, sh, sw, pt, pl, dh, dw, depthwise, bias
    (1, 1, 28, 28, 16, 3, 3, 1, 1, 1, 1, 1, 1, False, True),
    (1, 16, 14, 14, 32, 3, 3, 1, 1, 1, 1, 1, 1, False, True),
    (2, 3, 33, 31, 32, 3, 3, 2, 2, 1, 1, 1, 1, False, True),
    (1, 24, 20, 20, 144, 1, 1, 1, 1, 0, 0, 1, 1, False, False),
    (2, 144, 10, 10, 144, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (1, 32, 9, 9, 32, 3, 3, 1, 1, 2, 2, 2, 2, True, False),
    (3, 40, 7, 9, 70, 5, 3, 1, 2, 2, 1, 1, 1, False, True),
    (1, 160, 7, 7, 960, 1, 1, 1, 1, 0, 0, 1, 1, False, True),
    # 1 x 1 at stride 1 on whole 16-byte rows: the GEMM form W x per image (two
    # row tiles of channels, a batch; a K split with its per-channel bias)
    (3, 32, 8, 16, 200, 1, 1, 1, 1, 0, 0, 1, 1, False, True),
    (1, 2048, 4, 4, 40, 1, 1, 1, 1, 0, 0, 1, 1, False, True),
    # depthwise: warp-per-plane windows (stride 1 / 2, pads 0..2, W above a warp,
    # an input row no output reads), shared-memory planes (larger windows, 5x5)
    (3, 24, 14, 14, 24, 3, 3, 1, 1, 1, 1, 1, 1, True, True),
    (2, 20, 14, 12, 20, 3, 3, 2, 2, 0, 0, 1, 1, True, True),
    (2, 9, 5, 40, 9, 3, 3, 1, 1, 2, 1, 1, 1, True, False),
    (1, 17, 7, 7, 17, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (2, 6, 40, 37, 6, 3, 3, 1, 1, 1, 1, 1, 1, True, True),
    (2, 6, 45, 44, 6, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    # depthwise 3x3 on rows of whole 16-byte words (vector-staged windows):
    # stride 1 / 2, pads 0 / 1 / 2, odd heights, a plane per CTA and several
    (2, 16, 16, 24, 16, 3, 3, 1, 1, 1, 1, 1, 1, True, True),
    (1, 8, 32, 32, 8, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (2, 4, 9, 16, 4, 3, 3, 1, 1, 0, 0, 1, 1, True, False),
    (1, 3, 9, 8, 3, 3, 3, 2, 2, 0, 0, 1, 1, True, True),
    (1, 5, 20, 112, 5, 3, 3, 2, 2, 2, 2, 1, 1, True, True),
    (1, 5, 30, 30, 5, 5, 5, 1, 1, 2, 2, 1, 1, True, True),
    # depthwise 3x3 as runs of eight outputs: whole planes read as one range
    # (H W of 49 / 196 / 143 / 784 elements: units of 8 / 2 / 8 / 1 planes, a
    # ragged last unit and last word), rows of whole words, strides 1 / 2, left
    # pads 0 / 1 with top pads 0..2, several row groups and runs per plane
    (3, 12, 7, 7, 12, 3, 3, 1, 1, 1, 1, 1, 1, True, True),
    (2, 13, 7, 7, 13, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (3, 10, 14, 14, 10, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (2, 33, 13, 11, 33, 3, 3, 1, 1, 0, 0, 1, 1, True, True),
    (1, 70, 28, 28, 70, 3, 3, 1, 1, 1, 1, 1, 1, True, False),
    (2, 9, 28, 28, 9, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (1, 6, 19, 17, 6, 3, 3, 2, 2, 0, 0, 1, 1, True, True),
    (1, 4, 11, 10, 4, 3, 3, 1, 1, 2, 1, 1, 1, True, True),
    (2, 3, 57, 56, 3, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (1, 2, 112, 112, 2, 3, 3, 1, 1, 1, 1, 1, 1, True, True),
    (1, 3, 112, 112, 3, 3, 3, 2, 2, 1, 1, 1, 1, True, True),
    (2, 5, 12, 40, 5, 3, 3, 2, 2, 0, 1, 1, 1, True, True),
]


@pytest.mark.parametrize("case", CONV_CASES)
@pytest.mark.parametrize("act", [0, 4, 8])
def test_conv_vs_oracle(ops, case, act):
    N, C, H, W, M, kh, kw, sh, sw, pt, pl, dh, dw, dwise, hb = case
    rng = np.random.default_rng(N + C * 3 + M * 5 + kh)
    oh = (H + 2 * pt - (dh * (kh - 1) + 1)) // sh + 1
    ow = (W + 2 * pl - (dw * (kw - 1) + 1)) // sw + 1
    x = rnd16(rng, (N, C, H, W), -256, 256)
    w = rnd16(rng, (M, 1 if dwise else C, kh, kw), -128, 128)
    b = rnd16(rng, (M,), -256, 256)
    y = torch.full((N * M * oh * ow,), -8531, dtype=torch.int16, device="cuda")
    ops.conv(dev(x.reshape(-1)), dev(w.reshape(-1)), dev(b) if hb else None, y, batch=N, in_ch=C, in_h=H, in_w=W,
             out_ch=M, out_h=oh, out_w=ow, kh=kh, kw=kw, stride_h=sh, stride_w=sw, dilation_h=dh, dilation_w=dw,
             pad_top=pt, pad_left=pl, has_bias=hb, is_depthwise=dwise, flags=2 | act)
    exp = spec.conv_raw(x, w, b if hb else None, sh, sw, pt, pl, dh, dw, oh, ow, dwise)
    if act == 4:
        exp = np.maximum(exp, 0)
    elif act == 8:
        exp = np.clip(exp, 0, 1536)
    assert np.array_equal(y.cpu().numpy().reshape(N, M, oh, ow), exp)


@pytest.mark.parametrize("wrap", [0, 1])
@pytest.mark.parametrize("shape", [(2, 6, 9, 10, 1), (1, 5, 16, 16, 2)], ids=["flat_s1", "rows_s2"])
def test_depthwise_full_range(ops, shape, wrap):
    """Depthwise 3x3 on full-range operands: channels whose sums can leave
    int32 (the 64-bit path) beside channels whose cannot (the 32-bit path) in
    one unit; without the wrap rule the exact sums saturate, with it the 32-bit
    sums wrap as the rule does."""
    N, C, H, W, s_ = shape
    rng = np.random.default_rng(31 + C + wrap)
    x = rnd16(rng, (N, C, H, W), -32768, 32768)
    w = rnd16(rng, (C, 1, 3, 3), -32768, 32768)
    w[::2] //= 4096  # even channels: small taps (the bound holds), odd ones full range
    b = rnd16(rng, (C,), -32768, 32768)
    oh, ow = (H + 2 - 3) // s_ + 1, (W + 2 - 3) // s_ + 1
    y = torch.full((N * C * oh * ow,), -8531, dtype=torch.int16, device="cuda")
    ops.conv(dev(x.reshape(-1)), dev(w.reshape(-1)), dev(b), y, batch=N, in_ch=C, in_h=H, in_w=W, out_ch=C,
             out_h=oh, out_w=ow, kh=3, kw=3, stride_h=s_, stride_w=s_, pad_top=1, pad_left=1, has_bias=1,
             is_depthwise=1, flags=2 | wrap)
    exp = spec.conv_raw(x, w, b, s_, s_, 1, 1, 1, 1, oh, ow, True, wrap=bool(wrap))
    assert np.array_equal(y.cpu().numpy().reshape(N, C, oh, ow), exp)


@pytest.mark.parametrize("wrap", [0, 1])
@pytest.mark.parametrize("shape", [(2, 3, 11, 13, 32, 3, 2), (1, 20, 6, 6, 24, 1, 1)], ids=["stem_3x3_s2", "pointwise"])
def test_small_k_full_range(ops, shape, wrap):
    """Short sums (K = C kh kw <= 32, few channels out: the CUDA-core kernel)
    on full-range operands: chunks of 16 channels whose sums can leave int32
    (the 64-bit path) beside chunks whose cannot (the 32-bit path); without
    the wrap rule the exact sums saturate, with it the 32-bit sums wrap."""
    N, C, H, W, M, k, s_ = shape
    rng = np.random.default_rng(41 + C + wrap)
    x = rnd16(rng, (N, C, H, W), -32768, 32768)
    w = rnd16(rng, (M, C, k, k), -32768, 32768)
    w[:16] //= 4096  # the first chunk: small taps (the bound holds); the rest full range
    b = rnd16(rng, (M,), -32768, 32768)
    p_ = k // 2
    oh, ow = (H + 2 * p_ - k) // s_ + 1, (W + 2 * p_ - k) // s_ + 1
    y = torch.full((N * M * oh * ow,), -8531, dtype=torch.int16, device="cuda")
    ops.conv(dev(x.reshape(-1)), dev(w.reshape(-1)), dev(b), y, batch=N, in_ch=C, in_h=H, in_w=W, out_ch=M,
             out_h=oh, out_w=ow, kh=k, kw=k, stride_h=s_, stride_w=s_, pad_top=p_, pad_left=p_, has_bias=1,
             flags=2 | wrap)
    exp = spec.conv_raw(x, w, b, s_, s_, p_, p_, 1, 1, oh, ow, False, wrap=bool(wrap))
    assert np.array_equal(y.cpu().numpy().reshape(N, M, oh, ow), exp)


def test_conv_wrap(ops):
    """Large operands: the exact sum leaves int32; CORM_F_WRAP32 wraps it."""
    rng = np.random.default_rng(9)
    x = rnd16(rng, (1, 64, 6, 6), 20000, 32767)
    w = rnd16(rng, (8, 64, 3, 3), 20000, 32767)
    for wrap in (0, 1):
        y = torch.zeros(8 * 16, dtype=torch.int16, device="cuda")
        ops.conv(dev(x.reshape(-1)), dev(w.reshape(-1)), None, y, batch=1, in_ch=64, in_h=6, in_w=6, out_ch=8,
                 out_h=4, out_w=4, kh=3, kw=3, flags=2 | wrap)
        exp = spec.conv_raw(x, w, None, 1, 1, 0, 0, 1, 1, 4, 4, False, wrap=bool(wrap))
        assert np.array_equal(y.cpu().numpy().reshape(1, 8, 4, 4), exp)


@pytest.mark.parametrize("op", [0, 1, 2, 3, 4, 5, 6, 7, 8, 9])
@pytest.mark.parametrize("act", [0, 1, 2, 3, 4, 5, 6])
def test_vectorop_vs_oracle(ops, op, act):
    rng = np.random.default_rng(op * 10 + act)
    size, outer = 1000, 37
    a = rnd16(rng, (outer * 1000 + 64,))
    b = rnd16(rng, (1000 + 64,))
    c_len = (outer - 1) * 1000 + 1000
    c = torch.full((c_len + 8,), -8531, dtype=torch.int16, device="cuda")
    regs = dict(size=size, op=op, outer=outer, a_inc=1000, b_inc=0, act=act, alpha=0x12345678)
    ops.vectorop(dev(a), dev(b), c, **regs)
    exp = np.full(c_len + 8, -8531, np.int16)
    spec.vectorop_job(a, b, exp, **regs)
    assert np.array_equal(c.cpu().numpy(), exp)


@pytest.mark.parametrize("n", [1, 7, 128, 255, 300, 384, 500, 512, 700, 768, 1000, 1024, 2048, 4096, 10000])
@pytest.mark.parametrize("mask", [0, "full", "causal"])
def test_softmax_rows(ops, n, mask):
    rng = np.random.default_rng(n)
    rows = 24
    W = (n + 7) // 8 * 8
    x = rng.integers(-2048, 2048, size=(rows, W)).astype(np.int16)
    cm, cs = spec.smx_scale_regs(8, 1.0)
    m = {0: 0, "full": n, "causal": max(1, n // 4) | (5 << 16)}[mask]
    regs = dict(size=n, op=10, outer=rows, a_inc=W, b_inc=W, smx_cm=cm, smx_cfg=cs | (8 << 8), smx_mask=m)
    c = torch.full((rows * W,), -8531, dtype=torch.int16, device="cuda")
    ops.vectorop(dev(x.reshape(-1)), None, c, **regs)
    exp = np.full(rows * W, -8531, np.int16)
    spec.vectorop_job(x.reshape(-1), None, exp, **regs)
    assert np.array_equal(c.cpu().numpy(), exp)


@pytest.mark.parametrize("keys", [1, 37, 128, 384, 1024, 4096])
@pytest.mark.parametrize("queries", [16, 50, 96])
def test_softmax_cols(ops, keys, queries):
    rng = np.random.default_rng(keys + queries)
    a_inc = (queries + 7) // 8 * 8
    W = (keys + 7) // 8 * 8
    s = rng.integers(-4096, 4096, size=(keys, a_inc)).astype(np.int16)
    cm, cs = spec.smx_scale_regs(10, 0.125)
    regs = dict(size=keys, op=11, outer=queries, a_inc=a_inc, b_inc=W, smx_cm=cm, smx_cfg=cs | (12 << 8),
                smx_mask=max(1, keys // 3) | (3 << 16))
    rows = queries & ~15
    c = torch.full((max(rows, 1) * W + 8,), -8531, dtype=torch.int16, device="cuda")
    ops.vectorop(dev(s.reshape(-1)), None, c, **regs)
    exp = np.full(max(rows, 1) * W + 8, -8531, np.int16)
    spec.vectorop_job(s.reshape(-1), None, exp, **regs)
    assert np.array_equal(c.cpu().numpy(), exp)


POOL_CASES = [  # N, C, H, W, ph, pw, sh, sw, pt, pl, dh, dw, type, lp, cip
    (2, 16, 28, 28, 2, 2, 2, 2, 0, 0, 1, 1, 0, 0, 0),
    (1, 5, 13, 11, 3, 3, 2, 2, 1, 1, 1, 1, 1, 0, 0),
    (1, 5, 13, 11, 3, 3, 2, 2, 1, 1, 1, 1, 1, 0, 1),
    (2, 3, 9, 9, 3, 2, 1, 2, 1, 0, 2, 1, 2, 1, 0),
    (2, 3, 9, 9, 3, 3, 2, 2, 1, 1, 1, 1, 2, 2, 0),
    (4, 1280, 7, 7, 7, 7, 1, 1, 0, 0, 1, 1, 1, 0, 0),
    (2, 64, 7, 7, 7, 7, 1, 1, 0, 0, 1, 1, 0, 0, 0),
    (2, 64, 8, 8, 8, 8, 1, 1, 0, 0, 1, 1, 2, 2, 0),
    (1, 3, 4, 4, 3, 3, 3, 3, 2, 2, 1, 1, 0, 0, 0),
]


@pytest.mark.parametrize("case", POOL_CASES)
def test_pool_vs_oracle(ops, case):
    N, C, H, W, ph, pw, sh, sw, pt, pl, dh, dw, typ, lp, cip = case
    rng = np.random.default_rng(C + H)
    oh = (H + 2 * pt - (dh * (ph - 1) + 1)) // sh + 1
    ow = (W + 2 * pl - (dw * (pw - 1) + 1)) // sw + 1
    x = rnd16(rng, (N, C, H, W))
    y = torch.full((N * C * oh * ow,), -8531, dtype=torch.int16, device="cuda")
    ops.pool(dev(x.reshape(-1)), y, batch=N, channels=C, in_h=H, in_w=W, out_h=oh, out_w=ow, pool_h=ph, pool_w=pw,
             stride_h=sh, stride_w=sw, pad_top=pt, pad_left=pl, dil_h=dh, dil_w=dw, pool_type=typ, lp_order=lp,
             count_include_pad=cip)
    exp = spec.pool_raw(x, ph, pw, sh, sw, pt, pl, dh, dw, oh, ow, typ, lp, cip)
    assert np.array_equal(y.cpu().numpy().reshape(N, C, oh, ow), exp)


def _param_block(rng, n, sa_max=8, sc_lo=8, sc_hi=30):
    pb = np.zeros((n, 16), np.uint8)
    g = rng.integers(1, 1 << 24, size=n).astype(np.int64)
    bq = rng.integers(-(1 << 21), 1 << 21, size=n).astype(np.int64)
    pb[:, 0:4] = (g & 0xFFFFFFFF).astype("<u4").view(np.uint8).reshape(n, 4)
    pb[:, 4:8] = (bq & 0xFFFFFFFF).astype("<u4").view(np.uint8).reshape(n, 4)
    pb[:, 8] = rng.integers(0, sa_max, size=n)
    pb[:, 9] = rng.integers(0, sa_max, size=n)
    pb[:, 10] = rng.integers(sc_lo, sc_hi, size=n)
    return pb.reshape(-1)


ROWOPS_JOBS = [  # op word, n, rows, blocks, kind bytes of a / c
    ("copy", 1 | spec.F_B_EN, 96, 5, 2),
    ("addx_i32", 2 | (1 << 4) | (0 << 6) | (1 << 8) | spec.F_B_EN | spec.F_RELU, 40, 3, 1),
    ("scale", 1 | spec.F_SCALE, 64, 4, 1),
    ("mulact", 4 | spec.F_B_EN, 256, 4, 1),
    ("gate", 10 | spec.F_B_EN, 100, 3, 1),
    ("dequant", 3 | (1 << 4) | (2 << 8), 48, 3, 1),
    ("rms", 5 | (1 << 4), 960, 3, 1),
    ("ln", 5 | spec.F_NORM_LN, 768, 3, 1),
    ("ln_bcast", 5 | spec.F_NORM_LN | spec.F_P_BCAST, 64, 6, 1),
    ("rope", 6, 192, 4, 1),
]


@pytest.mark.parametrize("job", ROWOPS_JOBS, ids=[j[0] for j in ROWOPS_JOBS])
def test_rowops_vs_oracle(ops, job):
    name, op, n, rows, _ = job
    rng = np.random.default_rng(len(name) * 31 + n)
    ak, ck = (op >> 4) & 3, (op >> 8) & 3
    nba = 2 if ak == 0 else 4
    row_b = (n * 4 + 15) // 16 * 16
    a = np.zeros(rows * row_b, np.uint8)
    for r in range(rows):
        vals = rng.integers(-30000, 30000, size=n) if nba == 2 else rng.integers(-(1 << 28), 1 << 28, size=n)
        a[r * row_b:r * row_b + n * nba] = vals.astype("<i2" if nba == 2 else "<i4").view(np.uint8)
    if name == "rope":
        HD = 64
        ang = rng.uniform(-3, 3, size=HD)
        tab = np.concatenate([np.rint(np.cos(ang) * 2 ** 23), np.rint(np.sin(ang) * 2 ** 23)]).astype("<i4")
        b = np.zeros(rows * row_b, np.uint8)
        b[:tab.nbytes] = tab.view(np.uint8)
        b_s1, aux = 0, HD
    else:
        b = rng.integers(0, 256, size=rows * row_b).astype(np.uint8)
        b_s1, aux = row_b, 0
    p = _param_block(rng, n, sa_max=4 if name in ("mulact", "gate") else 8,
                     sc_lo=20 if name in ("rms", "ln", "ln_bcast") else 8, sc_hi=40)
    eps = 12345 if name in ("rms", "ln", "ln_bcast") else 0
    c_len = rows * row_b
    mem = np.zeros(len(a) + len(b) + len(p) + c_len + 1024, np.uint8)
    oa, ob, op_, oc = 0, (len(a) + 255) // 256 * 256, 0, 0
    op_ = ob + (len(b) + 255) // 256 * 256
    oc = op_ + (len(p) + 255) // 256 * 256
    mem = np.zeros(oc + c_len + 256, np.uint8)
    mem[oa:oa + len(a)] = a
    mem[ob:ob + len(b)] = b
    mem[op_:op_ + len(p)] = p
    mem[oc:oc + c_len] = 0xDE
    regs = dict(op=op, n=n, rows=rows, blocks=1, a_s1=row_b, a_s2=0, b_s1=b_s1, b_s2=0, c_s1=row_b, c_s2=0, eps=eps,
                aux=aux, bq_sh=3)
    buf = dev(mem)
    ops.rowops(buf, buf, buf, buf, a_off=oa, b_off=ob, c_off=oc, p_off=op_, **regs)
    m = spec.RowOpsMem(mem.copy())
    spec.rowops_job(m, op, n, rows, 1, oa, row_b, 0, ob, b_s1, 0, oc, row_b, 0, op_, eps, aux, 3)
    assert np.array_equal(buf.cpu().numpy(), m.buf)


@pytest.mark.parametrize("size,inc", [(10, 10), (3, 3), (13, 14), (1000, 1001), (7, 8)])
@pytest.mark.parametrize("op", [0, 2, 10])
def test_rows_not_on_words(ops, size, inc, op):
    """Dense rows whose length is not a multiple of 8: the hardware writes rows
    in order, so a row's zero tail survives only where the next row's data
    does not land (the oracle writes them sequentially)."""
    rng = np.random.default_rng(size * 7 + inc + op)
    outer = 9
    n_in = outer * inc + 64
    a = rnd16(rng, (n_in,), -2048, 2048)
    b = rnd16(rng, (n_in,), -2048, 2048)
    if op == 10:
        regs = dict(size=size, op=10, outer=outer, a_inc=inc, b_inc=inc, smx_cm=12102203, smx_cfg=19 | (8 << 8),
                    smx_mask=size)
    else:
        regs = dict(size=size, op=op, outer=outer, a_inc=inc, b_inc=0, act=1)
    c_len = outer * inc + 32
    c = torch.full((c_len,), -8531, dtype=torch.int16, device="cuda")
    ops.vectorop(dev(a), dev(b), c, **regs)
    exp = np.full(c_len, -8531, np.int16)
    spec.vectorop_job(a, b, exp, **regs)
    assert np.array_equal(c.cpu().numpy(), exp)
