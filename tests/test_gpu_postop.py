"""corm_matmul_post / corm_conv_post: the VectorOP job fused into the MatMul /
Conv epilogue equals the two jobs run one after the other (the plain job,
then corm_vectorop on its output) on every path — tensor-core GEMM, its K
split, the GEMV kernel, the NCHW conv epilogue and both depthwise kernels —
for each operand mode, op and activation."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

COL, SAME, SCALAR = 0, 1, 2


@pytest.fixture(scope="module")
def ops():
    from cormorant_b200 import ops as o
    return o


def _two_jobs(ops, y, bfull, op, act, alpha, rev):
    """The reference composition: corm_vectorop over the whole output."""
    N = y.numel()
    c = torch.empty(N + 16, dtype=torch.int16, device="cuda")
    a, b = (bfull, y) if rev else (y, bfull)
    ops.vectorop(a, b, c, size=N, op=op, outer=1, act=act, alpha=alpha)
    return c[:N]


POSTS = [  # op, act, alpha, b_mode, rev
    (0, 0, 0, COL, 0), (0, 5, 0, COL, 0), (0, 3, 0x3333, SAME, 0), (1, 0, 0, SAME, 1), (1, 1, 0, COL, 0),
    (2, 4, 0, SCALAR, 0), (2, 6, 0, COL, 0), (0, 2, 0, SAME, 0),
]


def _bfull_matmul(b, mode, batch, n, m):
    if mode == COL:
        return b.repeat(batch * n)
    if mode == SCALAR:
        return b[:1].repeat(batch * n * m)
    return b


@pytest.mark.parametrize("shape", [(2, 300, 200, 96), (1, 64, 4096, 64), (3, 1, 512, 200), (2, 2, 4096, 40),
                                   (1, 130, 64, 300)], ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("post", POSTS, ids=lambda p: "op%d_act%d_b%d_r%d" % (p[0], p[1], p[3], p[4]))
def test_matmul_post(ops, shape, post):
    batch, n, k, m = shape
    op, act, alpha, mode, rev = post
    g = torch.Generator(device="cuda")
    g.manual_seed(batch * 1000 + n + k + m + op * 7 + act)
    A = torch.randint(-3000, 3000, (batch * n * k,), dtype=torch.int16, device="cuda", generator=g)
    B = torch.randint(-3000, 3000, (batch * k * m,), dtype=torch.int16, device="cuda", generator=g)
    nb = {COL: m, SAME: batch * n * m, SCALAR: 1}[mode]
    bv = torch.randint(-20000, 20000, (nb,), dtype=torch.int16, device="cuda", generator=g)
    regs = dict(n=n, k=k, m=m, batch=batch, a_batch_stride=n * k, b_batch_stride=k * m, c_batch_stride=n * m)
    y = torch.empty(batch * n * m, dtype=torch.int16, device="cuda")
    ops.matmul(A, B, y, **regs)
    want = _two_jobs(ops, y, _bfull_matmul(bv, mode, batch, n, m), op, act, alpha, rev)
    got = torch.full((batch * n * m,), -1234, dtype=torch.int16, device="cuda")
    ops.matmul(A, B, got, post=dict(b=bv, op=op, act=act, alpha=alpha, b_mode=mode, b_is_first=rev), **regs)
    assert torch.equal(got, want)


CONVS = [  # N, C, H, W, M, k, s, p, depthwise
    (2, 16, 14, 14, 24, 3, 1, 1, False),
    (1, 8, 20, 20, 300, 1, 1, 0, False),
    (3, 24, 14, 14, 24, 3, 1, 1, True),
    (2, 20, 14, 12, 20, 3, 2, 0, True),
    (2, 6, 40, 37, 6, 3, 1, 1, True),
    (1, 5, 30, 30, 5, 5, 1, 2, True),
    (2, 8, 16, 16, 8, 3, 2, 1, True),
    (2, 3, 12, 12, 24, 3, 1, 1, False),
    (3, 7, 7, 7, 7, 3, 1, 1, True),
]


@pytest.mark.parametrize("case", CONVS, ids=lambda c: "_".join(map(str, c)))
@pytest.mark.parametrize("post", POSTS[:6], ids=lambda p: "op%d_act%d_b%d_r%d" % (p[0], p[1], p[3], p[4]))
def test_conv_post(ops, case, post):
    N, C, H, W, M, k, s, p, dw = case
    op, act, alpha, mode, rev = post
    oh, ow = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    g = torch.Generator(device="cuda")
    g.manual_seed(N + C + H + M + op * 7 + act)
    x = torch.randint(-600, 600, (N * C * H * W,), dtype=torch.int16, device="cuda", generator=g)
    w = torch.randint(-300, 300, (M * (1 if dw else C) * k * k,), dtype=torch.int16, device="cuda", generator=g)
    bias = torch.randint(-900, 900, (M,), dtype=torch.int16, device="cuda", generator=g)
    P = oh * ow
    nb = {COL: M, SAME: N * M * P, SCALAR: 1}[mode]
    bv = torch.randint(-20000, 20000, (nb,), dtype=torch.int16, device="cuda", generator=g)
    regs = dict(batch=N, in_ch=C, in_h=H, in_w=W, out_ch=M, out_h=oh, out_w=ow, kh=k, kw=k, stride_h=s, stride_w=s,
                pad_top=p, pad_left=p, has_bias=1, is_depthwise=dw, flags=2)
    y = torch.empty(N * M * P, dtype=torch.int16, device="cuda")
    ops.conv(x, w, bias, y, **regs)
    if mode == COL:
        bfull = bv.view(1, M, 1).expand(N, M, P).reshape(-1).contiguous()
    elif mode == SCALAR:
        bfull = bv[:1].repeat(N * M * P)
    else:
        bfull = bv
    want = _two_jobs(ops, y, bfull, op, act, alpha, rev)
    got = torch.full((N * M * P,), -1234, dtype=torch.int16, device="cuda")
    ops.conv(x, w, bias, got, post=dict(b=bv, op=op, act=act, alpha=alpha, b_mode=mode, b_is_first=rev), **regs)
    assert torch.equal(got, want)


def test_post_rejects(ops):
    from cormorant_b200._lib import CormError
    A = torch.zeros(64, dtype=torch.int16, device="cuda")
    y = torch.zeros(64, dtype=torch.int16, device="cuda")
    for bad in (dict(op=3), dict(act=7), dict(b_mode=3)):
        q = dict(b=A, op=0, act=0, b_mode=0)
        q.update(bad)
        with pytest.raises(CormError):
            ops.matmul(A, A, y, n=8, k=8, m=8, post=q)
