"""The GEMM that reads int16 operands and splits them into the int8 planes
inside the kernel (row-major B, K and m multiples of 8, 16-byte rows)
against the oracle: partial row / column / K tiles, batches with shared
operands (stride 0), the K split, the int32 wrap, full-range values."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import spec  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from cormorant_b200 import ops as o
    return o


CASES = [  # batch, n, k, m, a_shared, b_shared, flags, lo, hi
    (1, 3, 8, 8, False, False, 0, -32768, 32768),
    (1, 200, 136, 72, False, False, 0, -3000, 3000),
    (3, 130, 264, 136, False, True, 0, -32768, 32768),
    (2, 257, 520, 264, True, False, 1, -32768, 32768),
    (1, 64, 4096, 64, False, False, 0, -32768, 32768),
    (4, 384, 64, 384, False, False, 0, -600, 600),
    (2, 128, 384, 64, False, False, 1, -32768, 32768),
    (1, 400, 1024, 400, False, False, 0, -256, 256),
    (16, 8, 512, 256, False, False, 0, -32768, 32768),
]


@pytest.mark.parametrize("producers", ["tma", "ldg"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "b%d_n%d_k%d_m%d" % c[:4])
def test_direct_vs_oracle(ops, case, producers, monkeypatch):
    """Both producer forms: raw int16 tiles by TMA split in shared memory (the
    default) and plain loads split in registers (CORM_GEMM_LDG_PRODUCERS=1)."""
    if producers == "ldg":
        monkeypatch.setenv("CORM_GEMM_LDG_PRODUCERS", "1")
    batch, n, k, m, a_sh, b_sh, flags, lo, hi = case
    rng = np.random.default_rng(batch * 7 + n + k * 3 + m)
    A = rng.integers(lo, hi, size=(1 if a_sh else batch, n, k)).astype(np.int16)
    B = rng.integers(lo, hi, size=(1 if b_sh else batch, k, m)).astype(np.int16)
    C = torch.full((batch * n * m,), -8531, dtype=torch.int16, device="cuda")
    ops.matmul(torch.from_numpy(A.reshape(-1)).cuda(), torch.from_numpy(B.reshape(-1)).cuda(), C, n=n, k=k, m=m,
               batch=batch, a_batch_stride=0 if a_sh else n * k, b_batch_stride=0 if b_sh else k * m,
               c_batch_stride=n * m, flags=flags)
    want = spec.matmul_raw(np.broadcast_to(A, (batch, n, k)), np.broadcast_to(B, (batch, k, m)), wrap=bool(flags & 1))
    assert np.array_equal(C.cpu().numpy().reshape(batch, n, m), want)


def test_direct_unaligned_falls_back(ops):
    """An operand at an odd element offset (not 16-byte aligned) takes the
    plane-splitting path with the same result."""
    rng = np.random.default_rng(3)
    n, k, m = 40, 64, 48
    A = rng.integers(-32768, 32768, size=n * k + 1).astype(np.int16)
    B = rng.integers(-32768, 32768, size=(k, m)).astype(np.int16)
    Ad = torch.from_numpy(A).cuda()
    C = torch.empty(n * m, dtype=torch.int16, device="cuda")
    ops.matmul(Ad[1:], torch.from_numpy(B.reshape(-1)).cuda(), C, n=n, k=k, m=m)
    assert np.array_equal(C.cpu().numpy().reshape(n, m), spec.matmul_raw(A[1:].reshape(n, k), B))


@pytest.mark.parametrize("C,H,W", [(2048, 6, 5), (3640, 4, 4)])
def test_conv_large_k_int64_rule(ops, C, H, W):
    """Convolutions with K = in_ch kh kw of 18432 (the widening form of the
    rule) and 32760 (the general int64 form) on full-range values, against
    the oracle."""
    rng = np.random.default_rng(11)
    N, M = 1, 24
    x = rng.integers(-32768, 32768, size=(N, C, H, W)).astype(np.int16)
    w = rng.integers(-32768, 32768, size=(M, C, 3, 3)).astype(np.int16)
    b = rng.integers(-32768, 32768, size=(M,)).astype(np.int16)
    y = torch.full((N * M * H * W,), -8531, dtype=torch.int16, device="cuda")
    ops.conv(torch.from_numpy(x.reshape(-1)).cuda(), torch.from_numpy(w.reshape(-1)).cuda(),
             torch.from_numpy(b).cuda(), y, batch=N, in_ch=C, in_h=H, in_w=W, out_ch=M, out_h=H, out_w=W, kh=3,
             kw=3, pad_top=1, pad_left=1, has_bias=1, flags=2)
    want = spec.conv_raw(x, w, b, 1, 1, 1, 1, 1, 1, H, W, False)
    assert np.array_equal(y.cpu().numpy().reshape(N, M, H, W), want)


@pytest.mark.parametrize("k", [512, 2048, 4096])
@pytest.mark.parametrize("pattern", ["min_min", "min_max", "cancel"])
def test_extreme_accumulators(ops, k, pattern):
    """Operands at the int16 extremes: HH at its largest (-32768 * -32768 over
    the whole K), of both signs, and MID / LL pulling against HH — the
    epilogue's forms of floor(acc / 2^8) (int32, clamped HH, int64) agree
    with the oracle's exact sums."""
    rng = np.random.default_rng(k)
    n, m = 130, 72
    if pattern == "min_min":
        A = np.full((n, k), -32768, np.int16)
        B = np.full((k, m), -32768, np.int16)
    elif pattern == "min_max":
        A = np.full((n, k), -32768, np.int16)
        B = np.full((k, m), 32767, np.int16)
    else:  # hi bytes -128 with lo bytes 255 against lo bytes 0
        A = np.where(rng.random((n, k)) < 0.5, -32513, -32768).astype(np.int16)
        B = np.where(rng.random((k, m)) < 0.5, -32768, 255).astype(np.int16)
    C = torch.empty(n * m, dtype=torch.int16, device="cuda")
    # the int16-producer path (aligned operands, small n)
    ops.matmul(torch.from_numpy(A.reshape(-1)).cuda(), torch.from_numpy(B.reshape(-1)).cuda(), C, n=n, k=k, m=m)
    assert np.array_equal(C.cpu().numpy().reshape(n, m), spec.matmul_raw(A, B))
    # the plane path: the same sums through split planes and TMA (an unaligned B offset)
    Bp = np.concatenate([np.zeros(1, np.int16), B.reshape(-1)])
    ops.matmul(torch.from_numpy(A.reshape(-1)).cuda(), torch.from_numpy(Bp).cuda()[1:], C, n=n, k=k, m=m)
    assert np.array_equal(C.cpu().numpy().reshape(n, m), spec.matmul_raw(A, B))


@pytest.mark.parametrize("shape", [(1, 1024, 1536, 1024), (1, 1032, 2048, 1000)], ids=["n1024", "n1032"])
def test_plane_ksplit_vs_oracle(ops, shape):
    """Jobs large enough for the plane path with few tiles and a long K: the
    K split (int64 partial sums, then the rounding pass) on split planes."""
    batch, n, k, m = shape
    rng = np.random.default_rng(n + k)
    A = rng.integers(-32768, 32768, size=(batch, n, k)).astype(np.int16)
    B = rng.integers(-32768, 32768, size=(batch, k, m)).astype(np.int16)
    C = torch.empty(batch * n * m, dtype=torch.int16, device="cuda")
    ops.matmul(torch.from_numpy(A.reshape(-1)).cuda(), torch.from_numpy(B.reshape(-1)).cuda(), C, n=n, k=k, m=m,
               batch=batch, a_batch_stride=n * k, b_batch_stride=k * m, c_batch_stride=n * m)
    assert np.array_equal(C.cpu().numpy().reshape(batch, n, m), spec.matmul_raw(A, B))
