"""corm_matmul_groups (sibling projections in one launch, no reference
counterpart): one MatMul job over column-concatenated weights whose output
column groups land in separate buffers.  Each group equals the oracle's MatMul
of A with that group's weight slice, bit for bit: the int16-operand and the
split-plane forms, a K split, batches, the int32 wrap, a last group whose
width is not a multiple of 32; malformed groups are rejected."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import spec  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from cormorant_b200 import ops as o
    return o


CASES = [  # batch, n, k, widths, flags, value range
    (1, 64, 960, (960, 320, 320), 0, 3000),      # decode q / k / v: int16 operands
    (1, 64, 2560, (960, 64), 0, 32768),          # a K split (8 + 1 tiles, 20 K blocks)
    (2, 200, 264, (128, 96, 40), 1, 32768),      # batches, the wrap, a ragged last group
    (1, 2048, 512, (1024, 1024), 0, 32768),      # the split-plane form
    (1, 1032, 1536, (512, 488), 0, 32768),       # planes with a K split
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b%d_n%d_k%d_%s" % (c[0], c[1], c[2], "_".join(map(str, c[3]))))
def test_groups_vs_oracle(ops, case):
    batch, n, k, widths, flags, hi = case
    m = sum(widths)
    rng = np.random.default_rng(n + k + m)
    A = rng.integers(-hi, hi, size=(batch, n, k)).astype(np.int16)
    B = rng.integers(-hi, hi, size=(batch, k, m)).astype(np.int16)
    outs = [torch.full((batch * n * w,), -7777, dtype=torch.int16, device="cuda") for w in widths]
    ops.matmul_groups(torch.from_numpy(A.reshape(-1)).cuda(), torch.from_numpy(B.reshape(-1)).cuda(), outs,
                      list(widths), n=n, k=k, batch=batch, a_batch_stride=n * k, b_batch_stride=k * m, flags=flags)
    want = spec.matmul_raw(A, B, wrap=bool(flags & 1))
    c0 = 0
    for w, o in zip(widths, outs):
        got = o.cpu().numpy().reshape(batch, n, w)
        assert np.array_equal(got, want[:, :, c0:c0 + w]), f"group at column {c0}"
        c0 += w


def test_groups_rejects_unaligned_group(ops):
    from cormorant_b200._lib import CormError
    a = torch.zeros(64 * 64, dtype=torch.int16, device="cuda")
    b = torch.zeros(64 * 100, dtype=torch.int16, device="cuda")
    outs = [torch.empty(64 * 50, dtype=torch.int16, device="cuda") for _ in range(2)]
    with pytest.raises(CormError):
        ops.matmul_groups(a, b, outs, [50, 50], n=64, k=64)  # the first group is no run of 32 columns
