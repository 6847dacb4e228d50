"""corm_split_b_planes + corm_matmul_bplanes (a constant weight split into its
planes once; no counterpart in the reference): the MatMul job against the
planes equals the oracle's MatMul bit for bit — few rows, a ragged row count
and column count, a K split, the wrap flag, a batch sharing the weight, the
fused ReLU flag, output column groups, the decode step's shapes under the
wrap rule — and equals corm_matmul."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import spec  # noqa: E402

pytestmark = pytest.mark.gpu

CASES = [  # batch, n, k, m, flags, range
    (1, 64, 960, 960, 0, 3000),
    (1, 37, 264, 100, 1, 32768),
    (1, 64, 2560, 960, 0, 32768),   # K split
    (3, 20, 512, 136, 0, 32768),    # one weight for every batch
    (1, 128, 128, 256, 4, 32768),   # F_ACT_RELU
    # the decode step's shapes under the wrap rule (M = 64 MMAs), a ragged batch with ReLU
    (1, 64, 960, 1600, 1, 32768),
    (1, 64, 2560, 960, 1, 32768),
    (1, 64, 960, 5120, 1, 32768),
    (2, 7, 64, 40, 5, 32768),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b%d_n%d_k%d_m%d_f%d" % c[:5])
def test_bplanes_vs_oracle(case):
    from cormorant_b200 import ops
    batch, n, k, m, flags, hi = case
    rng = np.random.default_rng(n * k + m)
    A = rng.integers(-hi, hi, size=(batch, n, k)).astype(np.int16)
    B = rng.integers(-hi, hi, size=(k, m)).astype(np.int16)
    Bd = torch.from_numpy(B.reshape(-1)).cuda()
    planes = ops.split_b_planes(Bd, k=k, m=m)
    C = torch.full((batch * n * m,), -5, dtype=torch.int16, device="cuda")
    ops.matmul_bplanes(torch.from_numpy(A.reshape(-1)).cuda(), planes, C, n=n, k=k, m=m, batch=batch,
                       a_batch_stride=n * k, c_batch_stride=n * m, flags=flags)
    want = spec.matmul_raw(A, np.broadcast_to(B, (batch, k, m)), wrap=bool(flags & 1))
    if flags & 4:
        want = np.maximum(want, 0)
    assert np.array_equal(C.cpu().numpy().reshape(batch, n, m), want)
    ref = torch.empty_like(C)
    ops.matmul(torch.from_numpy(A.reshape(-1)).cuda(), Bd, ref, n=n, k=k, m=m, batch=batch, a_batch_stride=n * k,
               b_batch_stride=0, c_batch_stride=n * m, flags=flags)
    assert torch.equal(C, ref)


@pytest.mark.parametrize("flags", [0, 1], ids=["exact", "wrap"])
def test_bplanes_groups_vs_oracle(flags):
    from cormorant_b200 import ops
    n, k, widths = 64, 960, (960, 320, 320)
    m = sum(widths)
    rng = np.random.default_rng(5)
    A = rng.integers(-3000, 3000, size=(n, k)).astype(np.int16)
    B = rng.integers(-3000, 3000, size=(k, m)).astype(np.int16)
    planes = ops.split_b_planes(torch.from_numpy(B.reshape(-1)).cuda(), k=k, m=m)
    outs = [torch.empty(n * w, dtype=torch.int16, device="cuda") for w in widths]
    ops.matmul_bplanes(torch.from_numpy(A.reshape(-1)).cuda(), planes, None, n=n, k=k, m=m, outs=outs,
                       widths=list(widths), flags=flags)
    want = spec.matmul_raw(A, B, wrap=bool(flags))
    c0 = 0
    for w, o in zip(widths, outs):
        assert np.array_equal(o.cpu().numpy().reshape(n, w), want[:, c0:c0 + w])
        c0 += w
