"""Parity at the timed size: every one of the 128 problems of the benchmark's
MatMul sweep (M {1, 8, 128, 2048} x K {64, 512, 1024,
4096} x N {32, 256, 1024, 4096} x batch {1, 16}, exactly the shapes
``bench.py`` times) through the C ABI (``ops.matmul``, the path the bench
graph replays), against the oracle's MatMul (``oracle.spec.matmul_raw``,
_simulate.py:620-633).  On the bench's distribution, jobs up to 2^30 MACs are
compared in full and larger ones at a seeded grid of at least 4096 outputs,
each recomputed exactly from its row of A and column of B
(``oracle.sampled``); on the full int16 range (which drives the saturating
and wide-sum forms of the epilogue), plain and under the int32-wrap rule of
the exponent path, every job with more than 4096 outputs is checked at such
a grid.  Bit-exact: no tolerance."""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", torch.cuda.current_device())


@pytest.mark.parametrize("dist", ["bench", "full", "full_wrap"])
def test_matmul_sweep_every_problem(dev, dist):
    from bench import sweep_problems
    from cormorant_b200 import ops
    from cormorant_b200._lib import F_WRAP32
    from oracle import sampled
    probs = sweep_problems()
    assert len(probs) == 128
    lo, hi = (-256, 256) if dist == "bench" else (-32768, 32768)
    flags = F_WRAP32 if dist == "full_wrap" else 0
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    checked = bad = full = 0
    for i, (b, m, k, n) in enumerate(probs):
        A = torch.randint(lo, hi, (b * m * k,), dtype=torch.int16, device=dev, generator=g)
        B = torch.randint(lo, hi, (b * k * n,), dtype=torch.int16, device=dev, generator=g)
        C = torch.full((b * m * n,), 0x5A5A, dtype=torch.int16, device=dev)
        ops.matmul(A, B, C, n=m, k=k, m=n, batch=b, a_batch_stride=m * k, b_batch_stride=k * n,
                   c_batch_stride=m * n, flags=flags)
        idx = sampled.plan(b, m, k, n, seed=i, full_macs=sampled.FULL_MACS if dist == "bench" else None)
        c_n, c_bad = sampled.check(*sampled.gather(A, B, C, b, m, k, n, idx), wrap=bool(flags))
        assert c_bad == 0, f"problem {i} (batch {b}, M {m}, K {k}, N {n}): {c_bad} of {c_n} outputs differ"
        checked += c_n
        full += int(c_n == b * m * n)
        bad += c_bad
        del A, B, C
    assert bad == 0
    assert full >= (64 if dist == "bench" else 32) and checked > 96 * 4096
    assert ops.device_status() == 0
