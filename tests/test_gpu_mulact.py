"""Gate / up pairs (corm_matmul_groups / corm_matmul_bplanes with mulact):
one GEMM over the gate and up weights interleaved in 16-column blocks whose
epilogue applies the row-ops MULACT (SiLU(g << sa) u rounded at sc) equals
the two MatMuls followed by the MULACT job — on the split-plane form (many
rows), the int16-operand form, the weight-planes form with 64 rows (MMAs of
M = 64) and with more, a K-split job (the MULACTs in the finish pass), with
and without the int32 wrap, with the 64-bit (sa <= 23) and the 128-bit SiLU
paths.  Bit-exact."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import ops as o
    return o


def _entry(sa, sc):
    e = np.zeros(16, np.uint8)
    e[8], e[10] = sa, sc
    return torch.from_numpy(e.view(np.int16).copy()).cuda()


@pytest.mark.parametrize("case", [(2048, 256, 512, 0, 14, 22, "groups"), (300, 96, 160, 1, 10, 24, "groups"),
                                  (64, 960, 2560, 1, 1, 23, "bplanes"), (200, 128, 96, 0, 30, 35, "bplanes"),
                                  (7, 64, 64, 0, 2, 20, "bplanes"), (40, 2048, 256, 1, 28, 40, "groups")],
                         ids=["planes", "int16", "bplanes_m64", "bplanes_slow", "bplanes_7rows", "int16_split"])
def test_mulact_pairs(ops, case):
    from cormorant_b200 import rowops_host as RH
    n, k, ffn, wrap, sa, sc, form = case
    g_ = torch.Generator(device="cuda")
    g_.manual_seed(n + k + ffn)
    lim = 1 << 15 if wrap else 600
    A = torch.randint(-lim, lim, (n * k,), dtype=torch.int16, device="cuda", generator=g_)
    Wg = torch.randint(-lim, lim, (k * ffn,), dtype=torch.int16, device="cuda", generator=g_)
    Wu = torch.randint(-lim, lim, (k * ffn,), dtype=torch.int16, device="cuda", generator=g_)
    flags = 1 if wrap else 0  # CORM_F_WRAP32
    # the reference composition: both MatMuls, then the MULACT job with one broadcast entry
    gy = torch.empty(n * ffn, dtype=torch.int16, device="cuda")
    uy = torch.empty(n * ffn, dtype=torch.int16, device="cuda")
    for W, y in ((Wg, gy), (Wu, uy)):
        ops.matmul(A, W, y, n=n, k=k, m=ffn, flags=flags)
    want = torch.empty(n * ffn + 16, dtype=torch.int16, device="cuda")
    ops.rowops(gy, uy, want, _entry(sa, sc), op=RH.opword(RH.OP_MULACT, b_en=True, p_bcast=True), n=ffn, rows=n,
               a_s1=2 * ffn, b_s1=2 * ffn, c_s1=2 * ffn, win_hi=RH.NO_WINDOW)
    # the pair form
    cat = torch.stack([Wg.view(k, ffn // 16, 16), Wu.view(k, ffn // 16, 16)], dim=2).reshape(-1).contiguous()
    got = torch.full((n * ffn,), -7, dtype=torch.int16, device="cuda")
    if form == "groups":
        ops.matmul_groups(A, cat, [got], [ffn], n=n, k=k, flags=flags, mulact=(sa, sc))
    else:
        planes = ops.split_b_planes(cat, k=k, m=2 * ffn)
        ops.matmul_bplanes(A, planes, None, n=n, k=k, m=2 * ffn, flags=flags, outs=[got], widths=[ffn],
                           mulact=(sa, sc))
    torch.cuda.synchronize()
    assert torch.equal(got, want[:n * ffn])
