"""GPU parity against the reference's register-level known-answer fixtures
(hw/test_data, converted to tests/golden/hw_*.npz): every VectorOP, MatMul,
Conv, Pool and RowOps case, bit for bit, through the C ABI."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests import fixtures as fx  # noqa: E402

pytestmark = pytest.mark.gpu


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import ops as o
    return o


def test_vecop_fixtures(ops, golden):
    z = golden("hw_vecop.npz")
    fails, n = [], 0
    for label, regs, a, b, c_len, check in fx.vecop_cases(z):
        c = torch.full((max(c_len, 1) + 8,), -8531, dtype=torch.int16, device="cuda")
        ops.vectorop(dev(a), dev(b), c, **regs)
        bad = check(c.cpu().numpy())
        if bad:
            fails.append((label, bad[:3]))
        n += 1
    assert n == 212
    assert not fails, fails[:5]


def test_matmul_fixtures(ops, golden):
    z = golden("hw_matmul.npz")
    fails = []
    for label, regs, a, b, cv in fx.matmul_cases(z):
        c = torch.full((max(1, regs["batch"] * regs["c_batch_stride"]),), -8531, dtype=torch.int16, device="cuda")
        ops.matmul(dev(np.concatenate([a, np.zeros(8, np.int16)])), dev(np.concatenate([b, np.zeros(8, np.int16)])),
                   c, **regs)
        if not np.array_equal(c.cpu().numpy()[:len(cv)], cv):
            fails.append(label)
    assert not fails, fails


def test_conv_fixtures(ops, golden):
    z = golden("hw_conv.npz")
    fails = []
    for label, r, x, w, b, y in fx.conv_cases(z):
        P = r["out_h"] * r["out_w"]
        CS = r["y_cs"] or P
        offs = [((m % r["y_cn"]) * CS + (m // r["y_cn"]) * r["y_gs"] if r["y_cn"] else m * CS)
                for m in range(r["out_ch"])]
        span = r["batch"] * r["out_ch"] * P if not (r["y_cn"] or r["y_cs"]) else max(offs) + P
        yy = torch.full((span,), -8531, dtype=torch.int16, device="cuda")
        ops.conv(dev(x), dev(w), dev(b) if r["has_bias"] else None, yy, **r)
        got = yy.cpu().numpy()
        if r["y_cn"] or r["y_cs"]:
            ok = all(np.array_equal(got[o:o + P], y[m * P:(m + 1) * P]) for m, o in enumerate(offs))
        else:
            ok = np.array_equal(got, y)
        if not ok:
            fails.append(label)
    assert not fails, fails


def test_pool_fixtures(ops, golden):
    z = golden("hw_pool.npz")
    fails = []
    for label, r, x, y in fx.pool_cases(z):
        yy = torch.full((len(y),), -8531, dtype=torch.int16, device="cuda")
        ops.pool(dev(x), yy, **r)
        if not np.array_equal(yy.cpu().numpy(), y):
            fails.append(label)
    assert not fails, fails


def test_rowops_fixtures(ops, golden):
    z = golden("hw_rowops.npz")
    fails = []
    for label, r, a, b, p, cexp in fx.rowops_cases(z):
        mem, off = fx.rowops_memory(a, b, p, len(cexp))
        buf = dev(mem)
        regs = {("rows" if k == "c1" else "blocks" if k == "c2" else k): v for k, v in r.items()}
        ops.rowops(buf, buf, buf, buf, a_off=off["a"], b_off=off["b"], c_off=off["c"], p_off=off["p"], **regs)
        got = buf.cpu().numpy()[off["c"]:off["c"] + len(cexp)]
        if not np.array_equal(got, cexp):
            fails.append(label)
    assert not fails, fails
