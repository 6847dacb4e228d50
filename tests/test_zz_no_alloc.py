"""corm_matmul_noalloc — the MatMul entry point for callers that must not
allocate device memory once running (a project whose buffers all come from a
pool sized at start-up, or a host whose device memory belongs to another
allocator).  Its scratch is a fixed array compiled into the library.

Checks, through the C ABI: on two calls in a row with different operands (the
second call must not see the first call's leftovers in the shared scratch),
its output equals corm_matmul's bit for bit (the tolerance of every parity
test here: none) on the tensor-core path and on the small-n path with a K
split; the calls leave the device's free memory unchanged; a job larger than
the scratch is rejected with CORM_ELIMIT; a job whose bounded waits are made
to run out (a diagnostic wait limit of a few hundred cycles) returns, its
timeout is reported once by the status read and then cleared, and the next
call at the default limit is bit-exact again.  The file is named so that
pytest collects it last."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import _lib
    L = _lib.lib()
    assert L.corm_bind_device(torch.cuda.current_device()) == 0
    return _lib


def _desc(_lib, a, b, c, n, k, m, batch, flags=0, ws=None):
    d = _lib.MatmulDesc(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, k, m, batch, n * k, k * m, n * m, 0, 0, flags,
                        None, 0)
    if ws is not None:
        d.workspace, d.workspace_bytes = ws.data_ptr(), ws.numel()
    return d


def _run_both(_lib, n, k, m, batch, seed, flags=0):
    L = _lib.lib()
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    a = torch.randint(-32768, 32768, (batch * n * k,), dtype=torch.int16, device="cuda", generator=g)
    b = torch.randint(-32768, 32768, (batch * k * m,), dtype=torch.int16, device="cuda", generator=g)
    ref = torch.full((batch * n * m,), -1, dtype=torch.int16, device="cuda")
    out = torch.full((batch * n * m,), -2, dtype=torch.int16, device="cuda")
    need = C.c_size_t(0)
    dr = _desc(_lib, a, b, ref, n, k, m, batch, flags)
    assert L.corm_matmul_workspace_size(C.byref(dr), C.byref(need)) == 0
    ws = torch.empty(max(need.value, 256), dtype=torch.uint8, device="cuda")
    dr = _desc(_lib, a, b, ref, n, k, m, batch, flags, ws)
    stream = torch.cuda.current_stream().cuda_stream
    assert L.corm_matmul(C.byref(dr), stream) == 0, L.corm_last_error()
    dn = _desc(_lib, a, b, out, n, k, m, batch, flags)
    assert L.corm_matmul_noalloc(C.byref(dn), stream) == 0, L.corm_last_error()
    torch.cuda.synchronize()
    return ref.cpu().numpy(), out.cpu().numpy()


@pytest.mark.parametrize("shape", [(200, 640, 384, 2), (1, 4096, 96, 1), (7, 2048, 130, 3)],
                         ids=["tensor_path", "small_n_ksplit", "tensor_ksplit"])
def test_noalloc_matches_matmul_twice(lib, shape):
    n, k, m, batch = shape
    for call, seed in enumerate((11, 12)):
        ref, out = _run_both(lib, n, k, m, batch, seed, flags=call & 1)
        assert np.array_equal(out, ref), f"call {call + 1}"


@pytest.mark.parametrize("cbs", [0, 6 * 5, 6 * 5 + 13, 7], ids=["bcast", "dense", "gaps", "overlap"])
def test_k0_clears_outputs_only(lib, cbs):
    """K = 0: every output is floor(0) = 0, on both entry points; with a batch
    stride above n m the words between the batches' outputs are left as they
    were (one clearing call covers the batches)."""
    n, m, batch = 6, 5, 3
    L = lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    a = torch.zeros(8, dtype=torch.int16, device="cuda")
    span = (batch - 1) * cbs + n * m
    want = np.full(span + 8, 7, np.int16)
    for bt in range(batch):
        want[bt * cbs:bt * cbs + n * m] = 0
    for fn in (L.corm_matmul, L.corm_matmul_noalloc):
        c = torch.full((span + 8,), 7, dtype=torch.int16, device="cuda")
        d = lib.MatmulDesc(a.data_ptr(), a.data_ptr(), c.data_ptr(), n, 0, m, batch, 0, 0, cbs, 0, 0, 0, None, 0)
        assert fn(C.byref(d), stream) == 0, L.corm_last_error()
        torch.cuda.synchronize()
        assert np.array_equal(c.cpu().numpy(), want)


def test_noalloc_rejects_oversized(lib):
    L = lib.lib()
    a = torch.zeros(8, dtype=torch.int16, device="cuda")
    d = lib.MatmulDesc(a.data_ptr(), a.data_ptr(), a.data_ptr(), 4096, 4096, 4096, 4, 4096 * 4096, 4096 * 4096,
                       4096 * 4096, 0, 0, 0, None, 0)
    rc = L.corm_matmul_noalloc(C.byref(d), torch.cuda.current_stream().cuda_stream)
    assert rc == lib.CORM_ELIMIT
    assert b"static scratch" in L.corm_last_error()


def test_noalloc_leaves_free_memory_unchanged(lib):
    """The entry point's promise: after a first call per kernel (which may load
    the kernel's code), further calls take no device memory at all."""
    shapes = [(200, 640, 384, 2), (1, 4096, 96, 1), (7, 2048, 130, 3)]
    L = lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    bufs = []
    for n, k, m, batch in shapes:
        a = torch.randint(-32768, 32768, (batch * n * k,), dtype=torch.int16, device="cuda")
        b = torch.randint(-32768, 32768, (batch * k * m,), dtype=torch.int16, device="cuda")
        c = torch.empty(batch * n * m, dtype=torch.int16, device="cuda")
        bufs.append((a, b, c, n, k, m, batch))
    for a, b, c, n, k, m, batch in bufs:  # warm-up: every kernel these jobs use loaded once
        assert L.corm_matmul_noalloc(C.byref(_desc(lib, a, b, c, n, k, m, batch)), stream) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for a, b, c, n, k, m, batch in bufs:
            assert L.corm_matmul_noalloc(C.byref(_desc(lib, a, b, c, n, k, m, batch)), stream) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


@pytest.mark.parametrize("shape", [(256, 4096, 512, 1), (2048, 4096, 2048, 1)], ids=["int16_ksplit", "planes"])
def test_noalloc_timeout_reported_then_cleared(lib, shape):
    """A bounded wait that runs out: the launch returns, the status read reports
    the wait's code once and clears it, and the next job is exact."""
    n, k, m, batch = shape
    L = lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    code = C.c_int(-1)
    assert L.corm_matmul_noalloc_status(C.byref(code), stream) == 0  # start from a clear word
    a = torch.randint(-32768, 32768, (batch * n * k,), dtype=torch.int16, device="cuda")
    b = torch.randint(-32768, 32768, (batch * k * m,), dtype=torch.int16, device="cuda")
    out = torch.zeros(batch * n * m, dtype=torch.int16, device="cuda")
    try:
        # 200 cycles: far below one tile load's latency, so the first wait of
        # every CTA's epilogue runs out
        assert L.corm_set_wait_limit(200) == 0
        assert L.corm_matmul_noalloc(C.byref(_desc(lib, a, b, out, n, k, m, batch)), stream) == 0
        torch.cuda.synchronize()
    finally:
        assert L.corm_set_wait_limit(0) == 0
    assert L.corm_matmul_noalloc_status(C.byref(code), stream) == 0
    assert 101 <= code.value <= 109, code.value
    assert L.corm_matmul_noalloc_status(C.byref(code), stream) == 0
    assert code.value == 0  # read once, then cleared
    # corm_device_status reads (and clears) the word too
    try:
        assert L.corm_set_wait_limit(200) == 0
        assert L.corm_matmul_noalloc(C.byref(_desc(lib, a, b, out, n, k, m, batch)), stream) == 0
    finally:
        assert L.corm_set_wait_limit(0) == 0
    assert L.corm_device_status(C.byref(code)) == 0
    assert 101 <= code.value <= 109, code.value
    assert L.corm_matmul_noalloc_status(C.byref(code), stream) == 0
    assert code.value == 0
    # the default limit again: exact, and no timeout recorded
    ref, got = _run_both(lib, n, k, m, batch, 21)
    assert np.array_equal(got, ref)
    assert L.corm_matmul_noalloc_status(C.byref(code), stream) == 0
    assert code.value == 0
