"""The host's p12 softmax (LlmAttnSoftmaxNode, a decode step's) on the
device against the reference's node run through its _forward_pass
(tests/golden/sim_llm_smx_host.npz: a decode step, a prefill with n < T, a
sliding window, a logit scale): the oracle restatement and the product's exp
tables on the CPU, corm_llm_attn_softmax through GpuSimulator on the GPU, one
sequence and a batch of sequences side by side."""
import numpy as np
import pytest

from cormorant_b200 import attention as AT
from cormorant_b200 import nodes as N

G, C = 3, 64
CASES = ["dec", "pre", "win", "scl"]


@pytest.fixture(scope="module")
def z(golden):
    return golden("sim_llm_smx_host.npz")


def _regs(z, tag):
    T, pos, n, W = (int(v) for v in z[f"{tag}_regs"])
    return T, pos, (T if n < 0 else n), n >= 0, W, float(z[f"{tag}_scale"][0])


@pytest.mark.parametrize("tag", CASES)
def test_oracle_matches_reference(z, tag):
    from oracle import attn as A
    T, pos, n, _, W, scale = _regs(z, tag)
    P = A.attn_softmax_host(z[f"{tag}_s"], T=T, G=G, C=C, pos=pos, n_in=n, fs=z["fs"], fp=z["fp"], scale=scale,
                            window=W)
    assert np.array_equal(P, z[f"{tag}_p"])


def test_exp_tables_match_oracle():
    from oracle import attn as A
    for f, sc in ((10, 0.125), (-3, 1.0), (14, 0.2)):
        assert np.array_equal(AT.sexp_table(f, sc), A.sexp_table(f, sc))


def _graph(T, B, has_n, W, scale, fs, fp, C=C):
    ten = lambda name, shape, **kw: N.TensorInfo(name, list(shape), exp=np.asarray(0, np.int64), **kw)  # noqa: E731
    s, p = ten("s", (C, B * G * T)), ten("p", (B * G * T, C))
    pos, n = N.TensorInfo("pos", [1], host="i32"), N.TensorInfo("n", [1], host="i32")
    sn = N.LlmAttnSoftmaxNode(inputs=[s, pos] + ([n] if has_n else []), output=p, T=T, G=G, C=C, Q=16, group=1,
                              scale=scale, fs=fs, fp=fp, has_n=has_n, window=W, batch=B)
    return N.Graph(nodes=[sn], weight_tensors=[], input_tensors=[s, pos] + ([n] if has_n else []), output_tensors=[p])


@pytest.fixture(scope="module")
def sim_cls():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200.simulator import GpuSimulator
    return GpuSimulator


@pytest.mark.gpu
@pytest.mark.parametrize("tag", CASES)
def test_gpu_host_softmax(z, sim_cls, tag):
    T, pos, n, has_n, W, scale = _regs(z, tag)
    g = _graph(T, 1, has_n, W, scale, z["fs"], z["fp"])
    feeds = {"s": z[f"{tag}_s"].astype(np.float64), "pos": np.array([pos])}
    if has_n:
        feeds["n"] = np.array([n])
    out = sim_cls(g).simulate(feeds)["p"]
    assert np.array_equal(np.rint(out).astype(np.int64), z[f"{tag}_p"])


@pytest.mark.gpu
@pytest.mark.parametrize("T,pos,n,W", [(1, 37, 1, 0), (16, 100, 11, 0), (16, 40, 16, 9), (1, 700, 1, 0),
                                       (1, 1100, 1, 0)])
def test_gpu_host_softmax_batched(z, sim_cls, T, pos, n, W):
    """B sequences side by side (the decode batch), long key runs (the
    staged sum over several chunks), pos past the cache (n = 0)."""
    from oracle import attn as A
    B, Cb = 5, 1024
    rng = np.random.default_rng(T + pos)
    s = rng.integers(-9000, 9000, (Cb, B * G * T))
    g = _graph(T, B, True, W, 0.125, z["fs"], z["fp"], C=Cb)
    out = sim_cls(g).simulate({"s": s.astype(np.float64), "pos": np.array([pos]), "n": np.array([n])})["p"]
    got = np.rint(out).astype(np.int64).reshape(B, G * T, Cb)
    for b in range(B):
        want = A.attn_softmax_host(s[:, b * G * T:(b + 1) * G * T], T=T, G=G, C=Cb, pos=pos, n_in=n, fs=z["fs"],
                                   fp=z["fp"], scale=0.125, window=W)
        assert np.array_equal(got[b], want), b
