"""The prefill attention chain on the kernels — AttnPrepRoNode, LlmAttnConvNode
(q.K^T / P.V), LlmAttnSoftmaxVopNode, LlmAttnMergeNode — against the
reference's own node objects (built by its node factories) run through its
_forward_pass over seeded K / V caches (tests/golden/sim_llm_attn.npz):

* CPU: the host builders give the reference's parameter blocks and softmax
  registers; the oracle restatement reproduces every tensor and the caches;
  GpuSimulator's host logic (every job's registers, offsets and the state
  layout) reproduces them with its kernel calls replayed on the oracle's job
  models (a CPU device, no GPU);
* GPU: GpuSimulator on cuda reproduces them, and the static q.K^T row pieces
  / P.V with int32 wrap."""
import zlib

import numpy as np
import pytest

from cormorant_b200 import attention as AT
from cormorant_b200 import nodes as N
from cormorant_b200 import rowops_host as RH

T, H, KV, HD, C = 32, 6, 2, 64, 128
G = H // KV
CASES = {"a": 1, "b": 1, "c": 0, "d": 1}   # causal


@pytest.fixture(scope="module")
def z(golden):
    return golden("sim_llm_attn.npz")


def _chain(z, causal=1):
    ten = lambda name, shape, exp=None, **kw: N.TensorInfo(  # noqa: E731
        name, list(shape), exp=None if exp is None else np.asarray(exp, np.int64), **kw)
    q0, k0, v = ten("q0", (T, H * HD), z["fq0"]), ten("k0", (T, KV * HD), z["fk0"]), ten("v", (T, KV * HD), z["fv"])
    pos, n = ten("pos", (1,), host="i32"), ten("n", (1,), host="i32")
    ck = ten("ck", (C, KV * HD), z["fkc"], is_state=True, group_layout=(KV, HD))
    cv = ten("cv", (C, KV * HD), z["fvc"], is_state=True, group_layout=(KV, HD))
    nodes, pv = AT.prefill_layer("l0", T=T, H=H, KV=KV, HD=HD, C=C, fq0=z["fq0"], fk0=z["fk0"], fv=z["fv"],
                                 fq=z["fq"], fkc=z["fkc"][::HD], fvc=z["fvc"], fp=z["fp"], cos=z["cos"],
                                 sin=z["sin"], q0=q0, k0=k0, v=v, pos=pos, n=n, ck=ck, cv=cv, causal=causal)
    wts = list({t.onnx_name: t for nd in nodes for t in nd.inputs if t is not None and t.data is not None}.values())
    inter = [nd.output for nd in nodes]
    g = N.Graph(nodes=nodes, weight_tensors=wts, input_tensors=[q0, k0, v, pos, n], output_tensors=[pv],
                state_tensors=[ck, cv])
    return g, inter


def _feeds(z, tag):
    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
    pos, n = (int(x) for x in z[f"{tag}_posn"])
    feeds = {"q0": z[f"{tag}_q0"] / p2(z["fq0"]), "k0": z[f"{tag}_k0"] / p2(z["fk0"]), "v": z[f"{tag}_v"] / p2(z["fv"]),
             "pos": np.array([pos]), "n": np.array([n])}
    states = {"ck": z[f"{tag}_ck0"] / p2(z["fkc"]), "cv": z[f"{tag}_cv0"] / p2(z["fvc"])}
    return feeds, states


def _check(z, tag, arr, states):
    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
    raw = lambda a, e=0: np.rint(np.asarray(a) * (p2(e) if np.ndim(e) else 1.0)).astype(np.int64)  # noqa: E731
    assert np.array_equal(raw(arr["l0.qx"]).reshape(KV, HD, G * T), z[f"{tag}_qx"])
    for g in range(KV):
        for k in ("s", "p", "o"):
            assert np.array_equal(raw(arr[f"l0.{k}{g}"]), z[f"{tag}_{k}{g}"]), f"{k}{g}"
    assert np.array_equal(raw(arr["l0.pv"], z["fpv"]), z[f"{tag}_pv"])
    assert np.array_equal(raw(states["ck"], z["fkc"]), z[f"{tag}_ck"])
    assert np.array_equal(raw(states["cv"], z["fvc"]), z[f"{tag}_cv"])


# --------------------------------------------------------------------------- CPU
def test_builders_match_reference(z):
    sa, sb, sc = RH.rope_params(z["fq0"], H, HD, z["fq"])
    w, bc = RH.pblock(0, 0, sa, sb, sc, H * HD)
    assert np.array_equal(w, z["w_pq"]) and bc == bool(z["w_bc"][0])
    sa, sb, sc = RH.rope_params(z["fk0"], KV, HD, z["fkc"][::HD])
    w, bc = RH.pblock(0, 0, sa, sb, sc, KV * HD)
    assert np.array_equal(w, z["w_pk"]) and bc == bool(z["w_bc"][1])
    sa, sc = RH.vround_params(z["fv"], z["fvc"])
    w, bc = RH.pblock(0, 0, sa, 0, sc, KV * HD)
    assert np.array_equal(w, z["w_pvb"]) and bc == bool(z["w_bc"][2])
    words = RH.rope_table_words(z["cos"], z["sin"])
    assert zlib.crc32(words.astype("<i2").tobytes()) == int(z["w_rope_crc"][0])
    fs = AT.score_exp(z["fq"], z["fkc"][::HD], KV)
    assert np.array_equal(fs, z["fs"])
    regs = [AT.smx_regs(int(fs[h]), 1.0 / np.sqrt(HD), int(z["fp"][h])) for h in range(H)]
    assert np.array_equal(np.array(regs), z["w_smx"])


def test_attn_keys():
    assert AT.attn_keys(40, 27, 32, 128) == (27, 80)
    assert AT.attn_keys(0, 32, 32, 128) == (32, 32)
    assert AT.attn_keys(120, 32, 32, 128) == (8, 128)
    assert AT.attn_keys(128, 5, 32, 128) == (0, 128)
    assert AT.attn_keys(0, 0, 32, 128) == (0, 16)
    assert AT.attn_keys(3, 40, 32, 128) == (32, 48)


@pytest.mark.parametrize("tag", sorted(CASES))
def test_oracle_matches_reference(z, tag):
    from oracle import attn as A
    pos, n = (int(x) for x in z[f"{tag}_posn"])
    ck, cv = z[f"{tag}_ck0"].copy(), z[f"{tag}_cv0"].copy()
    out = A.prefill_layer(z[f"{tag}_q0"], z[f"{tag}_k0"], z[f"{tag}_v"], pos, n, T=T, H=H, KV=KV, HD=HD, C=C,
                          fq0=z["fq0"], fk0=z["fk0"], fv=z["fv"], fq=z["fq"], fkc=z["fkc"], fvc=z["fvc"],
                          cos=z["cos"], sin=z["sin"], ck=ck, cv=cv, cm=z["w_smx"][:, 0], cfg=z["w_smx"][:, 1],
                          causal=bool(CASES[tag]))
    for k in ("qx", "s0", "s1", "p0", "p1", "o0", "o1", "pv"):
        assert np.array_equal(out[k], z[f"{tag}_{k}"]), k
    assert np.array_equal(ck, z[f"{tag}_ck"]) and np.array_equal(cv, z[f"{tag}_cv"])


def test_oracle_static_matches_reference(z):
    from oracle import attn as A
    sr = A.attn_scores(z["st_ck"], z["st_qx"], 1, HD=HD, C=C, keys=C, r0=16, nr=48)
    assert np.array_equal(sr, z["st_sr"])
    assert np.array_equal(A.attn_pv(z["st_ps"], z["st_cv"], 0, HD=HD, keys=C), z["st_os"])


@pytest.fixture
def cpu_ops(monkeypatch):
    """ops.rowops / matmul / vectorop replayed on the oracle's job models over
    CPU tensors: the host logic of GpuSimulator without a GPU."""
    import torch

    from cormorant_b200 import ops
    from cormorant_b200._lib import F_WRAP32
    from cormorant_b200.simulator import GpuSimulator
    from oracle import spec

    def np16(t):
        return t.numpy() if t is not None else None

    def rowops(a, b, c, p, *, op, n, rows=1, blocks=1, a_s1=0, a_s2=0, b_s1=0, b_s2=0, c_s1=0, c_s2=0, eps=0, aux=0,
               bq_sh=0, win_lo=0, win_hi=0xFFFFFFFF, a_off=0, b_off=0, c_off=0, p_off=0):
        regions, base, addr = {}, 0, {}
        for nm, t, off in (("a", a, a_off), ("b", b, b_off), ("c", c, c_off), ("p", p, p_off)):
            if t is None:
                addr[nm] = 0
                continue
            st = t.untyped_storage()
            key = st.data_ptr()
            if key not in regions:
                regions[key] = (base, st)
                base += (st.nbytes() + 255) // 256 * 256 + 256
            addr[nm] = regions[key][0] + (t.data_ptr() - key) + off
        mem = np.zeros(base, np.uint8)
        for b0, st in regions.values():
            mem[b0:b0 + st.nbytes()] = np.frombuffer(bytes(st), np.uint8)
        m = spec.RowOpsMem(mem)
        spec.rowops_job(m, op, n, rows, blocks, addr["a"], a_s1, a_s2, addr["b"], b_s1, b_s2, addr["c"], c_s1, c_s2,
                        addr["p"], eps, aux, bq_sh, win_lo, win_hi)
        cst = c.untyped_storage()
        b0 = regions[cst.data_ptr()][0]
        cst.copy_(torch.frombuffer(bytearray(m.buf[b0:b0 + cst.nbytes()].tobytes()), dtype=torch.uint8).untyped_storage())

    def matmul(a, b, c, *, n, k, m, batch=1, a_batch_stride=0, b_batch_stride=0, c_batch_stride=0, b_packed=0,
               gemv_kw=0, flags=0, workspace=None, post=None):
        assert post is None
        spec.matmul_job(np16(a), np16(b), np16(c), n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride,
                        b_packed, gemv_kw, wrap=bool(flags & F_WRAP32))

    def vectorop(a, b, c, *, size, op, outer=1, a_inc=0, b_inc=0, act=0, alpha=0, smx_cm=0, smx_cfg=0, smx_mask=0):
        spec.vectorop_job(np16(a), np16(b), np16(c), size, op, outer, a_inc, b_inc, act, alpha, smx_cm, smx_cfg,
                          smx_mask)

    monkeypatch.setattr(ops, "rowops", rowops)
    monkeypatch.setattr(ops, "matmul", matmul)
    monkeypatch.setattr(ops, "vectorop", vectorop)
    monkeypatch.setattr(GpuSimulator, "_mm_ws", staticmethod(lambda *a: 0))
    return GpuSimulator


@pytest.mark.parametrize("tag", ["a", "c"])
def test_simulator_host_logic_cpu(z, cpu_ops, tag):
    g, _ = _chain(z, CASES[tag])
    feeds, states = _feeds(z, tag)
    arr = cpu_ops(g, device="cpu").forward_pass(feeds, states=states)
    _check(z, tag, arr, states)


# --------------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def sim_cls():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200.simulator import GpuSimulator
    return GpuSimulator


@pytest.mark.gpu
@pytest.mark.parametrize("tag", sorted(CASES))
def test_gpu_prefill_attention(z, sim_cls, tag):
    g, _ = _chain(z, CASES[tag])
    feeds, states = _feeds(z, tag)
    arr = sim_cls(g).forward_pass(feeds, states=states)
    _check(z, tag, arr, states)


@pytest.mark.gpu
def test_gpu_static_rows_and_pv(z, sim_cls):
    """A static q.K^T over the cache rows 16 .. 63 and a static P.V (keys = C)
    on full-range operands: int32 wrap and saturation."""
    ten = lambda name, shape, exp=None, **kw: N.TensorInfo(  # noqa: E731
        name, list(shape), exp=None if exp is None else np.asarray(exp, np.int64), **kw)
    ck = ten("ck", (C, KV * HD), z["fkc"], is_state=True, group_layout=(KV, HD))
    cv = ten("cv", (C, KV * HD), z["fvc"], is_state=True, group_layout=(KV, HD))
    qx, ps = ten("qx", (KV, HD, G * T), 0), ten("ps", (G * T, C), 0)
    sr, os_ = ten("sr", (48, G * T), 0), ten("os", (G * T, HD), 0)
    n1 = N.LlmAttnConvNode(inputs=[ck, qx], output=sr, kind="qk", group=1, T=T, H=H, KV=KV, HD=HD, C=C, static=True,
                           has_n=False, r0=16, nr=48)
    n2 = N.LlmAttnConvNode(inputs=[ps, cv], output=os_, kind="pv", group=0, T=T, H=H, KV=KV, HD=HD, C=C, static=True,
                           has_n=False)
    g = N.Graph(nodes=[n1, n2], weight_tensors=[], input_tensors=[qx, ps], output_tensors=[sr, os_],
                state_tensors=[ck, cv])
    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
    states = {"ck": z["st_ck"] / p2(z["fkc"]), "cv": z["st_cv"] / p2(z["fvc"])}
    arr = sim_cls(g).forward_pass({"qx": z["st_qx"].astype(np.float64), "ps": z["st_ps"].astype(np.float64)},
                                  states=states)
    assert np.array_equal(np.rint(arr["sr"]).astype(np.int64), z["st_sr"])
    assert np.array_equal(np.rint(arr["os"]).astype(np.int64), z["st_os"])
