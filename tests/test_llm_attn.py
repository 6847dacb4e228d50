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


@pytest.mark.parametrize("tag", ["a", "c"])
def test_simulator_host_logic_cpu(z, cpu_ops, tag):
    g, _ = _chain(z, CASES[tag])
    feeds, states = _feeds(z, tag)
    arr = cpu_ops(g, device="cpu").forward_pass(feeds, states=states)
    _check(z, tag, arr, states)


def _batched(z, B, tag="a"):
    """B sequences at case ``tag``'s pos / n: sequence b's inputs and caches
    are case tag's rolled by b rows (distinct data, one golden source)."""
    ten = lambda name, shape, exp=None, **kw: N.TensorInfo(  # noqa: E731
        name, list(shape), exp=None if exp is None else np.asarray(exp, np.int64), **kw)
    q0, k0, v = (ten("q0", (B * T, H * HD), z["fq0"]), ten("k0", (B * T, KV * HD), z["fk0"]),
                 ten("v", (B * T, KV * HD), z["fv"]))
    pos, n = ten("pos", (1,), host="i32"), ten("n", (1,), host="i32")
    ck = ten("ck", (B * C, KV * HD), z["fkc"], is_state=True, group_layout=(KV, HD))
    cv = ten("cv", (B * C, KV * HD), z["fvc"], is_state=True, group_layout=(KV, HD))
    regs = np.array([AT.smx_regs(int(f), 1.0 / np.sqrt(HD), int(p)) for f, p in
                     zip(AT.score_exp(z["fq"], z["fkc"][::HD], KV), z["fp"])])
    nodes, pv = AT.prefill_layer("l0", T=T, H=H, KV=KV, HD=HD, C=C, fq0=z["fq0"], fk0=z["fk0"], fv=z["fv"],
                                 fq=z["fq"], fkc=z["fkc"][::HD], fvc=z["fvc"], fp=z["fp"], cos=z["cos"],
                                 sin=z["sin"], q0=q0, k0=k0, v=v, pos=pos, n=n, ck=ck, cv=cv, batch=B)
    wts = list({t.onnx_name: t for nd in nodes for t in nd.inputs if t is not None and t.data is not None}.values())
    g = N.Graph(nodes=nodes, weight_tensors=wts, input_tensors=[q0, k0, v, pos, n], output_tensors=[pv],
                state_tensors=[ck, cv])
    roll = lambda a, b: np.roll(a, b, axis=0)  # noqa: E731
    raw = {k: np.concatenate([roll(z[f"{tag}_{k}"], b) for b in range(B)]) for k in ("q0", "k0", "v", "ck0", "cv0")}
    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
    posn = [int(x) for x in z[f"{tag}_posn"]]
    feeds = {"q0": raw["q0"] / p2(z["fq0"]), "k0": raw["k0"] / p2(z["fk0"]), "v": raw["v"] / p2(z["fv"]),
             "pos": np.array([posn[0]]), "n": np.array([posn[1]])}
    states = {"ck": raw["ck0"] / p2(z["fkc"]), "cv": raw["cv0"] / p2(z["fvc"])}
    return g, feeds, states, raw, posn, regs


def _check_batched(z, B, arr, states, raw, posn, regs):
    """Every sequence against the oracle run on its own."""
    from oracle import attn as A
    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
    pv = np.rint(arr["l0.pv"] * p2(z["fpv"])).astype(np.int64)
    ck = np.rint(states["ck"] * p2(z["fkc"])).astype(np.int64)
    cv = np.rint(states["cv"] * p2(z["fvc"])).astype(np.int64)
    for b in range(B):
        ck0, cv0 = raw["ck0"][b * C:(b + 1) * C].copy(), raw["cv0"][b * C:(b + 1) * C].copy()
        sl = slice(b * T, (b + 1) * T)
        out = A.prefill_layer(raw["q0"][sl], raw["k0"][sl], raw["v"][sl], posn[0], posn[1], T=T, H=H, KV=KV, HD=HD,
                              C=C, fq0=z["fq0"], fk0=z["fk0"], fv=z["fv"], fq=z["fq"], fkc=z["fkc"], fvc=z["fvc"],
                              cos=z["cos"], sin=z["sin"], ck=ck0, cv=cv0, cm=regs[:, 0], cfg=regs[:, 1])
        assert np.array_equal(pv[sl], out["pv"]), b
        assert np.array_equal(ck[b * C:(b + 1) * C], ck0) and np.array_equal(cv[b * C:(b + 1) * C], cv0), b
        qx = np.rint(arr["l0.qx"]).astype(np.int64).reshape(KV, B, HD, G * T)
        assert np.array_equal(qx[:, b], out["qx"]), b
        for g in range(KV):
            s = np.rint(arr[f"l0.s{g}"]).astype(np.int64).reshape(C, B, G * T)
            assert np.array_equal(s[:, b], out[f"s{g}"]), (b, g)
            p = np.rint(arr[f"l0.p{g}"]).astype(np.int64).reshape(B, G * T, C)
            assert np.array_equal(p[b], out[f"p{g}"]), (b, g)


def test_simulator_batched_cpu(z, cpu_ops):
    g, feeds, states, raw, posn, regs = _batched(z, 3)
    arr = cpu_ops(g, device="cpu").forward_pass(feeds, states=states)
    _check_batched(z, 3, arr, states, raw, posn, regs)


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


@pytest.mark.gpu
@pytest.mark.parametrize("tag,B", [("a", 5), ("d", 2)])
def test_gpu_prefill_attention_batched(z, sim_cls, tag, B):
    """B sequences in one pass (the batched launches) against the oracle run
    per sequence."""
    g, feeds, states, raw, posn, regs = _batched(z, B, tag)
    arr = sim_cls(g).forward_pass(feeds, states=states)
    _check_batched(z, B, arr, states, raw, posn, regs)
