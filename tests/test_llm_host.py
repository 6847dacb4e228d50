"""The float host operations of the LLM entries (scope row f2): LlmEmbed,
LlmDequant, LlmToHost, LlmResAdd, LlmRMSNorm (float32 rows and int16 head
rows), LlmSiluMul / LlmGeluMul and LlmAttnPrep's host form, against the
reference's own outputs (tests/golden/sim_llm_host.npz, made by
``make_golden.py --only llmhost`` from its node factories and _forward_pass).

CPU: the oracle restatement (oracle/llm_host.py) equals the golden.  GPU:
GpuSimulator on one-node graphs of this package's node classes (the
``corm_llm_*`` kernels) equals it bit for bit — float32 outputs compared as
float32, raw words exactly; and the batched host AttnPrep (two sequences side
by side) equals the single-sequence golden per sequence."""
import numpy as np
import pytest

from oracle import llm_host as LH


def _p2(e):
    return np.power(2.0, np.asarray(e, np.float64))[None, :]


def test_oracle_llm_host_vs_reference(golden):
    z = golden("sim_llm_host.npz")
    assert np.array_equal(LH.embed(z["emb_ids"], z["emb_tab"]), z["emb_f32_y"])
    assert np.array_equal(LH.embed(z["emb_ids"], z["emb_tab"], res32_f=15), z["emb_res32_y"])
    assert np.array_equal(LH.dequant(z["deq_x"], z["deq_fx"]), z["deq_y"])
    assert np.array_equal(LH.f32(z["toh_x"]), z["toh_y"])
    assert np.array_equal(LH.resadd(z["radd_h"], z["radd_d"], z["radd_fd"]), z["radd_y"])
    n = z["rms_gamma"].size
    assert np.array_equal(LH.rmsnorm(z["rms_h"], n, z["rms_gamma"], 1e-6, z["rms_fo"]), z["rms_y"])
    h16 = z["rms16_h"] / _p2(z["rms16_fh"])
    assert np.array_equal(LH.rmsnorm(h16, n, z["rms_gamma"], 1e-5, z["rms16_fo"], W=2 * n), z["rms16_y"])
    for kind in ("silu", "gelu"):
        got = LH.act_mul(kind, z["act_g"], z["act_u"], z["act_fg"], z["act_fu"], z["act_fa"])
        assert np.array_equal(got, z[f"{kind}_y"]), kind
    H, KV, HD, C = 6, 2, 32, 64
    for tag in ("pre", "dec"):
        T, pos, nn = (int(v) for v in z[f"prep_{tag}_regs"])
        qx, ck, cv = LH.attn_prep(z[f"prep_{tag}_q0"], z[f"prep_{tag}_k0"], z[f"prep_{tag}_v"], z[f"prep_{tag}_ck0"],
                                  z[f"prep_{tag}_cv0"], pos, T if nn < 0 else nn, T=T, H=H, KV=KV, HD=HD, C=C, Q=16,
                                  fq0=z["prep_fq0"], fk0=z["prep_fk0"], fv=z["prep_fv"], fkc=z["prep_fkc"],
                                  fvc=z["prep_fvc"], fq=z["prep_fq"], cos=z["prep_cos"], sin=z["prep_sin"])
        assert np.array_equal(qx, z[f"prep_{tag}_qx"]), tag
        assert np.array_equal(ck, z[f"prep_{tag}_ck"]) and np.array_equal(cv, z[f"prep_{tag}_cv"]), tag


def _gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import nodes as N
    from cormorant_b200.simulator import GpuSimulator
    return torch, N, GpuSimulator


def _one(N, node, inputs, weights=(), states=()):
    return N.Graph(nodes=[node], weight_tensors=list(weights), input_tensors=list(inputs),
                   output_tensors=[node.output], state_tensors=list(states))


@pytest.mark.gpu
def test_gpu_llm_host_ops_vs_reference(golden):
    torch, N, Sim = _gpu()
    z = golden("sim_llm_host.npz")
    T = N.TensorInfo
    rows, n = z["deq_x"].shape
    # LlmEmbed: float32 rows; the int32 residual (ids past the table clamp)
    V, d = z["emb_tab"].shape
    ids = z["emb_ids"]
    for tag, y_t, res32 in (("emb_f32", T("y", [ids.size, d], host="f32"), False),
                            ("emb_res32", T("y", [ids.size, d], exp=np.asarray(15), dma="i32"), True)):
        it = T("ids", [ids.size], host="i32")
        node = N.LlmEmbedNode(inputs=[it], output=y_t, rows=V, d=d, n=ids.size, res32=res32,
                              table=N.HostTable("tab", "f32", z["emb_tab"]))
        out = Sim(_one(N, node, [it])).forward_pass({"ids": ids})["y"]
        got = out if not res32 else np.rint(out * 2.0 ** 15).astype(np.int64)
        assert np.array_equal(got.reshape(z[f"{tag}_y"].shape), z[f"{tag}_y"]), tag
    # LlmDequant / LlmToHost
    x = T("x", [rows, n], exp=z["deq_fx"])
    y = T("y", [rows, n], host="f32")
    out = Sim(_one(N, N.LlmDequantNode(inputs=[x], output=y, count=rows * n), [x])).forward_pass(
        {"x": z["deq_x"] / _p2(z["deq_fx"])})["y"]
    assert np.array_equal(out, z["deq_y"])
    x = T("x", [rows, n], dma="f32")
    out = Sim(_one(N, N.LlmToHostNode(inputs=[x], output=y, count=rows * n), [x])).forward_pass(
        {"x": z["toh_x"]})["y"]
    assert np.array_equal(out, z["toh_y"])
    # LlmResAdd on the float32 residual
    h, dt = T("h", [rows, n], host="f32"), T("d", [rows, n], exp=z["radd_fd"])
    out = Sim(_one(N, N.LlmResAddNode(inputs=[h, dt], output=y, rows=rows, n=n), [h, dt])).forward_pass(
        {"h": z["radd_h"], "d": z["radd_d"] / _p2(z["radd_fd"])})["y"]
    assert np.array_equal(out, z["radd_y"])
    # LlmRMSNorm: float32 rows, int16 head rows
    yo = T("y", [rows, n], exp=z["rms_fo"])
    node = N.LlmRMSNormNode(inputs=[h], output=yo, rows=rows, n=n, W=n, eps=1e-6, gamma=z["rms_gamma"])
    out = Sim(_one(N, node, [h])).forward_pass({"h": z["rms_h"]})["y"]
    assert np.array_equal(np.rint(out * _p2(z["rms_fo"])).astype(np.int64), z["rms_y"])
    W = 2 * n
    h16, y16 = T("h", [rows, W], exp=z["rms16_fh"]), T("y", [rows, W], exp=z["rms16_fo"])
    node = N.LlmRMSNormNode(inputs=[h16], output=y16, rows=rows * 2, n=n, W=W, i16=True, eps=1e-5,
                            gamma=z["rms_gamma"])
    out = Sim(_one(N, node, [h16])).forward_pass({"h": z["rms16_h"] / _p2(z["rms16_fh"])})["y"]
    assert np.array_equal(np.rint(out * _p2(z["rms16_fo"])).astype(np.int64), z["rms16_y"])
    # LlmSiluMul / LlmGeluMul
    g, u = T("g", [rows, n], exp=z["act_fg"]), T("u", [rows, n], exp=z["act_fu"])
    ya = T("y", [rows, n], exp=z["act_fa"])
    for cls, tag in ((N.LlmSiluMulNode, "silu"), (N.LlmGeluMulNode, "gelu")):
        out = Sim(_one(N, cls(inputs=[g, u], output=ya, rows=rows, n=n), [g, u])).forward_pass(
            {"g": z["act_g"] / _p2(z["act_fg"]), "u": z["act_u"] / _p2(z["act_fu"])})["y"]
        assert np.array_equal(np.rint(out * _p2(z["act_fa"])).astype(np.int64), z[f"{tag}_y"]), tag


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["pre", "dec"])
@pytest.mark.parametrize("B", [1, 2])
def test_gpu_attn_prep_host_vs_reference(golden, tag, B):
    """The host AttnPrep for B sequences side by side (each with the golden's
    inputs and caches) equals the reference's single sequence per sequence."""
    torch, N, Sim = _gpu()
    z = golden("sim_llm_host.npz")
    T_ = N.TensorInfo
    H, KV, HD, C = 6, 2, 32, 64
    G = H // KV
    T, pos, nn = (int(v) for v in z[f"prep_{tag}_regs"])
    has_n = nn >= 0
    q0 = T_("q0", [B * T, H * HD], exp=z["prep_fq0"])
    k0 = T_("k0", [B * T, KV * HD], exp=z["prep_fk0"])
    v = T_("v", [B * T, KV * HD], exp=z["prep_fv"])
    pt, nt = T_("pos", [1], host="i32"), T_("n", [1], host="i32")
    ck = T_("ck", [B * C, KV * HD], exp=z["prep_fkc"], is_state=True, group_layout=(KV, HD))
    cv = T_("cv", [B * C, KV * HD], exp=z["prep_fvc"], is_state=True, group_layout=(KV, HD))
    qx = T_("qx", [KV, B, HD, G * T], exp=np.asarray(0))
    ins = [q0, k0, v, pt] + ([nt] if has_n else []) + [ck, cv]
    node = N.LlmAttnPrepNode(inputs=ins, output=qx, T=T, H=H, KV=KV, HD=HD, C=C, Q=16, has_n=has_n, fq=z["prep_fq"],
                             cos=z["prep_cos"], sin=z["prep_sin"], batch=B)
    graph = _one(N, node, [q0, k0, v, pt] + ([nt] if has_n else []), states=[ck, cv])
    rep = lambda a: np.concatenate([a] * B, axis=0)  # noqa: E731
    feeds = {"q0": rep(z[f"prep_{tag}_q0"]) / _p2(z["prep_fq0"]), "k0": rep(z[f"prep_{tag}_k0"]) / _p2(z["prep_fk0"]),
             "v": rep(z[f"prep_{tag}_v"]) / _p2(z["prep_fv"]), "pos": np.array([pos], np.int32)}
    if has_n:
        feeds["n"] = np.array([nn], np.int32)
    states = {"ck": rep(z[f"prep_{tag}_ck0"]) / _p2(z["prep_fkc"]), "cv": rep(z[f"prep_{tag}_cv0"]) / _p2(z["prep_fvc"])}
    out = Sim(graph).forward_pass(feeds, states=states)
    got_qx = np.rint(out["qx"]).astype(np.int64).reshape(KV, B, HD, G * T)
    for b in range(B):
        assert np.array_equal(got_qx[:, b], z[f"prep_{tag}_qx"]), b
        assert np.array_equal(np.rint(states["ck"][b * C:(b + 1) * C] * _p2(z["prep_fkc"])).astype(np.int64),
                              z[f"prep_{tag}_ck"]), b
        assert np.array_equal(np.rint(states["cv"][b * C:(b + 1) * C] * _p2(z["prep_fvc"])).astype(np.int64),
                              z[f"prep_{tag}_cv"]), b
