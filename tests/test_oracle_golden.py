"""Pin the CPU oracle (oracle/spec.py) against the reference's own golden
vectors: the register-level hw fixtures and the reference simulator outputs."""
import numpy as np
import pytest

from oracle import spec
from tests import fixtures as fx


def test_vecop_fixtures(golden):
    z = golden("hw_vecop.npz")
    fails = []
    n = 0
    for label, regs, a, b, c_len, check in fx.vecop_cases(z):
        c = np.full(max(c_len, 1), -8531, np.int16)          # 0xDEAD poison
        spec.vectorop_job(a, b, c, **regs)
        bad = check(c)
        n += 1
        if bad:
            fails.append((label, bad[:3]))
    assert n == 212
    assert not fails, fails[:5]


def test_matmul_fixtures(golden):
    z = golden("hw_matmul.npz")
    n = 0
    for label, regs, a, b, cv in fx.matmul_cases(z):
        c = np.zeros(regs["batch"] * regs["c_batch_stride"], np.int16)
        spec.matmul_job(a, b, c, **regs)
        assert np.array_equal(c, cv), label
        n += 1
    assert n == 50


def test_conv_fixtures(golden):
    z = golden("hw_conv.npz")
    n = 0
    for label, regs, x, w, b, y in fx.conv_cases(z):
        wi = spec.conv_weight_index(regs["out_ch"], regs["in_ch"], regs["kh"], regs["kw"], bool(regs["is_depthwise"]))
        ww = w.astype(np.int64)[wi]
        xx = x.astype(np.int64).reshape(regs["batch"], regs["in_ch"], regs["in_h"], regs["in_w"])
        bb = b.astype(np.int64)[:regs["out_ch"]] if regs["has_bias"] else None
        got = spec.conv_raw(xx, ww, bb, regs["stride_h"], regs["stride_w"], regs["pad_top"], regs["pad_left"],
                            regs["dilation_h"], regs["dilation_w"], regs["out_h"], regs["out_w"],
                            bool(regs["is_depthwise"]))
        assert np.array_equal(got.reshape(-1), y.astype(np.int64)), label
        # the board-image job writes the same values at the y channel pattern
        if regs["y_cn"] or regs["y_cs"]:
            P = regs["out_h"] * regs["out_w"]
            CS = regs["y_cs"] or P
            span = max(((m % regs["y_cn"]) * CS + (m // regs["y_cn"]) * regs["y_gs"] if regs["y_cn"] else m * CS) + P
                       for m in range(regs["out_ch"]))
            yy = np.zeros(span, np.int16)
            spec.conv_job(x, w, b, yy, **regs)
            for m in range(regs["out_ch"]):
                o = (m % regs["y_cn"]) * CS + (m // regs["y_cn"]) * regs["y_gs"] if regs["y_cn"] else m * CS
                assert np.array_equal(yy[o:o + P], y[m * P:(m + 1) * P]), label
        n += 1
    assert n == 66


def test_pool_fixtures(golden):
    z = golden("hw_pool.npz")
    n = 0
    for label, r, x, y in fx.pool_cases(z):
        xx = x.astype(np.int64).reshape(r["batch"], r["channels"], r["in_h"], r["in_w"])
        got = spec.pool_raw(xx, r["pool_h"], r["pool_w"], r["stride_h"], r["stride_w"], r["pad_top"], r["pad_left"],
                            r["dil_h"], r["dil_w"], r["out_h"], r["out_w"], r["pool_type"], r["lp_order"],
                            r["count_include_pad"])
        assert np.array_equal(got.reshape(-1), y.astype(np.int64)), label
        n += 1
    assert n == 45


def test_rowops_fixtures(golden):
    z = golden("hw_rowops.npz")
    n = 0
    fails = []
    for label, r, a, b, p, cexp in fx.rowops_cases(z):
        mem, off = fx.rowops_memory(a, b, p, len(cexp))
        m = spec.RowOpsMem(mem)
        spec.rowops_job(m, r["op"], r["n"], r["c1"], r["c2"], off["a"], r["a_s1"], r["a_s2"], off["b"], r["b_s1"],
                        r["b_s2"], off["c"], r["c_s1"], r["c_s2"], off["p"], r["eps"], r["aux"], r["bq_sh"],
                        r["win_lo"], r["win_hi"])
        got = mem[off["c"]:off["c"] + len(cexp)]
        if not np.array_equal(got, cexp):
            fails.append(label)
        n += 1
    assert n == 43
    assert not fails, fails


def test_rowops_tables(golden):
    z = golden("hw_rowops.npz")
    assert np.array_equal(np.frombuffer(spec.table_image(), np.uint8), z["tables"])
    s = golden("sim_rowops.npz")
    assert np.array_equal(spec.sigmoid_table(), s["sig_table"])
    assert np.array_equal(spec.rsqrt_table(), s["rsqrt_table"])
    for D, (rm, sh) in zip(s["rsqrt_D"], s["rsqrt_R"]):
        assert spec.rsqrt_bf(int(D)) == (int(rm), int(sh))


def test_act_tables(golden):
    z = golden("sim_act.npz")
    for act in (spec.ACT_SILU, spec.ACT_GELU, spec.ACT_GELU_TANH):
        assert np.array_equal(spec.act_table(act), z[f"act{act}"]), act
    for alpha in (0, 655, 6554, 16384, 32768, 65535):
        assert np.array_equal(spec.act_table(spec.ACT_LEAKY_RELU, alpha), z[f"leaky{alpha}"]), alpha


def test_softmax_spec(golden):
    z = golden("sim_smx.npz")
    cm, cs = int(z["cm"]), int(z["cs"])
    assert (cm, cs) == (12102203, 19)
    assert spec.smx_scale_regs(8, 1.0) == (cm, cs)
    for n in (1, 13, 128, 384, 1024):
        x = z[f"row{n}_x"]
        assert np.array_equal(spec.softmax_rows(x, n, cm, cs, 8), z[f"row{n}_p"])
        assert np.array_equal(spec.softmax_rows(x, z[f"row{n}_vc"], cm, cs, 12), z[f"row{n}_pc"])
        assert np.array_equal(spec.softmax_rows(z[f"col{n}_s"].T, n, cm, cs, 8), z[f"col{n}_p"])
    for key in z.files:
        if key.startswith("regs_"):
            _, fs, sg = key.split("_")
            assert spec.smx_scale_regs(float(fs), float(sg)) == tuple(int(v) for v in z[key])


def test_sim_ops(golden):
    """The simulator's node branches (S:620-765) vs the oracle's raw kernels."""
    z = golden("sim_ops.npz")
    x = z["pool_x"]
    for ci in range(9):
        pt, lp, cip, ph, pw, sh, sw, pt_, pl, dh, dw, oh, ow = (int(v) for v in z[f"pool{ci}_params"])
        got = spec.pool_raw(x, ph, pw, sh, sw, pt_, pl, dh, dw, oh, ow, pt, lp, cip)
        assert np.array_equal(got, z[f"pool{ci}_y"]), ci
    x = z["conv_x"]
    for ci in range(6):
        M, kh, kw, sh, sw, pt_, pl, dh, dw, dwise, hb, oh, ow = (int(v) for v in z[f"conv{ci}_params"])
        got = spec.conv_raw(x, z[f"conv{ci}_w"], z[f"conv{ci}_b"] if hb else None, sh, sw, pt_, pl, dh, dw, oh, ow,
                            bool(dwise))
        assert np.array_equal(got, z[f"conv{ci}_y"]), ci
    for ci in range(4):
        assert np.array_equal(spec.matmul_raw(z[f"mm{ci}_a"], z[f"mm{ci}_b"]), z[f"mm{ci}_c"]), ci
    a, b = z["vop_a"], z["vop_b"]
    for op in range(10):
        for act in range(7):
            key = f"vop{op}_{act}"
            if key not in z.files:
                continue
            alpha = 6554 if (act == 3 or op == 6) else 0
            c = np.zeros(a.size, np.int16)
            if op <= 3:
                spec.vectorop_job(a.reshape(-1), b, c, 40, op, 12, 40, 0, act, alpha)
            else:
                spec.vectorop_job(a.reshape(-1), None, c, a.size, op, 1, 0, 0, act, alpha)
            assert np.array_equal(c.astype(np.int64).reshape(a.shape), z[key]), key


@pytest.mark.parametrize("seed", [1, 2])
def test_mnist_sim(golden, seed):
    z = golden(f"sim_mnist_s{seed}.npz")
    c1 = spec.conv_raw(z["x"], z["w1"], z["b1"], 1, 1, 1, 1, 1, 1, 28, 28, False)
    assert np.array_equal(c1, z["c1"])
    r1 = np.maximum(c1, 0)
    p1 = spec.pool_raw(r1, 2, 2, 2, 2, 0, 0, 1, 1, 14, 14, 0, 0, 0)
    assert np.array_equal(p1, z["p1"])
    c2 = spec.conv_raw(p1, z["w2"], z["b2"], 1, 1, 1, 1, 1, 1, 14, 14, False)
    assert np.array_equal(c2, z["c2"])
    p2 = spec.pool_raw(np.maximum(c2, 0), 2, 2, 2, 2, 0, 0, 1, 1, 7, 7, 0, 0, 0)
    assert np.array_equal(p2, z["p2"])
    mm = spec.matmul_raw(p2.reshape(1, 1568), z["wf"])
    assert np.array_equal(mm, z["mm"])
    logits = spec.sat16(mm + z["bf"])
    assert np.array_equal(logits, z["logits"])
    cm, cs = spec.smx_scale_regs(8, 1.0)
    assert np.array_equal(spec.softmax_rows(logits, 10, cm, cs, 8), z["prob"])


@pytest.mark.parametrize("name,build", [
    ("mnist_b2", lambda: __import__("cormorant_b200.workloads", fromlist=["x"]).mnist(seed=11, batch=2)),
    ("mbv2_r32_b2", lambda: __import__("cormorant_b200.workloads", fromlist=["x"]).mobilenet_v2(seed=13, batch=2,
                                                                                                 res=32)),
])
def test_graph_oracle_vs_reference(golden, name, build):
    """The oracle's forward pass over this package's workload graphs equals the
    reference simulator's _forward_pass over the same architecture built with
    its own node classes (tests/golden/sim_graph_*.npz), node by node."""
    from oracle import graph as og
    z = golden(f"sim_graph_{name}.npz")
    g, feeds, _ = build()
    arr = og.forward(g, feeds)
    for sn in g.nodes:
        key = "t_" + sn.output.onnx_name
        assert np.array_equal(arr[sn.output.onnx_name].reshape(z[key].shape), z[key]), key


def _bert_small():
    from cormorant_b200 import workloads as WL
    return WL.bert_base(seed=17, batch=2, seq=32, layers=2)


def test_bert_oracle_vs_reference(golden):
    """BERT-base widths (2 layers, 2 x 32 tokens): the oracle's pass equals the
    reference simulator's over the same graph built with the reference's own
    LayerNormRoNode / TransposeRoNode / SoftmaxVopNode classes — every
    intermediate by CRC-32 of its raw int16 bytes, the logits in full."""
    import zlib

    from oracle import graph as og
    z = golden("sim_graph_bert_l2_t32_b2.npz")
    g, feeds, _ = _bert_small()
    arr = og.forward(g, feeds)
    for sn in g.nodes:
        name = sn.output.onnx_name
        v = np.ascontiguousarray(arr[name].astype("<i2"))
        assert zlib.crc32(v.tobytes()) == int(z["c_" + name][0]), name
    assert np.array_equal(arr["qa_logits"].reshape(z["out_qa_logits"].shape), z["out_qa_logits"])


def test_bert_rowops_registers_vs_reference(golden):
    """The host builders of the row-ops jobs (cormorant_b200.rowops_host) give
    the registers and parameter words the reference's node layer derives
    (rowops_nodes.from_onnx_layernorm / transpose_job)."""
    z = golden("sim_graph_bert_l2_t32_b2.npz")
    g, _, _ = _bert_small()
    seen = {"LayerNormRoNode": 0, "TransposeRoNode": 0}
    for sn in g.nodes:
        k = type(sn).__name__
        if k not in seen:
            continue
        seen[k] += 1
        r = z["r_" + sn.output.onnx_name]
        if k == "LayerNormRoNode":
            assert [sn.g, sn.bb, sn.E, sn.rows, sn.n] == r.tolist()
            words = np.round(np.asarray(sn.inputs[1].data) * 256).astype(np.int64)
            assert np.array_equal(words, z["p_" + sn.output.onnx_name])
        else:
            assert [0 if sn.kind == "copy" else 1, sn.n, sn.rows, sn.blocks, *sn.strides] == r.tolist()
    assert seen["LayerNormRoNode"] == 5 and seen["TransposeRoNode"] == 10


def test_layer_norm_rows_edges():
    """Constant rows (V = 0: D = E, or 1 when eps = 0), full-scale int16 rows
    and n = 4096 through the int64 / Python-integer split of the oracle agree
    with a per-row Python-integer restatement."""
    from oracle import spec
    rng = np.random.default_rng(5)
    for n, x, gam, bet, eps in [
            (64, np.full((3, 64), 77), np.ones(64), np.zeros(64), 0.0),
            (64, np.full((2, 64), -3), np.full(64, 2.0), np.full(64, 0.5), 1e-5),
            (4096, rng.integers(-32768, 32768, (2, 4096)), 60 * rng.normal(size=4096), 2 * rng.normal(size=4096), 1e-5),
            (768, rng.integers(-300, 300, (4, 768)), 1 + 0.02 * rng.normal(size=768), 0.02 * rng.normal(size=768),
             1e-12)]:
        y = spec.layer_norm_rows(np.asarray(x), gam, bet, eps)
        g = spec.ln_gamma_scale(gam)
        G = np.rint(gam * 2.0 ** g).astype(np.int64)
        bb = spec.ln_beta_bits(bet)
        Bq = [int(v) << (24 + g - bb) for v in np.rint(bet * 2.0 ** bb).astype(np.int64)]
        E = int(round(eps * n * n * 2.0 ** 16))
        for r in range(len(x)):
            xs = [int(v) for v in x[r]]
            S1, S2 = sum(xs), sum(v * v for v in xs)
            D = max(n * S2 - S1 * S1 + E, 0) or 1
            Rm, sh = spec.rsqrt_bf(D)
            want = [max(min(spec._rne(((n * v - S1) * Rm >> (sh - 24)) * int(G[c]) + Bq[c], 24 + g - 8), 32767),
                        -32768) for c, v in enumerate(xs)]
            assert y[r].tolist() == want


def test_rowops_chain_fixtures_numpy(golden):
    """The reference's descriptor-chain fixtures (kernels/rowops_rtl/scripts/
    gen_fixtures.py: a prefill's RoPE / cache / q image jobs, a norm chain
    with a P_KEEP job) on the numpy job model with its parameter RAM."""
    from oracle import spec
    z = golden("hw_rowops.npz")
    cp = z["chain_params"]
    for ci in sorted(set(int(v) for v in cp[:, 0])):
        m, ps = spec.RowOpsMem(z[f"chain{ci}_mem"].copy()), spec.ParamRAM()
        for row in cp[cp[:, 0] == ci]:
            spec.rowops_job(m, *(int(v) for v in row[2:21]), ps=ps)
        assert np.array_equal(m.buf, z[f"chain{ci}_out"]), ci
