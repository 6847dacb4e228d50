#!/usr/bin/env python3
"""Generate the committed golden vectors under tests/golden/ (run in the build
container, where the reference checkout is mounted; the GPU box has no
reference, so everything the tests need is written here).

1. ``hw_<kernel>.npz`` — the reference's register-level known-answer fixtures
   (``hw/test_data/<kernel>_test_data/manifest.txt`` + ``test_NN_*.hex``,
   produced by its HLS C++ models and ``kernels/rowops_rtl/scripts/
   gen_fixtures.py``), converted verbatim to int16 / uint8 arrays.
2. ``sim_*.npz`` — outputs of the reference's own Python simulator
   (``inference-scheduler/src``: ``_SimulateMixin._forward_pass``,
   ``vectorop_act.kernel_table``, ``vectorop_smx.softmax_raw``,
   ``rowops_spec``) on seeded inputs, imported through the inert ``onnx``
   stand-in in ``_onnx_stub``.

    python tests/golden/make_golden.py [--ref /root/reference] [--only hw|sim|graph|llm|attn|smx|numeric|convexp|llmhost]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def read_words(path):
    """int16 words, one hex word per line (vecop / matmul / conv / pool)."""
    with open(path) as f:
        v = [int(x, 16) for x in f.read().split()]
    return np.array(v, np.uint16).view(np.int16)


def read_bytes(path):
    """16-byte words as 32 hex digits per line, byte 0 first (rowops)."""
    with open(path) as f:
        s = "".join(f.read().split())
    return np.frombuffer(bytes.fromhex(s), np.uint8).copy()


def manifest(path):
    rows = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line or line.startswith("#"):
                continue
            rows.append(line.split())
    return rows


def convert_hw(ref, out):
    base = os.path.join(ref, "hw", "test_data")
    specs = {
        "vecop": ("vecop_test_data", ["a", "b", "c"], read_words, 11),
        "matmul": ("matmul_test_data", ["a", "b", "c"], read_words, 9),
        "conv": ("conv_test_data", ["x", "w", "b", "y"], read_words, 21),
        "pool": ("pool_test_data", ["x", "y"], read_words, 18),
        "rowops": ("rowops_test_data", ["a", "b", "p", "c"], read_bytes, 16),
    }
    for name, (d, parts, reader, nint) in specs.items():
        rows = manifest(os.path.join(base, d, "manifest.txt"))
        arrays, params, labels = {}, [], []
        for r in rows:
            idx = int(r[0])
            params.append([int(v) for v in r[:nint]])
            labels.append(r[nint] if len(r) > nint else "")
            for p in parts:
                fn = os.path.join(base, d, f"test_{idx:02d}_{p}.hex")
                arrays[f"c{idx}_{p}"] = reader(fn) if os.path.exists(fn) else np.zeros(0, np.int16)
        arrays["params"] = np.array(params, np.int64)
        arrays["labels"] = np.array(labels)
        if name == "rowops":
            arrays["tables"] = read_bytes(os.path.join(base, d, "tables.hex"))
            chains = manifest(os.path.join(base, d, "chains", "manifest.txt"))
            arrays["chain_params"] = np.array([[int(v) for v in c[:21]] for c in chains], np.int64)
            for ci in sorted({int(c[0]) for c in chains}):
                for p in ("mem", "out"):
                    arrays[f"chain{ci}_{p}"] = read_bytes(os.path.join(base, d, "chains", f"chain_{ci:02d}_{p}.hex"))
        np.savez_compressed(os.path.join(out, f"hw_{name}.npz"), **arrays)
        print(f"hw_{name}.npz: {len(rows)} cases")


# --------------------------------------------------------------------------- simulator goldens
def _import_reference(ref):
    sys.path[:0] = [os.path.join(HERE, "_onnx_stub"), os.path.join(ref, "inference-scheduler")]
    import src.codegen._simulate as sim  # noqa: F401
    return sim


class _Graph:
    def __init__(self, nodes, weights, inputs, outputs):
        self.nodes, self.weight_tensors = nodes, weights
        self.input_tensors, self.output_tensors = inputs, outputs
        self.state_tensors = []


def _shim(sim, dtype, graph):
    """A minimal object carrying what ``_SimulateMixin._forward_pass`` reads."""
    class Shim(sim._SimulateMixin):
        pass
    s = Shim()
    s._dtype, s._graph = dtype, graph
    s.initial_states = lambda: {}
    return s


def q88(rng, shape, lo, hi):
    """raw Q8.8 of uniform values in [lo, hi), rounded half to even."""
    return np.clip(np.round(rng.uniform(lo, hi, size=shape) * 256.0), -32768, 32767).astype(np.int64)


def make_mnist(sim, seed):
    """Config 1: Conv 1->16 +bias, Relu, MaxPool, Conv 16->32 +bias, Relu,
    MaxPool, flatten, MatMul 1568x10, Add bias, Softmax (row, Q8.8)."""
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as T
    from src import nodes as N
    import onnx
    rng = np.random.default_rng(seed)
    x = q88(rng, (1, 1, 28, 28), -1, 1)
    w1, b1 = q88(rng, (16, 1, 3, 3), -0.25, 0.25), q88(rng, (16,), -0.25, 0.25)
    w2, b2 = q88(rng, (32, 16, 3, 3), -0.25, 0.25), q88(rng, (32,), -0.25, 0.25)
    wf, bf = q88(rng, (1568, 10), -0.25, 0.25), q88(rng, (1, 10), -0.25, 0.25)
    t = {}

    def ten(name, shape, data=None):
        t[name] = T(onnx_name=name, shape=list(shape), dtype="float32", data=None if data is None else data / 256.0)
        return t[name]
    X = ten("x", x.shape)
    W1, B1, W2, B2 = ten("w1", w1.shape, w1), ten("b1", b1.shape, b1), ten("w2", w2.shape, w2), ten("b2", b2.shape, b2)
    WF, BF = ten("wf", wf.shape, wf), ten("bf", bf.shape, bf)
    c1, r1, p1 = ten("c1", (1, 16, 28, 28)), ten("r1", (1, 16, 28, 28)), ten("p1", (1, 16, 14, 14))
    c2, r2, p2 = ten("c2", (1, 32, 14, 14)), ten("r2", (1, 32, 14, 14)), ten("p2", (1, 32, 7, 7))
    fl, mm, ad = ten("flat", (1, 1568)), ten("mm", (1, 10)), ten("logits", (1, 10))
    nd = onnx.NodeProto()
    nodes = [
        N.ConvNode(onnx_node=nd, inputs=[X, W1, B1], output=c1, batch=1, in_ch=1, in_h=28, in_w=28, out_ch=16,
                   out_h=28, out_w=28, kh=3, kw=3, pad_top=1, pad_left=1, has_bias=True),
        N.ScheduledNode(onnx_node=nd, op_code=N.OP_RELU, arity=1, inputs=[c1], output=r1),
        N.PoolNode(onnx_node=nd, inputs=[r1], output=p1, batch=1, channels=16, in_h=28, in_w=28, out_h=14,
                   out_w=14, pool_h=2, pool_w=2, stride_h=2, stride_w=2, pool_type=N.POOL_MAX),
        N.ConvNode(onnx_node=nd, inputs=[p1, W2, B2], output=c2, batch=1, in_ch=16, in_h=14, in_w=14, out_ch=32,
                   out_h=14, out_w=14, kh=3, kw=3, pad_top=1, pad_left=1, has_bias=True),
        N.ScheduledNode(onnx_node=nd, op_code=N.OP_RELU, arity=1, inputs=[c2], output=r2),
        N.PoolNode(onnx_node=nd, inputs=[r2], output=p2, batch=1, channels=32, in_h=14, in_w=14, out_h=7,
                   out_w=7, pool_h=2, pool_w=2, stride_h=2, stride_w=2, pool_type=N.POOL_MAX),
        N.ReshapeNode(onnx_node=nd, inputs=[p2], output=fl),
        N.MatmulNode(onnx_node=nd, inputs=[fl, WF], output=mm, n=1, k=1568, m=10, batch=1),
        N.ScheduledNode(onnx_node=nd, op_code=N.OP_ADD, arity=2, inputs=[mm, BF], output=ad),
    ]
    g = _Graph(nodes, [W1, B1, W2, B2, WF, BF], [X], [ad])
    arrays = _shim(sim, D, g)._forward_pass({"x": x / 256.0})
    from src import vectorop_smx as VS
    cm, cs = VS.scale_regs(8, 1.0)
    logits = np.round(arrays["logits"] * 256).astype(np.int64)
    prob = VS.softmax_raw(logits, 10, cm, cs, 8)
    out = dict(x=x, w1=w1, b1=b1, w2=w2, b2=b2, wf=wf, bf=bf, prob=prob)
    for k in ("c1", "r1", "p1", "c2", "r2", "p2", "mm", "logits"):
        out[k] = np.round(arrays[k] * 256).astype(np.int64)
    return out


def make_sim(ref, out):
    sim = _import_reference(ref)
    from src import vectorop_act as VA, vectorop_smx as VS, rowops_spec as RS
    from src.nodes import ACT_SILU, ACT_GELU, ACT_GELU_TANH, ACT_LEAKY_RELU
    # activation tables over every Q8.8 input
    tabs = {f"act{a}": np.round(VA.kernel_table(a) * 256).astype(np.int16)
            for a in (ACT_SILU, ACT_GELU, ACT_GELU_TANH)}
    from src.dtype import AP_FIXED_16_8 as D
    xs = np.arange(-32768, 32768, dtype=np.float64) / 256.0
    for alpha in (0, 655, 6554, 16384, 32768, 65535):
        tabs[f"leaky{alpha}"] = np.round(VA.apply(ACT_LEAKY_RELU, xs, D, alpha) * 256).astype(np.int16)
    np.savez_compressed(os.path.join(out, "sim_act.npz"), **tabs)
    # softmax spec on seeded scores, row and column mode, causal masks
    rng = np.random.default_rng(7)
    cm, cs = VS.scale_regs(8, 1.0)
    smx = {"cm": np.array(cm), "cs": np.array(cs)}
    for n in (1, 13, 128, 384, 1024):
        x = rng.integers(-2048, 2048, size=(8, n))
        smx[f"row{n}_x"] = x
        smx[f"row{n}_p"] = VS.softmax_raw(x, n, cm, cs, 8)
        v = VS.causal_valid(8, max(1, n // 3), 4, n)
        smx[f"row{n}_pc"] = VS.softmax_raw(x, v, cm, cs, 12)
        smx[f"row{n}_vc"] = v
        s = rng.integers(-4096, 4096, size=(n, 16))
        smx[f"col{n}_s"] = s
        smx[f"col{n}_p"] = VS.softmax_cols(s, n, cm, cs, 8)
    for fs, sg in ((8, 1.0), (10, 0.125), (6, 0.5), (12, 1.0 / 8.0)):
        smx[f"regs_{fs}_{sg}"] = np.array(VS.scale_regs(fs, sg))
    np.savez_compressed(os.path.join(out, "sim_smx.npz"), **smx)
    # row-ops spec functions
    rng = np.random.default_rng(11)
    ro = {}
    h = rng.integers(-(1 << 20), 1 << 20, size=(6, 960))
    gam = rng.normal(1.0, 0.1, size=960)
    ro["rms_h"], ro["rms_g"] = h, gam
    ro["rms_y"] = RS.rms_norm(h, 15, gam, 1e-5, 10)
    x = rng.integers(-4096, 4096, size=(6, 768))
    bet = rng.normal(0.0, 0.2, size=768)
    ro["ln_x"], ro["ln_g"], ro["ln_b"] = x, gam[:768], bet
    ro["ln_y"] = RS.layer_norm(x, 8, gam[:768], bet, 1e-12, 9)
    g = rng.integers(-8000, 8000, size=(5, 256))
    u = rng.integers(-8000, 8000, size=(5, 256))
    ro["silu_g"], ro["silu_u"], ro["silu_y"] = g, u, RS.silu_mul(g, 10, u, 10, 11)
    xr = rng.integers(-6000, 6000, size=(4, 3, 64))
    ang = np.arange(4)[:, None] * (100000.0 ** (-np.arange(32) / 32.0))[None, :]
    cos = np.concatenate([np.cos(ang), np.cos(ang)], axis=1).astype(np.float32)
    sin = np.concatenate([np.sin(ang), np.sin(ang)], axis=1).astype(np.float32)
    cr, sr = RS.rope_tables_raw(cos, sin)
    ro["rope_x"], ro["rope_c"], ro["rope_s"] = xr, cr, sr
    ro["rope_y"] = RS.rope(xr, 11, cr, sr, 11)
    ro["sig_table"], ro["rsqrt_table"] = RS.sigmoid_table(), RS.rsqrt_table()
    ro["table_image"] = np.frombuffer(RS.table_image(), np.uint8)
    D_ = rng.integers(1, 1 << 62, size=64, dtype=np.int64)
    ro["rsqrt_D"] = D_
    ro["rsqrt_R"] = np.array([RS.rsqrt_bf(int(d)) for d in D_], np.int64)
    np.savez_compressed(os.path.join(out, "sim_rowops.npz"), **ro)
    # the simulator's forward pass: MNIST config, two seeds
    for seed in (1, 2):
        np.savez_compressed(os.path.join(out, f"sim_mnist_s{seed}.npz"), **make_mnist(sim, seed))
    # the simulator's pool / conv / matmul / vectorop branches on small seeded cases
    np.savez_compressed(os.path.join(out, "sim_ops.npz"), **make_ops(sim))
    print("sim goldens written")


def make_ops(sim):
    """Single-node graphs through ``_forward_pass`` (Q8.8 and exponent paths)."""
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as T
    from src import nodes as N
    import onnx
    nd = onnx.NodeProto()
    rng = np.random.default_rng(5)
    out = {}

    def run(nodes, weights, inputs, feeds):
        g = _Graph(nodes, weights, inputs, [nodes[-1].output])
        return _shim(sim, D, g)._forward_pass({k: v / 256.0 for k, v in feeds.items()})

    # pools: every type on one input
    x = q88(rng, (2, 5, 9, 11), -4, 4)
    out["pool_x"] = x
    cases = [(0, 0, 0, 2, 2, 2, 2, 0, 0, 1, 1), (1, 0, 0, 3, 3, 2, 2, 1, 1, 1, 1), (1, 0, 1, 3, 3, 2, 2, 1, 1, 1, 1),
             (2, 1, 0, 2, 3, 1, 2, 0, 1, 1, 1), (2, 2, 0, 3, 3, 2, 2, 1, 1, 1, 1), (2, 2, 0, 2, 2, 1, 1, 0, 0, 2, 2),
             (1, 0, 0, 9, 11, 1, 1, 0, 0, 1, 1), (2, 2, 0, 9, 11, 1, 1, 0, 0, 1, 1), (0, 0, 0, 3, 3, 3, 3, 2, 2, 1, 1)]
    for ci, (pt, lp, cip, ph, pw, sh, sw, pt_, pl, dh, dw) in enumerate(cases):
        oh = (9 + 2 * pt_ - (dh * (ph - 1) + 1)) // sh + 1
        ow = (11 + 2 * pl - (dw * (pw - 1) + 1)) // sw + 1
        X, Y = T(onnx_name="x", shape=[2, 5, 9, 11], dtype="float32"), T(onnx_name="y", shape=[2, 5, oh, ow], dtype="float32")
        n = N.PoolNode(onnx_node=nd, inputs=[X], output=Y, batch=2, channels=5, in_h=9, in_w=11, out_h=oh, out_w=ow,
                       pool_h=ph, pool_w=pw, stride_h=sh, stride_w=sw, pad_top=pt_, pad_left=pl, dil_h=dh, dil_w=dw,
                       pool_type=pt, lp_order=lp, count_include_pad=cip)
        out[f"pool{ci}_params"] = np.array([pt, lp, cip, ph, pw, sh, sw, pt_, pl, dh, dw, oh, ow])
        out[f"pool{ci}_y"] = np.round(run([n], [], [X], {"x": x})["y"] * 256).astype(np.int64)
    # conv Q8.8: standard and depthwise, stride / dilation / padding
    x = q88(rng, (2, 6, 10, 9), -1, 1)
    out["conv_x"] = x
    ccases = [(8, 3, 3, 1, 1, 1, 1, 1, 1, False, True), (4, 3, 3, 2, 2, 1, 1, 1, 1, False, False),
              (6, 3, 3, 1, 2, 1, 1, 2, 1, True, True), (6, 5, 5, 2, 1, 2, 2, 1, 1, True, False),
              (5, 1, 1, 1, 1, 0, 0, 1, 1, False, True), (3, 7, 7, 2, 2, 3, 3, 1, 1, False, True)]
    for ci, (M, kh, kw, sh, sw, pt_, pl, dh, dw, dwise, hb) in enumerate(ccases):
        oh = (10 + 2 * pt_ - (dh * (kh - 1) + 1)) // sh + 1
        ow = (9 + 2 * pl - (dw * (kw - 1) + 1)) // sw + 1
        w = q88(rng, (M, 1 if dwise else 6, kh, kw), -0.5, 0.5)
        b = q88(rng, (M,), -1, 1)
        X = T(onnx_name="x", shape=[2, 6, 10, 9], dtype="float32")
        W = T(onnx_name="w", shape=list(w.shape), dtype="float32", data=w / 256.0)
        B = T(onnx_name="b", shape=[M], dtype="float32", data=b / 256.0)
        Y = T(onnx_name="y", shape=[2, M, oh, ow], dtype="float32")
        n = N.ConvNode(onnx_node=nd, inputs=[X, W, B] if hb else [X, W], output=Y, batch=2, in_ch=6, in_h=10, in_w=9,
                       out_ch=M, out_h=oh, out_w=ow, kh=kh, kw=kw, stride_h=sh, stride_w=sw, dilation_h=dh,
                       dilation_w=dw, pad_top=pt_, pad_left=pl, has_bias=hb, is_depthwise=dwise)
        out[f"conv{ci}_params"] = np.array([M, kh, kw, sh, sw, pt_, pl, dh, dw, int(dwise), int(hb), oh, ow])
        out[f"conv{ci}_w"], out[f"conv{ci}_b"] = w, b
        out[f"conv{ci}_y"] = np.round(run([n], [W, B] if hb else [W], [X], {"x": x})["y"] * 256).astype(np.int64)
    # matmul Q8.8, with saturation, and a batched case
    for ci, (bt, n_, k_, m_, lo, hi) in enumerate([(1, 7, 33, 5, -1, 1), (1, 16, 64, 24, -8, 8), (3, 5, 40, 9, -2, 2),
                                                    (1, 1, 1568, 10, -1, 1)]):
        a = q88(rng, (bt, n_, k_), lo, hi)
        bb = q88(rng, (bt, k_, m_), lo, hi)
        A, B, C = T(onnx_name="a", shape=[bt, n_, k_], dtype="float32"), T(onnx_name="b", shape=[bt, k_, m_], dtype="float32"), T(onnx_name="c", shape=[bt, n_, m_], dtype="float32")
        node = N.MatmulNode(onnx_node=nd, inputs=[A, B], output=C, n=n_, k=k_, m=m_, batch=bt)
        out[f"mm{ci}_a"], out[f"mm{ci}_b"] = a, bb
        out[f"mm{ci}_c"] = np.round(run([node], [], [A, B], {"a": a, "b": bb})["c"] * 256).astype(np.int64)
    # vectorop: every op with every act, broadcast b
    a = q88(rng, (4, 3, 40), -3, 3)
    b = q88(rng, (40,), -3, 3)
    b = np.where(b == 0, 1, b)
    out["vop_a"], out["vop_b"] = a, b
    for op in range(10):
        for act in range(7):
            if op >= 6 and act:
                continue
            A = T(onnx_name="a", shape=[4, 3, 40], dtype="float32")
            Bt = T(onnx_name="b", shape=[40], dtype="float32")
            C = T(onnx_name="c", shape=[4, 3, 40], dtype="float32")
            arity = 2 if op <= 3 else 1
            node = N.ScheduledNode(onnx_node=nd, op_code=op, arity=arity, inputs=[A, Bt] if arity == 2 else [A], output=C)
            node.act, node.alpha = act, 6554 if (act == 3 or op == 6) else 0
            feeds = {"a": a, "b": b} if arity == 2 else {"a": a}
            out[f"vop{op}_{act}"] = np.round(run([node], [], [A, Bt] if arity == 2 else [A], feeds)["c"] * 256).astype(np.int64)
    return out


def make_graph_goldens(ref, out):
    """The benchmark architectures (cormorant_b200.workloads) instantiated with
    the reference's own node classes and run through its _forward_pass."""
    sim = _import_reference(ref)
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from cormorant_b200 import workloads as WL
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as T
    from src import nodes as RN, smx_nodes as SN, rowops_nodes as RON, rowops_spec as RS
    from src.host_nodes import _collapse
    import onnx

    class RefFactory(WL.NodeFactory):
        def tensor(self, name, shape, data=None):
            t = T(onnx_name=name, shape=list(shape), dtype="float32", data=data)
            self.tensors[name] = t
            if data is not None:
                self.weights.append(t)
            return t

        def conv(self, x, w, b, y, **geo):
            self.nodes.append(RN.ConvNode(onnx_node=onnx.NodeProto(), inputs=[x, w] + ([b] if b is not None else []),
                                          output=y, has_bias=b is not None, **geo))

        def vop(self, op, ins, y, act=0):
            n = RN.ScheduledNode(onnx_node=onnx.NodeProto(), op_code=op, arity=len(ins), inputs=ins, output=y)
            n.act = act
            self.nodes.append(n)

        def pool(self, x, y, **geo):
            self.nodes.append(RN.PoolNode(onnx_node=onnx.NodeProto(), inputs=[x], output=y, **geo))

        def reshape(self, x, y):
            self.nodes.append(RN.ReshapeNode(onnx_node=onnx.NodeProto(), inputs=[x], output=y))

        def matmul(self, a, b, y, n, k, m):
            self.nodes.append(RN.MatmulNode(onnx_node=onnx.NodeProto(), inputs=[a, b], output=y, n=n, k=k, m=m,
                                            batch=1))

        def softmax(self, x, y, rows, n, cm, cfg):
            self.nodes.append(SN.SoftmaxVopNode(onnx_node=onnx.NodeProto(), inputs=[x], output=y, rows=rows, n=n,
                                                cm=cm, cfg=cfg))

        # the row-ops nodes exactly as rowops_nodes.from_onnx_layernorm /
        # from_onnx_transpose build them (registers from the reference's own spec)
        def layernorm(self, x, y, rows, n, gamma, beta, eps):
            G, g, _bq, E = RS.norm_params(gamma, n, eps, 8, beta=beta)
            bb = RS.beta_bits(beta)
            words = RS.param_block(G, np.rint(beta * 2.0 ** bb).astype(np.int64), 0, 0, RS.P1_BITS + g - 8)
            p = RON.param_tensor(self.tensors, f"{y.onnx_name}__rowops_p", words)
            self.weights.append(p)
            self.nodes.append(RON.LayerNormRoNode(onnx_node=onnx.NodeProto(), inputs=[x, p, self._tables()], output=y,
                                                  F=8, rows=rows, n=n, eps=eps, g=int(g), bb=int(bb), E=int(E),
                                                  gamma=np.asarray(gamma, np.float64),
                                                  beta=np.asarray(beta, np.float64)))

        def _tables(self):
            had = RON.TABLES_NAME in self.tensors
            t = RON.tables_tensor(self.tensors)
            if not had:
                self.weights.append(t)
            return t

        def transpose(self, x, y, in_shape, perm):
            src = [int(np.prod(in_shape[i + 1:])) for i in range(len(in_shape))]
            dims, sstr = _collapse([in_shape[p] for p in perm], [src[p] for p in perm])
            kind, n, rows, blocks, strides = RON.transpose_job(dims, sstr, 2)
            had = RON.ZERO_P_NAME in self.tensors
            pz = RON.zero_param_tensor(self.tensors)
            if not had:
                self.weights.append(pz)
            self.nodes.append(RON.TransposeRoNode(onnx_node=onnx.NodeProto(), inputs=[x, pz, self._tables()],
                                                  output=y, F=8, kind=kind, n=n, rows=rows, blocks=blocks,
                                                  strides=strides, perm=list(perm), pz=pz))

        def graph(self, inputs, outputs):
            return _Graph(self.nodes, self.weights, inputs, outputs)

    for name, build in (("mnist_b2", lambda f: WL.mnist(seed=11, batch=2, factory=f)),
                        ("mbv2_r32_b2", lambda f: WL.mobilenet_v2(seed=13, batch=2, res=32, factory=f)),
                        ("bert_l2_t32_b2", lambda f: WL.bert_base(seed=17, batch=2, seq=32, layers=2, factory=f))):
        g, feeds, _ = build(RefFactory())
        arrays = _shim(sim, D, g)._forward_pass(feeds)
        outs = {}
        for t in g.output_tensors:
            outs["out_" + t.onnx_name] = np.round(arrays[t.onnx_name] * 256).astype(np.int64)
        # every intermediate too (the fused ones are compared where materialised)
        for sn in g.nodes:
            outs["t_" + sn.output.onnx_name] = np.round(arrays[sn.output.onnx_name] * 256).astype(np.int64)
        for sn in g.nodes:                   # the row-ops registers the reference derived
            if type(sn).__name__ == "LayerNormRoNode":
                outs["r_" + sn.output.onnx_name] = np.array([sn.g, sn.bb, sn.E, sn.rows, sn.n], np.int64)
                outs["p_" + sn.output.onnx_name] = np.round(np.asarray(sn.inputs[1].data) * 256).astype(np.int64)
            elif type(sn).__name__ == "TransposeRoNode":
                outs["r_" + sn.output.onnx_name] = np.array([0 if sn.kind == "copy" else 1, sn.n, sn.rows, sn.blocks,
                                                             *sn.strides], np.int64)
        if name.startswith("bert"):
            # intermediates as CRC-32 of their raw int16 bytes (C order), the
            # outputs in full: a few KB instead of every activation
            outs = {(("c" + k[1:]) if k.startswith("t_") else k):
                    (np.array([zlib.crc32(np.ascontiguousarray(v.astype("<i2")).tobytes())], np.int64)
                     if k.startswith("t_") else v.astype(np.int16) if k.startswith("out_") else v)
                    for k, v in outs.items()}
        np.savez_compressed(os.path.join(out, f"sim_graph_{name}.npz"), **outs)
        print(f"sim_graph_{name}.npz: {len(g.nodes)} nodes")


def make_llm_nodes(ref, out):
    """The LLM kernel nodes on seeded single-node graphs — ResAddRoNode,
    RMSNormRoNode, WidenRoNode, SiluMulRoNode (rowops_nodes.py:400-583) with
    their parameter blocks built as the from_llm_* constructors build them,
    and VitGeluVopNode (vit_nodes.py:580-668) — run through the reference's
    _forward_pass.  Saved: inputs and outputs as raw integers at their
    exponents, the parameter words and registers."""
    sim = _import_reference(ref)
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as T
    from src import rowops_nodes as RON, rowops_spec as RS, vit_nodes as VN
    import onnx
    rng = np.random.default_rng(41)
    res = {}

    def run(node, ins, feeds):
        g = _Graph([node], [t for t in node.inputs if t.data is not None], ins, [node.output])
        return _shim(sim, D, g)._forward_pass(feeds)[node.output.onnx_name]

    def ten(name, shape, exp=None, dma=None, data=None):
        return T(onnx_name=name, shape=list(shape), dtype="float32", data=data,
                 exp=None if exp is None else np.asarray(exp, np.int64), dma=dma)

    rows, n = 6, 64
    # ResAdd: h int32 at 2^-15, d int16 at per-channel exponents <= 15
    fr, fd = 15, rng.integers(8, 16, n)
    hraw = rng.integers(-(1 << 28), 1 << 28, (rows, n))
    draw = rng.integers(-32768, 32768, (rows, n))
    tens = {}
    h, d, y = ten("h", (rows, n), fr, "i32"), ten("d", (rows, n), fd), ten("y", (rows, n), fr, "i32")
    pt, bc = RON._pblock(tens, "y__p", 0, 0, 0, fr - fd, 0, n)
    node = RON.ResAddRoNode(onnx_node=onnx.NodeProto(), inputs=[h, d, pt, RON.tables_tensor(tens)], output=y,
                            F=8, rows=rows, n=n, fr=fr, bcast=bc)
    yv = run(node, [h, d], {"h": hraw / 2.0 ** fr, "d": draw / np.power(2.0, fd)[None, :]})
    res.update(resadd_h=hraw, resadd_d=draw, resadd_fd=fd, resadd_y=np.rint(yv * 2.0 ** fr).astype(np.int64),
               resadd_p=np.rint(np.asarray(pt.data, np.float64) * 256).astype(np.int64), resadd_bc=np.array([bc]))
    # RMSNorm: int32 rows at 2^-15 -> int16 at per-channel exponents (one per channel of a row)
    gamma = 1.0 + 0.1 * rng.standard_normal(n)
    fo = rng.integers(10, 13, n)
    hraw = rng.integers(-(1 << 24), 1 << 24, (rows, n))
    h, y = ten("h", (rows, n), fr, "i32"), ten("y", (rows, n), fo)
    G, g, _bq, E = RS.norm_params(gamma, n, 1e-5, fr, rms=True)
    pt, bc = RON._pblock(tens, "y__p2", G, 0, 0, 0, RS.P1_BITS + g - fo, n)
    node = RON.RMSNormRoNode(onnx_node=onnx.NodeProto(), inputs=[h, pt, RON.tables_tensor(tens)], output=y, F=8,
                             rows=rows, n=n, fr=fr, eps=1e-5, g=int(g), E=int(E), bcast=bc, gamma=gamma)
    yv = run(node, [h], {"h": hraw / 2.0 ** fr})
    res.update(rms_h=hraw, rms_gamma=gamma, rms_fo=fo, rms_y=np.rint(yv * np.power(2.0, fo)[None, :]).astype(np.int64),
               rms_p=np.rint(np.asarray(pt.data, np.float64) * 256).astype(np.int64),
               rms_regs=np.array([int(bc), int(g), int(E)], np.int64))
    # Widen: int16 at fx[c] -> int32 at 12
    fx, fy = rng.integers(4, 13, n), 12
    xraw = rng.integers(-32768, 32768, (rows, n))
    x, y = ten("x", (rows, n), fx), ten("y", (rows, n), fy, "i32")
    pt, bc = RON._pblock(tens, "y__p3", 0, 0, fy - fx, 0, 0, n)
    node = RON.WidenRoNode(onnx_node=onnx.NodeProto(), inputs=[x, pt, RON.tables_tensor(tens)], output=y, F=8,
                           rows=rows, n=n, bcast=bc)
    yv = run(node, [x], {"x": xraw / np.power(2.0, fx)[None, :]})
    res.update(widen_x=xraw, widen_fx=fx, widen_y=np.rint(yv * 2.0 ** fy).astype(np.int64),
               widen_p=np.rint(np.asarray(pt.data, np.float64) * 256).astype(np.int64))
    # SiluMul: g at fg[c] <= 14, u at fu[c], a at fa[c]
    fg, fu, fa = rng.integers(6, 15, n), rng.integers(8, 13, n), rng.integers(8, 13, n)
    graw = rng.integers(-32768, 32768, (rows, n))
    uraw = rng.integers(-32768, 32768, (rows, n))
    gt, ut, y = ten("g", (rows, n), fg), ten("u", (rows, n), fu), ten("y", (rows, n), fa)
    pt, bc = RON._pblock(tens, "y__p4", 0, 0, RS.G_BITS - fg, 0, RS.SILU_BITS + fu - fa, n)
    node = RON.SiluMulRoNode(onnx_node=onnx.NodeProto(), inputs=[gt, ut, pt, RON.tables_tensor(tens)], output=y, F=8,
                             rows=rows, n=n, bcast=bc)
    yv = run(node, [gt, ut], {"g": graw / np.power(2.0, fg)[None, :], "u": uraw / np.power(2.0, fu)[None, :]})
    res.update(silu_g=graw, silu_u=uraw, silu_fg=fg, silu_fu=fu, silu_fa=fa,
               silu_y=np.rint(yv * np.power(2.0, fa)[None, :]).astype(np.int64),
               silu_p=np.rint(np.asarray(pt.data, np.float64) * 256).astype(np.int64))
    # VitGelu: f at ff[c], ba / sc raw rows; erf and tanh
    ff = rng.integers(6, 12, n)
    fraw = rng.integers(-32768, 32768, (rows, n))
    ba = rng.integers(-4000, 4000, n)
    sc = rng.integers(1, 600, n)
    for erf in (False, True):
        f = ten("f", (rows, n), ff)
        bat, sct = ten("ba", (n,), data=(ba / 256.0).astype(np.float32)), ten("sc", (n,), data=(sc / 256.0).astype(np.float32))
        y = ten("y", (rows, n))
        node = VN.VitGeluVopNode(onnx_node=onnx.NodeProto(), inputs=[f, bat, sct], output=y, rows=rows, n=n, F=8,
                                 erf=erf)
        yv = run(node, [f], {"f": fraw / np.power(2.0, ff)[None, :]})
        res[f"vit_y_{int(erf)}"] = np.rint(yv * 256).astype(np.int64)
    res.update(vit_f=fraw, vit_ff=ff, vit_ba=ba, vit_sc=sc)
    np.savez_compressed(os.path.join(out, "sim_llm_nodes.npz"), **res)
    print("sim_llm_nodes.npz:", len(res), "arrays")


class _Attr:
    def __init__(self, name, value):
        self.name, self.value = name, value


class _Node:
    """What the reference's node factories read of an onnx NodeProto."""
    def __init__(self, op_type, inputs, outputs, name="", **attrs):
        self.op_type, self.input, self.output, self.name = op_type, list(inputs), list(outputs), name
        self.attribute = [_Attr(k, v) for k, v in attrs.items()]


def make_llm_attn(ref, out):
    """The prefill attention chain of one layer on the kernels, as the
    reference's node factories build it from LlmAttnPrep (rowops = 1) /
    LlmAttnScores / LlmAttnSoftmax (vsmx = 1) / LlmAttnPV / LlmAttnMerge
    nodes (rowops_nodes.py:1146-1234, llm_nodes.py:1253-1310, 1457-1491,
    1618-1636) — AttnPrepRoNode, LlmAttnConvNode, LlmAttnSoftmaxVopNode,
    LlmAttnMergeNode — run through the reference's _forward_pass over seeded
    K / V caches.  Cases: a prefill at pos > 0 (runtime keys), one from pos
    0 with n = T, a non-causal softmax, and the static q.K^T row pieces /
    P.V of an encoder.  Saved: every input, state and output as raw
    integers, and the registers the factories derived."""
    sim = _import_reference(ref)
    import onnx.helper
    onnx.helper.get_attribute_value = lambda a: a.value
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as TI
    from src import _rowops_hw_config, _vectorop_hw_config
    from src import llm_nodes as LN, rowops_nodes as RON
    from src.host_nodes import HostContext
    _rowops_hw_config.ROWOPS_UNIT = True
    _vectorop_hw_config.VECTOROP_SOFTMAX = True
    rng = np.random.default_rng(43)
    res = {}
    T, H, KV, HD, C = 32, 6, 2, 64, 128
    G = H // KV

    def ten(name, shape, exp=None, **kw):
        return TI(onnx_name=name, shape=list(shape), dtype="float32",
                  exp=None if exp is None else np.asarray(exp, np.int64), **kw)

    # exponents: q0 / k0 per channel (the rotation pairs at different ones), the
    # caches one per KV head (K) / per channel (V), v per channel
    fq0 = rng.integers(9, 13, H * HD)
    fk0 = rng.integers(9, 13, KV * HD)
    fv = rng.integers(9, 13, KV * HD)
    fq = rng.integers(10, 13, H)
    fkc = np.repeat(rng.integers(10, 13, KV), HD)
    fvc = rng.integers(9, 13, KV * HD)
    fs = fq + fkc[::HD][np.arange(H) // G] - 8
    fp = rng.integers(12, 15, H)
    fpv = np.repeat(fp, HD) + np.tile(fvc.reshape(KV, HD), (1, G)).reshape(-1)[:H * HD] - 8
    ang = np.outer(np.arange(C), 1.0 / (10000.0 ** (np.arange(HD // 2) * 2.0 / HD)))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    res.update(fq0=fq0, fk0=fk0, fv=fv, fq=fq, fkc=fkc, fvc=fvc, fs=fs, fp=fp, fpv=fpv, cos=cos, sin=sin)

    def chain(tag, pos, n, causal=1):
        tens = {}
        q0, k0, v = ten("q0", (T, H * HD), fq0), ten("k0", (T, KV * HD), fk0), ten("v", (T, KV * HD), fv)
        post, nt = ten("pos", (1,), host="i32"), ten("n", (1,), host="i32")
        ck = ten("ck", (C, KV * HD), fkc, is_state=True, group_layout=(KV, HD))
        cv = ten("cv", (C, KV * HD), fvc, is_state=True, group_layout=(KV, HD))
        qs, ks = ten("qs", (T, H * HD), 0, is_state=True), ten("ks", (T, KV * HD), 0, is_state=True)
        vs = ten("vs", (T, KV * HD), 0, is_state=True)
        qx = ten("qx", (KV, HD, G * T), 0)
        for t in (q0, k0, v, post, nt, ck, cv, qs, ks, vs, qx):
            tens[t.onnx_name] = t
        tens["cos"], tens["sin"] = ten("cos", cos.shape, data=cos), ten("sin", sin.shape, data=sin)
        ctx = HostContext(opset=17, consts={"cos": cos, "sin": sin}, frac_bits=8)
        common = dict(num_heads=H, num_kv_heads=KV, head_dim=HD, key_quantum=16)
        nodes = [RON.from_llm_attn_prep(
            _Node("LlmAttnPrep", ["q0", "k0", "v", "pos", "n", "ck", "cv", "cos", "sin", "qs", "ks", "vs"], ["qx"],
                  qk_kw=1, q_exp=[int(x) for x in fq], rowops=1, first=1, **common), tens, 0, 8, ctx)]
        for g in range(KV):
            for nm, shp in ((f"s{g}", (C, G * T)), (f"p{g}", (G * T, C)), (f"o{g}", (G * T, HD))):
                tens[nm] = ten(nm, shp, 0)
            nodes.append(LN.LlmAttnConvNode.from_onnx_node(
                _Node("LlmAttnScores", ["ck", "qx", "pos", "n"], [f"s{g}"], group=g, qk_kw=1, **common), tens, 0, 8,
                ctx))
            hs = slice(g * G, (g + 1) * G)
            nodes.append(LN.LlmAttnSoftmaxNode.from_onnx_node(
                _Node("LlmAttnSoftmax", [f"s{g}", "pos", "n"], [f"p{g}"], group=g, s_exp=[int(x) for x in fs[hs]],
                      p_exp=[int(x) for x in fp[hs]], vsmx=1, causal=causal, **common), tens, 0, 8, ctx))
            nodes.append(LN.LlmAttnConvNode.from_onnx_node(
                _Node("LlmAttnPV", [f"p{g}", "cv", "pos", "n"], [f"o{g}"], group=g, **common), tens, 0, 8, ctx))
        tens["pv"] = ten("pv", (T, H * HD), fpv)
        nodes.append(LN.LlmAttnMergeNode.from_onnx_node(
            _Node("LlmAttnMerge", [f"o{g}" for g in range(KV)], ["pv"], **common), tens, 0, 8, ctx))
        wts = list({t.onnx_name: t for nd in nodes for t in nd.inputs if t is not None and t.data is not None}.values())
        g_ = _Graph(nodes, wts, [q0, k0, v, post, nt], [tens["pv"]])
        g_.state_tensors = [ck, cv, qs, ks, vs]
        q0r = rng.integers(-700, 700, (T, H * HD))
        k0r = rng.integers(-700, 700, (T, KV * HD))
        vr = rng.integers(-1500, 1500, (T, KV * HD))
        ckr = rng.integers(-700, 700, (C, KV * HD))
        cvr = rng.integers(-1500, 1500, (C, KV * HD))
        p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
        states = {"ck": ckr / p2(fkc), "cv": cvr / p2(fvc), "qs": np.zeros((T, H * HD)),
                  "ks": np.zeros((T, KV * HD)), "vs": np.zeros((T, KV * HD))}
        feeds = {"q0": q0r / p2(fq0), "k0": k0r / p2(fk0), "v": vr / p2(fv), "pos": np.array([pos], np.int32),
                 "n": np.array([n], np.int32)}
        arr = _shim(sim, D, g_)._forward_pass(feeds, states=states)
        r = lambda a, e=0: np.rint(np.asarray(a, np.float64) * (p2(e) if np.ndim(e) else 2.0 ** e)).astype(np.int64)  # noqa: E731
        res.update({f"{tag}_q0": q0r, f"{tag}_k0": k0r, f"{tag}_v": vr, f"{tag}_ck0": ckr, f"{tag}_cv0": cvr,
                    f"{tag}_posn": np.array([pos, n]), f"{tag}_qx": r(arr["qx"]).reshape(KV, HD, G * T),
                    f"{tag}_ck": r(states["ck"], fkc), f"{tag}_cv": r(states["cv"], fvc),
                    f"{tag}_pv": r(arr["pv"], fpv)})
        for g in range(KV):
            res.update({f"{tag}_s{g}": r(arr[f"s{g}"]), f"{tag}_p{g}": r(arr[f"p{g}"]), f"{tag}_o{g}": r(arr[f"o{g}"])})
        if tag == "a":
            prep, smx = nodes[0], nodes[2]
            for nm in ("pq", "pk", "pvb"):
                t = getattr(prep, nm)
                res[f"w_{nm}"] = np.rint(np.asarray(t.data, np.float64) * 256).astype(np.int64)
            res["w_bc"] = np.array([prep.pq_bc, prep.pk_bc, prep.pv_bc, prep.v_direct], np.int64)
            res["w_rope_crc"] = np.array([zlib.crc32(np.rint(np.asarray(prep.raw.data, np.float64) * 256)
                                                     .astype("<i2").tobytes())], np.int64)
            res["w_smx"] = np.array([[nd.cm[h], nd.cfg[h]] for nd in nodes[2::3][:KV] for h in range(G)], np.int64)
            res["w_keys"] = np.array([nd_.C for nd_ in nodes[1:2]], np.int64)
        print(f"attn {tag}: pos {pos} n {n} keys {LN.attn_keys(pos, n, T, C)[1]}")

    chain("a", 40, 27)          # a prefill at pos 40: keys = roundup(67, 16) = 80
    chain("b", 0, T)            # from pos 0, every row valid: keys 32
    chain("c", 60, 20, causal=0)  # an encoder's rows: every row over keys < pos + n
    chain("d", 120, 32)         # n clamped at the cache end: keys = C

    # static q.K^T row pieces and a static P.V (an encoder's attention, keys = C)
    tens = {}
    ctx = HostContext(opset=17, consts={}, frac_bits=8)
    common = dict(num_heads=H, num_kv_heads=KV, head_dim=HD, key_quantum=16)
    ck = ten("ck", (C, KV * HD), fkc, is_state=True, group_layout=(KV, HD))
    cv = ten("cv", (C, KV * HD), fvc, is_state=True, group_layout=(KV, HD))
    qx = ten("qx", (KV, HD, G * T), 0)
    for t in (ck, cv, qx):
        tens[t.onnx_name] = t
    tens["sr"], tens["ps"], tens["os"] = ten("sr", (48, G * T), 0), ten("ps", (G * T, C), 0), ten("os", (G * T, HD), 0)
    n1 = LN.LlmAttnConvNode.from_onnx_node(_Node("LlmAttnScores", ["ck", "qx"], ["sr"], group=1, rows=[16, 48],
                                                 **common), tens, 0, 8, ctx)
    n2 = LN.LlmAttnConvNode.from_onnx_node(_Node("LlmAttnPV", ["ps", "cv"], ["os"], group=0, **common), tens, 0, 8, ctx)
    g_ = _Graph([n1, n2], [], [qx, tens["ps"]], [tens["sr"], tens["os"]])
    g_.state_tensors = [ck, cv]
    # full-range operands: sums beyond int32 (the wrap) as well as saturated outputs
    ckr = rng.integers(-32768, 32768, (C, KV * HD)) >> rng.integers(0, 6, (C, 1))
    cvr = rng.integers(-32768, 32768, (C, KV * HD)) >> rng.integers(0, 6, (C, 1))
    qxr = rng.integers(-32768, 32768, (KV, HD, G * T)) >> rng.integers(0, 6, (1, 1, G * T))
    psr = rng.integers(0, 32768, (G * T, C)) >> rng.integers(0, 8, (G * T, 1))
    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
    states = {"ck": ckr / p2(fkc), "cv": cvr / p2(fvc)}
    arr = _shim(sim, D, g_)._forward_pass({"qx": qxr.astype(np.float64), "ps": psr.astype(np.float64)}, states=states)
    res.update(st_ck=ckr, st_cv=cvr, st_qx=qxr, st_ps=psr, st_sr=np.rint(arr["sr"]).astype(np.int64),
               st_os=np.rint(arr["os"]).astype(np.int64))
    np.savez_compressed(os.path.join(out, "sim_llm_attn.npz"), **res)
    print("sim_llm_attn.npz:", len(res), "arrays")


def make_llm_smx_host(ref, out):
    """LlmAttnSoftmaxNode (llm_nodes.py:1426-1557, the host's p12 softmax of a
    decode step or a prefill without the unit) from the reference's node
    factory, run through its _forward_pass on seeded scores: a decode step
    (T = 1, no n), a prefill (T = 8, n = 5) and a sliding window (W = 6).
    Saved: the scores, pos / n, the exponents and P as raw integers."""
    sim = _import_reference(ref)
    import onnx.helper
    onnx.helper.get_attribute_value = lambda a: a.value
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as TI
    from src import llm_nodes as LN
    from src.host_nodes import HostContext
    rng = np.random.default_rng(47)
    res = {}
    H, KV, HD, C = 6, 2, 64, 64
    G = H // KV
    fs = rng.integers(9, 13, G)
    fp = rng.integers(12, 15, G)
    res.update(fs=fs, fp=fp)
    cases = {"dec": (1, 37, None, 0, None), "pre": (8, 20, 5, 0, None), "win": (8, 30, 8, 6, None),
             "scl": (8, 10, 8, 0, 0.2)}
    for tag, (T, pos, n, W, scale) in cases.items():
        tens = {}
        s = TI(onnx_name="s", shape=[C, G * T], dtype="float32", exp=np.asarray(0, np.int64))
        y = TI(onnx_name="p", shape=[G * T, C], dtype="float32", exp=np.asarray(0, np.int64))
        post = TI(onnx_name="pos", shape=[1], dtype="float32", host="i32")
        nt = TI(onnx_name="n", shape=[1], dtype="float32", host="i32")
        for t in (s, y, post, nt):
            tens[t.onnx_name] = t
        attrs = dict(num_heads=H, num_kv_heads=KV, head_dim=HD, key_quantum=16, group=1,
                     s_exp=[int(v) for v in fs], p_exp=[int(v) for v in fp])
        if W:
            attrs["window"] = W
        if scale is not None:
            attrs["logit_scale"] = repr(float(scale))
        ins = ["s", "pos"] + (["n"] if n is not None else [""])
        node = LN.LlmAttnSoftmaxNode.from_onnx_node(_Node("LlmAttnSoftmax", ins, ["p"], **attrs), tens, 0, 8,
                                                   HostContext(opset=17, consts={}, frac_bits=8))
        sraw = rng.integers(-6000, 6000, (C, G * T))
        sraw[:, :1] = rng.integers(-32768, 32768, (C, 1))      # a full-range column
        g_ = _Graph([node], [], [s, post] + ([nt] if n is not None else []), [y])
        feeds = {"s": sraw.astype(np.float64), "pos": np.array([pos], np.int32)}
        if n is not None:
            feeds["n"] = np.array([n], np.int32)
        arr = _shim(sim, D, g_)._forward_pass(feeds)
        res.update({f"{tag}_s": sraw, f"{tag}_p": np.rint(arr["p"]).astype(np.int64),
                    f"{tag}_regs": np.array([T, pos, -1 if n is None else n, W], np.int64),
                    f"{tag}_scale": np.array([node.scale])})
    np.savez_compressed(os.path.join(out, "sim_llm_smx_host.npz"), **res)
    print("sim_llm_smx_host.npz:", len(res), "arrays")


def make_llm_host(ref, out):
    """The LLM host ops (llm_nodes.py:466-1790) from the reference's node
    factories, run through its _forward_pass on seeded inputs: LlmEmbed (into
    float32 host rows and into the int32 residual), LlmDequant, LlmToHost,
    LlmResAdd (float32 residual), LlmRMSNorm (float32 rows; int16 head rows at
    per-channel exponents), LlmSiluMul / LlmGeluMul (libm tables per gate
    exponent) and LlmAttnPrep in its host form (float RoPE with the float32
    tables: a prefill with n, a decode step without).  Saved: inputs and
    outputs (raw integers at their exponents, float32 as float64)."""
    sim = _import_reference(ref)
    import onnx.helper
    onnx.helper.get_attribute_value = lambda a: a.value
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as TI
    from src import llm_nodes as LN
    from src.host_nodes import HostContext
    rng = np.random.default_rng(53)
    res = {}

    def ten(name, shape, exp=None, **kw):
        return TI(onnx_name=name, shape=list(shape), dtype="float32",
                  exp=None if exp is None else np.asarray(exp, np.int64), **kw)

    def run(factory, op, ins, outs, tens, feeds, consts=None, states=None, st_tens=(), **attrs):
        ctx = HostContext(opset=17, consts=consts or {}, frac_bits=8)
        node = factory(_Node(op, ins, outs, **attrs), tens, 0, 8, ctx)
        g_ = _Graph([node], [], [tens[i] for i in ins if i and i in feeds], [tens[o] for o in outs])
        g_.state_tensors = list(st_tens)
        arr = _shim(sim, D, g_)._forward_pass(feeds, states=states) if states is not None else \
            _shim(sim, D, g_)._forward_pass(feeds)
        return node, arr

    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))  # noqa: E731
    rows, n, V = 5, 48, 40
    # LlmEmbed: float32 rows, and the int32 residual at 2^-15 (ids past the table clamp)
    tab = (rng.standard_normal((V, n)) * 0.05).astype(np.float32)
    ids = np.array([3, 0, 39, 17, 45, -2], np.int32)
    for tag, yk in (("emb_f32", dict(host="f32")), ("emb_res32", dict(exp=15, dma="i32"))):
        tens = {"ids": ten("ids", (ids.size,), host="i32"), "tab": ten("tab", tab.shape, data=tab),
                "y": ten("y", (ids.size, n), **yk)}
        _, arr = run(LN.LlmEmbedNode.from_onnx_node, "LlmEmbed", ["ids", "tab"], ["y"], tens, {"ids": ids},
                     consts={"tab": tab})
        y = np.asarray(arr["y"], np.float64)
        res[f"{tag}_y"] = y if tag == "emb_f32" else np.rint(y * 2.0 ** 15).astype(np.int64)
    res.update(emb_tab=tab, emb_ids=ids)
    # LlmDequant: int16 at per-channel exponents -> float32
    fx = rng.integers(4, 20, n)
    xr = rng.integers(-32768, 32768, (rows, n))
    tens = {"x": ten("x", (rows, n), fx), "y": ten("y", (rows, n), host="f32")}
    _, arr = run(LN.LlmDequantNode.from_onnx_node, "LlmDequant", ["x"], ["y"], tens, {"x": xr / p2(fx)[None, :]})
    res.update(deq_x=xr, deq_fx=fx, deq_y=np.asarray(arr["y"], np.float64))
    # LlmToHost: a float32 DMA tensor to the host
    xf = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    tens = {"x": ten("x", (rows, n), dma="f32"), "y": ten("y", (rows, n), host="f32")}
    _, arr = run(LN.LlmToHostNode.from_onnx_node, "LlmToHost", ["x"], ["y"], tens, {"x": xf.astype(np.float64)})
    res.update(toh_x=xf, toh_y=np.asarray(arr["y"], np.float64))
    # LlmResAdd: float32 residual + int16 delta at per-channel exponents
    h = (rng.standard_normal((rows, n)) * 4).astype(np.float32)
    fd = rng.integers(8, 16, n)
    dr = rng.integers(-32768, 32768, (rows, n))
    tens = {"h": ten("h", (rows, n), host="f32"), "d": ten("d", (rows, n), fd), "y": ten("y", (rows, n), host="f32")}
    _, arr = run(LN.LlmResAddNode.from_onnx_node, "LlmResAdd", ["h", "d"], ["y"], tens,
                 {"h": h.astype(np.float64), "d": dr / p2(fd)[None, :]})
    res.update(radd_h=h, radd_d=dr, radd_fd=fd, radd_y=np.asarray(arr["y"], np.float64))
    # LlmRMSNorm on float32 rows -> int16 at per-channel exponents
    gamma = (1.0 + 0.2 * rng.standard_normal(n)).astype(np.float32)
    fo = rng.integers(10, 14, n)
    tens = {"h": ten("h", (rows, n), host="f32"), "gamma": ten("gamma", (n,), data=gamma), "y": ten("y", (rows, n), fo)}
    _, arr = run(LN.LlmRMSNormNode.from_onnx_node, "LlmRMSNorm", ["h", "gamma"], ["y"], tens,
                 {"h": h.astype(np.float64)}, consts={"gamma": gamma}, axi_eps=b"1e-06")
    res.update(rms_h=h, rms_gamma=gamma, rms_fo=fo, rms_y=np.rint(np.asarray(arr["y"]) * p2(fo)[None, :]).astype(np.int64))
    # LlmRMSNorm on int16 head rows: rows of W = 2 n (two heads of n), exponents per channel of W
    W = 2 * n
    fh = rng.integers(8, 13, W)
    fo2 = rng.integers(10, 14, W)
    hr = rng.integers(-20000, 20000, (rows, W))
    tens = {"h": ten("h", (rows, W), fh), "gamma": ten("gamma", (n,), data=gamma), "y": ten("y", (rows, W), fo2)}
    node, arr = run(LN.LlmRMSNormNode.from_onnx_node, "LlmRMSNorm", ["h", "gamma"], ["y"], tens,
                    {"h": hr / p2(fh)[None, :]}, consts={"gamma": gamma}, epsilon=1e-5)
    assert node.i16
    res.update(rms16_h=hr, rms16_fh=fh, rms16_fo=fo2,
               rms16_y=np.rint(np.asarray(arr["y"]) * p2(fo2)[None, :]).astype(np.int64))
    # LlmSiluMul / LlmGeluMul: gate at 2-3 exponents, up and out per channel
    fg = rng.choice([9, 11, 13], n)
    fu, fa = rng.integers(8, 13, n), rng.integers(9, 14, n)
    gr = rng.integers(-32768, 32768, (rows, n))
    ur = rng.integers(-32768, 32768, (rows, n))
    for tag, fac, op in (("silu", LN.LlmSiluMulNode.from_onnx_node, "LlmSiluMul"),
                         ("gelu", LN.LlmGeluMulNode.from_onnx_node, "LlmGeluMul")):
        tens = {"g": ten("g", (rows, n), fg), "u": ten("u", (rows, n), fu), "y": ten("y", (rows, n), fa)}
        _, arr = run(fac, op, ["g", "u"], ["y"], tens, {"g": gr / p2(fg)[None, :], "u": ur / p2(fu)[None, :]})
        res[f"{tag}_y"] = np.rint(np.asarray(arr["y"]) * p2(fa)[None, :]).astype(np.int64)
    res.update(act_g=gr, act_u=ur, act_fg=fg, act_fu=fu, act_fa=fa)
    # LlmAttnPrep (host): RoPE in float64 with the float32 tables, the caches'
    # rows at their exponents, the q.K^T image at f_q per head
    H, KV, HD, C = 6, 2, 32, 64
    G = H // KV
    fq0, fk0, fv = rng.integers(9, 13, H * HD), rng.integers(9, 13, KV * HD), rng.integers(9, 13, KV * HD)
    fq = rng.integers(10, 13, H)
    fkc, fvc = np.repeat(rng.integers(10, 13, KV), HD), rng.integers(9, 13, KV * HD)
    ang = np.outer(np.arange(C), 1.0 / (10000.0 ** (np.arange(HD // 2) * 2.0 / HD)))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    res.update(prep_fq0=fq0, prep_fk0=fk0, prep_fv=fv, prep_fq=fq, prep_fkc=fkc, prep_fvc=fvc, prep_cos=cos,
               prep_sin=sin)
    for tag, T, pos, nn in (("pre", 8, 20, 5), ("dec", 1, 37, None)):
        tens = {"q0": ten("q0", (T, H * HD), fq0), "k0": ten("k0", (T, KV * HD), fk0),
                "v": ten("v", (T, KV * HD), fv), "pos": ten("pos", (1,), host="i32"), "n": ten("n", (1,), host="i32"),
                "ck": ten("ck", (C, KV * HD), fkc, is_state=True, group_layout=(KV, HD)),
                "cv": ten("cv", (C, KV * HD), fvc, is_state=True, group_layout=(KV, HD)),
                "qx": ten("qx", (KV, HD, G * T), 0), "cos": ten("cos", cos.shape, data=cos),
                "sin": ten("sin", sin.shape, data=sin)}
        q0r = rng.integers(-20000, 20000, (T, H * HD))
        k0r = rng.integers(-20000, 20000, (T, KV * HD))
        vr = rng.integers(-20000, 20000, (T, KV * HD))
        ckr = rng.integers(-700, 700, (C, KV * HD))
        cvr = rng.integers(-1500, 1500, (C, KV * HD))
        states = {"ck": ckr / p2(fkc)[None, :], "cv": cvr / p2(fvc)[None, :]}
        feeds = {"q0": q0r / p2(fq0)[None, :], "k0": k0r / p2(fk0)[None, :], "v": vr / p2(fv)[None, :],
                 "pos": np.array([pos], np.int32)}
        if nn is not None:
            feeds["n"] = np.array([nn], np.int32)
        _, arr = run(LN.LlmAttnPrepNode.from_onnx_node, "LlmAttnPrep",
                     ["q0", "k0", "v", "pos", "n" if nn is not None else "", "ck", "cv", "cos", "sin"], ["qx"], tens,
                     feeds, consts={"cos": cos, "sin": sin}, states=states, st_tens=[tens["ck"], tens["cv"]],
                     num_heads=H, num_kv_heads=KV, head_dim=HD, q_exp=[int(x) for x in fq], qk_kw=1, key_quantum=16)
        res.update({f"prep_{tag}_q0": q0r, f"prep_{tag}_k0": k0r, f"prep_{tag}_v": vr, f"prep_{tag}_ck0": ckr,
                    f"prep_{tag}_cv0": cvr, f"prep_{tag}_regs": np.array([T, pos, -1 if nn is None else nn]),
                    f"prep_{tag}_qx": np.rint(np.asarray(arr["qx"], np.float64)).astype(np.int64),
                    f"prep_{tag}_ck": np.rint(states["ck"] * p2(fkc)[None, :]).astype(np.int64),
                    f"prep_{tag}_cv": np.rint(states["cv"] * p2(fvc)[None, :]).astype(np.int64)})
    np.savez_compressed(os.path.join(out, "sim_llm_host.npz"), **res)
    print("sim_llm_host.npz:", len(res), "arrays")


def make_numeric(ref, out):
    """The exponent planner: the reference's weight encodings
    (src/numeric.py encode_matmul_weights / encode_conv_weights) on MatMul and
    Conv nodes with per-tensor and per-channel exponents, and its Llama
    formats lookups (src/llama.py Formats: K / V caches, P.V, scores, the
    residual).  Weights are seeded float32; the fixture keeps the inputs and
    the encoded raw words, exponents and saturation counts (for the large
    MatMul, which crosses the row-block boundary, CRCs of them)."""
    _import_reference(ref)
    import types
    import onnx
    from src import numeric as NU, nodes as N
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as T
    from src.graph_builder import score_exp
    from src.llama import Formats
    nd = onnx.NodeProto()
    rng = np.random.default_rng(11)
    res = {}
    mm_cases = [  # tag, batch, K, M, f_in (scalar or [K]), f_out, weight scale
        ("mm_t", 1, 24, 40, 11, 10, 0.05),
        ("mm_ch", 1, 32, 48, rng.integers(6, 14, 32), rng.integers(8, 13, 48), 0.2),
        ("mm_wide", 2, 16, 24, rng.integers(-3, 20, 16), rng.integers(-10, 25, 24), 1.5),
        ("mm_sat", 1, 20, 12, 4, 14, 3.0),
    ]
    for tag, bt, K, M, fi, fo, sc in mm_cases:
        w = (rng.standard_normal((bt, K, M) if bt > 1 else (K, M)) * sc).astype(np.float32)
        A = T(onnx_name="a", shape=[1, 5, K], dtype="float32", exp=np.asarray(fi))
        B = T(onnx_name="w_" + tag, shape=list(w.shape), dtype="float32", data=w.copy())
        C = T(onnx_name="c", shape=[1, 5, M], dtype="float32", exp=np.asarray(fo))
        node = N.MatmulNode(onnx_node=nd, inputs=[A, B], output=C, n=5, k=K, m=M, batch=bt)
        sat = NU.encode_matmul_weights([node], D)
        res[f"{tag}_w"], res[f"{tag}_fin"], res[f"{tag}_fout"] = w, np.asarray(fi), np.asarray(fo)
        res[f"{tag}_raw"] = np.round(B.data.astype(np.float64) * 256).astype(np.int64)
        res[f"{tag}_wexp"] = np.asarray(B.wexp)
        res[f"{tag}_wexp_dtype"] = np.array([np.dtype(B.wexp.dtype).itemsize])
        res[f"{tag}_sat"] = np.array([sat["w_" + tag]])
    # a weight of 2^21 elements: two row blocks of the encoding
    K, M = 2048, 1024
    brng = np.random.default_rng(12345)  # its own stream: the test regenerates the weight
    w = (brng.standard_normal((K, M)) * 0.03).astype(np.float32)
    fi, fo = brng.integers(9, 13, K), brng.integers(9, 12, M)
    B = T(onnx_name="w_big", shape=[K, M], dtype="float32", data=w.copy())
    node = N.MatmulNode(onnx_node=nd, inputs=[T(onnx_name="a", shape=[1, 2, K], dtype="float32", exp=fi), B],
                        output=T(onnx_name="c", shape=[1, 2, M], dtype="float32", exp=fo), n=2, k=K, m=M, batch=1)
    sat = NU.encode_matmul_weights([node], D)
    raw = np.round(B.data.astype(np.float64) * 256).astype(np.int16)
    res["mm_big_seed"] = np.array([12345])
    res["mm_big_crc"] = np.array([zlib.crc32(raw.tobytes()), zlib.crc32(np.ascontiguousarray(B.wexp).tobytes()),
                                  sat["w_big"], np.dtype(B.wexp.dtype).itemsize], np.int64)
    res["mm_big_fin"], res["mm_big_fout"] = fi, fo
    res["mm_big_w_crc"] = np.array([zlib.crc32(w.tobytes())], np.int64)
    # convs: per tensor / per channel, standard / depthwise, with bias
    conv_cases = [  # tag, C, M, kh, kw, depthwise, fx, fy (scalars: exp; vectors: chexp)
        ("cv_t", 6, 8, 3, 3, False, 11, 10),
        ("cv_tdw", 8, 8, 3, 3, True, 12, 9),
        ("cv_ch", 6, 5, 1, 3, False, rng.integers(8, 13, 6), rng.integers(7, 12, 5)),
        ("cv_chdw", 7, 7, 3, 1, True, rng.integers(8, 13, 7), rng.integers(7, 12, 7)),
        ("cv_sat", 4, 3, 1, 1, False, 6, 14),
    ]
    for tag, C, M, kh, kw, dw, fx, fy in conv_cases:
        w = (rng.standard_normal((M, 1 if dw else C, kh, kw)) * (2.0 if tag == "cv_sat" else 0.1)).astype(np.float32)
        b = (rng.standard_normal(M) * 0.5).astype(np.float32)
        per_ch = np.ndim(fx) > 0
        X = T(onnx_name="x", shape=[1, C, 4, 6], dtype="float32", **({"chexp": np.asarray(fx)} if per_ch else {"exp": np.asarray(fx)}))
        Y = T(onnx_name="y", shape=[1, M, 4 - kh + 1, 6 - kw + 1], dtype="float32",
              **({"chexp": np.asarray(fy)} if per_ch else {"exp": np.asarray(fy)}))
        W = T(onnx_name="w_" + tag, shape=list(w.shape), dtype="float32", data=w.copy())
        Bt = T(onnx_name="b_" + tag, shape=[M], dtype="float32", data=b.copy())
        node = N.ConvNode(onnx_node=nd, inputs=[X, W, Bt], output=Y, batch=1, in_ch=C, in_h=4, in_w=6, out_ch=M,
                          out_h=4 - kh + 1, out_w=6 - kw + 1, kh=kh, kw=kw, stride_h=1, stride_w=1, dilation_h=1,
                          dilation_w=1, pad_top=0, pad_left=0, has_bias=True, is_depthwise=dw)
        sat = NU.encode_conv_weights([node], D)
        res[f"{tag}_w"], res[f"{tag}_b"] = w, b
        res[f"{tag}_fx"], res[f"{tag}_fy"] = np.asarray(fx), np.asarray(fy)
        res[f"{tag}_wraw"] = np.round(W.data.astype(np.float64) * 256).astype(np.int64).reshape(w.shape)
        res[f"{tag}_braw"] = np.round(Bt.data.astype(np.float64) * 256).astype(np.int64).reshape(-1)[:M]
        res[f"{tag}_wexp"], res[f"{tag}_bexp"] = np.asarray(W.wexp), np.asarray(Bt.wexp)
        res[f"{tag}_sat"] = np.array([sat["w_" + tag], sat["b_" + tag]])
    # Llama formats lookups on a table with per-head and per-channel entries
    cfg = types.SimpleNamespace(L=2, H=6, KV=2, HD=4)
    exps = {"q@0": [10, 11, 10, 9, 10, 12], "k@0": [10, 11], "p@0": 12, "v@0": 13, "x@0": 12,
            "q@1": 10, "k@1": [9, 10], "p@1": [12, 12, 11, 12, 13, 12], "v@1": list(range(8, 16)),
            "vc@1": [9] * 8, "s@1": [3, 4, 5, 6, 7, 8], "pv@1": list(range(24)), "res@2": 16}
    fm = Formats({"exponents": exps, "policy": "test"}, cfg)
    res["fm_exps"] = np.frombuffer(json.dumps(exps).encode(), np.uint8)
    for li in range(2):
        res[f"fm_k{li}"], res[f"fm_v{li}"], res[f"fm_pv{li}"] = fm.k_cache(li), fm.v_cache(li), fm.pv(li)
        res[f"fm_s{li}"] = (fm.heads("s", li, 6) if f"s@{li}" in fm.exp
                            else score_exp(fm.heads("q", li, 6), fm.heads("k", li, 2), 2))
    res["fm_res"] = np.array([fm.res_bits])
    np.savez_compressed(os.path.join(out, "sim_numeric.npz"), **res)
    print("sim_numeric.npz:", len(res), "arrays")


def make_conv_exp(ref, out):
    """Convs on tensors with power-of-two exponents (``_SimulateMixin._conv_exp``
    + ``_conv2d_int``, _simulate.py:784-812, 198-220): weights and biases
    encoded by the reference's ``numeric.encode_conv_weights``
    (numeric.py:258-307: f_w = f_y + F - f_x, the bias at f_y), inputs on their
    exponents' grids, run through the reference's ``_forward_pass``.  Per-tensor
    and per-channel (chexp) exponents, standard and depthwise, stride /
    padding / dilation, with and without bias, and cases whose int32
    accumulator wraps.  The fixture keeps the raw inputs, the encoded raw
    weight / bias words with their exponents, and the raw outputs."""
    sim = _import_reference(ref)
    import onnx
    from src import numeric as NU, nodes as N
    from src.dtype import AP_FIXED_16_8 as D
    from src.tensor import TensorInfo as T
    nd = onnx.NodeProto()
    rng = np.random.default_rng(23)
    res = {}
    # tag: C, M, H, W, kh, kw, stride, pad, dil, depthwise, bias, fx, fy, x range, weight sigma
    cases = [
        ("t3", 6, 8, 9, 7, 3, 3, 1, 1, 1, False, True, 11, 10, 2.0, 0.1),
        ("tdw", 8, 8, 10, 10, 3, 3, 2, 1, 1, True, True, 12, 9, 1.0, 0.3),
        ("t1nb", 16, 12, 5, 6, 1, 1, 1, 0, 1, False, False, 10, 11, 3.0, 0.2),
        ("ch1", 6, 5, 4, 6, 1, 1, 1, 0, 1, False, True, rng.integers(8, 13, 6), rng.integers(7, 12, 5), 2.0, 0.1),
        ("ch3s2", 5, 7, 11, 9, 3, 3, 2, 1, 1, False, True, rng.integers(8, 13, 5), rng.integers(7, 12, 7), 2.0, 0.1),
        ("chdw", 7, 7, 8, 9, 3, 3, 1, 2, 2, True, True, rng.integers(8, 13, 7), rng.integers(7, 12, 7), 2.0, 0.2),
        ("chdw51", 6, 6, 9, 8, 5, 1, 1, 2, 1, True, False, rng.integers(6, 12, 6), rng.integers(9, 13, 6), 4.0, 0.5),
        # the int32 accumulator wraps: raw inputs near full scale, saturated weights
        ("wrap", 64, 4, 6, 6, 3, 3, 1, 1, 1, False, True, 6, 14, 500.0, 0.8),
        ("wrapdw", 4, 4, 7, 7, 7, 7, 1, 3, 1, True, True, 6, 14, 500.0, 0.8),
        ("wrapch", 32, 6, 5, 5, 3, 3, 1, 1, 1, False, True, rng.integers(5, 8, 32), rng.integers(12, 15, 6), 400.0,
         0.9),
    ]
    for (tag, C, M, H, W_, kh, kw, st, pad, dil, dw, hb, fx, fy, xr, sig) in cases:
        oh = (H + 2 * pad - (dil * (kh - 1) + 1)) // st + 1
        ow = (W_ + 2 * pad - (dil * (kw - 1) + 1)) // st + 1
        per_ch = np.ndim(fx) > 0
        w = (rng.standard_normal((M, 1 if dw else C, kh, kw)) * sig).astype(np.float32)
        b = (rng.standard_normal(M) * 0.5).astype(np.float32)
        fxv = np.asarray(fx, np.int64).reshape(-1) if per_ch else np.full(C, int(fx))
        xraw = np.clip(np.round(rng.uniform(-xr, xr, size=(2, C, H, W_)) * np.power(2.0, fxv)[None, :, None, None]),
                       -32768, 32767).astype(np.int64)
        ekw = (lambda f: {"chexp": np.asarray(f, np.int8)}) if per_ch else (lambda f: {"exp": np.asarray(f)})
        X = T(onnx_name="x", shape=[2, C, H, W_], dtype="float32", **ekw(fx))
        Y = T(onnx_name="y", shape=[2, M, oh, ow], dtype="float32", **ekw(fy))
        Wt = T(onnx_name="w_" + tag, shape=list(w.shape), dtype="float32", data=w.copy())
        Bt = T(onnx_name="b_" + tag, shape=[M], dtype="float32", data=b.copy())
        node = N.ConvNode(onnx_node=nd, inputs=[X, Wt, Bt] if hb else [X, Wt], output=Y, batch=2, in_ch=C, in_h=H,
                          in_w=W_, out_ch=M, out_h=oh, out_w=ow, kh=kh, kw=kw, stride_h=st, stride_w=st,
                          dilation_h=dil, dilation_w=dil, pad_top=pad, pad_left=pad, has_bias=hb, is_depthwise=dw)
        NU.encode_conv_weights([node], D)
        g = _Graph([node], [Wt, Bt] if hb else [Wt], [X], [Y])
        xv = xraw / np.power(2.0, fxv)[None, :, None, None]
        yv = _shim(sim, D, g)._forward_pass({"x": xv})["y"]
        fyv = np.asarray(fy, np.float64).reshape(1, -1, 1, 1) if per_ch else float(fy)
        yraw = np.round(yv * np.power(2.0, fyv)).astype(np.int64)
        res[f"{tag}_geo"] = np.array([C, M, H, W_, kh, kw, st, pad, dil, int(dw), int(hb), oh, ow, int(per_ch)])
        res[f"{tag}_fx"], res[f"{tag}_fy"] = np.asarray(fx), np.asarray(fy)
        res[f"{tag}_x"] = xraw
        res[f"{tag}_wraw"] = np.round(Wt.data.astype(np.float64) * 256).astype(np.int64).reshape(w.shape)
        res[f"{tag}_wexp"] = np.asarray(Wt.wexp, np.int64)
        if hb:
            res[f"{tag}_braw"] = np.round(Bt.data.astype(np.float64) * 256).astype(np.int64).reshape(-1)[:M]
            res[f"{tag}_bexp"] = np.asarray(Bt.wexp, np.int64)
        res[f"{tag}_y"] = yraw
        print(f"  {tag}: y {yraw.shape}, max |raw| {int(np.abs(yraw).max())}")
    res["tags"] = np.array([c[0] for c in cases])
    np.savez_compressed(os.path.join(out, "sim_conv_exp.npz"), **res)
    print("sim_conv_exp.npz:", len(cases), "cases")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", choices=["hw", "sim", "graph", "llm", "attn", "smx", "numeric", "convexp", "llmhost"])
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if args.only in (None, "hw"):
        convert_hw(args.ref, args.out)
    if args.only in (None, "sim"):
        make_sim(args.ref, args.out)
    if args.only in (None, "graph"):
        make_graph_goldens(args.ref, args.out)
    if args.only in (None, "llm"):
        make_llm_nodes(args.ref, args.out)
    if args.only in (None, "attn"):
        make_llm_attn(args.ref, args.out)
    if args.only in (None, "smx"):
        make_llm_smx_host(args.ref, args.out)
    if args.only in (None, "numeric"):
        make_numeric(args.ref, args.out)
    if args.only in (None, "convexp"):
        make_conv_exp(args.ref, args.out)
    if args.only in (None, "llmhost"):
        make_llm_host(args.ref, args.out)


if __name__ == "__main__":
    main()
