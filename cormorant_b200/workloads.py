"""Graph builders for the benchmark configurations:
the MNIST-shaped CNN (config 1) and MobileNetV2-1.0 (config 3), as node
graphs the simulator runs, with seeded synthetic Q8.8 weights and inputs.

The builders go through a ``NodeFactory`` so the same architecture can be
instantiated with this package's descriptors (``NodeFactory``) or with the
reference's own node classes (the golden-vector generator subclasses it), and
the GPU result compared with the reference simulator's on identical weights.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np

from . import nodes as N
from . import rowops_host as RH


def q88_uniform(rng, shape, lo, hi) -> np.ndarray:
    """Q8.8 values of uniform reals in [lo, hi), rounded half to even."""
    return np.clip(np.round(rng.uniform(lo, hi, size=shape) * 256.0), -32768, 32767) / 256.0


def he_normal_q88(rng, shape, fan_in) -> np.ndarray:
    """He-normal weights (sigma = sqrt(2 / fan_in)) quantised to Q8.8 with
    saturation."""
    return np.clip(np.round(rng.normal(0.0, np.sqrt(2.0 / fan_in), size=shape) * 256.0), -32768, 32767) / 256.0


def unit_rng(seed: int, i: int) -> np.random.Generator:
    """The input stream of unit ``i`` (an image, a sequence) of a seeded
    configuration.  Weights come from the configuration's own stream, inputs
    from one stream per unit, so a rank that runs units [first, first +
    batch) of a sharded batch holds exactly those units' inputs, with the
    same weights, whatever the split."""
    return np.random.default_rng([seed, 0x5EED, i])


def _per_unit(seed: int, first: int, batch: int, draw) -> np.ndarray:
    return np.stack([draw(unit_rng(seed, first + i)) for i in range(batch)])


class NodeFactory:
    """Builds graph pieces with cormorant_b200.nodes descriptors."""

    def __init__(self):
        self.tensors: Dict[str, N.TensorInfo] = {}
        self.nodes: list = []
        self.weights: List[N.TensorInfo] = []

    def tensor(self, name, shape, data=None):
        t = N.TensorInfo(onnx_name=name, shape=list(shape), data=data)
        self.tensors[name] = t
        if data is not None:
            self.weights.append(t)
        return t

    def conv(self, x, w, b, y, **geo):
        self.nodes.append(N.ConvNode(inputs=[x, w] + ([b] if b is not None else []), output=y,
                                     has_bias=b is not None, **geo))

    def vop(self, op, ins, y, act=0):
        self.nodes.append(N.ScheduledNode(op_code=op, inputs=ins, output=y, act=act))

    def pool(self, x, y, **geo):
        self.nodes.append(N.PoolNode(inputs=[x], output=y, **geo))

    def reshape(self, x, y):
        self.nodes.append(N.ReshapeNode(inputs=[x], output=y))

    def matmul(self, a, b, y, n, k, m):
        self.nodes.append(N.MatmulNode(inputs=[a, b], output=y, n=n, k=k, m=m, batch=1))

    def softmax(self, x, y, rows, n, cm, cfg):
        self.nodes.append(N.SoftmaxVopNode(inputs=[x], output=y, rows=rows, n=n, cm=cm, cfg=cfg))

    def layernorm(self, x, y, rows, n, gamma, beta, eps):
        """LayerNorm on the row-ops unit: the parameter block (words as Q8.8
        values, rowops_nodes.py:96-102) and the registers of the job."""
        words, g, bb, E = RH.layernorm_job(gamma, beta, n, eps)
        p = self.tensor(f"{y.onnx_name}__rowops_p", (words.size,), words / 256.0)
        self.nodes.append(N.LayerNormRoNode(inputs=[x, p], output=y, rows=rows, n=n, eps=eps, g=g, bb=bb, E=E,
                                            gamma=np.asarray(gamma, np.float64), beta=np.asarray(beta, np.float64)))

    def transpose(self, x, y, in_shape, perm):
        """A Transpose as one row-ops COPY / TRANSPOSE job (rowops_nodes.py:318-346)."""
        job = RH.transpose_job(in_shape, perm)
        if job is None:
            raise ValueError(f"transpose {in_shape} perm {perm}: not a row-ops job")
        kind, n, rows, blocks, strides = job
        pz = self.tensors.get("__rowops_zero_p")
        if pz is None:
            pz = self.tensor("__rowops_zero_p", (8,), RH.param_block(0, 0, 0, 0, 0) / 256.0)
        self.nodes.append(N.TransposeRoNode(inputs=[x, pz], output=y, kind=kind, n=n, rows=rows, blocks=blocks,
                                            strides=strides, perm=list(perm)))

    def graph(self, inputs, outputs):
        return N.Graph(nodes=self.nodes, weight_tensors=self.weights, input_tensors=inputs, output_tensors=outputs)


# ---------------------------------------------------------------- config 1: MNIST CNN
def mnist(seed: int = 1, batch: int = 1, factory: NodeFactory = None, first: int = 0):
    """Conv3x3 1->16 +bias, Relu, MaxPool 2x2, Conv3x3 16->32 +bias, Relu,
    MaxPool 2x2, flatten 1568, MatMul 1568x10, Add bias, Softmax (row, Q8.8).
    Images [first, first + batch) of the seeded input set.
    Returns (graph, {input: values}, macs_per_image)."""
    f = factory or NodeFactory()
    rng = np.random.default_rng(seed)
    x = _per_unit(seed, first, batch, lambda r: q88_uniform(r, (1, 28, 28), -1, 1))
    w1, b1 = q88_uniform(rng, (16, 1, 3, 3), -0.25, 0.25), q88_uniform(rng, (16,), -0.25, 0.25)
    w2, b2 = q88_uniform(rng, (32, 16, 3, 3), -0.25, 0.25), q88_uniform(rng, (32,), -0.25, 0.25)
    wf, bf = q88_uniform(rng, (1568, 10), -0.25, 0.25), q88_uniform(rng, (1, 10), -0.25, 0.25)
    X = f.tensor("x", x.shape)
    W1, B1, W2, B2 = f.tensor("w1", w1.shape, w1), f.tensor("b1", b1.shape, b1), f.tensor("w2", w2.shape, w2), \
        f.tensor("b2", b2.shape, b2)
    WF, BF = f.tensor("wf", wf.shape, wf), f.tensor("bf", bf.shape, bf)
    c1, r1, p1 = f.tensor("c1", (batch, 16, 28, 28)), f.tensor("r1", (batch, 16, 28, 28)), f.tensor("p1", (batch, 16, 14, 14))
    c2, r2, p2 = f.tensor("c2", (batch, 32, 14, 14)), f.tensor("r2", (batch, 32, 14, 14)), f.tensor("p2", (batch, 32, 7, 7))
    fl, mm, lg, pr = f.tensor("flat", (batch, 1568)), f.tensor("mm", (batch, 10)), f.tensor("logits", (batch, 10)), \
        f.tensor("prob", (batch, 10))
    g3 = dict(kh=3, kw=3, pad_top=1, pad_left=1)
    f.conv(X, W1, B1, c1, batch=batch, in_ch=1, in_h=28, in_w=28, out_ch=16, out_h=28, out_w=28, **g3)
    f.vop(N.OP_RELU, [c1], r1)
    f.pool(r1, p1, batch=batch, channels=16, in_h=28, in_w=28, out_h=14, out_w=14, pool_h=2, pool_w=2, stride_h=2,
           stride_w=2, pool_type=N.POOL_MAX)
    f.conv(p1, W2, B2, c2, batch=batch, in_ch=16, in_h=14, in_w=14, out_ch=32, out_h=14, out_w=14, **g3)
    f.vop(N.OP_RELU, [c2], r2)
    f.pool(r2, p2, batch=batch, channels=32, in_h=14, in_w=14, out_h=7, out_w=7, pool_h=2, pool_w=2, stride_h=2,
           stride_w=2, pool_type=N.POOL_MAX)
    f.reshape(p2, fl)
    f.matmul(fl, WF, mm, batch, 1568, 10)
    f.vop(N.OP_ADD, [mm, BF], lg)
    f.softmax(lg, pr, batch, 10, 12102203, 19 | (8 << 8))
    macs = 16 * 9 * 784 + 32 * 16 * 9 * 196 + 1568 * 10
    return f.graph([X], [pr]), {"x": x}, macs


# ---------------------------------------------------------------- config 3: MobileNetV2-1.0
MBV2_BLOCKS = [(1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2), (6, 96, 3, 1), (6, 160, 3, 2),
               (6, 320, 1, 1)]  # (expansion t, channels c, repeats n, first stride s)


def mobilenet_v2(seed: int = 3, batch: int = 1, res: int = 224, classes: int = 1000, factory: NodeFactory = None,
                 first: int = 0):
    """MobileNetV2-1.0: stem Conv3x3 s2 3->32 + Clip(0,6); inverted residuals
    (1x1 expand x t + Clip, depthwise 3x3 + Clip, 1x1 project, residual Add
    when shapes match); Conv1x1 320->1280 + Clip; GlobalAveragePool; MatMul
    1280 x classes + Add bias.  Batch-norm folded into the conv biases (small
    seeded values).  Images [first, first + batch) of the seeded input set.
    Returns (graph, {input: values}, macs_per_image)."""
    f = factory or NodeFactory()
    rng = np.random.default_rng(seed)
    x = _per_unit(seed, first, batch, lambda r: q88_uniform(r, (3, res, res), -1, 1))
    X = f.tensor("x", x.shape)
    macs = 0
    counter = [0]

    def name(p):
        counter[0] += 1
        return f"{p}{counter[0]}"

    def conv(t, cin, h, w, cout, k, s, dw=False, act=True):
        nonlocal macs
        pad = k // 2
        oh, ow = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
        fan = k * k * (1 if dw else cin)
        wv = he_normal_q88(rng, (cout, 1 if dw else cin, k, k), fan)
        bv = q88_uniform(rng, (cout,), -0.0625, 0.0625)
        W, B = f.tensor(name("w"), wv.shape, wv), f.tensor(name("b"), bv.shape, bv)
        y = f.tensor(name("conv"), (batch, cout, oh, ow))
        f.conv(t, W, B, y, batch=batch, in_ch=cin, in_h=h, in_w=w, out_ch=cout, out_h=oh, out_w=ow, kh=k, kw=k,
               stride_h=s, stride_w=s, pad_top=pad, pad_left=pad, is_depthwise=dw)
        macs += cout * oh * ow * fan
        if act:
            z = f.tensor(name("clip"), (batch, cout, oh, ow))
            f.vop(N.OP_RELU6, [y], z)
            y = z
        return y, oh, ow

    t, h, w = conv(X, 3, res, res, 32, 3, 2)
    cin = 32
    for tt, c, n, s in MBV2_BLOCKS:
        for r in range(n):
            stride = s if r == 0 else 1
            inp = t
            hid = cin * tt
            u, hh, ww = (conv(t, cin, h, w, hid, 1, 1) if tt != 1 else (t, h, w))
            u, hh, ww = conv(u, hid, hh, ww, hid, 3, stride, dw=True)
            u, hh, ww = conv(u, hid, hh, ww, c, 1, 1, act=False)
            if stride == 1 and cin == c:
                z = f.tensor(name("add"), (batch, c, hh, ww))
                f.vop(N.OP_ADD, [inp, u], z)
                u = z
            t, h, w, cin = u, hh, ww, c
    t, h, w = conv(t, cin, h, w, 1280, 1, 1)
    gp = f.tensor(name("gap"), (batch, 1280, 1, 1))
    f.pool(t, gp, batch=batch, channels=1280, in_h=h, in_w=w, out_h=1, out_w=1, pool_h=h, pool_w=w,
           pool_type=N.POOL_AVG)
    fl = f.tensor(name("flat"), (batch, 1280))
    f.reshape(gp, fl)
    wf = he_normal_q88(rng, (1280, classes), 1280)
    bf = q88_uniform(rng, (1, classes), -0.0625, 0.0625)
    WF, BF = f.tensor("wfc", wf.shape, wf), f.tensor("bfc", bf.shape, bf)
    mm = f.tensor(name("fc"), (batch, classes))
    f.matmul(fl, WF, mm, batch, 1280, classes)
    lg = f.tensor("logits", (batch, classes))
    f.vop(N.OP_ADD, [mm, BF], lg)
    macs += 1280 * classes
    return f.graph([X], [lg]), {"x": x}, macs


# ---------------------------------------------------------------- config 4: BERT-base encoder
SMX_Q88 = (12102203, 19 | (8 << 8))      # softmax unit registers at Q8.8 (vectorop_smx.scale_regs(8, 1.0))


def normal_q88(rng, shape, sigma) -> np.ndarray:
    """N(0, sigma) reals quantised RNE + saturate to Q8.8 (per-tensor exponent 8)."""
    return np.clip(np.round(rng.normal(0.0, sigma, size=shape) * 256.0), -32768, 32767) / 256.0


def bert_base(seed: int = 4, batch: int = 1, seq: int = 384, layers: int = 12, hidden: int = 768, heads: int = 12,
              ffn: int = 3072, vocab: int = 30522, qa_head: bool = True, factory: NodeFactory = None, first: int = 0):
    """BERT-base encoder on the kernels, the scheduler's partition of
    bertsquad (ap_fixed<16,8> throughout): per layer Q / K / V = x W + b
    (MatMul, VectorOP ADD), head split and K^T as row-ops COPY / TRANSPOSE
    jobs, scores Q K^T (batched MatMul), MUL 1/8, softmax on the VectorOP unit
    (row mode), context P V, head merge (COPY), output projection + bias,
    residual ADD, LayerNorm on the row-ops unit, FFN x W1 + b1 with GELU (erf)
    fused into the ADD, x W2 + b2, residual ADD, LayerNorm; then the SQuAD
    head (start / end logits).

    Layout: the batch's sequences are stacked, hidden states [batch * seq][768];
    the heads are head-major over the whole batch ([heads][batch * seq][64], one
    COPY job), so every per-(head, sequence) tensor is a contiguous slice and
    K^T is one TRANSPOSE job over heads * batch blocks.  Full-length
    sequences (no padding mask).  The word-embedding gather is the
    reference's host op: the graph input is the gathered rows (ids uniform
    over ``vocab``); position and token-type embeddings are added on
    VectorOP.  Weights N(0, 0.02) quantised to Q8.8; LayerNorm gamma =
    1 + N(0, 0.02), beta = N(0, 0.02) (encoded by the parameter block).
    Sequences [first, first + batch) of the seeded input set.
    Returns (graph, {input: values}, macs_per_token)."""
    f = factory or NodeFactory()
    rng = np.random.default_rng(seed)
    T, D, H, dh = seq, hidden, heads, hidden // heads
    R = batch * T
    word = normal_q88(rng, (vocab, D), 0.02)
    ids = _per_unit(seed, first, batch, lambda r: r.integers(0, vocab, size=T))
    x = word[ids]
    cnt = [0]

    def nm(p):
        cnt[0] += 1
        return f"{p}{cnt[0]}"

    def act(shape, p="t"):
        return f.tensor(nm(p), shape)

    def weight(shape, sigma=0.02, p="w"):
        v = normal_q88(rng, shape, sigma)
        return f.tensor(nm(p), v.shape, v)

    def linear(t, k, m):
        W, B = weight((k, m)), weight((m,), p="b")
        mm, y = act((R, m), "mm"), act((R, m), "lin")
        f.matmul(t, W, mm, R, k, m)
        return mm, B, y

    def ln(t):
        y = act((R, D), "ln")
        f.layernorm(t, y, R, D, 1.0 + rng.normal(0.0, 0.02, D), rng.normal(0.0, 0.02, D), 1e-12)
        return y

    X = f.tensor("x", (batch, T, D))
    pos, typ = weight((T, D)), weight((D,))
    e1, e2 = act((batch, T, D), "emb"), act((R, D), "emb")
    f.vop(N.OP_ADD, [X, pos], e1)
    f.vop(N.OP_ADD, [e1, typ], e2)
    h = ln(e2)
    scale = f.tensor("attn_scale", (1,), np.array([0.125]))
    for _ in range(layers):
        heads_out = []
        for p in ("q", "k", "v"):
            mm, B, y = linear(h, D, D)
            f.vop(N.OP_ADD, [mm, B], y)
            y3 = act((R, H, dh), p + "3")
            f.reshape(y, y3)
            hs = act((H * batch, T, dh), p + "h")
            f.transpose(y3, hs, (R, H, dh), (1, 0, 2))
            heads_out.append(hs)
        qh, kh, vh = heads_out
        kt = act((H * batch, dh, T), "kt")
        f.transpose(kh, kt, (H * batch, T, dh), (0, 2, 1))
        sc, ss, pr = act((H * batch, T, T), "sc"), act((H * batch, T, T), "ss"), act((H * batch, T, T), "pr")
        f.matmul(qh, kt, sc, T, dh, T)
        f.vop(N.OP_MUL, [sc, scale], ss)
        f.softmax(ss, pr, H * batch * T, T, *SMX_Q88)
        ctx = act((H * batch, T, dh), "ctx")
        f.matmul(pr, vh, ctx, T, T, dh)
        ctx3 = act((H, R, dh), "ctx3")
        f.reshape(ctx, ctx3)
        mg = act((R, H, dh), "merge")
        f.transpose(ctx3, mg, (H, R, dh), (1, 0, 2))
        mg2 = act((R, D), "mflat")
        f.reshape(mg, mg2)
        mm, B, y = linear(mg2, D, D)
        f.vop(N.OP_ADD, [mm, B], y)
        r1 = act((R, D), "res")
        f.vop(N.OP_ADD, [h, y], r1)
        h1 = ln(r1)
        mm, B, y = linear(h1, D, ffn)
        f.vop(N.OP_ADD, [mm, B], y, act=N.ACT_GELU)
        mm, B, y2 = linear(y, ffn, D)
        f.vop(N.OP_ADD, [mm, B], y2)
        r2 = act((R, D), "res")
        f.vop(N.OP_ADD, [h1, y2], r2)
        h = ln(r2)
    outs = [h]
    if qa_head:
        mm, B, y = linear(h, D, 2)
        lg = f.tensor("qa_logits", (R, 2))
        f.vop(N.OP_ADD, [mm, B], lg)
        outs = [lg]
    macs = layers * (4 * D * D + 2 * D * ffn + 2 * T * D) + (2 * D if qa_head else 0)
    return f.graph([X], outs), {"x": x}, macs


def graph_macs(graph) -> int:
    """Int16 MACs of one pass: sum over Conv (N M oH oW (C/groups) kh kw) and
    MatMul (batch n k m) nodes."""
    total = 0
    for sn in graph.nodes:
        k = type(sn).__name__
        if k == "ConvNode":
            total += sn.batch * sn.out_ch * sn.out_h * sn.out_w * (1 if sn.is_depthwise else sn.in_ch) * sn.kh * sn.kw
        elif k in ("MatmulNode", "MatmulConvNode"):
            a = sn.inputs[0].shape
            total += int(np.prod(a[:-1])) * a[-1] * sn.inputs[1].shape[-1]
    return total


def shapes_summary(graph) -> List[Tuple[str, list]]:
    return [(type(sn).__name__, list(sn.output.shape)) for sn in graph.nodes]


# exponents of the Llama prefill (per tensor): the int32 residual, RMSNorm
# outputs, projections, the rotated q / the caches, P, the attention output,
# the MLP's, the logits
LLAMA_EXP = dict(fr=15, fx=12, fq0=13, fk0=13, fv=13, fq=10, fkc=10, fvc=9, fp=12, fo=13, fg=13, fu=13, fa=13,
                 fd=13, fl=11)
# the formats-table class of each (src/llama.py:413-455): x serves x, x2 and xf
_LLAMA_CLASS = dict(fr="res", fx="x", fq0="q0", fk0="k0", fv="v", fq="q", fkc="k", fvc="vc", fp="p", fo="o", fg="g",
                    fu="u", fa="a", fd="d", fl="logits")


class LlamaModel:
    """A Llama-family decoder on the kernels (SmolLM2-360M shape by default):
    its weights, KV-cache states and embedding table, and the node graphs of a
    prefill (``prefill_graph``) and of one decode step (``decode_graph``) that
    share them, as the scheduler's LLM entries lower the model with the
    row-ops unit (src/llama.py:329-402 with rowops = 1): per layer RMSNorm
    (the int32 residual -> int16), the q / k / v projections (MatMul), the
    attention chain (AttnPrepRoNode: RoPE and the KV-cache rows; per KV group
    q.K^T, the softmax and P.V; the head merge), the output projection,
    ResAdd, RMSNorm, gate / up, SiLU(g) u, down, ResAdd; then the final
    RMSNorm and the LM head.  The prefill runs the softmax on VectorOP's unit
    (vsmx = 1) and ends with the last valid row of every sequence
    (LlmSelectRowNode); a decode step (one row, no n) runs the host's p12
    softmax, as the reference's decode entries do.

    ``batch`` sequences side by side (the nodes' batch layouts: sequences
    [first, first + batch) of the seeded input set), ``seq`` prefill tokens
    at pos 0, KV caches of ``cache`` rows (default seq + 128)
    as group-major states.  The embedding lookup is the reference's host op:
    a graph input is the gathered rows of a N(0, 0.02) table as the int32
    residual.  Weights N(0, 0.02) (norm weights 1) at the rank-1 exponents the
    per-tensor activation exponents ``exps`` give."""

    def __init__(self, seed: int = 5, batch: int = 1, seq: int = 512, layers: int = 32, hidden: int = 960,
                 heads: int = 15, kv_heads: int = 5, head_dim: int = 64, ffn: int = 2560, vocab: int = 49152,
                 theta: float = 1e5, cache: int = None, eps: float = 1e-5, exps: dict = None, first: int = 0):
        from . import attention as AT
        from . import numeric as NU
        E = dict(LLAMA_EXP, **(exps or {}))
        per_class = {_LLAMA_CLASS[k]: v for k, v in E.items()}
        per_class.update(x2=E["fx"], xf=E["fx"])
        # the exponent table the lowering reads (one exponent per tensor class)
        self.formats = fm = NU.LlamaFormats.per_tensor(per_class, L=layers, H=heads, KV=kv_heads, HD=head_dim)
        self.E = E
        rng = np.random.default_rng(seed)
        self.B, self.T, self.D, self.H, self.KV, self.HD = batch, seq, hidden, heads, kv_heads, head_dim
        self.L, self.ffn, self.vocab, self.eps = layers, ffn, vocab, eps
        C = seq + 128 if cache is None else cache
        self.C = C = -(-C // AT.KEY_QUANTUM) * AT.KEY_QUANTUM
        D, nq, nk = hidden, heads * head_dim, kv_heads * head_dim
        self.w = []
        for li in range(layers):
            lw = {}
            # each weight at wexp[i][j] = f_out[j] + 8 - f_in[i] from the table
            # (the o projection reads the P.V output, f_p + f_vc - 8 per channel)
            for nm, (k, m, f_in, f_out) in dict(
                    q0=(D, nq, fm.get("x", li, D), fm.get("q0", li, nq)),
                    k0=(D, nk, fm.get("x", li, D), fm.get("k0", li, nk)),
                    v=(D, nk, fm.get("x", li, D), fm.get("v", li, nk)),
                    o=(nq, D, fm.pv(li), fm.get("o", li, D)),
                    g=(D, ffn, fm.get("x2", li, D), fm.get("g", li, ffn)),
                    u=(D, ffn, fm.get("x2", li, D), fm.get("u", li, ffn)),
                    d=(ffn, D, fm.get("a", li, ffn), fm.get("d", li, D))).items():
                data, _, _ = NU.encode_matmul_weight(rng.normal(0.0, 0.02, (k, m)), f_in, f_out)
                lw[nm] = N.TensorInfo(f"l{li}.{nm}.w", [k, m], data=data)
            self.w.append(lw)
        data, _, _ = NU.encode_matmul_weight(rng.normal(0.0, 0.02, (D, vocab)), fm.get("xf", layers, D),
                                             fm.get("logits", layers, vocab))
        self.w_lm = N.TensorInfo("logits.w", [D, vocab], data=data)
        self.states = []
        for li in range(layers):
            for nm, f in (("ck", E["fkc"]), ("cv", E["fvc"])):
                self.states.append(N.TensorInfo(f"l{li}.{nm}", [batch * C, nk], exp=np.asarray(f, np.int64),
                                                is_state=True, group_layout=(kv_heads, head_dim)))
        inv = 1.0 / theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
        ang = np.outer(np.arange(C, dtype=np.float64), inv)
        self.cos, self.sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        self.emb = rng.normal(0.0, 0.02, (vocab, D))
        self.first = first
        self.ids = _per_unit(seed, first, batch, lambda r: r.integers(0, vocab, size=seq))
        self.prefill_graph = self._graph(seq, prefill=True)
        self.decode_graph = self._graph(1, prefill=False)
        self.prefill_feeds = {"h0": self.emb[self.ids].reshape(batch * seq, D), "pos": np.array([0]),
                              "n": np.array([seq])}

    def _graph(self, T: int, prefill: bool):
        from . import attention as AT
        E, B, D, H, KV, HD, C = self.E, self.B, self.D, self.H, self.KV, self.HD, self.C
        nq, nk, ffn, R = H * HD, KV * HD, self.ffn, B * T
        weights: List[N.TensorInfo] = []
        nodes: list = []
        tag = "p" if prefill else "d"

        def ten(name, shape, exp=None, **kw):
            return N.TensorInfo(f"{tag}.{name}", list(shape), exp=None if exp is None else np.asarray(exp, np.int64),
                                **kw)

        def param(name, words):
            t = N.TensorInfo(name, [len(words)], data=np.asarray(words, np.float64) / 256.0)
            weights.append(t)
            return t

        def linear(name, x, w, f_out, rows=R):
            weights.append(w)
            k, m = w.shape
            y = ten(name, (rows, m), f_out)
            nodes.append(N.MatmulNode(inputs=[x, w], output=y, n=rows, k=k, m=m, batch=1))
            return y

        def rmsnorm(name, h, f_out, rows=R):
            words, bc, g, Ev = RH.rmsnorm_job(np.ones(D), self.eps, E["fr"], np.full(D, f_out))
            y = ten(name, (rows, D), f_out)
            nodes.append(N.RMSNormRoNode(inputs=[h, param("rms.p", words)], output=y, rows=rows, n=D, fr=E["fr"],
                                         eps=self.eps, g=g, E=Ev, bcast=bc, gamma=np.ones(D)))
            return y

        def resadd(name, h, d, f_d):
            words, bc = RH.resadd_job(E["fr"], np.full(D, f_d), D)
            y = ten(name, (R, D), E["fr"], dma="i32")
            nodes.append(N.ResAddRoNode(inputs=[h, d, param(f"resadd{f_d}.p", words)], output=y, rows=R, n=D,
                                        fr=E["fr"], bcast=bc))
            return y

        h = h0 = N.TensorInfo("h0" if prefill else "h_step", [R, D], exp=np.asarray(E["fr"], np.int64), dma="i32")
        pos = N.TensorInfo("pos", [1], host="i32")
        n_t = N.TensorInfo("n", [1], host="i32") if prefill else None
        for li in range(self.L):
            lw = self.w[li]
            x = rmsnorm(f"l{li}.x", h, E["fx"])
            q0 = linear(f"l{li}.q0", x, lw["q0"], E["fq0"])
            k0 = linear(f"l{li}.k0", x, lw["k0"], E["fk0"])
            v = linear(f"l{li}.v", x, lw["v"], E["fv"])
            ck, cv = self.states[2 * li], self.states[2 * li + 1]
            chain, pv = AT.prefill_layer(f"{tag}.l{li}.attn", T=T, H=H, KV=KV, HD=HD, C=C, fq0=np.full(nq, E["fq0"]),
                                         fk0=np.full(nk, E["fk0"]), fv=np.full(nk, E["fv"]), fq=np.full(H, E["fq"]),
                                         fkc=np.full(KV, E["fkc"]), fvc=np.full(KV, E["fvc"]),
                                         fp=np.full(H, E["fp"]), cos=self.cos, sin=self.sin, q0=q0, k0=k0, v=v,
                                         pos=pos, n=n_t, ck=ck, cv=cv, batch=B,
                                         softmax="unit" if prefill else "host")
            for nd in chain:
                for t in nd.inputs:
                    if t is not None and t.data is not None and all(t is not w for w in weights):
                        weights.append(t)
            nodes += chain
            o = linear(f"l{li}.o", pv, lw["o"], E["fo"])
            h1 = resadd(f"l{li}.h1", h, o, E["fo"])
            x2 = rmsnorm(f"l{li}.x2", h1, E["fx"])
            g = linear(f"l{li}.g", x2, lw["g"], E["fg"])
            u = linear(f"l{li}.u", x2, lw["u"], E["fu"])
            words, bc = RH.silu_mul_job(np.full(ffn, E["fg"]), np.full(ffn, E["fu"]), np.full(ffn, E["fa"]), ffn)
            a = ten(f"l{li}.a", (R, ffn), E["fa"])
            nodes.append(N.SiluMulRoNode(inputs=[g, u, param("silumul.p", words)], output=a, rows=R, n=ffn,
                                         bcast=bc))
            d = linear(f"l{li}.d", a, lw["d"], E["fd"])
            h = resadd(f"l{li}.h2", h1, d, E["fd"])
        if prefill:
            last = ten("h_last", (B, D), E["fr"], dma="i32")
            nodes.append(N.LlmSelectRowNode(inputs=[h, n_t], output=last, rows=T, n=D, res32=True, batch=B))
            h = last
        xf = rmsnorm("xf", h, E["fx"], rows=B)
        logits = linear("logits", xf, self.w_lm, E["fl"], rows=B)
        ins = [h0, pos] + ([n_t] if prefill else [])
        weights = list({w.onnx_name: w for w in weights}.values())
        return N.Graph(nodes=nodes, weight_tensors=weights, input_tensors=ins, output_tensors=[logits],
                       state_tensors=list(self.states))

    def macs_per_token(self, keys: int, prefill: bool = True) -> float:
        """Int16 MACs per token of a pass: the projections, the attention at
        ``keys`` keys (masked keys included, as the kernels run them) and the
        LM head (once per sequence in a prefill of T tokens)."""
        D, H, KV, HD, ffn = self.D, self.H, self.KV, self.HD, self.ffn
        nq, nk = H * HD, KV * HD
        per_layer = D * (nq + 2 * nk) + nq * D + 3 * D * ffn + 2 * H * keys * HD
        return self.L * per_layer + D * self.vocab / (self.T if prefill else 1)


def llama_prefill(seed: int = 5, batch: int = 1, seq: int = 512, layers: int = 32, hidden: int = 960, heads: int = 15,
                  kv_heads: int = 5, head_dim: int = 64, ffn: int = 2560, vocab: int = 49152, theta: float = 1e5,
                  cache: int = None, eps: float = 1e-5, exps: dict = None, first: int = 0):
    """The prefill of ``LlamaModel``: (graph, {input: values}, macs_per_token)."""
    from . import attention as AT
    m = LlamaModel(seed=seed, batch=batch, seq=seq, layers=layers, hidden=hidden, heads=heads, kv_heads=kv_heads,
                   head_dim=head_dim, ffn=ffn, vocab=vocab, theta=theta, cache=cache, eps=eps, exps=exps, first=first)
    keys = -(-seq // AT.KEY_QUANTUM) * AT.KEY_QUANTUM
    return m.prefill_graph, m.prefill_feeds, m.macs_per_token(keys)
