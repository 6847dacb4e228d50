"""CPU forward pass of the LLM graphs on the kernels (raw integers at
per-tensor exponents) — TEST INFRASTRUCTURE: the checker for GpuSimulator on
the Llama configuration.  Row-ops nodes run as the jobs their emit_call
issues on the oracle's job model (spec.rowops_job); the prefill attention as
oracle.attn per sequence; MatMul as the exact sum wrapped to int32.

Reference files (phoenix367/cormorant inference-scheduler/src):
  S  = codegen/_simulate.py   RO = rowops_nodes.py   LN = llm_nodes.py
"""
from __future__ import annotations

import numpy as np

from . import attn as A
from . import spec

I16, I32 = 0, 1
OP_COPY, OP_ADDX, OP_MULACT, OP_NORM = 1, 2, 4, 5
F_B_EN, F_P_BCAST = 1 << 12, 1 << 13


def _op(op, ak, bk, ck, b_en=False, bcast=False):
    return op | (ak << 4) | (bk << 6) | (ck << 8) | (F_B_EN if b_en else 0) | (F_P_BCAST if bcast else 0)


def rowops_rows(op: int, n: int, rows: int, a, a_kind: int, b, b_kind: int, p_words, c_kind: int, eps: int = 0):
    """One row-ops job over dense rows (strides = the rows' bytes) on the job
    model; returns C [rows][n] as int64."""
    enc = lambda v, k: np.asarray(v, np.int64).astype("<i2" if k == I16 else "<i4").tobytes()  # noqa: E731
    parts = [enc(a, a_kind), enc(b, b_kind) if b is not None else b"",
             np.asarray(p_words, np.int64).astype("<i2").tobytes(), bytes((2 if c_kind == I16 else 4) * n * rows)]
    offs, cur = [], 0
    for pb in parts:
        offs.append(cur)
        cur += (len(pb) + 255) // 256 * 256 + 256
    mem = np.zeros(cur, np.uint8)
    for o, pb in zip(offs, parts):
        mem[o:o + len(pb)] = np.frombuffer(pb, np.uint8)
    m = spec.RowOpsMem(mem)
    nb = lambda k: 2 if k == I16 else 4  # noqa: E731
    spec.rowops_job(m, op, n, rows, 1, offs[0], nb(a_kind) * n, 0, offs[1], nb(b_kind) * n, 0, offs[3],
                    nb(c_kind) * n, 0, offs[2], eps, 0, 0, 0, 0xFFFFFFFF)
    out = m.buf[offs[3]:offs[3] + nb(c_kind) * n * rows].tobytes()
    return np.frombuffer(out, "<i2" if c_kind == I16 else "<i4").astype(np.int64).reshape(rows, n)


def _words(t):
    return np.round(np.asarray(t.data, np.float64) * 256.0).astype(np.int64)


def forward(graph, raw_inputs: dict, raw_states: dict, weights: dict = None) -> dict:
    """{name: raw int64 array} of every tensor; ``raw_states`` (logical raw
    arrays) are updated in place; host ints (pos, n) pass through.
    ``weights``: a dict that keeps the weights' raw words between passes of
    graphs sharing weights.  The words are kept as integer-valued float64 (the
    MatMul sums read them so; every word is exact in float64)."""
    arr = {k: np.asarray(v, np.int64) for k, v in raw_inputs.items()}
    arr.update(raw_states)
    wc = {} if weights is None else weights
    for t in graph.weight_tensors:
        if getattr(t, "data", None) is not None and t.onnx_name not in arr:
            if t.onnx_name not in wc:
                v = np.clip(np.asarray(t.data, np.float64).reshape(t.shape), -128.0, 127.99609375)
                wc[t.onnx_name] = np.round(v * 256.0)
            arr[t.onnx_name] = wc[t.onnx_name]
    hi = lambda t: int(np.asarray(arr[t.onnx_name]).reshape(-1)[0])  # noqa: E731
    for sn in graph.nodes:
        k = type(sn).__name__
        ins = [arr.get(t.onnx_name) if t is not None else None for t in sn.inputs]
        if k == "MatmulNode":                                               # S:814-835
            a = ins[0].reshape(-1, sn.inputs[0].shape[-1])
            y = spec.matmul_raw(a, ins[1], True)
        elif k == "RMSNormRoNode":                                          # RO:492-497
            y = rowops_rows(_op(OP_NORM, I32, I16, I16, bcast=sn.bcast), sn.n, sn.rows, ins[0], I32, None, I16,
                            _words(sn.inputs[1]), I16, int(sn.E))
        elif k == "ResAddRoNode":                                           # RO:437-446
            y = rowops_rows(_op(OP_ADDX, I32, I16, I32, b_en=True, bcast=sn.bcast), sn.n, sn.rows, ins[0], I32,
                            ins[1], I16, _words(sn.inputs[2]), I32)
        elif k == "SiluMulRoNode":                                          # RO:578-583
            y = rowops_rows(_op(OP_MULACT, I16, I16, I16, b_en=True, bcast=sn.bcast), sn.n, sn.rows, ins[0], I16,
                            ins[1], I16, _words(sn.inputs[2]), I16)
        elif k == "WidenRoNode":                                            # RO:533-537
            y = rowops_rows(_op(OP_COPY, I16, I16, I32, bcast=sn.bcast), sn.n, sn.rows, ins[0], I16, None, I16,
                            _words(sn.inputs[1]), I32)
        elif k == "AttnPrepRoNode":                                         # RO:1112-1143
            B, T, C, nq, nk = sn.batch, sn.T, sn.C, sn.H * sn.HD, sn.KV * sn.HD
            e = lambda t, w: np.broadcast_to(np.asarray(8 if t.exp is None else t.exp, np.int64), (w,))  # noqa: E731
            ck, cv = arr[sn.ck.onnx_name], arr[sn.cv.onnx_name]
            qx = []
            for b in range(B):
                rs = slice(b * T, (b + 1) * T)
                ckb, cvb = ck[b * C:(b + 1) * C], cv[b * C:(b + 1) * C]
                qx.append(A.attn_prep(arr[sn.q0.onnx_name].reshape(-1, nq)[rs], arr[sn.k0.onnx_name].reshape(-1, nk)[rs],
                                      arr[sn.v.onnx_name].reshape(-1, nk)[rs], hi(sn.pos),
                                      hi(sn.n_t) if sn.has_n else T, T=T, H=sn.H, KV=sn.KV, HD=sn.HD, C=C,
                                      fq0=e(sn.q0, nq), fk0=e(sn.k0, nk), fv=e(sn.v, nk), fq=sn.fq, fkc=e(sn.ck, nk),
                                      fvc=e(sn.cv, nk), cos=sn.cos, sin=sn.sin, ck=ckb, cv=cvb, Q=sn.Q))
            y = np.stack(qx, axis=1)                                        # [KV][B][HD][G T]
        elif k == "LlmAttnConvNode":                                        # LN:1407-1423
            B, C, HD, g = sn.batch, sn.C, sn.HD, sn.group
            GT = sn.H // sn.KV * sn.T
            keys = C if sn.static else A.attn_keys(hi(sn.inputs[2]), hi(sn.inputs[3]) if sn.has_n else sn.T,
                                                   sn.T, C, sn.Q)[1]
            cache = ins[0] if sn.kind == "qk" else ins[1]
            cache = cache.reshape(B, C, -1)
            outs = []
            for b in range(B):
                if sn.kind == "qk":
                    qx = ins[1].reshape(sn.KV, B, HD, GT)[:, b]
                    outs.append(A.attn_scores(cache[b], qx, g, HD=HD, C=C, keys=keys, r0=sn.r0, nr=sn.nr))
                else:
                    outs.append(A.attn_pv(ins[0].reshape(B, GT, C)[b], cache[b], g, HD=HD, keys=keys))
            y = np.concatenate(outs, axis=1) if sn.kind == "qk" else np.concatenate(outs, axis=0)
        elif k == "LlmAttnSoftmaxVopNode":                                  # SN:320-338
            B, C, GT = sn.batch, sn.C, sn.G * sn.T
            pos = hi(sn.inputs[1])
            n, keys = A.attn_keys(pos, hi(sn.inputs[2]) if sn.has_n else sn.T, sn.T, C, sn.Q)
            s = ins[0].reshape(C, B, GT)
            y = np.concatenate([A.attn_softmax(s[:, b], T=sn.T, G=sn.G, C=C, keys=keys, pos=pos, n=n,
                                               causal=sn.causal, prefix_lm=sn.prefix_lm, cm=sn.cm, cfg=sn.cfg)
                                for b in range(B)], axis=0)
        elif k == "LlmAttnSoftmaxNode":                                     # LN:1532-1557
            B, C, GT = sn.batch, sn.C, sn.G * sn.T
            s = ins[0].reshape(C, B, GT)
            y = np.concatenate([A.attn_softmax_host(s[:, b], T=sn.T, G=sn.G, C=C, pos=hi(sn.inputs[1]),
                                                    n_in=hi(sn.inputs[2]) if sn.has_n else sn.T, fs=sn.fs, fp=sn.fp,
                                                    scale=sn.scale, window=sn.window, Q=sn.Q) for b in range(B)],
                               axis=0)
        elif k == "LlmAttnMergeNode":                                       # LN:1645-1657
            B, T, HD, G = sn.batch, sn.T, sn.HD, sn.H // sn.KV
            y = np.concatenate([A.attn_merge([o.reshape(B, G * T, HD)[b] for o in ins], T=T, H=sn.H, KV=sn.KV, HD=HD)
                                for b in range(B)], axis=0)
        elif k == "LlmSelectRowNode":                                       # LN:1713-1717
            r = min(max(hi(sn.inputs[1]), 1), sn.rows) - 1
            y = ins[0].reshape(sn.batch, sn.rows, sn.n)[:, r]
        elif k == "ReshapeNode":
            y = ins[0]
        else:
            raise NotImplementedError(k)
        arr[sn.output.onnx_name] = np.asarray(y, np.int64).reshape(sn.output.shape)
    return arr


def greedy_decode(model, raw_states: dict, prefill_logits: np.ndarray, steps: int, weights: dict = None):
    """Greedy decode steps on the oracle after a prefill (the states already
    hold its cache rows): the first argmax of each sequence's logits, its
    embedding row as the int32 residual (RNE at the residual's exponent), one
    decode-step pass at pos = T + i.  Returns (ids [steps][B], logits of every
    step).  ``weights``: the raw-word cache of ``forward`` (shared with the
    prefill's pass, so the weights are converted once)."""
    g = model.decode_graph
    out = g.output_tensors[0].onnx_name
    emb_raw = np.rint(model.emb * 2.0 ** model.E["fr"]).astype(np.int64)
    lg = np.asarray(prefill_logits, np.int64)
    ids, logits = [], []
    wc = {} if weights is None else weights
    for i in range(steps):
        nxt = lg.argmax(axis=1)
        ids.append(nxt)
        arr = forward(g, {"h_step": emb_raw[nxt], "pos": np.array([model.T + i])}, raw_states, wc)
        lg = arr[out]
        logits.append(lg)
    return np.stack(ids), logits
