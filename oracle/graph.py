"""CPU forward pass over node graphs (cormorant_b200.nodes or the reference's
own node objects) with the oracle's raw-integer kernels — TEST
INFRASTRUCTURE: the checker for GpuSimulator and the CPU baseline of the
model configurations.  Restates phoenix367/cormorant
inference-scheduler/src/codegen/_simulate.py:541-769 (``_forward_pass``) on
raw int64 arrays at Q8.8.
"""
from __future__ import annotations

import numpy as np

from . import spec


def forward_raw(graph, raw_inputs):
    """{name: raw int64 array (logical shape)} for every tensor visited."""
    arr = {k: np.asarray(v, np.int64) for k, v in raw_inputs.items()}
    for t in graph.weight_tensors:
        if getattr(t, "data", None) is not None:
            v = np.clip(np.asarray(t.data, np.float64).reshape(t.shape), -128.0, 127.99609375)
            arr[t.onnx_name] = np.round(v * 256.0).astype(np.int64)         # _simulate.py:531-539
    for sn in graph.nodes:
        k = type(sn).__name__
        out = sn.output
        if k in ("MatmulNode", "MatmulConvNode"):                            # :620-633, :814-835
            wrap = any(getattr(t, a, None) is not None for t in (sn.inputs[0], sn.inputs[1], out)
                       for a in ("exp", "wexp"))
            y = spec.matmul_raw(arr[sn.inputs[0].onnx_name], arr[sn.inputs[1].onnx_name], wrap)
        elif k == "ConvNode":                                                # :635-660, :784-812
            x = arr[sn.inputs[0].onnx_name].reshape(sn.batch, sn.in_ch, sn.in_h, sn.in_w)
            w = arr[sn.inputs[1].onnx_name]
            exp = any(getattr(t, a, None) is not None for t in (sn.inputs[0], sn.inputs[1], out)
                      for a in ("exp", "wexp", "chexp"))
            b = None
            if sn.has_bias:
                b = arr[sn.inputs[2].onnx_name].reshape(-1)[:sn.out_ch]
                if exp and getattr(sn.inputs[2], "wexp", None) is None:
                    # a Q8.8 bias on an exponent conv: its value at f_y (S:805-806)
                    b = spec.rne_int(b * _conv_fy(out, sn.out_ch) / 256.0)
            y = spec.conv_raw(x, w, b, sn.stride_h, sn.stride_w, sn.pad_top, sn.pad_left, sn.dilation_h,
                              sn.dilation_w, sn.out_h, sn.out_w, bool(sn.is_depthwise), wrap=exp)
        elif k == "ReshapeNode":                                             # :662-665
            y = arr[sn.inputs[0].onnx_name]
        elif k == "PoolNode":                                                # :701-719
            x = arr[sn.inputs[0].onnx_name].reshape(sn.batch, sn.channels, sn.in_h, sn.in_w)
            y = spec.pool_raw(x, sn.pool_h, sn.pool_w, sn.stride_h, sn.stride_w, sn.pad_top, sn.pad_left, sn.dil_h,
                              sn.dil_w, sn.out_h, sn.out_w, sn.pool_type, sn.lp_order, int(bool(sn.count_include_pad)))
        elif k == "SoftmaxVopNode":                                          # smx_nodes.py:121-134
            x = arr[sn.inputs[0].onnx_name].reshape(sn.rows, sn.n)
            y = spec.softmax_rows(x, sn.n, sn.cm, sn.cfg & 63, (sn.cfg >> 8) & 31)
        elif k == "ScheduledNode":                                           # :721-765
            a = arr[sn.inputs[0].onnx_name].reshape(-1)
            op = sn.op_code
            N = int(np.prod(out.shape))
            c = np.zeros(N + 16, np.int16)
            if op <= 3:
                # the broadcast operand repeats (trailing-contiguous, nodes.py:226-305):
                # elementwise, so it is tiled to the output's length
                b = arr[sn.inputs[1].onnx_name].reshape(-1)
                a = np.tile(a, N // a.size) if a.size != N else a
                b = np.tile(b, N // b.size) if b.size != N else b
                spec.vectorop_job(a, b, c, N, op, 1, 0, 0, getattr(sn, "act", 0), getattr(sn, "alpha", 0))
            else:
                spec.vectorop_job(a, None, c, N, op, 1, 0, 0, getattr(sn, "act", 0), getattr(sn, "alpha", 0))
            y = c[:N].astype(np.int64)
        elif k == "LayerNormRoNode":                                         # rowops_nodes.py:188-192
            x = arr[sn.inputs[0].onnx_name].reshape(sn.rows, sn.n)
            y = spec.layer_norm_rows(x, np.ones(sn.n) if sn.gamma is None else sn.gamma,
                                     np.zeros(sn.n) if sn.beta is None else sn.beta, sn.eps, sn.F, sn.F)
        elif k == "TransposeRoNode":                                         # rowops_nodes.py:296-298
            y = np.transpose(arr[sn.inputs[0].onnx_name].reshape(sn.inputs[0].shape), sn.perm)
        else:
            raise NotImplementedError(k)
        arr[out.onnx_name] = np.asarray(y, np.int64).reshape(out.shape)
    return arr


def _conv_fy(t, out_ch):
    """2^f_y per output channel of an exponent conv's output (chexp or exp;
    Q8.8 without either)."""
    if getattr(t, "chexp", None) is not None:
        f = np.asarray(t.chexp, np.float64).reshape(-1)
    else:
        f = np.full(out_ch, 8.0 if getattr(t, "exp", None) is None else float(np.asarray(t.exp)))
    return np.power(2.0, f)


def forward(graph, inputs):
    """Values in (float64, on the Q8.8 grid), every tensor's raw out."""
    raw = {k: np.round(np.asarray(v, np.float64) * 256.0).astype(np.int64) for k, v in inputs.items()}
    return forward_raw(graph, raw)
