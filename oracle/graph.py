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
        if k in ("MatmulNode", "MatmulConvNode"):                            # :620-633
            y = spec.matmul_raw(arr[sn.inputs[0].onnx_name], arr[sn.inputs[1].onnx_name])
        elif k == "ConvNode":                                                # :643-660
            x = arr[sn.inputs[0].onnx_name].reshape(sn.batch, sn.in_ch, sn.in_h, sn.in_w)
            w = arr[sn.inputs[1].onnx_name]
            b = arr[sn.inputs[2].onnx_name].reshape(-1) if sn.has_bias else None
            y = spec.conv_raw(x, w, b, sn.stride_h, sn.stride_w, sn.pad_top, sn.pad_left, sn.dilation_h,
                              sn.dilation_w, sn.out_h, sn.out_w, bool(sn.is_depthwise))
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
            a = arr[sn.inputs[0].onnx_name]
            op = sn.op_code
            N = out.numel if hasattr(out, "numel") else int(np.prod(out.shape))
            c = np.zeros(N + 16, np.int16)
            if op <= 3:
                b = arr[sn.inputs[1].onnx_name]
                na, nb = a.size, b.size
                size = nb if nb != N else na
                a_inc, b_inc = (size, 0) if nb != N else (0, size)
                for o in range(N // size):   # row by row: rows need not be 8-lane aligned here
                    cc = np.zeros(size + 16, np.int16)
                    spec.vectorop_job(a.reshape(-1)[o * a_inc: o * a_inc + size + (0 if a_inc else 0)],
                                      b.reshape(-1)[o * b_inc: o * b_inc + size], cc, size, op, 1, 0, 0,
                                      getattr(sn, "act", 0), getattr(sn, "alpha", 0))
                    c[o * size:(o + 1) * size] = cc[:size]
            else:
                spec.vectorop_job(a.reshape(-1), None, c, N, op, 1, 0, 0, getattr(sn, "act", 0),
                                  getattr(sn, "alpha", 0))
            y = c[:N].astype(np.int64)
        else:
            raise NotImplementedError(k)
        arr[out.onnx_name] = np.asarray(y, np.int64).reshape(out.shape)
    return arr


def forward(graph, inputs):
    """Values in (float64, on the Q8.8 grid), every tensor's raw out."""
    raw = {k: np.round(np.asarray(v, np.float64) * 256.0).astype(np.int64) for k, v in inputs.items()}
    return forward_raw(graph, raw)
