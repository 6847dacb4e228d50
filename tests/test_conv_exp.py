"""Conv with power-of-two exponents (scope row a6): the reference's
``_SimulateMixin._conv_exp`` + ``_conv2d_int`` (inference-scheduler/src/
codegen/_simulate.py:784-812, 198-220), with weights and biases encoded by its
``numeric.encode_conv_weights`` (numeric.py:258-307).  The golden
(``tests/golden/sim_conv_exp.npz``, ``make_golden.py --only convexp``) holds
the reference's own outputs on per-tensor and per-channel (chexp) exponents,
standard and depthwise convs, strides / padding / dilation, with and without
bias, and cases whose int32 accumulator wraps.

CPU: the oracle (``oracle/graph.py``) equals the golden on every case, and the
wrap cases do wrap.  GPU: ``GpuSimulator`` (the kernel with ``CORM_F_WRAP32``
and the bias at the output's exponent) equals the golden bit for bit."""
import numpy as np
import pytest


def _case(z, tag):
    """This package's node objects for one golden case, and its raw input."""
    from cormorant_b200 import nodes as N
    C, M, H, W, kh, kw, st, pad, dil, dw, hb, oh, ow, per_ch = (int(v) for v in z[f"{tag}_geo"])
    fx, fy = z[f"{tag}_fx"], z[f"{tag}_fy"]
    ekw = (lambda f: {"chexp": np.asarray(f)}) if per_ch else (lambda f: {"exp": np.asarray(f)})
    X = N.TensorInfo("x", [2, C, H, W], **ekw(fx))
    Y = N.TensorInfo("y", [2, M, oh, ow], **ekw(fy))
    Wt = N.TensorInfo("w_" + tag, list(z[f"{tag}_wraw"].shape), data=z[f"{tag}_wraw"] / 256.0,
                      wexp=z[f"{tag}_wexp"])
    ins, weights = [X, Wt], [Wt]
    if hb:
        Bt = N.TensorInfo("b_" + tag, [M], data=z[f"{tag}_braw"] / 256.0, wexp=z[f"{tag}_bexp"])
        ins.append(Bt)
        weights.append(Bt)
    node = N.ConvNode(inputs=ins, output=Y, batch=2, in_ch=C, in_h=H, in_w=W, out_ch=M, out_h=oh, out_w=ow, kh=kh,
                      kw=kw, stride_h=st, stride_w=st, dilation_h=dil, dilation_w=dil, pad_top=pad, pad_left=pad,
                      has_bias=bool(hb), is_depthwise=bool(dw))
    g = N.Graph(nodes=[node], weight_tensors=weights, input_tensors=[X], output_tensors=[Y])
    return g, z[f"{tag}_x"], per_ch


def _tags(z):
    return [str(t) for t in z["tags"]]


def test_oracle_conv_exp_vs_reference(golden):
    from oracle import graph as og
    from oracle import spec
    z = golden("sim_conv_exp.npz")
    wrapped = 0
    for tag in _tags(z):
        g, x, _ = _case(z, tag)
        got = og.forward_raw(g, {"x": x})["y"]
        assert np.array_equal(got, z[f"{tag}_y"]), tag
        if tag.startswith("wrap"):
            sn = g.nodes[0]
            b = z[f"{tag}_braw"] if sn.has_bias else None
            plain = spec.conv_raw(x, z[f"{tag}_wraw"], b, sn.stride_h, sn.stride_w, sn.pad_top, sn.pad_left,
                                  sn.dilation_h, sn.dilation_w, sn.out_h, sn.out_w, sn.is_depthwise, wrap=False)
            wrapped += int((plain != got).sum())
    assert wrapped > 0  # the wrap cases exercise the int32 wrap


@pytest.mark.gpu
@pytest.mark.parametrize("fuse", [False, True])
def test_gpu_simulator_conv_exp_vs_reference(golden, fuse):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200.simulator import GpuSimulator
    z = golden("sim_conv_exp.npz")
    for tag in _tags(z):
        g, x, per_ch = _case(z, tag)
        fx = z[f"{tag}_fx"]
        f = np.asarray(fx, np.float64).reshape(1, -1, 1, 1) if per_ch else float(fx)
        out = GpuSimulator(g, fuse=fuse).simulate({"x": x / np.power(2.0, f)})
        fy = z[f"{tag}_fy"]
        fyv = np.asarray(fy, np.float64).reshape(1, -1, 1, 1) if per_ch else float(fy)
        got = np.round(out["y"] * np.power(2.0, fyv)).astype(np.int64)
        assert np.array_equal(got, z[f"{tag}_y"]), tag
