"""BERT-base widths on the device: GpuSimulator over the encoder graph
(LayerNorm and head transposes as row-ops jobs, softmax on the VectorOP unit,
batched MatMuls) against the reference simulator's pass (CRC-32 of every
intermediate, tests/golden/sim_graph_bert_l2_t32_b2.npz) and against the
oracle on a longer sequence."""
import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(g, feeds, fuse=True):
    from cormorant_b200.simulator import GpuSimulator
    sim = GpuSimulator(g, fuse=fuse)
    raw = {"x": sim._to_raw(g.input_tensors[0], feeds["x"])}
    res, meta = sim.forward_raw(raw)
    return {k: v[:meta[k].numel].cpu().numpy().astype(np.int64).reshape(meta[k].shape) for k, v in res.items()}


@pytest.mark.parametrize("fuse", [True, False])
def test_bert_small_vs_reference(golden, fuse):
    from cormorant_b200 import workloads as WL
    z = golden("sim_graph_bert_l2_t32_b2.npz")
    g, feeds, _ = WL.bert_base(seed=17, batch=2, seq=32, layers=2)
    out = _run(g, feeds, fuse)
    missing = 0
    for sn in g.nodes:
        name = sn.output.onnx_name
        if name not in out:  # folded into its producer's epilogue
            assert fuse
            missing += 1
            continue
        crc = zlib.crc32(np.ascontiguousarray(out[name].astype("<i2")).tobytes())
        assert crc == int(z["c_" + name][0]), name
    assert np.array_equal(out["qa_logits"].reshape(z["out_qa_logits"].shape), z["out_qa_logits"])
    assert (missing > 0) == fuse


def test_bert_seq384_one_layer_vs_oracle():
    """Full BERT-base shapes per layer (384 tokens, 2 sequences, one layer):
    every tensor equal to the oracle's."""
    from cormorant_b200 import workloads as WL
    from oracle import graph as og
    g, feeds, _ = WL.bert_base(seed=21, batch=2, seq=384, layers=1)
    out = _run(g, feeds)
    ref = og.forward(g, feeds)
    for sn in g.nodes:
        name = sn.output.onnx_name
        if name in out:
            assert np.array_equal(out[name], ref[name].reshape(out[name].shape)), name


def test_bert_lean_keep():
    """The lean pass (``keep``) returns the outputs unchanged."""
    from cormorant_b200 import workloads as WL
    from cormorant_b200.simulator import GpuSimulator
    g, feeds, _ = WL.bert_base(seed=17, batch=2, seq=32, layers=2)
    full = _run(g, feeds)
    sim = GpuSimulator(g)
    res = sim.simulate(feeds)
    assert np.array_equal(np.round(res["qa_logits"] * 256).astype(np.int64), full["qa_logits"])
