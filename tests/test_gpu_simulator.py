"""GpuSimulator (the _forward_pass twin) on the benchmark architectures vs
the reference simulator's own forward pass (tests/golden/sim_graph_*.npz,
made by running the reference's _SimulateMixin._forward_pass on the same
graphs built with its node classes) — every materialised tensor bit-exact,
with and without epilogue fusion — and vs the CPU oracle at full size."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sim_cls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200.simulator import GpuSimulator
    return GpuSimulator


def _builders():
    from cormorant_b200 import workloads as WL
    return {"mnist_b2": lambda: WL.mnist(seed=11, batch=2),
            "mbv2_r32_b2": lambda: WL.mobilenet_v2(seed=13, batch=2, res=32)}


@pytest.mark.parametrize("name", ["mnist_b2", "mbv2_r32_b2"])
@pytest.mark.parametrize("fuse", [False, True])
def test_graph_vs_reference(sim_cls, golden, name, fuse):
    z = golden(f"sim_graph_{name}.npz")
    g, feeds, _ = _builders()[name]()
    sim = sim_cls(g, fuse=fuse)
    arr = sim.forward_pass(feeds)
    checked = 0
    for sn in g.nodes:
        nm = sn.output.onnx_name
        if nm not in arr:
            continue  # fused intermediate
        got = np.round(arr[nm] * 256).astype(np.int64)
        assert np.array_equal(got.reshape(z["t_" + nm].shape), z["t_" + nm]), nm
        checked += 1
    assert checked >= (len(g.nodes) // 2 if fuse else len(g.nodes))
    out = sim.simulate(feeds)
    for t in g.output_tensors:
        assert np.array_equal(np.round(out[t.onnx_name] * 256).astype(np.int64), z["out_" + t.onnx_name])


def test_mobilenet_v2_224_vs_oracle(sim_cls):
    """Full-resolution MobileNetV2-1.0 (2 images) against the CPU oracle."""
    from cormorant_b200 import workloads as WL
    from oracle import graph as og
    g, feeds, _ = WL.mobilenet_v2(seed=21, batch=2, res=224)
    out = sim_cls(g).simulate(feeds)
    ref = og.forward(g, feeds)
    assert np.array_equal(np.round(out["logits"] * 256).astype(np.int64), ref["logits"])
