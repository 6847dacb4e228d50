"""Parity at the configurations' timed sizes (the benchmark's own builders and
seeds; rank 0's units, and for the Llama model two sequences of a batch):

* BERT-base: 12 layers x 384 tokens, 2 sequences — the SQuAD
  logits equal the CPU oracle's forward pass (``oracle/graph.py``, the
  reference's ``_forward_pass`` restated and pinned to its goldens);
* MobileNetV2-1.0 at 224 x 224: 4 images, the logits;
* MNIST: 64 images, the softmax output;
* the SmolLM2-360M-shaped Llama: 32 layers, a 512-token prefill
  and all 128 greedy decode steps, run as the benchmark runs it (a batch of
  sequences side by side, the decode steps captured and replayed as CUDA
  graphs), against the oracle's goldens of sequences 0 and 8
  (``tests/golden/llama_full_s*.npz``, ``make_llama_full.py``): the greedy
  ids of every step, the CRC-32 of the prefill logits and of every step's
  logits, and the CRC-32 of every layer's K / V cache after the last step.
Bit-exact: no tolerance."""
import zlib

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


def _crc16(a) -> int:
    return zlib.crc32(np.ascontiguousarray(np.asarray(a, np.int64).astype("<i2")).tobytes())


@pytest.mark.parametrize("name", ["bert_base_384_l12_b2", "mobilenet_v2_224_b4", "mnist_b64"])
def test_config_vs_oracle(sim_cls, name):
    from cormorant_b200 import workloads as WL
    from oracle import graph as og
    g, feeds, _ = {"bert_base_384_l12_b2": lambda: WL.bert_base(seed=4, batch=2, seq=384),
                   "mobilenet_v2_224_b4": lambda: WL.mobilenet_v2(seed=3, batch=4, res=224),
                   "mnist_b64": lambda: WL.mnist(seed=1, batch=64)}[name]()
    out_t = g.output_tensors[0]
    sim = sim_cls(g)
    raw = {t.onnx_name: sim._to_raw(t, feeds[t.onnx_name]) for t in g.input_tensors}
    res, _ = sim.forward_raw(raw, keep=[out_t.onnx_name])
    got = res[out_t.onnx_name][:out_t.numel].cpu().numpy().astype(np.int64)
    ref = og.forward(g, feeds)[out_t.onnx_name].reshape(-1)
    assert np.array_equal(got, ref)


def test_llama_full_prefill_decode_vs_golden(golden):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import workloads as WL
    from cormorant_b200.llm_runner import LlamaRunner
    seqs, steps = (0, 8), 128
    zs = {s: golden(f"llama_full_s{s}.npz") for s in seqs}
    B = 9
    m = WL.LlamaModel(seed=int(zs[0]["seed"][0]), batch=B, seq=512)
    assert m.L == 32 and m.vocab == 49152
    r = LlamaRunner(m)
    stream = torch.cuda.Stream()
    ids = torch.empty((steps, B), dtype=torch.int32, device=r.device)
    with torch.cuda.stream(stream):
        lg0 = r.prefill()
        pre = lg0[:B * m.vocab].clone()
        r.decode_step(lg0, steps - 1)  # the largest key count: sized before capture
    torch.cuda.synchronize()
    pool = torch.cuda.graph_pool_handle()
    graphs, lg, outs = [], lg0, []
    for i in range(steps):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream, pool=pool):
            lg = r.decode_step(lg, i, ids[i])
        graphs.append(gr)
        outs.append(lg)
    step_logits = []
    with torch.cuda.stream(stream):
        for i, gr in enumerate(graphs):
            gr.replay()
            step_logits.append(outs[i][:B * m.vocab].clone())
    torch.cuda.synchronize()
    pre = pre.cpu().numpy().reshape(B, m.vocab)
    idv = ids.cpu().numpy()
    cache = {t.onnx_name: np.rint(r.pre.state_values(t, r.states[t.onnx_name]) *
                                  np.power(2.0, np.asarray(t.exp, np.float64))).astype(np.int64)
             for t in m.prefill_graph.state_tensors}
    for s in seqs:
        z = zs[s]
        assert _crc16(pre[s]) == int(z["crc_prefill_logits"][0]), f"sequence {s}: prefill logits"
        assert np.array_equal(idv[:, s], z["ids"][:steps]), f"sequence {s}: greedy ids"
        for i in range(steps):
            lgi = step_logits[i].cpu().numpy().reshape(B, m.vocab)[s]
            assert _crc16(lgi) == int(z["crc_step_logits"][i]), f"sequence {s}: logits of step {i}"
        C = m.C
        for name, crc in zip(z["cache_names"], z["crc_cache"]):
            assert _crc16(cache[str(name)][s * C:(s + 1) * C]) == int(crc), f"sequence {s}: cache {name}"
    del graphs
