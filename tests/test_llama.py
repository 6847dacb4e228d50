"""The Llama prefill graph (workloads.llama_prefill: RMSNorm / projections /
the prefill attention chain / ResAdd / SiLU(g) u / the LM head on the
kernels) on the GPU against the CPU oracle (oracle.llm: the row-ops jobs on
the job model, the attention restatement per sequence), every tensor
bit-exact, the KV caches included."""
import numpy as np
import pytest


def _raw_inputs(g, feeds):
    tm = {t.onnx_name: t for t in g.input_tensors}
    out = {}
    for k, v in feeds.items():
        t = tm[k]
        f = 0.0 if t.host else np.asarray(t.exp, np.float64)
        out[k] = np.asarray(v) if t.host else np.rint(np.asarray(v, np.float64) * 2.0 ** f).astype(np.int64)
    return out


def test_llama_oracle_runs_small():
    """The builder and the CPU oracle on a tiny configuration (no GPU)."""
    from cormorant_b200 import workloads as WL
    from oracle import llm
    g, feeds, macs = WL.llama_prefill(seed=7, batch=2, seq=16, layers=1, hidden=64, heads=4, kv_heads=2,
                                      head_dim=16, ffn=128, vocab=50)
    states = {t.onnx_name: np.zeros(t.shape, np.int64) for t in g.state_tensors}
    arr = llm.forward(g, _raw_inputs(g, feeds), states)
    lg = arr[g.output_tensors[0].onnx_name]
    assert lg.shape == (2, 50) and np.abs(lg).max() > 0 and (np.abs(lg) < 32767).mean() > 0.9
    assert macs > 0


def _compare(g, arr, ref, states, rstates):
    checked = 0
    for sn in g.nodes:
        t = sn.output
        if t.onnx_name not in arr:
            continue
        f = np.asarray(8 if t.exp is None else t.exp, np.float64)
        got = np.rint(np.asarray(arr[t.onnx_name]) * np.power(2.0, f)).astype(np.int64)
        assert np.array_equal(got.reshape(ref[t.onnx_name].shape), ref[t.onnx_name]), t.onnx_name
        checked += 1
    assert checked >= len(g.nodes) // 2
    for t in g.state_tensors:
        got = np.rint(states[t.onnx_name] * np.power(2.0, np.asarray(t.exp, np.float64))).astype(np.int64)
        assert np.array_equal(got, rstates[t.onnx_name]), t.onnx_name


@pytest.mark.parametrize("seq", [16, 144])
def test_llama_host_logic_cpu(cpu_ops, seq):
    """GpuSimulator's host logic on the Llama graph (every job's registers,
    the batched attention's strides, the states) with its kernel calls
    replayed on the oracle's job models, against the oracle's forward pass;
    at 288 rows the gate / up pair and its SiluMul run as one job (the
    interleaved weights, the MULACT shifts from the parameter words)."""
    from cormorant_b200 import workloads as WL
    from oracle import llm
    g, feeds, _ = WL.llama_prefill(seed=8, batch=2, seq=seq, layers=1, hidden=64, heads=4, kv_heads=2, head_dim=16,
                                   ffn=128, vocab=50)
    states = {t.onnx_name: np.zeros(t.shape) for t in g.state_tensors}
    arr = cpu_ops(g, device="cpu").forward_pass(feeds, states=states)
    rstates = {t.onnx_name: np.zeros(t.shape, np.int64) for t in g.state_tensors}
    ref = llm.forward(g, _raw_inputs(g, feeds), rstates)
    _compare(g, arr, ref, states, rstates)


def test_llama_lean_prefill_cpu(cpu_ops):
    """The lean prefill (only the logits kept): the q image and the scores
    held transposed, the softmax by rows — with the kernel calls replayed on
    the oracle's job models, the logits and the caches equal the oracle's."""
    from cormorant_b200 import workloads as WL
    from oracle import llm
    g, feeds, _ = WL.llama_prefill(seed=9, batch=2, seq=32, layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16,
                                   ffn=128, vocab=50)
    out = g.output_tensors[0].onnx_name
    sim = cpu_ops(g, device="cpu")
    states = {t.onnx_name: np.zeros(t.shape) for t in g.state_tensors}
    arr = sim.forward_pass(feeds, states=states, keep=[out])
    assert sim._tr, "no transposed attention in the lean pass"
    rstates = {t.onnx_name: np.zeros(t.shape, np.int64) for t in g.state_tensors}
    ref = llm.forward(g, _raw_inputs(g, feeds), rstates)
    t = g.output_tensors[0]
    got = np.rint(np.asarray(arr[out]) * np.power(2.0, np.asarray(t.exp, np.float64))).astype(np.int64)
    assert np.array_equal(got.reshape(ref[out].shape), ref[out])
    for st in g.state_tensors:
        v = np.rint(states[st.onnx_name] * np.power(2.0, np.asarray(st.exp, np.float64))).astype(np.int64)
        assert np.array_equal(v, rstates[st.onnx_name]), st.onnx_name


@pytest.mark.gpu
@pytest.mark.parametrize("fuse", [False, True])
def test_gpu_llama_prefill_vs_oracle(fuse):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import workloads as WL
    from cormorant_b200.simulator import GpuSimulator
    from oracle import llm
    g, feeds, _ = WL.llama_prefill(seed=9, batch=2, seq=32, layers=2, vocab=1000)
    sim = GpuSimulator(g, fuse=fuse)
    states = {t.onnx_name: np.zeros(t.shape) for t in g.state_tensors}
    arr = sim.forward_pass(feeds, states=states)
    rstates = {t.onnx_name: np.zeros(t.shape, np.int64) for t in g.state_tensors}
    ref = llm.forward(g, _raw_inputs(g, feeds), rstates)
    _compare(g, arr, ref, states, rstates)
    # lean mode (only the logits observed: the parts past the key count left unwritten)
    st2 = {t.onnx_name: np.zeros(t.shape) for t in g.state_tensors}
    out = g.output_tensors[0].onnx_name
    lean = sim.forward_pass(feeds, states=st2, keep=[out])
    assert np.array_equal(np.rint(lean[out] * 2.0 ** 11).astype(np.int64), ref[out])
    for t in g.state_tensors:
        assert np.array_equal(st2[t.onnx_name], states[t.onnx_name]), t.onnx_name


def _decode_vs_oracle(runner, model, steps):
    from oracle import llm
    ids = runner.generate(steps)
    rstates = {t.onnx_name: np.zeros(t.shape, np.int64) for t in model.prefill_graph.state_tensors}
    ref = llm.forward(model.prefill_graph, _raw_inputs(model.prefill_graph, model.prefill_feeds), rstates)
    rids, rlog = llm.greedy_decode(model, rstates, ref[model.prefill_graph.output_tensors[0].onnx_name], steps)
    assert np.array_equal(np.stack(ids), rids)
    last = runner.last_logits[:model.B * model.vocab].cpu().numpy().astype(np.int64).reshape(model.B, model.vocab)
    assert np.array_equal(last, rlog[-1])
    for t in model.prefill_graph.state_tensors:
        got = runner.pre.state_values(t, runner.states[t.onnx_name])
        got = np.rint(got * np.power(2.0, np.asarray(t.exp, np.float64))).astype(np.int64)
        assert np.array_equal(got, rstates[t.onnx_name]), t.onnx_name


def test_llama_decode_host_logic_cpu(cpu_ops):
    """Prefill then greedy decode steps (the decode-step graph with the host
    softmax, the device greedy step) with the kernel calls replayed on the
    oracle's job models, against the oracle's own loop."""
    from cormorant_b200 import workloads as WL
    from cormorant_b200.llm_runner import LlamaRunner
    m = WL.LlamaModel(seed=12, batch=3, seq=16, layers=1, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=128,
                      vocab=50)  # 3 sequences: the step's q / k / v and gate / up run as column groups
    _decode_vs_oracle(LlamaRunner(m, device="cpu"), m, 3)


@pytest.mark.gpu
def test_gpu_llama_decode_vs_oracle():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import workloads as WL
    from cormorant_b200.llm_runner import LlamaRunner
    m = WL.LlamaModel(seed=13, batch=3, seq=32, layers=2, vocab=1000)  # 3 rows: column-group projections
    _decode_vs_oracle(LlamaRunner(m), m, 4)


@pytest.mark.gpu
@pytest.mark.parametrize("dims", [dict(hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=128),
                                  dict(hidden=256, heads=8, kv_heads=1, head_dim=32, ffn=256),
                                  dict(hidden=640, heads=10, kv_heads=2, head_dim=64, ffn=256)],
                         ids=["g2_hd16", "g8_hd32", "g5_hd64"])
def test_gpu_llama_decode_heads_vs_oracle(dims):
    """The decode attention launch at other group sizes and head widths (2
    heads of 16, 8 heads of 32, 5 heads of 64 per KV group: the compiled
    64-wide form at two CTAs an SM, its P.V sums reduced head by head)
    against the oracle's loop."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cormorant_b200 import workloads as WL
    from cormorant_b200.llm_runner import LlamaRunner
    m = WL.LlamaModel(seed=21, batch=3, seq=16, layers=1, vocab=300, **dims)
    _decode_vs_oracle(LlamaRunner(m), m, 3)


def test_sibling_groups_host_logic():
    """Which MatMuls the simulator runs as one column-group launch: per Llama
    layer q / k / v and gate / up (same A, constant weights, widths in runs of
    32); none in BERT, whose projections carry a fused bias job; none at two
    rows or fewer (the GEMV path); none with fusion off."""
    from cormorant_b200 import workloads as WL
    from cormorant_b200.simulator import GpuSimulator
    m = WL.LlamaModel(seed=3, batch=3, seq=16, layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=128,
                      vocab=256)
    for g in (m.prefill_graph, m.decode_graph):
        s = GpuSimulator(g, device="cpu")
        names = sorted(tuple(g.nodes[j].output.onnx_name.split(".")[-1] for j in v) for v in s._groups.values())
        assert names == [("g", "u")] * 2 + [("q0", "k0", "v")] * 2
        assert not GpuSimulator(g, fuse=False, device="cpu")._groups
    bert = WL.bert_base(seed=4, batch=1, seq=32, layers=1)[0]
    assert not GpuSimulator(bert, device="cpu")._groups
    m1 = WL.LlamaModel(seed=3, batch=2, seq=16, layers=1, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=128,
                       vocab=256)
    assert not GpuSimulator(m1.decode_graph, device="cpu")._groups  # 2 rows: the GEMV path
