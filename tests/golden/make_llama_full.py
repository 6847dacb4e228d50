#!/usr/bin/env python3
"""Golden of configuration 5 at its full size, made by the CPU oracle (test
infrastructure; run in the build container, where it takes tens of minutes
per sequence, so the GPU box only compares):

    python tests/golden/make_llama_full.py --seqs 0 8 16 ... [--steps 128]

For each sequence s: ``workloads.LlamaModel(seed=5, batch=1, seq=512,
layers=32, first=s)`` — the SmolLM2-360M shape the benchmark runs, sequence s
of its seeded input set — prefilled by ``oracle.llm.forward`` (the reference's
LLM entries restated: _simulate.py:541-769 on the row-ops / VectorOP / MatMul
job models, llm_nodes.py attention) and then ``steps`` greedy decode steps
(``oracle.llm.greedy_decode``).  ``llama_full_s<s>.npz`` keeps the greedy ids
of every step, the CRC-32 of the prefill's and of every step's int16 logits,
and the CRC-32 of every layer's K and V cache (int16, logical [rows][KV HD])
after the last step.
"""
from __future__ import annotations

import argparse
import os
import sys
import time
import zlib

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
SEED, SEQ, LAYERS = 5, 512, 32


def crc16(a) -> int:
    import numpy as np
    return zlib.crc32(np.ascontiguousarray(np.asarray(a, np.int64).astype("<i2")).tobytes())


def make_one(s: int, steps: int, out: str) -> None:
    import numpy as np
    sys.path.insert(0, ROOT)
    from cormorant_b200 import workloads as WL
    from oracle import llm
    t0 = time.time()
    m = WL.LlamaModel(seed=SEED, batch=1, seq=SEQ, layers=LAYERS, first=s)
    g = m.prefill_graph
    tm = {t.onnx_name: t for t in g.input_tensors}
    raw = {k: (np.asarray(v) if tm[k].host else np.rint(np.asarray(v) * 2.0 ** float(tm[k].exp)).astype(np.int64))
           for k, v in m.prefill_feeds.items()}
    states = {t.onnx_name: np.zeros(t.shape, np.int64) for t in g.state_tensors}
    wc = {}
    ref = llm.forward(g, raw, states, wc)
    lg0 = ref[g.output_tensors[0].onnx_name]
    print(f"s={s}: prefill {time.time() - t0:.0f} s", flush=True)
    ids, logits = llm.greedy_decode(m, states, lg0, steps, wc)
    res = {"seed": np.array([SEED]), "seq": np.array([s]), "steps": np.array([steps]),
           "ids": np.asarray(ids, np.int64).reshape(steps),
           "crc_prefill_logits": np.array([crc16(lg0)], np.int64),
           "crc_step_logits": np.array([crc16(x) for x in logits], np.int64),
           "crc_cache": np.array([crc16(states[t.onnx_name]) for t in g.state_tensors], np.int64),
           "cache_names": np.array([t.onnx_name for t in g.state_tensors])}
    np.savez_compressed(os.path.join(out, f"llama_full_s{s}.npz"), **res)
    print(f"s={s}: done in {time.time() - t0:.0f} s, ids {res['ids'][:8].tolist()}", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seqs", type=int, nargs="+", default=[0])
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--procs", type=int, default=0, help="parallel processes (default: one per sequence)")
    a = ap.parse_args()
    if len(a.seqs) == 1:
        make_one(a.seqs[0], a.steps, a.out)
        return
    import multiprocessing as mp
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    ctx = mp.get_context("spawn")
    with ctx.Pool(a.procs or len(a.seqs)) as pool:
        pool.starmap(make_one, [(s, a.steps, a.out) for s in a.seqs])


if __name__ == "__main__":
    main()
