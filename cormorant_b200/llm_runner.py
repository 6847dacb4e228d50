"""Prefill and greedy decode of a ``workloads.LlamaModel`` on the device: the
prefill graph, then decode steps, each one pass of the decode-step graph at
pos = T + i over the same KV-cache states, with the token chosen on the
device between them (``corm_greedy_embed``: the first argmax of each
sequence's logits and its embedding row as the next input) — the loop the
reference's host runs between its LLM entries (the prefill entry, then a
decode entry per token, with LlmDequant / argmax / LlmEmbed on the host).
"""
from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch

from . import ops
from .simulator import GpuSimulator


class LlamaRunner:
    def __init__(self, model, device=None, fuse: bool = True):
        self.m = model
        self.pre = GpuSimulator(model.prefill_graph, device=device, fuse=fuse)
        self.dec = GpuSimulator(model.decode_graph, device=self.pre.device, fuse=fuse, share=self.pre)
        self.device = self.pre.device
        self.states = self.pre.states_to_device()
        self.out_pre = model.prefill_graph.output_tensors[0].onnx_name
        self.out_dec = model.decode_graph.output_tensors[0].onnx_name
        emb = np.rint(model.emb * 2.0 ** model.E["fr"]).astype(np.int32)
        self.table = torch.from_numpy(emb).to(self.device)
        self.h = torch.empty(model.B * model.D + 4, dtype=torch.int32, device=self.device)
        self.raw_pre = None

    def prefill(self, feeds=None) -> torch.Tensor:
        """The prefill pass (lean: only the logits kept); returns the int16
        logits [B][vocab] on the device."""
        feeds = self.m.prefill_feeds if feeds is None else feeds
        if self.raw_pre is None:
            g = self.m.prefill_graph
            self.raw_pre = {t.onnx_name: (np.asarray(feeds[t.onnx_name]).astype(np.int64).reshape(-1) if t.host
                                          else self.pre._to_raw(t, feeds[t.onnx_name])) for t in g.input_tensors}
        res, _ = self.pre.forward_raw(self.raw_pre, keep=[self.out_pre], states=self.states)
        return res[self.out_pre]

    def decode_step(self, logits: torch.Tensor, i: int, ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Decode step i (pos = T + i) after ``logits``: the next tokens'
        embedding rows, then one decode-step pass; returns its logits."""
        m = self.m
        ops.greedy_embed(logits, self.table, self.h, ids, batch=m.B, vocab=m.vocab, dim=m.D)
        res, _ = self.dec.forward_raw({"h_step": self.h, "pos": np.array([m.T + i])}, keep=[self.out_dec],
                                      states=self.states)
        return res[self.out_dec]

    def generate(self, steps: int) -> List[np.ndarray]:
        """Prefill then ``steps`` greedy steps; returns the token ids chosen
        before every step ([B] each)."""
        lg = self.prefill()
        ids = torch.empty((steps, self.m.B), dtype=torch.int32, device=self.device)
        for i in range(steps):
            lg = self.decode_step(lg, i, ids[i])
        self.last_logits = lg
        return [r for r in ids.cpu().numpy()]
