"""GpuSimulator — the B200 twin of the reference simulator's forward pass
(phoenix367/cormorant inference-scheduler/src/codegen/_simulate.py:382-403
``simulate`` and :541-769 ``_forward_pass``).

Same surface: ``simulate(inputs)`` takes float64 value arrays in logical
shapes and returns the graph outputs as float64 values; ``forward_pass(inputs,
states=None, keep=None)`` returns every tensor visited (or only ``keep``).
Inside, every tensor lives on the device as its int16 storage integers (raw =
value * 2^f, f = 8 for Q8.8 or the tensor's exponent): values are converted
once at entry (round half to even, the inputs being on their grid by the
reference's convention) and once at exit, and every node runs as one or more
launches of the sm_100a kernels through the C ABI (cormorant_b200.ops).  There
is no CPU path: a node type without a kernel here raises NotImplementedError.

Numerics per node type, all bit-exact with the reference's branch:
  MatmulNode / MatmulConvNode  sat16(floor(sum / 2^8)); int32 wrap first when
                               any operand carries an exponent (:620-633, :814-835)
  ConvNode                     bias << 8 seeded, same rule (:643-660, :784-812)
  PoolNode                     MAX / AVG / LP (:701-719, :230-358)
  ScheduledNode                op, saturation, fused act (:721-765); DIV follows
                               the kernel (b = 0 gives 0), the float path of the
                               reference gives +-max / NaN there
  SoftmaxVopNode               the softmax unit, row mode (smx_nodes.py:121-134)
  LayerNormRoNode, TransposeRoNode, ResAddRoNode, RMSNormRoNode, WidenRoNode,
  SiluMulRoNode                one row-ops job each, the registers of the
                               node's emit_call (rowops_nodes.py:162-583);
                               int32 DMA tensors (dma "i32") held as int32
  VitGeluVopNode               two VectorOP jobs (vit_nodes.py:580-668)
  ReshapeNode / SpaceToDepth   views / reorders (:662-665, :692-699)

Graph fusion (``fuse=True``): a ScheduledNode whose input is a Conv / MatMul
output read by nothing else is folded into that kernel's epilogue, and the
intermediate tensor is not materialised: a Relu / Clip(0,6) as an act flag
(CORM_F_ACT_RELU / RELU6 — max(sat16(v), 0) is what the separate node
computes), an ADD / SUB / MUL (with its fused act) against a bias row, a
scalar or a same-shaped tensor as a fused VectorOP job (corm_matmul_post /
corm_conv_post, bit-exact with the two jobs).
"""
from __future__ import annotations

from typing import Dict, Iterable, Optional

import numpy as np
import torch

from . import ops
from ._lib import F_ACT_RELU, F_ACT_RELU6, F_WEIGHT_LOGICAL, F_WRAP32

_ACT_FOR_OP = {4: 1, 5: 2, 6: 3, 7: 4, 8: 5, 9: 6}


def _kind(node) -> str:
    return type(node).__name__


def _exp_of(t, frac_bits: int = 8):
    """The tensor's exponent(s) for raw <-> value: scalar f, or an array
    broadcastable to its logical shape (chexp on axis 1)."""
    if getattr(t, "chexp", None) is not None:
        ce = np.asarray(t.chexp, np.float64).reshape(-1)
        shape = [1] * max(len(t.shape), 2)
        shape[1] = ce.size
        return ce.reshape(shape)
    e = getattr(t, "exp", None)
    if e is None:
        return frac_bits
    e = np.asarray(e, np.float64)
    return float(e) if e.ndim == 0 else e


def _is_f32(t) -> bool:
    """A float32 tensor (the float residual stream, a DEQUANT output): its
    buffer holds values, not raw words at an exponent."""
    return getattr(t, "host", None) == "f32" or getattr(t, "dma", None) == "f32"


def _chan(t, n: int, frac_bits: int = 8) -> np.ndarray:
    """The exponent of each of the n channels of t's last axis (int64)."""
    if getattr(t, "chexp", None) is not None:
        e = np.asarray(t.chexp, np.int64).reshape(-1)
    elif getattr(t, "exp", None) is not None:
        e = np.asarray(t.exp, np.int64).reshape(-1)
    else:
        e = np.array([frac_bits], np.int64)
    return np.broadcast_to(e, (n,)) if e.size == 1 else e[:n]


def _has_exp(*ts) -> bool:
    return any(getattr(t, a, None) is not None for t in ts for a in ("exp", "wexp", "chexp"))


class GpuSimulator:
    """Forward pass of a node graph on the current CUDA device."""

    def __init__(self, graph, fuse: bool = True, device=None, share=None):
        """``share``: another GpuSimulator whose device weights (and tables)
        this one reuses — the prefill and decode graphs of one model."""
        self._graph = graph
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.fuse = fuse
        self._weights: Dict[str, torch.Tensor] = share._weights if share is not None else {}
        self._ws: Optional[torch.Tensor] = None
        self._plan = self._fusion_plan() if fuse else {}
        self._groups = self._sibling_groups() if fuse else {}
        self._pairs = self._rowops_pairs() if fuse else {}
        self._mulacts = self._mulact_pairs() if fuse else {}

    # ------------------------------------------------------------ tensors
    def _alloc(self, numel: int) -> torch.Tensor:
        # every buffer padded to whole 8-lane words (+ one word): the kernels
        # write the tail lanes of the last word, as the hardware does
        return torch.empty((numel + 7) // 8 * 8 + 8, dtype=torch.int16, device=self.device)

    def _alloc32(self, numel: int) -> torch.Tensor:
        """An int32 DMA tensor (the LLM residual stream), padded to whole
        16-byte words (+ one word)."""
        return torch.empty((numel + 3) // 4 * 4 + 4, dtype=torch.int32, device=self.device)

    def _alloc_f32(self, numel: int) -> torch.Tensor:
        """A float32 tensor (padded to whole 16-byte words, plus one)."""
        return torch.empty((numel + 3) // 4 * 4 + 4, dtype=torch.float32, device=self.device)

    def _to_raw(self, t, values) -> torch.Tensor:
        if _is_f32(t):  # values as they are, in float32
            buf = self._alloc_f32(t.numel)
            buf[:t.numel].copy_(torch.from_numpy(np.asarray(values, np.float32).reshape(-1)))
            return buf
        f = _exp_of(t)
        v = np.round(np.asarray(values, np.float64).reshape(t.shape) * np.power(2.0, f))
        if getattr(t, "dma", None) == "i32":
            raw = np.clip(v, -2147483648.0, 2147483647.0).astype(np.int32)
            buf = self._alloc32(t.numel)
        else:
            raw = np.clip(v, -32768, 32767).astype(np.int16)
            buf = self._alloc(t.numel)
        buf[:t.numel].copy_(torch.from_numpy(raw.reshape(-1)))
        return buf

    def _weight_raw(self, t) -> torch.Tensor:
        """_simulate.py:531-539: weights quantised RNE + saturate at Q8.8; a
        rank-1 exponent weight keeps the same raw integers."""
        if t.onnx_name not in self._weights:
            v = np.clip(np.asarray(t.data, np.float64).reshape(t.shape), -128.0, 127.99609375)
            raw = np.round(v * 256.0).astype(np.int16)
            buf = self._alloc(t.numel)
            buf[:t.numel].copy_(torch.from_numpy(raw.reshape(-1)))
            self._weights[t.onnx_name] = buf
        return self._weights[t.onnx_name]

    def _bias_raw(self, node, t) -> torch.Tensor:
        """Conv bias as the kernel adds it: raw at the output's exponent
        (_simulate.py:805; Q8.8: the quantised value's raw)."""
        key = ("bias", t.onnx_name, node.output.onnx_name)
        if key not in self._weights:
            v = np.clip(np.asarray(t.data, np.float64).reshape(-1), -128.0, 127.99609375)
            if getattr(t, "wexp", None) is not None:
                # encoded at its exponent (numeric.py:258-307: f_b = f_y): data holds
                # raw / 2^8, the value raw / 2^f_b, so at f_y the raw is round(data 2^8)
                # 2^(f_y - f_b) — the stored word itself when f_b = f_y
                M = node.out_ch
                fy = np.broadcast_to(np.asarray(_exp_of(node.output), np.float64).reshape(-1), (M,))
                fb = np.broadcast_to(np.asarray(t.wexp, np.float64).reshape(-1), (M,))
                raw = np.round(np.round(v[:M] * 256.0) * np.power(2.0, fy - fb))
            elif _has_exp(node.output):
                fy = _exp_of(node.output)
                fy = np.asarray(fy, np.float64).reshape(-1) if np.ndim(fy) else fy
                raw = np.round(np.round(v * 256.0) / 256.0 * np.power(2.0, fy))
            else:
                raw = np.round(v * 256.0)
            buf = self._alloc(raw.size)
            buf[:raw.size].copy_(torch.from_numpy(np.clip(raw, -32768, 32767).astype(np.int16)))
            self._weights[key] = buf
        return self._weights[key]

    def _workspace(self, nbytes: int) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
        return self._ws

    # ------------------------------------------------------------ fusion
    def _fusion_plan(self):
        """{consumer node index: (producer index, act flag, post)} for the
        ScheduledNodes folded into a Conv / MatMul epilogue: Relu / Clip(0,6)
        as an act flag; ADD / SUB / MUL with a bias row (MatMul), a scalar or
        a same-shaped tensor as a fused VectorOP job (corm_*_post)."""
        nodes = self._graph.nodes
        readers: Dict[str, int] = {}
        for sn in nodes:
            for t in sn.inputs:
                if t is not None:
                    readers[t.onnx_name] = readers.get(t.onnx_name, 0) + 1
        outs = {t.onnx_name for t in self._graph.output_tensors}
        producer = {getattr(sn, "output", None).onnx_name: i for i, sn in enumerate(nodes)
                    if getattr(sn, "output", None) is not None}
        plan = {}
        taken = set()
        for i, sn in enumerate(nodes):
            if _kind(sn) != "ScheduledNode":
                continue
            op, act = sn.op_code, getattr(sn, "act", 0)
            if op in (4, 5) and act == 0:
                cands = [(0, None)]
            elif op in (0, 1, 2) and len(sn.inputs) == 2:
                cands = [(0, sn.inputs[1]), (1, sn.inputs[0])]
            else:
                continue
            for pos, other in cands:
                src = sn.inputs[pos].onnx_name
                j = producer.get(src)
                if j is None or j in taken or readers.get(src, 0) != 1 or src in outs:
                    continue
                pk = _kind(nodes[j])
                if pk not in ("ConvNode", "MatmulNode", "MatmulConvNode"):
                    continue
                if other is None:
                    plan[i] = (j, F_ACT_RELU if op == 4 else F_ACT_RELU6, None)
                    taken.add(j)
                    break
                # the other operand must exist when the producer runs
                po = producer.get(other.onnx_name)
                if po is not None and po > j:
                    continue
                N, no = sn.output.numel, other.numel
                if sn.inputs[pos].numel != N:
                    continue
                if no == N:
                    mode = 1
                elif no == 1:
                    mode = 2
                elif pk != "ConvNode" and no == int(sn.output.shape[-1]) and N % no == 0:
                    mode = 0
                else:
                    continue
                post = dict(other=other, op=op, act=act, alpha=getattr(sn, "alpha", 0), b_mode=mode,
                            b_is_first=1 if (op == 1 and pos == 1) else 0)
                plan[i] = (j, 0, post)
                taken.add(j)
                break
        return plan

    # ------------------------------------------------------------ forward
    def simulate(self, inputs: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
        """_simulate.py:382-403: float64 values in, graph outputs out."""
        arrays = self.forward_pass(inputs, keep=[t.onnx_name for t in self._graph.output_tensors])
        return {t.onnx_name: arrays[t.onnx_name] for t in self._graph.output_tensors}

    def forward_pass(self, input_arrays: Dict[str, np.ndarray], states=None,
                     keep: Optional[Iterable[str]] = None) -> Dict[str, np.ndarray]:
        """_simulate.py:541-769 on the device; returns float64 values of every
        tensor visited (or only ``keep``, plus the states).  ``states``
        ({name: float64 logical array}) are updated IN PLACE, as the
        reference's are; None: fresh copies of the initial values."""
        tmap = {t.onnx_name: t for t in self._graph.input_tensors}
        raw_in = {}
        for name, v in input_arrays.items():
            t = tmap[name]
            if getattr(t, "host", None) == "f32":     # float32 host rows: on the device as float32
                raw_in[name] = self._to_raw(t, v)
            elif getattr(t, "host", None) is not None:   # a host int (pos, n, ids): stays on the host
                if t.host != "i32":
                    raise NotImplementedError(f"GpuSimulator: host tensor kind {t.host}")
                raw_in[name] = np.asarray(v).astype(np.int64).reshape(-1)
            else:
                raw_in[name] = self._to_raw(t, v)
        dev_states = self.states_to_device(states)
        raw, meta = self.forward_raw(raw_in, keep=keep, states=dev_states)
        names = set(keep) if keep is not None else set(raw)
        out = {}
        for name in names:
            if name not in raw or name in dev_states:
                continue
            t = meta[name]
            if isinstance(raw[name], np.ndarray):
                out[name] = raw[name].astype(np.float64).reshape(t.shape)
                continue
            v = raw[name][:t.numel].cpu().numpy().astype(np.float64).reshape(t.shape)
            out[name] = v if _is_f32(t) else v / np.power(2.0, _exp_of(t))
        for t in self._graph.state_tensors:
            vals = self.state_values(t, dev_states[t.onnx_name])
            if states is not None:
                states[t.onnx_name][...] = vals.reshape(np.shape(states[t.onnx_name]))
            out[t.onnx_name] = vals
        return out

    # ------------------------------------------------------------ states
    def initial_states(self) -> Dict[str, np.ndarray]:
        """_simulate.py:775-782: fresh float64 copies of every state's initial value."""
        return {t.onnx_name: (np.zeros(t.shape) if getattr(t, "init_data", None) is None
                              else np.array(t.init_data, np.float64).reshape(t.shape))
                for t in self._graph.state_tensors}

    @staticmethod
    def _group_major(t, raw: np.ndarray, to_device: bool) -> np.ndarray:
        """A group-major state (group_layout (G, D)): logical [R][G D] <->
        storage [G][R][D]."""
        gl = getattr(t, "group_layout", None)
        if not gl:
            return raw
        G, D = int(gl[0]), int(gl[1])
        R = t.numel // (G * D)
        if to_device:
            return np.ascontiguousarray(raw.reshape(R, G, D).transpose(1, 0, 2))
        return np.ascontiguousarray(raw.reshape(G, R, D).transpose(1, 0, 2)).reshape(t.shape)

    def states_to_device(self, states=None) -> Dict[str, torch.Tensor]:
        """The states' storage integers on the device ({name: buffer}; a KV
        cache group-major), from value arrays (default: the initial values)."""
        vals = self.initial_states() if states is None else states
        out = {}
        for t in self._graph.state_tensors:
            f = _exp_of(t)
            v = np.round(np.asarray(vals[t.onnx_name], np.float64).reshape(t.shape) * np.power(2.0, f))
            if getattr(t, "dma", None) == "i32":
                raw = np.clip(v, -2147483648.0, 2147483647.0).astype(np.int32)
                buf = self._alloc32(t.numel)
            else:
                raw = np.clip(v, -32768, 32767).astype(np.int16)
                buf = self._alloc(t.numel)
            buf[:t.numel].copy_(torch.from_numpy(self._group_major(t, raw, True).reshape(-1)))
            out[t.onnx_name] = buf
        return out

    def state_values(self, t, buf: torch.Tensor) -> np.ndarray:
        """A device state back as its logical float64 values."""
        raw = buf[:t.numel].cpu().numpy().astype(np.float64)
        raw = self._group_major(t, raw, False).reshape(t.shape)
        return raw / np.power(2.0, _exp_of(t))

    def forward_raw(self, raw_inputs: Dict[str, torch.Tensor], keep: Optional[Iterable[str]] = None,
                    states: Optional[Dict[str, torch.Tensor]] = None):
        """The pass on int16 device tensors (no host conversion): returns
        ({name: raw tensor}, {name: TensorInfo}).  With ``keep`` (the lean
        mode of _simulate.py:573-592) every other tensor is released after its
        last reader, so the allocator reuses its memory.  ``states``: the
        device states (``states_to_device``), updated in place; host int
        inputs (pos, n) are numpy arrays."""
        raw: Dict[str, torch.Tensor] = dict(raw_inputs)
        # lean mode: a tensor outside ``keep`` is never observed, so parts no
        # reader takes (the scores / P past the key count) need not be zeroed
        self._observed = None if keep is None else set(keep)
        snames = {t.onnx_name for t in self._graph.state_tensors}
        if snames:
            if states is None:
                states = self.states_to_device()
            raw.update({k: states[k] for k in snames})
        dying: Dict[int, list] = {}
        if keep is not None:
            keep = set(keep)
            last: Dict[str, int] = {}
            for i, sn in enumerate(self._graph.nodes):
                for t in sn.inputs:
                    if t is not None:
                        last[t.onnx_name] = i
                last.setdefault(sn.output.onnx_name, i)
            # a fused decode attention reads its blocks' inputs at the merge
            for mi, info in (self._decode_attn_plan(keep) if self.fuse else {}).items():
                for j in info["nodes"]:
                    for t in self._graph.nodes[j].inputs:
                        if t is not None:
                            last[t.onnx_name] = max(last.get(t.onnx_name, mi), mi)
            wnames = {t.onnx_name for t in self._graph.weight_tensors}
            for name, i in last.items():
                if name not in keep and name not in wnames and name not in snames:
                    dying.setdefault(i, []).append(name)
        meta = {t.onnx_name: t for t in self._graph.input_tensors}
        meta.update({t.onnx_name: t for t in self._graph.state_tensors})
        for t in self._graph.weight_tensors:
            if getattr(t, "data", None) is not None:
                meta[t.onnx_name] = t
        fused_into = {j: (i, flag, post) for i, (j, flag, post) in self._plan.items()}
        skip = set(self._plan)
        for members in self._groups.values():  # run at their group's first member
            skip |= set(members[1:])
        attn_fused = self._decode_attn_plan(keep) if (self.fuse and keep is not None) else {}
        for _mi, info in attn_fused.items():
            skip |= set(info["nodes"])
        # prefill attention with the q image and the scores in their transposed
        # layouts where nobody observes them (the names of the tensors held so)
        self._tr = self._attn_transpose_plan(keep) if (self.fuse and keep is not None) else set()
        skip |= set(self._pairs.values())
        skip |= set(self._mulacts.values())

        def get(t):
            if t.onnx_name not in raw:
                raw[t.onnx_name] = self._weight_raw(t)
            return raw[t.onnx_name]

        for i, sn in enumerate(self._graph.nodes):
            if i in skip:  # folded into its producer's launch
                for name in dying.get(i, ()):
                    raw.pop(name, None)
                continue
            kind = _kind(sn)
            out_t = sn.output
            flag, alias_t, post = 0, None, None
            if i in fused_into:
                ri, flag, pspec = fused_into[i]
                alias_t = self._graph.nodes[ri].output
                if pspec is not None:
                    post = self._post_of(pspec, get)
            if i in self._mulacts:  # gate / up and their SiLU(g) u in one launch
                sm = self._graph.nodes[self._mulacts[i]]
                y = self._matmul_mulact(self._groups[i], sm, get)
                out_t = sm.output
            elif i in self._groups:
                ys = self._matmul_group(self._groups[i], get)
                for j, yj in zip(self._groups[i][1:], ys[1:]):
                    t = self._graph.nodes[j].output
                    raw[t.onnx_name] = yj
                    meta[t.onnx_name] = t
                y = ys[0]
            elif kind in ("MatmulNode", "MatmulConvNode"):
                y = self._matmul(sn, get(sn.inputs[0]), get(sn.inputs[1]), flag, post)
            elif kind == "ConvNode":
                y = self._conv(sn, get(sn.inputs[0]), get(sn.inputs[1]),
                               self._bias_raw(sn, sn.inputs[2]) if sn.has_bias else None, flag, post)
            elif kind == "ReshapeNode":
                y = get(sn.inputs[0])
            elif kind == "PoolNode":
                y = self._pool(sn, get(sn.inputs[0]))
            elif kind == "SpaceToDepthNode":
                bs = sn.blocksize
                x = get(sn.inputs[0])[:sn.inputs[0].numel].view(sn.batch, sn.in_ch, sn.in_h // bs, bs, sn.in_w // bs, bs)
                y = self._alloc(out_t.numel)
                y[:out_t.numel].view(sn.batch, bs, bs, sn.in_ch, sn.in_h // bs, sn.in_w // bs).copy_(
                    x.permute(0, 3, 5, 1, 2, 4))
            elif kind == "SoftmaxVopNode":
                y = self._alloc(out_t.numel)
                ops.vectorop(get(sn.inputs[0]), None, y, size=sn.n, op=10, outer=sn.rows, a_inc=sn.n, b_inc=sn.n,
                             smx_cm=sn.cm, smx_cfg=sn.cfg, smx_mask=sn.n)
            elif kind == "ScheduledNode":
                y = self._vectorop(sn, get)
            elif kind == "LayerNormRoNode":
                y = self._layernorm(sn, get(sn.inputs[0]), get(sn.inputs[1]))
            elif kind == "TransposeRoNode":
                y = self._transpose(sn, get(sn.inputs[0]), get(sn.inputs[1]))
            elif kind == "ResAddRoNode" and i in self._pairs:
                nn = self._graph.nodes[self._pairs[i]]
                y, y2 = self._resadd_norm(sn, nn, get)
                raw[nn.output.onnx_name] = y2
                meta[nn.output.onnx_name] = nn.output
            elif kind in ("ResAddRoNode", "RMSNormRoNode", "WidenRoNode", "SiluMulRoNode"):
                y = self._llm_rowops(sn, kind, get)
            elif kind == "VitGeluVopNode":
                y = self._vit_gelu(sn, get)
            elif kind == "AttnPrepRoNode":
                y = self._attn_prep(sn, get)
            elif kind == "LlmAttnConvNode":
                y = self._attn_conv(sn, get)
            elif kind == "LlmAttnSoftmaxVopNode":
                y = self._attn_softmax(sn, get)
            elif kind == "LlmAttnSoftmaxNode":
                y = self._attn_softmax_host(sn, get)
            elif kind == "LlmAttnMergeNode" and i in attn_fused:
                y = self._decode_attn(sn, attn_fused[i], get)
            elif kind == "LlmAttnMergeNode":
                y = self._attn_merge(sn, get)
            elif kind == "LlmSelectRowNode":
                y = self._select_row(sn, get)
            elif kind in ("LlmEmbedNode", "LlmDequantNode", "LlmToHostNode", "LlmResAddNode", "LlmRMSNormNode",
                          "LlmSiluMulNode", "LlmGeluMulNode"):
                y = self._llm_host(sn, kind, get)
            elif kind == "LlmAttnPrepNode":
                y = self._attn_prep_host(sn, get)
            else:
                raise NotImplementedError(f"GpuSimulator: no sm_100a kernel for node type {kind}")
            if alias_t is not None:  # the fused intermediate is not materialised
                raw[alias_t.onnx_name] = y
                meta[alias_t.onnx_name] = alias_t
            else:
                raw[out_t.onnx_name] = y
                meta[out_t.onnx_name] = out_t
            for name in dying.get(i, ()):
                raw.pop(name, None)
        return raw, meta

    # ------------------------------------------------------------ node kernels
    def _post_of(self, pspec, get):
        """The corm_postop of a fused VectorOP node: its other operand on the
        device (a small weight broadcast as one scalar, a bias row or a full
        tensor at the output's offsets)."""
        return dict(b=get(pspec["other"]), op=pspec["op"], act=pspec["act"], alpha=pspec["alpha"],
                    b_mode=pspec["b_mode"], b_is_first=pspec["b_is_first"])

    def _matmul(self, sn, a, b, flag, post=None):
        A, B, Y = sn.inputs[0], sn.inputs[1], sn.output
        wrap = F_WRAP32 if _has_exp(A, B, Y) else 0
        ash, bsh = list(A.shape), list(B.shape)
        if len(bsh) == 2 and len(ash) > 2:  # a weight: A's leading dims are rows
            ash = [int(np.prod(ash[:-1])), ash[-1]]
        if len(bsh) == 1:
            bsh = [bsh[0], 1]
        if len(ash) == 1:
            ash = [1, ash[0]]
        n, k, m = ash[-2], ash[-1], bsh[-1]
        lead_a, lead_b = ash[:-2], bsh[:-2]
        L = max(len(lead_a), len(lead_b))
        lead_a = [1] * (L - len(lead_a)) + lead_a
        lead_b = [1] * (L - len(lead_b)) + lead_b
        lead = [max(x, z) for x, z in zip(lead_a, lead_b)]
        y = self._alloc(Y.numel)
        # the broadcast leading dims: an outer loop over the dims where one side is 1
        # ahead of the innermost run of dims both sides share (nodes.py:632-660)
        total = int(np.prod(lead)) if lead else 1
        a_strides = np.cumprod([1] + lead_a[::-1])[::-1][1:] if L else []
        b_strides = np.cumprod([1] + lead_b[::-1])[::-1][1:] if L else []
        # innermost batch run: dims from the end where both agree (no broadcast)
        inner = 1
        d = L - 1
        while d >= 0 and lead_a[d] == lead_b[d]:
            inner *= lead[d]
            d -= 1
        a_bs = n * k if inner > 1 else 0
        b_bs = k * m if inner > 1 else 0
        if (len(bsh) == 2 and len(sn.inputs[1].shape) == 2 and getattr(B, "data", None) is not None and post is None
                and total == 1 and self._use_bplanes(n, k) and (a.data_ptr() % 16) == 0):
            ws = self._workspace(self._mm_ws(n, k, m, 1, 0, 0))
            ops.matmul_bplanes(a, self._planes(B.onnx_name, b, k, m), y, n=n, k=k, m=m, c_batch_stride=n * m,
                               flags=wrap | flag, workspace=ws)
            return y
        for o in range(total // inner):
            idx = np.unravel_index(o * inner, lead) if L else ()
            ao = sum((0 if lead_a[q] == 1 else int(idx[q])) * int(a_strides[q]) for q in range(L)) * n * k
            bo = sum((0 if lead_b[q] == 1 else int(idx[q])) * int(b_strides[q]) for q in range(L)) * k * m
            ws = self._workspace(self._mm_ws(n, k, m, inner, a_bs, b_bs))
            po = post
            if post is not None and post["b_mode"] == 1:  # a full operand: the slice at this output's offset
                po = dict(post, b=post["b"][o * inner * n * m:])
            ops.matmul(a[ao:], b[bo:], y[o * inner * n * m:], n=n, k=k, m=m, batch=inner, a_batch_stride=a_bs,
                       b_batch_stride=b_bs, c_batch_stride=n * m, flags=wrap | flag, workspace=ws, post=po)
        return y

    def _sibling_groups(self) -> Dict[int, list]:
        """MatMuls that read the same A with constant 2-D weights of the same K
        and run no fused job (a layer's q / k / v, its gate / up): runs of up to
        4, in graph order, all widths but a run's last multiples of 32, and
        n > 2 rows.  {first index: member indices}; each run is one
        corm_matmul_groups launch over the column-concatenated weights, at
        its first member (A and the weights exist there), every output the
        same as its own MatMul's."""
        nodes = self._graph.nodes
        fused_producers = {j for (j, _f, _p) in self._plan.values()}
        wnames = {t.onnx_name for t in self._graph.weight_tensors}
        by_a: Dict[tuple, list] = {}
        for i, sn in enumerate(nodes):
            if _kind(sn) != "MatmulNode" or i in fused_producers or len(sn.inputs) != 2:
                continue
            A, B, Y = sn.inputs[0], sn.inputs[1], sn.output
            if B.onnx_name not in wnames or getattr(B, "data", None) is None or len(B.shape) != 2 or len(A.shape) < 2:
                continue
            n, k = int(np.prod(A.shape[:-1])), int(A.shape[-1])
            if n <= 2 or k != int(B.shape[0]):
                continue
            by_a.setdefault((A.onnx_name, k, _has_exp(A, B, Y)), []).append(i)
        groups: Dict[int, list] = {}
        for idx in by_a.values():
            run: list = []
            for i in idx + [None]:
                if i is not None:
                    run.append(i)
                if i is None or int(nodes[i].inputs[1].shape[1]) % 32 or len(run) == 4:
                    if len(run) >= 2:
                        groups[run[0]] = list(run)
                    run = []
        return groups

    def _matmul_group(self, members, get):
        """One corm_matmul_groups launch for a run of sibling MatMuls: their
        outputs, in member order."""
        sns = [self._graph.nodes[j] for j in members]
        A = sns[0].inputs[0]
        n, k = int(np.prod(A.shape[:-1])), int(A.shape[-1])
        widths = [int(sn.inputs[1].shape[1]) for sn in sns]
        m = sum(widths)
        key = ("group",) + tuple(sn.inputs[1].onnx_name for sn in sns)
        if key not in self._weights:  # the weights side by side, once
            cat = self._alloc(k * m)
            cat[:k * m].view(k, m).copy_(torch.cat([get(sn.inputs[1])[:k * w].view(k, w)
                                                    for sn, w in zip(sns, widths)], dim=1))
            self._weights[key] = cat
        ys = [self._alloc(sn.output.numel) for sn in sns]
        wrap = F_WRAP32 if _has_exp(A, sns[0].inputs[1], sns[0].output) else 0
        ws = self._workspace(self._mm_ws(n, k, m, 1, 0, 0))
        if self._use_bplanes(n, k):
            ops.matmul_bplanes(get(A), self._planes(key, self._weights[key], k, m), None, n=n, k=k, m=m, flags=wrap,
                               workspace=ws, outs=ys, widths=widths)
        else:
            ops.matmul_groups(get(A), self._weights[key], ys, widths, n=n, k=k, flags=wrap, workspace=ws)
        return ys

    def _mulact_pairs(self) -> Dict[int, int]:
        """Sibling pairs (gate, up) whose two outputs only a SiluMulRoNode
        reads, with one broadcast parameter entry: {the pair's first index:
        the SiluMul index}.  The pair runs as one GEMM over the gate / up
        weights interleaved in 16-column blocks whose epilogue applies the
        MULACT (corm_matmul_groups with mulact)."""
        nodes, out = self._graph.nodes, {}
        readers: Dict[str, int] = {}
        for sn in nodes:
            for t in sn.inputs:
                if t is not None:
                    readers[t.onnx_name] = readers.get(t.onnx_name, 0) + 1
        for first, members in self._groups.items():
            if len(members) != 2:
                continue
            g, u = (nodes[j] for j in members)
            wg, wu = int(g.inputs[1].shape[1]), int(u.inputs[1].shape[1])
            A = g.inputs[0]
            n, k = int(np.prod(A.shape[:-1])), int(A.shape[-1])
            # few rows (a decode step): the pair GEMM has few tiles and each
            # epilogue thread would run all its row's MULACTs; the separate
            # row-ops job spreads them (measured 32.9 against 29.0 us a layer;
            # 8 layers of the decode step 0.97 against 0.91 ms)
            if wg != wu or wg % 16 or self._use_bplanes(n, k):
                continue
            for j in range(members[1] + 1, len(nodes)):
                sm = nodes[j]
                if _kind(sm) != "SiluMulRoNode":
                    continue
                if (sm.inputs[0].onnx_name == g.output.onnx_name and sm.inputs[1].onnx_name == u.output.onnx_name and
                        bool(getattr(sm, "bcast", False)) and readers.get(g.output.onnx_name) == 1 and
                        readers.get(u.output.onnx_name) == 1 and sm.n == wg):
                    out[first] = j
                break
        return out

    def _matmul_mulact(self, members, sm, get):
        """The gate / up pair and the SiluMul job of their outputs as one
        launch: the weights interleaved in 16-column blocks (gate block i,
        then up block i), once; the MULACT entry's shifts from its parameter
        words (byte 8 sa, byte 10 sc)."""
        sg, su = (self._graph.nodes[j] for j in members)
        A = sg.inputs[0]
        n, k = int(np.prod(A.shape[:-1])), int(A.shape[-1])
        ffn = int(sg.inputs[1].shape[1])
        key = ("mulact", sg.inputs[1].onnx_name, su.inputs[1].onnx_name)
        if key not in self._weights:
            wg = get(sg.inputs[1])[:k * ffn].view(k, ffn // 16, 16)
            wu = get(su.inputs[1])[:k * ffn].view(k, ffn // 16, 16)
            cat = self._alloc(2 * k * ffn)
            cat[:2 * k * ffn].view(k, ffn // 16, 2, 16).copy_(torch.stack([wg, wu], dim=2))
            self._weights[key] = cat
        pw = np.round(np.asarray(sm.inputs[2].data, np.float64).reshape(-1)[:8] * 256.0).astype(np.int16)
        words = pw.view(np.uint8)  # (host data: no device read, so the pass can be captured as a graph)
        sa, sc = int(words[8]) & 63, int(words[10]) & 63
        y = self._alloc(sm.output.numel)
        wrap = F_WRAP32 if _has_exp(A, sg.inputs[1], sg.output) else 0
        ws = self._workspace(self._mm_ws(n, k, 2 * ffn, 1, 0, 0))
        if self._use_bplanes(n, k):
            ops.matmul_bplanes(get(A), self._planes(key, self._weights[key], k, 2 * ffn), None, n=n, k=k, m=2 * ffn,
                               flags=wrap, workspace=ws, outs=[y], widths=[ffn], mulact=(sa, sc))
        else:
            ops.matmul_groups(get(A), self._weights[key], [y], [ffn], n=n, k=k, flags=wrap, workspace=ws,
                              mulact=(sa, sc))
        return y

    # few rows against a constant weight: the weight split into its planes once
    # (cached beside it) and only A split inside each job
    BPLANES_MAX_ROWS = 256

    @classmethod
    def _use_bplanes(cls, n, k) -> bool:
        return 2 < n <= cls.BPLANES_MAX_ROWS and k % 8 == 0

    def _planes(self, key, w, k, m):
        pk = ("planes",) + (key if isinstance(key, tuple) else (key,))
        if pk not in self._weights:
            self._weights[pk] = ops.split_b_planes(w, k=k, m=m)
        return self._weights[pk]

    @staticmethod
    def _mm_ws(n, k, m, batch, a_bs, b_bs) -> int:
        import ctypes as C

        from . import _lib
        d = _lib.MatmulDesc(0, 0, 0, n, k, m, batch, a_bs, b_bs, n * m, 0, 0, 0, None, 0)
        need = C.c_size_t(0)
        _lib.check(_lib.lib().corm_matmul_workspace_size(C.byref(d), C.byref(need)))
        return need.value

    def _conv(self, sn, x, w, b, flag, post=None):
        wrap = F_WRAP32 if _has_exp(sn.inputs[0], sn.inputs[1], sn.output) else 0
        y = self._alloc(sn.output.numel)
        regs = dict(batch=sn.batch, in_ch=sn.in_ch, in_h=sn.in_h, in_w=sn.in_w, out_ch=sn.out_ch, out_h=sn.out_h,
                    out_w=sn.out_w, kh=sn.kh, kw=sn.kw, stride_h=sn.stride_h, stride_w=sn.stride_w,
                    dilation_h=sn.dilation_h, dilation_w=sn.dilation_w, pad_top=sn.pad_top, pad_left=sn.pad_left,
                    has_bias=int(bool(sn.has_bias)), is_depthwise=int(bool(sn.is_depthwise)))
        need = self._conv_ws(regs, F_WEIGHT_LOGICAL | wrap | flag)
        ops.conv(x, w, b, y, flags=F_WEIGHT_LOGICAL | wrap | flag,
                 workspace=self._workspace(need) if need else None, post=post, **regs)
        return y

    @staticmethod
    def _conv_ws(regs, flags) -> int:
        """Bytes of scratch the library asks for the conv job (its split planes
        and K-split partial sums)."""
        import ctypes as C

        from . import _lib
        d = _lib.ConvDesc(0, 0, 0, 0, *(int(regs[k]) for k in (
            "batch", "in_ch", "in_h", "in_w", "out_ch", "out_h", "out_w", "kh", "kw", "stride_h", "stride_w",
            "dilation_h", "dilation_w", "pad_top", "pad_left", "has_bias", "is_depthwise")), 0, 0, 0, flags, None, 0)
        need = C.c_size_t(0)
        _lib.check(_lib.lib().corm_conv_workspace_size(C.byref(d), C.byref(need)))
        return need.value

    def _pool(self, sn, x):
        y = self._alloc(sn.output.numel)
        ops.pool(x, y, batch=sn.batch, channels=sn.channels, in_h=sn.in_h, in_w=sn.in_w, out_h=sn.out_h,
                 out_w=sn.out_w, pool_h=sn.pool_h, pool_w=sn.pool_w, stride_h=sn.stride_h, stride_w=sn.stride_w,
                 pad_top=sn.pad_top, pad_left=sn.pad_left, dil_h=sn.dil_h, dil_w=sn.dil_w, pool_type=sn.pool_type,
                 lp_order=sn.lp_order, count_include_pad=int(bool(sn.count_include_pad)))
        return y

    def _layernorm(self, sn, x, P):
        """One NORM job (rowops_nodes.py:238-242): eps register E, Bq' shifted by
        24 + g - bb; rows of n int16 at 2n-byte strides."""
        from . import rowops_host as RH
        y = self._alloc(sn.output.numel)
        ops.rowops(x, None, y, P, op=RH.opword(RH.OP_NORM, ln=True), n=sn.n, rows=sn.rows, blocks=1,
                   a_s1=2 * sn.n, c_s1=2 * sn.n, eps=int(sn.E), bq_sh=RH.P1_BITS + sn.g - sn.bb,
                   win_lo=0, win_hi=RH.NO_WINDOW)
        return y

    def _transpose(self, sn, x, pz):
        """The node's COPY (a zero P_BCAST entry) or TRANSPOSE (8-row tiles) job
        (rowops_nodes.py:309-316)."""
        from . import rowops_host as RH
        y = self._alloc(sn.output.numel)
        s1, s2, b1, b2, c1, c2 = sn.strides
        copy = sn.kind == "copy"
        op = RH.opword(RH.OP_COPY, p_bcast=True) if copy else RH.opword(RH.OP_XPOSE)
        ops.rowops(x, None, y, pz if copy else None, op=op, n=sn.n, rows=sn.rows, blocks=sn.blocks,
                   a_s1=s1, a_s2=s2, b_s1=b1, b_s2=b2, c_s1=c1, c_s2=c2, aux=0 if copy else RH.QIMAGE_R,
                   win_lo=0, win_hi=RH.NO_WINDOW, a_off=getattr(sn, "a_off", 0))
        return y

    def _llm_rowops(self, sn, kind, get):
        """The one row-ops job of an LLM row-ops node, with the registers its
        emit_call() issues (rowops_nodes.py:437-446, 492-497, 533-537,
        578-583); rows of n elements at their element widths."""
        from . import rowops_host as RH
        n, rows, bc = sn.n, sn.rows, bool(getattr(sn, "bcast", False))
        I16, I32 = RH.K_I16, RH.K_I32
        if kind == "ResAddRoNode":
            y = self._alloc32(sn.output.numel)
            ops.rowops(get(sn.inputs[0]), get(sn.inputs[1]), y, get(sn.inputs[2]),
                       op=RH.opword(RH.OP_ADDX, I32, I16, I32, b_en=True, p_bcast=bc), n=n, rows=rows,
                       a_s1=4 * n, b_s1=2 * n, c_s1=4 * n, win_hi=RH.NO_WINDOW)
        elif kind == "RMSNormRoNode":
            y = self._alloc(sn.output.numel)
            ops.rowops(get(sn.inputs[0]), None, y, get(sn.inputs[1]),
                       op=RH.opword(RH.OP_NORM, I32, I16, I16, p_bcast=bc), n=n, rows=rows, a_s1=4 * n,
                       c_s1=2 * n, eps=int(sn.E), win_hi=RH.NO_WINDOW)
        elif kind == "WidenRoNode":
            y = self._alloc32(sn.output.numel)
            ops.rowops(get(sn.inputs[0]), None, y, get(sn.inputs[1]),
                       op=RH.opword(RH.OP_COPY, I16, I16, I32, p_bcast=bc), n=n, rows=rows, a_s1=2 * n,
                       c_s1=4 * n, win_hi=RH.NO_WINDOW)
        else:  # SiluMulRoNode
            y = self._alloc(sn.output.numel)
            ops.rowops(get(sn.inputs[0]), get(sn.inputs[1]), y, get(sn.inputs[2]),
                       op=RH.opword(RH.OP_MULACT, I16, I16, I16, b_en=True, p_bcast=bc), n=n, rows=rows,
                       a_s1=2 * n, b_s1=2 * n, c_s1=2 * n, win_hi=RH.NO_WINDOW)
        return y

    def _rowops_pairs(self) -> Dict[int, int]:
        """ResAdd nodes followed at once by the RMSNorm of their sum (a Llama
        layer's two residual adds): {ResAdd index: RMSNorm index}.  The pair
        runs as a two-job descriptor chain, which the library executes in one
        pass over the rows (both outputs written)."""
        nodes, pairs = self._graph.nodes, {}
        for i in range(len(nodes) - 1):
            a, b = nodes[i], nodes[i + 1]
            if (_kind(a) == "ResAddRoNode" and _kind(b) == "RMSNormRoNode" and
                    b.inputs[0].onnx_name == a.output.onnx_name and a.n == b.n and a.rows == b.rows):
                pairs[i] = i + 1
        return pairs

    def _resadd_norm(self, sa, sb, get):
        """The ResAdd job and the RMSNorm job of its sum as one chain (the
        registers of ``_llm_rowops``); returns (the sum, the normed rows)."""
        from . import rowops_host as RH
        n, rows = sa.n, sa.rows
        I16, I32 = RH.K_I16, RH.K_I32
        h = self._alloc32(sa.output.numel)
        y = self._alloc(sb.output.numel)
        ops.rowops_chain([
            dict(a=get(sa.inputs[0]), b=get(sa.inputs[1]), c=h, p=get(sa.inputs[2]), n=n, rows=rows,
                 op=RH.opword(RH.OP_ADDX, I32, I16, I32, b_en=True, p_bcast=bool(getattr(sa, "bcast", False))),
                 a_s1=4 * n, b_s1=2 * n, c_s1=4 * n, win_hi=RH.NO_WINDOW),
            dict(a=h, c=y, p=get(sb.inputs[1]), n=n, rows=rows,
                 op=RH.opword(RH.OP_NORM, I32, I16, I16, p_bcast=bool(getattr(sb, "bcast", False))),
                 a_s1=4 * n, c_s1=2 * n, eps=int(sb.E), win_hi=RH.NO_WINDOW)])
        return h, y

    def _vit_gelu(self, sn, get):
        """VitGelu (vit_nodes.py:649-655): ADD f + ba, then MUL by sc with the
        GELU act, in place, rows runs of n with the [n] rows repeated."""
        y = self._alloc(sn.output.numel)
        geo = dict(size=sn.n, outer=sn.rows, a_inc=sn.n, b_inc=0)
        ops.vectorop(get(sn.inputs[0]), get(sn.inputs[1]), y, op=0, act=0, **geo)
        ops.vectorop(y, get(sn.inputs[2]), y, op=2, act=5 if getattr(sn, "erf", False) else 6, **geo)
        return y

    # ------------------------------------------------------------ prefill attention
    def _seen(self, t) -> bool:
        """Whether the pass returns tensor t (every tensor outside lean mode)."""
        obs = getattr(self, "_observed", None)
        return obs is None or t.onnx_name in obs

    @staticmethod
    def _host_int(get, t) -> int:
        return int(np.asarray(get(t)).reshape(-1)[0])

    def _keys(self, sn, get, i_pos: int):
        """(n, keys) of a runtime key count from the host inputs pos / n
        (llm_nodes.py:1409-1410; the C run function's llm_keys)."""
        from .attention import attn_keys
        pos = self._host_int(get, sn.inputs[i_pos])
        n = self._host_int(get, sn.inputs[i_pos + 1]) if sn.has_n else sn.T
        return (pos,) + attn_keys(pos, n, sn.T, sn.C, sn.Q)

    def _attn_prep(self, sn, get):
        """AttnPrepRoNode (rowops_nodes.py:985-1037, 1112-1143) for B
        sequences at one pos / n: ROPE jobs q0 -> qs and k0 -> ks over the rows
        t < n of every sequence (the cos / sin rows of pos + t), v re-rounded
        -> vs (a COPY job), then the cache rows [pos, pos + n) of the
        group-major states written in place and the q image qx[g][b][d][h' T
        + t] gathered (corm_copy_nd).  The staging rows are this pass's own,
        zeroed, so the image's columns t >= n are 0."""
        from . import rowops_host as RH
        from .attention import attn_keys
        if int(getattr(sn, "F", 8)) != 8:
            raise NotImplementedError("AttnPrepRoNode: F != 8")
        T, H, KV, HD, C = sn.T, sn.H, sn.KV, sn.HD, sn.C
        B = int(getattr(sn, "batch", 1))
        G = H // KV
        nq, nk = H * HD, KV * HD
        pos = self._host_int(get, sn.pos)
        n, _keys = attn_keys(pos, self._host_int(get, sn.n_t) if sn.has_n else T, T, C, sn.Q)
        qx = self._alloc(sn.output.numel)
        qs = self._alloc(B * T * nq)
        if n < T:  # rows t >= n of the image stay 0 (every row below n is written)
            qs.zero_()
        NW = RH.NO_WINDOW
        if n > 0:
            ks = self._alloc(B * T * nk)
            tab = get(sn.raw)
            I16, I32 = RH.K_I16, RH.K_I32
            rope = RH.opword(RH.OP_ROPE, I16, I32, I16, b_en=True)
            for src, dst, p_t, bc, w in ((get(sn.q0), qs, sn.pq, sn.pq_bc, nq), (get(sn.k0), ks, sn.pk, sn.pk_bc, nk)):
                ops.rowops(src, tab, dst, get(p_t), op=rope | (RH.F_P_BCAST if bc else 0), n=w, rows=n, blocks=B,
                           a_s1=2 * w, a_s2=2 * w * T, b_s1=8 * HD, c_s1=2 * w, c_s2=2 * w * T, aux=HD,
                           b_off=pos * 8 * HD, win_hi=NW)
            vsrc = get(sn.v)
            if not sn.v_direct:
                vs = self._alloc(B * T * nk)
                ops.rowops(vsrc, None, vs, get(sn.pvb), op=RH.opword(RH.OP_COPY, p_bcast=bool(sn.pv_bc)), n=nk,
                           rows=n, blocks=B, a_s1=2 * nk, a_s2=2 * nk * T, c_s1=2 * nk, c_s2=2 * nk * T, win_hi=NW)
                vsrc = vs
            for src, cache in ((ks, get(sn.ck)), (vsrc, get(sn.cv))):
                ops.copy_nd(src, cache, (KV, B, n, HD), (HD, T * nk, nk, 1), (B * C * HD, C * HD, HD, 1),
                            dst_off=pos * HD)
        GT = G * T
        if sn.output.onnx_name in getattr(self, "_tr", ()):  # [KV][B][G T][HD]: rows of HD as ROPE wrote them
            ops.copy_nd(qs, qx, (KV, B, G, T, HD), (G * HD, T * nq, HD, nq, 1), (B * GT * HD, GT * HD, T * HD, HD, 1))
            return qx
        ops.copy_nd(qs, qx, (KV, B, G, T, HD), (G * HD, T * nq, HD, nq, 1), (B * HD * GT, HD * GT, T, 1, GT))
        return qx

    def _attn_conv(self, sn, get):
        """q.K^T of every sequence of group g in one strided batch: the K
        cache rows [r0, r0 + keys) (group-major [KV][B][C][HD]) @ the
        sequence's q image [HD][G T] -> its G T columns of the scores [C][B G
        T], rows keys .. C 0; P.V: P rows [G T][keys] (row stride C) @ the V
        cache rows [0, keys).  The MatMul rule with the int32 wrap
        (llm_nodes.py:1407-1423)."""
        if int(getattr(sn, "F", 8)) != 8:
            raise NotImplementedError("LlmAttnConvNode: F != 8")
        T, HD, C, g = sn.T, sn.HD, sn.C, sn.group
        B = int(getattr(sn, "batch", 1))
        GT = (sn.H // sn.KV) * T
        keys = C if sn.static else self._keys(sn, get, 2)[2]
        w, x = get(sn.inputs[0]), get(sn.inputs[1])
        y = self._alloc(sn.output.numel)
        if sn.kind == "qk" and sn.output.onnx_name in getattr(self, "_tr", ()):
            # the scores transposed, [B G T][C]: per sequence the q image rows
            # [G T][HD] @ the K cache rows [0, keys) as B transposed
            self._ws = ops.gemm_strided(x[g * B * GT * HD:], w[g * B * C * HD:], y, n=GT, k=HD, m=keys, batch=B,
                                        lda=HD, ldb=HD, ldc=C, b_trans=True, a_batch_stride=GT * HD,
                                        b_batch_stride=C * HD, c_batch_stride=GT * C, flags=F_WRAP32,
                                        workspace=self._ws)
            return y
        if sn.kind == "qk":
            rows, r0 = (sn.nr, sn.r0) if sn.nr else (keys, 0)
            self._ws = ops.gemm_strided(w[(g * B * C + r0) * HD:], x[g * B * HD * GT:], y, n=rows, k=HD, m=GT, batch=B,
                             lda=HD, ldb=GT, ldc=B * GT, a_batch_stride=C * HD, b_batch_stride=HD * GT,
                             c_batch_stride=GT, flags=F_WRAP32, workspace=self._ws)
            if not sn.nr and keys < C and self._seen(sn.output):
                y[keys * B * GT:C * B * GT].zero_()
            return y
        self._ws = ops.gemm_strided(w, x[g * B * C * HD:], y, n=GT, k=keys, m=HD, batch=B, lda=C, ldb=HD, ldc=HD,
                                    a_batch_stride=GT * C, b_batch_stride=C * HD, c_batch_stride=GT * HD,
                                    flags=F_WRAP32, workspace=self._ws)
        return y

    def _attn_softmax(self, sn, get):
        """The column-mode softmax calls (smx_nodes.py:362-383) over s [C][B G
        T]: P rows at stride C over the first keys columns (the rest 0); the
        mask register valid0 = pos + 1, period T (causal; column b G T + h' T
        + t has t = column mod T) or one valid length.  One call for the whole
        group when its heads share the registers, else one per sequence and
        head."""
        T, G, C = sn.T, sn.G, sn.C
        B = int(getattr(sn, "batch", 1))
        GT = G * T
        pos, n, keys = self._keys(sn, get, 1)
        if sn.causal:
            mask = ((pos + 1) & 0xFFFF) | (T << 16)
        else:
            mask = max(min(keys, pos + n) - int(bool(sn.prefix_lm)), 1) & 0xFFFF
        s = get(sn.inputs[0])
        y = self._alloc(sn.output.numel)
        if keys < C and self._seen(sn.output):
            y.zero_()
        regs = [(int(sn.cm[h]), int(sn.cfg[h])) for h in range(G)]
        if sn.inputs[0].onnx_name in getattr(self, "_tr", ()):  # transposed scores: the same P by rows
            ops.vectorop(s, None, y, size=keys, op=10, outer=B * GT, a_inc=C, b_inc=C, smx_cm=regs[0][0],
                         smx_cfg=regs[0][1], smx_mask=mask)
            return y
        if all(r == regs[0] for r in regs):
            ops.vectorop(s, None, y, size=keys, op=11, outer=B * GT, a_inc=B * GT, b_inc=C, smx_cm=regs[0][0],
                         smx_cfg=regs[0][1], smx_mask=mask)
            return y
        for b in range(B):
            for h in range(G):
                ops.vectorop(s[b * GT + h * T:], None, y[(b * GT + h * T) * C:], size=keys, op=11, outer=T,
                             a_inc=B * GT, b_inc=C, smx_cm=regs[h][0], smx_cfg=regs[h][1], smx_mask=mask)
        return y

    def _attn_softmax_host(self, sn, get):
        """The host's p12 softmax on the device (corm_llm_attn_softmax): the
        float64 exp tables of the group's score exponents (built once on the
        host with libm, as the generated code's init does) and 2^f_p."""
        from .attention import sexp_table
        if not sn.causal:
            raise NotImplementedError("LlmAttnSoftmaxNode: causal = 0 / 2 run on the softmax unit only")
        B = int(getattr(sn, "batch", 1))
        fs = tuple(int(v) for v in np.asarray(sn.fs).reshape(-1))
        fp = tuple(int(v) for v in np.asarray(sn.fp).reshape(-1))
        key = ("sexp", fs, fp, float(sn.scale))
        if key not in self._weights:
            tab = np.concatenate([sexp_table(f, float(sn.scale)) for f in fs])
            self._weights[key] = (torch.from_numpy(tab).to(self.device),
                                  torch.tensor([2.0 ** f for f in fp], dtype=torch.float64, device=self.device))
        tab, ip = self._weights[key]
        pos = self._host_int(get, sn.inputs[1])
        n = self._host_int(get, sn.inputs[2]) if sn.has_n else sn.T
        y = self._alloc(sn.output.numel)
        ops.llm_attn_softmax(get(sn.inputs[0]), y, tab, ip, pos=pos, n=max(n, 0), T=sn.T, G=sn.G, rows=sn.C, Q=sn.Q,
                             window=int(getattr(sn, "window", 0)), batch=B)
        return y

    def _attn_transpose_plan(self, keep) -> set:
        """Names of the prefill attention tensors held transposed in a lean
        pass: a q image qx [KV][B][HD][G T] as [KV][B][G T][HD] (the ROPE
        rows copied without a transposition) when every reader of it is a
        q.K^T over all its keys (no row pieces, not static) and nobody
        observes it; those q.K^T's scores [C][B G T] as [B G T][C] when their
        one reader is the unit's column softmax with the same registers for
        every head, which then runs in row mode (the same P: a column of the
        scores is a row of their transpose)."""
        key = frozenset(keep)
        cache = self.__dict__.setdefault("_tr_plans", {})
        if key in cache:
            return cache[key]
        nodes = self._graph.nodes
        readers: Dict[str, list] = {}
        for i, sn in enumerate(nodes):
            for t in sn.inputs:
                if t is not None:
                    readers.setdefault(t.onnx_name, []).append(i)
        out = set()
        for sn in nodes:
            if _kind(sn) != "AttnPrepRoNode" or sn.output.onnx_name in key:
                continue
            qn = sn.output.onnx_name
            convs = [nodes[i] for i in readers.get(qn, [])]
            ok = bool(convs)
            scores = []
            for cn in convs:
                if (_kind(cn) != "LlmAttnConvNode" or cn.kind != "qk" or cn.static or cn.nr or
                        cn.inputs[1].onnx_name != qn or cn.output.onnx_name in key):
                    ok = False
                    break
                rs = [nodes[i] for i in readers.get(cn.output.onnx_name, [])]
                if (len(rs) != 1 or _kind(rs[0]) != "LlmAttnSoftmaxVopNode" or
                        len({(int(c), int(f)) for c, f in zip(rs[0].cm, rs[0].cfg)}) != 1):
                    ok = False
                    break
                scores.append(cn.output.onnx_name)
            if ok:
                out.add(qn)
                out.update(scores)
        cache[key] = out
        return out

    def _decode_attn_plan(self, keep) -> dict:
        """{merge node index: plan} for the decode steps' attention blocks whose
        intermediates nobody observes: per KV group a q.K^T (T = 1, no n, all
        keys), the host softmax and the P.V, merged — run as one
        corm_llm_decode_attn launch at the merge."""
        key = frozenset(keep)
        cache = self.__dict__.setdefault("_attn_plans", {})
        if key in cache:
            return cache[key]
        nodes = self._graph.nodes
        producer = {sn.output.onnx_name: i for i, sn in enumerate(nodes)}
        readers: Dict[str, int] = {}
        for sn in nodes:
            for t in sn.inputs:
                if t is not None:
                    readers[t.onnx_name] = readers.get(t.onnx_name, 0) + 1
        plans = {}
        for mi, mn in enumerate(nodes):
            if _kind(mn) != "LlmAttnMergeNode" or int(getattr(mn, "R", 1)) != 1 or mn.T != 1:
                continue
            idx, qks, smxs, pvs, ok = [], [], [], [], True
            for g, o in enumerate(mn.inputs):
                pi = producer.get(o.onnx_name)
                pv = nodes[pi] if pi is not None else None
                if pv is None or _kind(pv) != "LlmAttnConvNode" or pv.kind != "pv" or pv.group != g:
                    ok = False
                    break
                si = producer.get(pv.inputs[0].onnx_name)
                sm = nodes[si] if si is not None else None
                if sm is None or _kind(sm) != "LlmAttnSoftmaxNode" or sm.group != g or not sm.causal:
                    ok = False
                    break
                qi = producer.get(sm.inputs[0].onnx_name)
                qk = nodes[qi] if qi is not None else None
                if qk is None or _kind(qk) != "LlmAttnConvNode" or qk.kind != "qk" or qk.group != g or qk.nr:
                    ok = False
                    break
                for nd in (qk, sm, pv):
                    if nd.T != 1 or getattr(nd, "has_n", True) or getattr(nd, "static", False) or \
                            nd.output.onnx_name in keep or readers.get(nd.output.onnx_name, 0) != 1:
                        ok = False
                if qks and (qk.inputs[1].onnx_name != qks[0].inputs[1].onnx_name or
                            qk.inputs[0].onnx_name != qks[0].inputs[0].onnx_name or
                            pv.inputs[1].onnx_name != pvs[0].inputs[1].onnx_name or
                            sm.window != smxs[0].window or sm.scale != smxs[0].scale):
                    ok = False
                idx += [qi, si, pi]
                qks.append(qk)
                smxs.append(sm)
                pvs.append(pv)
            if ok and qks and len(qks) == mn.KV:
                plan = {"nodes": idx, "qk": qks, "smx": smxs, "pv": pvs}
                # the step's AttnPrep too, when its q image feeds only this block
                qx = qks[0].inputs[1].onnx_name
                ri = producer.get(qx)
                pr = nodes[ri] if ri is not None else None
                if pr is not None and _kind(pr) == "AttnPrepRoNode" and pr.T == 1 and not pr.has_n and \
                        int(getattr(pr, "batch", 1)) == int(getattr(smxs[0], "batch", 1)) and qx not in keep and \
                        readers.get(qx, 0) == len(qks) and pr.ck.onnx_name == qks[0].inputs[0].onnx_name and \
                        pr.cv.onnx_name == pvs[0].inputs[1].onnx_name and pr.HD % 16 == 0:
                    plan["prep"] = pr
                    plan["nodes"] = idx + [ri]
                plans[mi] = plan
        cache[key] = plans
        return plans

    def _decode_attn(self, mn, plan, get):
        """The fused decode attention (corm_llm_decode_attn) of a plan: the
        exp tables of every head's score exponent, 2^f_p per head."""
        from .attention import sexp_table
        qk0, sm0 = plan["qk"][0], plan["smx"][0]
        G, B = sm0.G, int(getattr(sm0, "batch", 1))
        fs = tuple(int(v) for sm in plan["smx"] for v in np.asarray(sm.fs).reshape(-1))
        fp = tuple(int(v) for sm in plan["smx"] for v in np.asarray(sm.fp).reshape(-1))
        key = ("sexp", fs, fp, float(sm0.scale))
        if key not in self._weights:
            tab = np.concatenate([sexp_table(f, float(sm0.scale)) for f in fs])
            self._weights[key] = (torch.from_numpy(tab).to(self.device),
                                  torch.tensor([2.0 ** f for f in fp], dtype=torch.float64, device=self.device))
        tab, ip = self._weights[key]
        pos = self._host_int(get, qk0.inputs[2])
        y = self._alloc(mn.output.numel)
        prep, qx = None, None
        pr = plan.get("prep")
        if pr is not None:
            prep = dict(q0=get(pr.q0), k0=get(pr.k0), v0=get(pr.v), ldq=pr.H * pr.HD, ldk=pr.KV * pr.HD,
                        ldv=pr.KV * pr.HD, rope=get(pr.raw), pq=get(pr.pq), pk=get(pr.pk),
                        pv=None if pr.v_direct else get(pr.pvb), pq_bc=pr.pq_bc, pk_bc=pr.pk_bc, pv_bc=pr.pv_bc,
                        v_direct=pr.v_direct)
        else:
            qx = get(qk0.inputs[1])
        ops.llm_decode_attn(qx, get(qk0.inputs[0]), get(plan["pv"][0].inputs[1]), tab, ip, y, pos=pos, B=B, KV=mn.KV,
                            G=G, HD=mn.HD, rows=qk0.C, Q=qk0.Q, window=int(getattr(sm0, "window", 0)),
                            o_stride=mn.H * mn.HD, prep=prep)
        return y

    def _attn_merge(self, sn, get):
        """o_g -> pv in head order (llm_nodes.py:1645-1657): one strided copy
        per input, pv[b][t][(g G + h') HD + d] = o_g[b][h'][t][d]."""
        T, H, KV, HD = sn.T, sn.H, sn.KV, sn.HD
        R = int(getattr(sn, "R", 1))
        B = int(getattr(sn, "batch", 1))
        G = H // KV
        nq = H * HD
        y = self._alloc(sn.output.numel)
        if R > 1:
            if B != 1:
                raise NotImplementedError("LlmAttnMergeNode: row splits of a batch")
            rows = T // R
            for i, t in enumerate(sn.inputs):
                g, r = divmod(i, R)
                ops.copy_nd(get(t), y, (rows, HD), (HD, 1), (nq, 1), dst_off=r * rows * nq + g * HD)
            return y
        for g, t in enumerate(sn.inputs):
            ops.copy_nd(get(t), y, (B, G, T, HD), (G * T * HD, T * HD, HD, 1), (T * nq, HD, nq, 1), dst_off=g * G * HD)
        return y

    def _exps8(self, key, e) -> torch.Tensor:
        """An exponent vector as a cached int8 device tensor."""
        k = ("exps8", key, tuple(int(x) for x in e))
        if k not in self._weights:
            a = np.asarray(e, np.int64)
            if (a < -127).any() or (a > 127).any():
                raise NotImplementedError("exponent outside the int8 range")
            self._weights[k] = torch.from_numpy(a.astype(np.int8)).to(self.device)
        return self._weights[k]

    def _llm_host(self, sn, kind, get):
        """The float host ops of the LLM entries on the device (llm_host.cu):
        LlmEmbed, LlmDequant, LlmToHost, LlmResAdd, LlmRMSNorm, LlmSiluMul /
        LlmGeluMul (llm_nodes.py:466-791, 1722-1777)."""
        from .attention import act_table
        out_t = sn.output
        N = out_t.numel
        if kind == "LlmEmbedNode":
            if int(getattr(sn, "image_rows", 0)):
                raise NotImplementedError("LlmEmbedNode: image rows")
            tb = sn.table
            res32 = bool(sn.res32)
            f = 0
            if res32:
                fo = _chan(out_t, sn.d)
                if (fo != fo[0]).any():
                    raise NotImplementedError("LlmEmbedNode: the residual at per-channel exponents")
                f = int(fo[0])
            key = ("embed", tb.name, tb.kind)
            if key not in self._weights:
                data = np.asarray(tb.data)
                vals = (data.astype(np.float64) / 2.0 ** f) if tb.kind == "i16" else data
                self._weights[key] = torch.from_numpy(np.asarray(vals, np.float32).reshape(-1).copy()).to(self.device)
            ids = torch.from_numpy(np.asarray(get(sn.inputs[0])).astype(np.int32).reshape(-1)).to(self.device)
            y = self._alloc32(N) if res32 else self._alloc_f32(N)
            ops.llm_embed(ids, self._weights[key], y, n=sn.n, rows=sn.rows, d=sn.d, res32=res32, f=f,
                          scale=float(getattr(sn, "scale", 1.0)))
            return y
        if kind == "LlmDequantNode":
            x = sn.inputs[0]
            n = int(x.shape[-1])
            y = self._alloc_f32(N)
            ops.llm_dequant(get(x), y, self._exps8(x.onnx_name, _chan(x, n)), count=sn.count, n=n)
            return y
        if kind == "LlmToHostNode":
            src = get(sn.inputs[0])
            y = self._alloc_f32(N)
            ops.copy_nd(src.view(torch.int16), y.view(torch.int16), (2 * N,), (1,), (1,))
            return y
        if kind == "LlmResAddNode":
            d_t = sn.inputs[1]
            y = self._alloc_f32(N)
            ops.llm_resadd(get(sn.inputs[0]), get(d_t), y, self._exps8(d_t.onnx_name, _chan(d_t, sn.n)), rows=sn.rows,
                           n=sn.n)
            return y
        if kind == "LlmRMSNormNode":
            h_t = sn.inputs[0]
            W = int(getattr(sn, "W", sn.n))
            gk = ("gamma", out_t.onnx_name)
            if gk not in self._weights:
                self._weights[gk] = torch.from_numpy(np.asarray(sn.gamma, np.float32).reshape(-1).copy()).to(self.device)
            y = self._alloc(N)
            fy = self._exps8(out_t.onnx_name, _chan(out_t, W))
            fh = None if _is_f32(h_t) else self._exps8(h_t.onnx_name, _chan(h_t, W))
            ops.llm_rmsnorm(get(h_t), y, self._weights[gk], fy, rows=sn.rows, n=sn.n, W=W, eps=float(sn.eps), fh=fh)
            return y
        # LlmSiluMulNode / LlmGeluMulNode
        g_t, u_t = sn.inputs[0], sn.inputs[1]
        fg = _chan(g_t, sn.n)
        act = "gelu" if kind == "LlmGeluMulNode" else "silu"
        uniq = sorted(set(int(v) for v in fg))
        tk = ("acttab", act, tuple(uniq))
        if tk not in self._weights:
            self._weights[tk] = torch.from_numpy(np.concatenate([act_table(act, f) for f in uniq])).to(self.device)
        ok = ("acttab_of", act, tuple(int(v) for v in fg))
        if ok not in self._weights:
            self._weights[ok] = torch.from_numpy(np.array([uniq.index(int(v)) for v in fg], np.uint8)).to(self.device)
        y = self._alloc(N)
        ops.llm_act_mul(get(g_t), get(u_t), y, self._weights[tk], self._weights[ok],
                        self._exps8(u_t.onnx_name, _chan(u_t, sn.n)), self._exps8(out_t.onnx_name, _chan(out_t, sn.n)),
                        rows=sn.rows, n=sn.n)
        return y

    def _attn_prep_host(self, sn, get):
        """LlmAttnPrep's host form (llm_nodes.py:1012-1169) for B sequences:
        the K / V cache rows pos + t (t < n) of the group-major states written in
        place and the q image qx[g][b][d][h' T + t] (corm_llm_attn_prep_host)."""
        from .attention import attn_keys
        T, H, KV, HD, C = sn.T, sn.H, sn.KV, sn.HD, sn.C
        B = int(getattr(sn, "batch", 1))
        if int(getattr(sn, "kw", 1)) != 1:
            raise NotImplementedError("LlmAttnPrepNode: a q image for qk_kw > 1")
        q0, k0, v = sn.inputs[0], sn.inputs[1], sn.inputs[2]
        pos = self._host_int(get, sn.inputs[3])
        n_in = self._host_int(get, sn.inputs[4]) if sn.has_n else T
        n, _keys = attn_keys(pos, n_in, T, C, sn.Q)
        ck, cv = sn.inputs[-2], sn.inputs[-1]
        tk = ("rope_f32", id(sn.cos), id(sn.sin))
        if tk not in self._weights:
            self._weights[tk] = (torch.from_numpy(np.asarray(sn.cos, np.float32).reshape(-1).copy()).to(self.device),
                                 torch.from_numpy(np.asarray(sn.sin, np.float32).reshape(-1).copy()).to(self.device))
        cos_t, sin_t = self._weights[tk]
        qx = self._alloc(sn.output.numel)
        e = lambda t, w: self._exps8(t.onnx_name, _chan(t, w))  # noqa: E731
        ops.llm_attn_prep_host(get(q0), get(k0), get(v), get(ck), get(cv), qx, cos_t, sin_t, e(q0, H * HD),
                               e(k0, KV * HD), e(v, KV * HD), e(ck, KV * HD), e(cv, KV * HD),
                               self._exps8(("fq", sn.output.onnx_name), np.asarray(sn.fq, np.int64)),
                               pos=pos, n=n, T=T, H=H, KV=KV, HD=HD, C_=C, Q=sn.Q, batch=B)
        return qx

    def _select_row(self, sn, get):
        """h[n - 1], n clamped to [1, rows] (llm_nodes.py:1713-1717), of every
        sequence: one strided copy (an int32 row as int16 halves)."""
        B = int(getattr(sn, "batch", 1))
        r = min(max(self._host_int(get, sn.inputs[1]), 1), sn.rows) - 1
        wide = 2 if (sn.res32 or getattr(sn.output, "dma", None) == "i32") else 1
        y = self._alloc32(B * sn.n) if wide == 2 else self._alloc(B * sn.n)
        w = sn.n * wide
        ops.copy_nd(get(sn.inputs[0]).view(torch.int16), y.view(torch.int16), (B, w), (sn.rows * w, 1), (w, 1),
                    src_off=r * w)
        return y

    def _tiled_weight(self, t, size: int) -> torch.Tensor:
        """A small broadcast weight repeated to ``size`` elements: the same
        elementwise job with longer rows (a scalar would give rows of one)."""
        key = ("tiled", t.onnx_name, size)
        if key not in self._weights:
            w = self._weight_raw(t)[:t.numel]
            buf = self._alloc(size)
            buf[:size].copy_(w.repeat(size // t.numel))
            self._weights[key] = buf
        return self._weights[key]

    def _vectorop(self, sn, get):
        """The node's kernel call(s): one operand may be a repeating chunk
        (nodes.py:226-305 trailing-contiguous broadcast): outer = numel /
        chunk, that operand's stride 0."""
        op = sn.op_code
        out_t = sn.output
        N = out_t.numel
        y = self._alloc(N)
        a_t = sn.inputs[0]
        a = get(a_t)
        act, alpha = getattr(sn, "act", 0), getattr(sn, "alpha", 0)
        if op > 3:
            ops.vectorop(a, None, y, size=N, op=op, outer=1, act=act, alpha=alpha)
            return y
        b_t = sn.inputs[1]
        b = get(b_t)
        na, nb = a_t.numel, b_t.numel
        if na == N and nb == N:
            ops.vectorop(a, b, y, size=N, op=op, outer=1, act=act, alpha=alpha)
            return y
        if na != N and nb != N:
            raise NotImplementedError("VectorOP: both operands broadcast")
        size = nb if nb != N else na
        small_t = b_t if nb != N else a_t
        if size < 1024 and getattr(small_t, "data", None) is not None:
            r = 1
            while size * r * 2 <= 2048 and N % (size * r * 2) == 0:
                r *= 2
            if r > 1:
                size *= r
                if nb != N:
                    b = self._tiled_weight(b_t, size)
                else:
                    a = self._tiled_weight(a_t, size)
        outer = N // size
        a_inc, b_inc = (size, 0) if nb != N else (0, size)
        # rows need not be on 8-lane words: the kernel writes a row's tail lanes
        # only where the next row's data does not land (the hardware's order)
        ops.vectorop(a, b, y, size=size, op=op, outer=outer, a_inc=a_inc, b_inc=b_inc, act=act, alpha=alpha)
        return y
