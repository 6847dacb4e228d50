"""Op descriptors of the simulator's graph, field-compatible with the
reference's node layer (phoenix367/cormorant inference-scheduler/src/nodes.py,
tensor.py, smx_nodes.py): ``GpuSimulator`` reads only these attribute names,
so it accepts either these dataclasses or the reference's own node objects
(``ScheduledNode``, ``MatmulNode``, ``MatmulConvNode``, ``ConvNode``,
``PoolNode``, ``ReshapeNode``, ``SpaceToDepthNode``, ``SoftmaxVopNode``)
unchanged.

Op / act codes are the kernel register values (nodes.py:88-164).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_RELU, OP_RELU6 = range(6)
OP_LEAKY_RELU, OP_SILU, OP_GELU, OP_GELU_TANH, OP_SOFTMAX, OP_SOFTMAX_T = range(6, 12)
ACT_NONE, ACT_RELU, ACT_RELU6, ACT_LEAKY_RELU, ACT_SILU, ACT_GELU, ACT_GELU_TANH = range(7)
POOL_MAX, POOL_AVG, POOL_LP = 0, 1, 2


@dataclass
class TensorInfo:
    """tensor.py:49-120: logical shape, optional weight data (values), and the
    power-of-two exponent metadata (exp per tensor / channel, chexp per
    channel on axis 1, wexp the rank-1 weight exponent)."""
    onnx_name: str
    shape: List[int]
    dtype: str = "float32"
    data: Optional[np.ndarray] = field(default=None, repr=False)
    exp: Optional[np.ndarray] = field(default=None, repr=False)
    chexp: Optional[np.ndarray] = field(default=None, repr=False)
    wexp: Optional[np.ndarray] = field(default=None, repr=False)
    is_state: bool = False
    init_data: Optional[np.ndarray] = field(default=None, repr=False)
    dma: Optional[str] = None  # "i32": an int32 DMA tensor at ``exp`` (the LLM residual stream)
    host: Optional[str] = None  # "i32": a host-memory int32 input (a position, a row count)
    # (G, D): a state of logical shape [R][G*D] stored group-major [G][R][D] (a KV
    # cache, every KV head's rows contiguous); group_kw > 1 is the board's row
    # interleave of the V cache, which the B200 layout does not need (tensor.py:99-111)
    group_layout: Optional[tuple] = None
    group_kw: int = 1

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def is_host(self) -> bool:
        return self.host is not None


@dataclass
class ScheduledNode:
    """VectorOPKernel node (nodes.py:311-598): op_code, fused act / alpha."""
    op_code: int
    inputs: List[TensorInfo]
    output: TensorInfo
    act: int = ACT_NONE
    alpha: int = 0
    onnx_node: object = None


@dataclass
class MatmulNode:
    """MatmulKernel node (nodes.py:632-1109): logical A [.., n, k] @ B [.., k, m]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    n: int = 0
    k: int = 0
    m: int = 0
    batch: int = 1
    onnx_node: object = None


@dataclass
class ConvNode:
    """ConvKernel node (nodes.py:1154-1590): NCHW x, logical weight
    [M][C or 1][kh][kw], bias [M]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    batch: int = 1
    in_ch: int = 0
    in_h: int = 0
    in_w: int = 0
    out_ch: int = 0
    out_h: int = 0
    out_w: int = 0
    kh: int = 1
    kw: int = 1
    stride_h: int = 1
    stride_w: int = 1
    dilation_h: int = 1
    dilation_w: int = 1
    pad_top: int = 0
    pad_left: int = 0
    has_bias: bool = False
    is_depthwise: bool = False
    onnx_node: object = None


@dataclass
class PoolNode:
    """PoolingKernel node (nodes.py:1800-2141)."""
    inputs: List[TensorInfo]
    output: TensorInfo
    batch: int = 1
    channels: int = 0
    in_h: int = 0
    in_w: int = 0
    out_h: int = 0
    out_w: int = 0
    pool_h: int = 1
    pool_w: int = 1
    stride_h: int = 1
    stride_w: int = 1
    pad_top: int = 0
    pad_left: int = 0
    dil_h: int = 1
    dil_w: int = 1
    pool_type: int = POOL_MAX
    lp_order: int = 0
    count_include_pad: int = 0
    onnx_node: object = None


@dataclass
class ReshapeNode:
    """Pure view (nodes.py:2144)."""
    inputs: List[TensorInfo]
    output: TensorInfo
    onnx_node: object = None


@dataclass
class SpaceToDepthNode:
    """ONNX SpaceToDepth channel order (nodes.py:2267; _simulate.py:692-699)."""
    inputs: List[TensorInfo]
    output: TensorInfo
    blocksize: int = 2
    batch: int = 1
    in_ch: int = 0
    in_h: int = 0
    in_w: int = 0
    onnx_node: object = None


@dataclass
class SoftmaxVopNode:
    """Softmax on VectorOPKernel's unit, row mode, Q8.8 in and out
    (smx_nodes.py:121-134): rows x n, registers cm and cfg = Cs | f_p << 8."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    cm: int = 0
    cfg: int = 0
    F: int = 8
    onnx_node: object = None


@dataclass
class LayerNormRoNode:
    """LayerNorm on the row-ops unit, Q8.8 in and out (rowops_nodes.py:162-220):
    rows x n, NORM with NORM_LN; inputs [x, P (parameter words as Q8.8
    values), tables]; eps register E, gamma at 2^-g, Bq' at 2^-bb."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    eps: float = 1e-5
    g: int = 0
    bb: int = 20
    E: int = 0
    gamma: Optional[np.ndarray] = field(default=None, repr=False)
    beta: Optional[np.ndarray] = field(default=None, repr=False)
    F: int = 8
    onnx_node: object = None


@dataclass
class TransposeRoNode:
    """Transpose of an int16 tensor as one row-ops job (rowops_nodes.py:265-316):
    kind "copy" (rows kept: COPY with a zero P_BCAST entry) or "xpose" (K^T:
    TRANSPOSE of 8-row tiles); strides in bytes (a_s1, a_s2, b_s1, b_s2, c_s1,
    c_s2); inputs [x, zero P, tables]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    kind: str = "copy"
    n: int = 0
    rows: int = 0
    blocks: int = 1
    a_off: int = 0
    strides: tuple = (0, 0, 0, 0, 0, 0)
    perm: list = field(default_factory=list)
    onnx_node: object = None


@dataclass
class ResAddRoNode:
    """LlmResAdd on the row-ops unit (rowops_nodes.py:400-446): h1 = sat32(h +
    d << (fr - f_d)), h / h1 int32 DMA tensors at 2^-fr, d int16 at its
    per-channel exponents; one ADDX job.  inputs [h, d, P]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    fr: int = 15
    bcast: bool = True
    F: int = 8
    onnx_node: object = None


@dataclass
class RMSNormRoNode:
    """LlmRMSNorm on the row-ops unit (rowops_nodes.py:449-497): the int32
    residual at 2^-fr -> int16 at the output's per-channel exponents, NORM
    (rms); inputs [h, P]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    fr: int = 15
    eps: float = 1e-5
    g: int = 0
    E: int = 0
    bcast: bool = False
    gamma: Optional[np.ndarray] = field(default=None, repr=False)
    F: int = 8
    onnx_node: object = None


@dataclass
class WidenRoNode:
    """LlmWiden on the row-ops unit (rowops_nodes.py:500-537): int16 at
    per-channel exponents -> the int32 DMA tensor at one exponent, COPY;
    inputs [x, P]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    bcast: bool = True
    F: int = 8
    onnx_node: object = None


@dataclass
class SiluMulRoNode:
    """LlmSiluMul on the row-ops unit (rowops_nodes.py:540-583): a = silu(g) *
    u, MULACT; inputs [g, u, P]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    bcast: bool = False
    F: int = 8
    onnx_node: object = None


@dataclass
class VitGeluVopNode:
    """VitGelu on VectorOPKernel (vit_nodes.py:580-668): ADD f + ba, then MUL
    by sc with act GELU (erf) / GELU_TANH, rows runs of n with the [n]
    operands repeated; inputs [f, ba, sc] (ba / sc constant raw rows),
    output at 2^-8."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    F: int = 8
    erf: bool = False
    onnx_node: object = None


@dataclass
class AttnPrepRoNode:
    """LlmAttnPrep of a prefill on the row-ops unit (rowops_nodes.py:893-1145):
    RoPE of q0 / k0 (cos / sin rows of positions pos + t from the ``raw``
    table, B offset pos 8 HD), v re-rounded to the V cache's exponents, the
    q.K^T image qx [KV][HD][G T] (TRANSPOSE of 8-row tiles), and the rows
    [pos, pos + n) of both caches (group-major states, written in place).
    inputs = [q0, k0, v, pos, (n), ck, cv, qs, ks, (vs), raw, pq, pk, (pvb),
    pz, tables]; the named fields point into them.

    ``batch`` B > 1 (no counterpart in the reference, whose entries run one
    sequence): B sequences at the same pos / n, stacked — q0 / k0 / v
    [B T][..], the caches [B C][KV HD] (stored [KV][B][C][HD]), qx
    [KV][B][HD][G T]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    T: int = 1
    H: int = 1
    KV: int = 1
    HD: int = 16
    C: int = 16
    Q: int = 16
    K: int = 1
    first: bool = False
    has_n: bool = True
    v_direct: bool = False
    pq_bc: bool = False
    pk_bc: bool = False
    pv_bc: bool = True
    fq: Optional[np.ndarray] = field(default=None, repr=False)
    cos: Optional[np.ndarray] = field(default=None, repr=False)
    sin: Optional[np.ndarray] = field(default=None, repr=False)
    q0: Optional[TensorInfo] = field(default=None, repr=False)
    k0: Optional[TensorInfo] = field(default=None, repr=False)
    v: Optional[TensorInfo] = field(default=None, repr=False)
    pos: Optional[TensorInfo] = field(default=None, repr=False)
    n_t: Optional[TensorInfo] = field(default=None, repr=False)
    ck: Optional[TensorInfo] = field(default=None, repr=False)
    cv: Optional[TensorInfo] = field(default=None, repr=False)
    qs: Optional[TensorInfo] = field(default=None, repr=False)
    ks: Optional[TensorInfo] = field(default=None, repr=False)
    vs: Optional[TensorInfo] = field(default=None, repr=False)
    raw: Optional[TensorInfo] = field(default=None, repr=False)
    pq: Optional[TensorInfo] = field(default=None, repr=False)
    pk: Optional[TensorInfo] = field(default=None, repr=False)
    pvb: Optional[TensorInfo] = field(default=None, repr=False)
    pz: Optional[TensorInfo] = field(default=None, repr=False)
    F: int = 8
    batch: int = 1
    onnx_node: object = None

    @property
    def G(self) -> int:
        return self.H // self.KV


@dataclass
class LlmAttnConvNode:
    """One q.K^T (``kind`` "qk") or P.V ("pv") call of KV group ``group``
    (llm_nodes.py:1183-1423) over keys = roundup(pos + n, Q) — a runtime
    count from the host inputs pos / n — or keys = C (``static``; a static
    q.K^T over the cache rows r0 .. r0 + nr - 1 when nr > 0): raw int16
    operands, the int32 sum wraps, floor / 2^8, saturated.  inputs = [weight,
    x, pos, (n)] or [weight, x].  ``batch`` B: B sequences side by side —
    scores [C][B G T] (sequence b's columns at b G T), P [B G T][C], o
    [B G T][HD]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    kind: str = "qk"
    group: int = 0
    T: int = 1
    H: int = 1
    KV: int = 1
    HD: int = 16
    C: int = 16
    Q: int = 16
    F: int = 8
    static: bool = False
    has_n: bool = True
    r0: int = 0
    nr: int = 0
    batch: int = 1
    onnx_node: object = None

    @property
    def G(self) -> int:
        return self.H // self.KV


@dataclass
class LlmAttnSoftmaxVopNode:
    """The prefill softmax of KV group ``group`` on VectorOP's unit, column
    mode (smx_nodes.py:284-340): per head h' < G one call over s [C][G T]
    (columns h' T ..) -> P rows h' T .. over keys = roundup(pos + n, Q), row
    t valid over j < min(keys, pos + 1 + t) (``causal``), else every row over
    j < max(min(keys, pos + n) - prefix_lm, 1); registers cm[h'], cfg[h'].
    inputs = [s, pos, (n)]; ``batch`` B: s [C][B G T] -> P [B G T][C]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    T: int = 1
    G: int = 1
    C: int = 16
    Q: int = 16
    group: int = 0
    has_n: bool = True
    causal: bool = True
    prefix_lm: bool = False
    cm: List[int] = field(default_factory=list)
    cfg: List[int] = field(default_factory=list)
    F: int = 8
    batch: int = 1
    onnx_node: object = None


@dataclass
class LlmAttnSoftmaxNode:
    """The host's p12 softmax of KV group ``group`` (llm_nodes.py:1426-1557; a
    decode step's, or a prefill's without the softmax unit): s [C][G T] ->
    P [G T][C], rows t < n over keys j <= pos + t (window W: j > pos + t -
    W), exp tables of the score exponents fs[h'] at ``scale``, P at fp[h'].
    inputs = [s, pos, (n)]; ``batch`` B: s [C][B G T] -> P [B G T][C]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    T: int = 1
    G: int = 1
    C: int = 16
    Q: int = 16
    group: int = 0
    scale: float = 1.0
    fs: Optional[np.ndarray] = field(default=None, repr=False)
    fp: Optional[np.ndarray] = field(default=None, repr=False)
    has_n: bool = True
    causal: bool = True
    prefix_lm: bool = False
    window: int = 0
    F: int = 8
    batch: int = 1
    onnx_node: object = None


@dataclass
class LlmAttnMergeNode:
    """The P.V outputs o_g [G T][HD] (raw) -> pv [T][H HD] in head order,
    pv[t][(g G + h') HD + d] = o_g[h' T + t][d], a raw copy
    (llm_nodes.py:1560-1660); R row splits with G = 1.  ``batch`` B: o_g
    [B G T][HD] -> pv [B T][H HD]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    T: int = 1
    H: int = 1
    KV: int = 1
    HD: int = 16
    R: int = 1
    F: int = 8
    batch: int = 1
    onnx_node: object = None


@dataclass
class LlmSelectRowNode:
    """y = h[n - 1] with n clamped to [1, rows] — the last valid row of a
    padded prefill (llm_nodes.py:1663-1718); ``res32``: h / y int32 DMA
    tensors.  inputs = [h, n].  ``batch`` B: h [B rows][d] -> y [B][d], one
    row per sequence."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    res32: bool = False
    F: int = 8
    batch: int = 1
    onnx_node: object = None


@dataclass
class HostTable:
    """A host-side constant table of an LLM node (llm_nodes.py HostTable):
    kind f32 / bf16 (float32 values) or i16 (raw words at the output's
    exponent)."""
    name: str
    kind: str
    data: np.ndarray = field(repr=False)


@dataclass
class LlmEmbedNode:
    """h[t] = table[clamp(ids[t], 0, rows - 1)] (llm_nodes.py:466-570): float32
    rows, or with ``res32`` the int32 residual (round half to even at its
    exponent); ``scale`` a float32 factor.  inputs = [ids] (host int32)."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    d: int = 1
    n: int = 1
    image_rows: int = 0
    res32: bool = False
    scale: float = 1.0
    table: Optional[HostTable] = field(default=None, repr=False)
    F: int = 8
    onnx_node: object = None


@dataclass
class LlmDequantNode:
    """y = float32(raw 2^-f[c]) (llm_nodes.py:1722-1750)."""
    inputs: List[TensorInfo]
    output: TensorInfo
    count: int = 1
    F: int = 8
    onnx_node: object = None


@dataclass
class LlmToHostNode:
    """A float32 DMA tensor handed to the host unchanged (llm_nodes.py:1753-1777)."""
    inputs: List[TensorInfo]
    output: TensorInfo
    count: int = 1
    F: int = 8
    onnx_node: object = None


@dataclass
class LlmResAddNode:
    """y = float32((double) h + d) on the float32 residual (llm_nodes.py:572-603)."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    F: int = 8
    onnx_node: object = None


@dataclass
class LlmRMSNormNode:
    """y = (h r) gamma, r = 1 / sqrt(sum(h^2) / n + eps) per row of n
    (llm_nodes.py:618-694): h float32, or int16 rows of W (``i16``: W / n
    head rows each); y int16 at its per-channel exponents."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    W: int = 1
    i16: bool = False
    eps: float = 1e-5
    gamma: Optional[np.ndarray] = field(default=None, repr=False)
    F: int = 8
    onnx_node: object = None


@dataclass
class LlmSiluMulNode:
    """a = silu(g) u with silu from a libm table over g's raw word per gate
    exponent (llm_nodes.py:697-746).  inputs = [g, u]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    rows: int = 1
    n: int = 1
    F: int = 8
    onnx_node: object = None


@dataclass
class LlmGeluMulNode(LlmSiluMulNode):
    """a = gelu_tanh(g) u, the table form of llm_nodes.py:749-791."""


@dataclass
class LlmAttnPrepNode:
    """LlmAttnPrep's host form (llm_nodes.py:1012-1169): RoPE in float64 with
    the float32 tables, the K / V cache rows pos + t (t < n) at their
    exponents, the q.K^T image qx [KV][HD][G T] at fq per head.  inputs =
    [q0, k0, v, pos, (n), cache_k, cache_v]; ``batch`` B sequences: q0 / k0 /
    v [B T][..], caches [KV][B][C][HD], qx [KV][B][HD][G T]."""
    inputs: List[TensorInfo]
    output: TensorInfo
    T: int = 1
    H: int = 1
    KV: int = 1
    HD: int = 16
    C: int = 16
    kw: int = 1
    Q: int = 16
    has_n: bool = True
    fq: Optional[np.ndarray] = field(default=None, repr=False)
    cos: Optional[np.ndarray] = field(default=None, repr=False)
    sin: Optional[np.ndarray] = field(default=None, repr=False)
    F: int = 8
    batch: int = 1
    onnx_node: object = None

    @property
    def ck(self):
        return self.inputs[-2]

    @property
    def cv(self):
        return self.inputs[-1]


@dataclass
class Graph:
    """What the simulator reads of the reference's OnnxGraph: nodes in
    topological order, weights (with data), graph inputs / outputs, states."""
    nodes: list
    weight_tensors: List[TensorInfo]
    input_tensors: List[TensorInfo]
    output_tensors: List[TensorInfo]
    state_tensors: List[TensorInfo] = field(default_factory=list)
