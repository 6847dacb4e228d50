"""Exponent plans for tensors stored at power-of-two scales.

A tensor "at exponent f" stores the integer raw = value * 2^f in int16 (the
LLM residual stream in int32).  f is one number for the whole tensor or one
number per channel of its last axis.  The kernels multiply raw integers,
add the products exactly and write floor(sum / 2^8), so everything about a
layer's scaling is settled by the exponents of its operands; this module
holds the two host-side pieces of that bookkeeping.

Calibration tables.  A calibration run writes one exponent entry per tensor
class and layer, under the key ``"<class>@<layer>"``; an entry is one int, a
list with one int per head, or a list with one int per channel.  ``ExponentTable``
reads such a table and hands out per-channel vectors of any requested width
(``expand_exp`` states the widening rule).  Asking for a class the table
never saw raises ``KeyError``: a silent default scale would make a typo in a
class name look like a numerics bug far downstream.  ``LlamaFormats`` adds the
derived quantities a decoder layer needs: the cache exponents, the q.K^T
score exponent and the P.V output exponent (phoenix367/cormorant
inference-scheduler/src/llama.py:92-132 and src/graph_builder.py:155-208
define what a table means; the semantics here are pinned to them by
``tests/golden/sim_numeric.npz``).

Weight encoding.  A constant operand is stored at whatever exponent makes the
kernel's output land on its consumer's grid: for C = A B with A at f_a
(per input channel i) and C at f_c (per output channel j), B[i][j] must sit
at f_c[j] + 8 - f_a[i]; for a convolution from x (f_x) to y (f_y) the weight
sits at f_y + 8 - f_x and the bias at f_y, because the kernel seeds its
accumulator with bias << 8 (src/numeric.py:199-307).  ``encode_matmul_weight``
and ``encode_conv_weight`` return the rounded, saturated raw words (as the
reference's node layer carries them: raw / 2^8 in float32), the exponent
array in the narrowest signed integer type that holds it, and how many
elements saturated.
"""
from __future__ import annotations

import json
from typing import Dict, Optional, Tuple

import numpy as np

F = 8             # the kernels' output shift: floor(sum / 2^F)
RES_BITS = 15     # the int32 residual's exponent when a table has no res@L entry
RAW_LO, RAW_HI = -32768, 32767
_CHUNK = 1 << 20  # weight elements encoded per pass (bounds the float64 temporaries)


class NumericError(ValueError):
    """A table entry or an encoding request that cannot be honoured."""


# ---------------------------------------------------------------- calibration tables
def expand_exp(v, n: int, what: str = "exponents") -> np.ndarray:
    """A table entry widened to ``n`` channels (int64): one value fills all of
    them; exactly n values are taken as they are; any other count that divides
    n is a per-head entry, each value covering a run of n / count channels."""
    vals = np.atleast_1d(np.asarray(v, np.int64)).ravel()
    if vals.size == 1:
        return np.full(n, vals[0], np.int64)
    if vals.size == n:
        return vals.copy()
    if vals.size and n % vals.size == 0:
        return np.repeat(vals, n // vals.size)
    raise NumericError(f"formats: {what} has {vals.size} values, {n} wanted")


class ExponentTable:
    """The exponent entries of a calibration (the ``exponents`` object of a
    formats JSON) and the name of the policy that wrote them."""

    def __init__(self, d: dict):
        if "exponents" not in d:
            raise NumericError("formats: no 'exponents' object")
        self.exp: Dict[str, object] = dict(d["exponents"])
        self.policy = d.get("policy", "")

    @classmethod
    def from_file(cls, path: str, **kw):
        with open(path) as fh:
            return cls(json.load(fh), **kw)

    def has(self, key: str) -> bool:
        return key in self.exp

    def lookup(self, key: str, n: int) -> np.ndarray:
        """The entry ``key`` over ``n`` channels; a missing entry is an error."""
        try:
            entry = self.exp[key]
        except KeyError:
            raise KeyError(f"formats: no exponent for {key} (policy {self.policy!r})") from None
        return expand_exp(entry, n, key)


def _kv_group(n_heads: int, groups: int) -> np.ndarray:
    """The KV group each of ``n_heads`` query heads reads (consecutive runs)."""
    return np.arange(n_heads) // (n_heads // groups)


def score_exp(fq, fk, groups: int) -> np.ndarray:
    """Exponent of each query head's q.K^T scores: the kernel's sum of
    raw q x raw k is at f_q + f_k, and its output shift takes F away."""
    fq = np.asarray(fq, np.int64).ravel()
    fk = np.asarray(fk, np.int64).ravel()
    return fq + fk[_kv_group(fq.size, groups)] - F


def pv_exp(fp, fv, groups: int, hd: int) -> np.ndarray:
    """Exponent of each channel of the P.V output ([heads * hd]): head h's
    probabilities (f_p[h]) times its KV group's value channels (f_v), less F."""
    fp = np.asarray(fp, np.int64).ravel()
    fv = np.asarray(fv, np.int64).reshape(groups, hd)
    return (fp[:, None] + fv[_kv_group(fp.size, groups)] - F).ravel()


class LlamaFormats(ExponentTable):
    """A calibration table read by a decoder's lowering.  Per layer ``li`` it
    holds the classes x, q0, k0, v, q, k, p (per head), o, x2, g, u, a, d and
    optionally vc (the V cache when it differs from v), s (scores) and pv;
    at layer ``L`` xf, logits and optionally res (the final norm, the LM head,
    the residual's exponent)."""

    def __init__(self, d: dict, *, L: int, H: int, KV: int, HD: int):
        super().__init__(d)
        self.L, self.H, self.KV, self.HD = L, H, KV, HD
        self.sink_k = d.get("sink_k_raw")
        self.sink_v = d.get("sink_v_raw")

    def get(self, cls_: str, layer: int, n: int) -> np.ndarray:
        return self.lookup(f"{cls_}@{layer}", n)

    def heads(self, cls_: str, layer: int, n_heads: int) -> np.ndarray:
        return self.get(cls_, layer, n_heads)

    @property
    def res_bits(self) -> int:
        entry = self.exp.get(f"res@{self.L}")
        return RES_BITS if entry is None else int(np.atleast_1d(np.asarray(entry))[0])

    def k_cache(self, li: int) -> np.ndarray:
        """The K cache's exponent per channel: each KV head's k entry over its HD channels."""
        return np.repeat(self.heads("k", li, self.KV), self.HD)

    def v_cache(self, li: int) -> np.ndarray:
        """The V cache's exponent per channel (the vc entry, else v's)."""
        cls_ = "vc" if self.has(f"vc@{li}") else "v"
        return self.get(cls_, li, self.KV * self.HD)

    def scores(self, li: int) -> np.ndarray:
        """Per query head: the calibrated s entry, else derived from q and k."""
        if self.has(f"s@{li}"):
            return self.heads("s", li, self.H)
        return score_exp(self.heads("q", li, self.H), self.heads("k", li, self.KV), self.KV)

    def pv(self, li: int) -> np.ndarray:
        """Per P.V output channel: the calibrated pv entry, else derived from p and the V cache."""
        if self.has(f"pv@{li}"):
            return self.get("pv", li, self.H * self.HD)
        return pv_exp(self.heads("p", li, self.H), self.v_cache(li), self.KV, self.HD)

    @classmethod
    def per_tensor(cls, e: Dict[str, int], *, L: int, H: int, KV: int, HD: int,
                   policy: str = "per-tensor") -> "LlamaFormats":
        """A table with one exponent per class, equal in every layer; ``e``
        maps class names to ints (res, xf and logits go to layer L)."""
        final = {"res", "xf", "logits"}
        table = {}
        for name, val in e.items():
            layers = [L] if name in final else range(L)
            table.update({f"{name}@{li}": int(val) for li in layers})
        return cls({"exponents": table, "policy": policy}, L=L, H=H, KV=KV, HD=HD)


# ---------------------------------------------------------------- weight encoding
def _narrowest(lo: int, hi: int):
    """The smallest signed numpy integer type holding [lo, hi]."""
    for t in (np.int8, np.int16, np.int32, np.int64):
        info = np.iinfo(t)
        if info.min <= lo and hi <= info.max:
            return t
    raise NumericError(f"exponents [{lo}, {hi}] exceed int64")


def _quantize(values: np.ndarray, exps: np.ndarray, lo: int, hi: int) -> Tuple[np.ndarray, int]:
    """RNE(values * 2^exps) saturated to [lo, hi] (float64 integers) and how
    many elements saturated; ``exps`` broadcasts against ``values``."""
    r = np.rint(np.asarray(values, np.float64) * np.exp2(np.asarray(exps, np.float64)))
    clipped = np.clip(r, lo, hi)
    return clipped, int(np.count_nonzero(clipped != r))


def _as_data(raw: np.ndarray, f: int) -> np.ndarray:
    """Raw words as the node layer's ``data`` convention: raw / 2^f in float32 (exact)."""
    return (raw / float(1 << f)).astype(np.float32)


def encode_matmul_weight(w: np.ndarray, f_in, f_out, f: int = F, lo: int = RAW_LO,
                         hi: int = RAW_HI) -> Tuple[np.ndarray, np.ndarray, int]:
    """Encode a MatMul's constant B ([..., K, M]) for A at ``f_in`` (a scalar
    or [K]) and C at ``f_out`` (a scalar or [M]): element (i, j) sits at
    f_out[j] + f - f_in[i].  Returns (data in w's shape, the exponent matrix
    [K][M] in its narrowest signed type, the number of saturated elements).
    Leading batch dims share the exponent matrix; the rows are encoded in
    chunks of about 2^20 elements."""
    w = np.asarray(w)
    if w.ndim < 2:
        raise NumericError("encode_matmul_weight: B needs at least 2 dims")
    K, M = w.shape[-2:]
    row_part = f - np.broadcast_to(np.asarray(f_in, np.int64), (K,))   # [K]
    col_part = np.broadcast_to(np.asarray(f_out, np.int64), (M,))      # [M]
    lo_e = int(row_part.min() + col_part.min())
    hi_e = int(row_part.max() + col_part.max())
    exps = (row_part[:, None] + col_part[None, :]).astype(_narrowest(lo_e, hi_e))
    slabs = w.reshape(-1, K, M)
    data = np.empty(slabs.shape, np.float32)
    saturated = 0
    rows_per_chunk = max(1, _CHUNK // max(1, slabs.shape[0] * M))
    for start in range(0, K, rows_per_chunk):
        sl = slice(start, min(K, start + rows_per_chunk))
        raw, n = _quantize(slabs[:, sl], exps[sl][None], lo, hi)
        data[:, sl] = _as_data(raw, f)
        saturated += n
    return data.reshape(w.shape), exps, saturated


def matmul_weight_raw(data: np.ndarray, f: int = F) -> np.ndarray:
    """The int16 words behind an encoded weight's ``data``."""
    return np.rint(np.asarray(data, np.float64) * (1 << f)).astype(np.int16)


def encode_conv_weight(w: np.ndarray, b: Optional[np.ndarray], fx, fy, *, depthwise: bool = False,
                       f: int = F, lo: int = RAW_LO, hi: int = RAW_HI):
    """Encode a convolution's weight ([M][C or 1][kh][kw]) and bias ([M]) for
    x at ``fx`` and y at ``fy`` (scalars, or per channel [C] / [M]).  With
    scalars the weight sits at fy + f - fx and the bias at fy; per channel,
    weight (m, c) at fy[m] + f - fx[c] (depthwise: fy[m] + f - fx[m]) and bias
    m at fy[m].  Returns ((weight data, its exponent, saturated count), the
    same for the bias or None).  A scalar exponent is typed int8 when it fits
    (else int64); per-channel exponents are int8."""
    w = np.asarray(w)
    M, C = w.shape[:2]
    if np.ndim(fx) == 0 and np.ndim(fy) == 0:
        w_exp = np.asarray(int(fy) + f - int(fx))
        b_exp = np.asarray(int(fy))
    else:
        fyv = np.broadcast_to(np.asarray(fy, np.int64), (M,))
        fxv = np.broadcast_to(np.asarray(fx, np.int64), (M if depthwise else C,))
        per_pair = (fyv + f)[:, None] - (fxv[:, None] if depthwise else fxv[None, :])   # [M][1] or [M][C]
        w_exp = per_pair[:, :, None, None]
        b_exp = fyv

    def encode(v, e):
        raw, n = _quantize(v, e, lo, hi)
        if e.ndim == 0:
            typed = e.astype(np.int8 if -128 <= int(e) <= 127 else np.int64)
        else:
            typed = e.astype(np.int8)
        return _as_data(raw, f), typed, n

    return encode(w, w_exp), (encode(np.asarray(b), b_exp) if b is not None else None)
