"""Power-of-two exponents on the host: the calibration's exponent tables and
the encoding of constant weights at the exponents their consumers give.

A tensor with exponent f carries raw int16 values at 2^-f (per tensor, or per
last-axis channel).  The kernels sum raw products exactly and write
floor(acc / 2^F) (F = 8), so a MatMul from x (f_in) to y (f_out) needs its
constant weight at f_w = f_out + F - f_in, per (input channel, output
channel) pair when the exponents are per channel, and a Conv's weight at
f_y + F - f_x with its bias at f_y (the kernel seeds the accumulator with
bias << F).  This module restates the reference's planner layer:

* ``expand_exp`` / ``ExponentTable`` — the formats table of a calibration,
  ``class@<layer>`` -> a scalar, a per-head or a per-channel vector
  (src/graph_builder.py:155-190); a class the table does not hold is an
  error, never a default.
* ``LlamaFormats`` — the Llama lowering's lookups on that table
  (src/llama.py:92-132): the residual's exponent, per-head q / k / p, the K
  and V caches' per-channel vectors, the P.V output's.
* ``score_exp`` / ``pv_exp`` — the exponents of q.K^T and P.V
  (src/graph_builder.py:197-208).
* ``encode_matmul_weight`` / ``encode_conv_weight`` — the weight encodings of
  src/numeric.py:199-307 on one weight: RNE(w 2^f_w) saturated to int16, the
  saturation count, the exponent array in the narrowest integer type, the
  data carried as raw / 2^F in float32 (the reference's convention for an
  encoded tensor's ``data``).

The workloads (``workloads.LlamaModel``) take their exponents from a
``LlamaFormats`` table and encode their weights with ``encode_matmul_weight``.
"""
from __future__ import annotations

import json
from typing import Dict, Optional, Tuple

import numpy as np

F = 8             # the kernels' output shift (floor(acc / 2^F)); ap_fixed<16,8>
RES_BITS = 15     # the int32 residual's exponent unless the table gives res@L
RAW_LO, RAW_HI = -32768, 32767
_ENCODE_BLOCK = 1 << 20   # weight elements per block of the MatMul encoding


class NumericError(ValueError):
    """An exponent table or an encoding request that cannot be honoured."""


def expand_exp(v, n: int, what: str = "exponents") -> np.ndarray:
    """int64 [n] of a calibrated value: a scalar broadcast, n values as they
    are, a per-head vector repeated over each head's n / heads channels
    (src/graph_builder.py:155-165)."""
    v = np.asarray(v, np.int64).reshape(-1)
    if v.size == 1:
        return np.full(n, int(v[0]), np.int64)
    if v.size == n:
        return v.copy()
    if v.size == 0 or n % v.size:
        raise NumericError(f"formats: {what} has {v.size} values, {n} wanted")
    return np.repeat(v, n // v.size)


class ExponentTable:
    """A calibration's exponents per ``class@<layer key>`` (the formats
    JSON's "exponents") and its policy string (src/graph_builder.py:168-190)."""

    def __init__(self, d: dict):
        if "exponents" not in d:
            raise NumericError("formats: no 'exponents' object")
        self.exp = dict(d["exponents"])
        self.policy = d.get("policy", "")

    @classmethod
    def from_file(cls, path: str, *args):
        with open(path) as f:
            return cls(json.load(f), *args)

    def has(self, key: str) -> bool:
        return key in self.exp

    def lookup(self, key: str, n: int) -> np.ndarray:
        if key not in self.exp:
            raise KeyError(f"formats: no exponent for {key} (policy {self.policy!r})")
        return expand_exp(self.exp[key], n, key)


def score_exp(fq, fk, groups: int) -> np.ndarray:
    """Per query head: the q.K^T scores' exponent f_q + f_k(its KV head) - F."""
    fq = np.asarray(fq, np.int64).reshape(-1)
    fk = np.asarray(fk, np.int64).reshape(-1)
    return fq + fk[np.arange(fq.size) // (fq.size // groups)] - F


def pv_exp(fp, fv, groups: int, hd: int) -> np.ndarray:
    """[H * hd]: the P.V output's exponent per channel, f_p(head) + f_v(channel
    of its KV head) - F."""
    fp = np.asarray(fp, np.int64).reshape(-1)
    grp = np.arange(fp.size) // (fp.size // groups)
    return (fp[:, None] + np.asarray(fv, np.int64).reshape(groups, hd)[grp] - F).reshape(-1)


class LlamaFormats(ExponentTable):
    """The Llama lowering's view of a formats table (src/llama.py:92-132):
    classes x, q0, k0, v, q, k, p (per head), s and pv (optional, derived
    otherwise), vc (optional, else v), o, x2, g, u, a, d per layer, and xf,
    logits, res at layer L (the final norm / LM head)."""

    def __init__(self, d: dict, *, L: int, H: int, KV: int, HD: int):
        super().__init__(d)
        self.L, self.H, self.KV, self.HD = L, H, KV, HD
        self.sink_k = d.get("sink_k_raw")
        self.sink_v = d.get("sink_v_raw")

    @property
    def res_bits(self) -> int:
        return int(np.asarray(self.exp.get(f"res@{self.L}", RES_BITS)).reshape(-1)[0])

    def get(self, cls_: str, layer: int, n: int) -> np.ndarray:
        return self.lookup(f"{cls_}@{layer}", n)

    def heads(self, cls_: str, layer: int, n_heads: int) -> np.ndarray:
        return self.get(cls_, layer, n_heads)

    def k_cache(self, li: int) -> np.ndarray:
        """[KV * HD]: the K cache exponent (per KV head) over the channels."""
        return np.repeat(self.heads("k", li, self.KV), self.HD)

    def v_cache(self, li: int) -> np.ndarray:
        key = "vc" if f"vc@{li}" in self.exp else "v"
        return self.get(key, li, self.KV * self.HD)

    def scores(self, li: int) -> np.ndarray:
        """Per query head: s@li when the table holds it, else f_q + f_k - F."""
        if f"s@{li}" in self.exp:
            return self.heads("s", li, self.H)
        return score_exp(self.heads("q", li, self.H), self.heads("k", li, self.KV), self.KV)

    def pv(self, li: int) -> np.ndarray:
        """P.V output exponent per channel of [H * HD]: f_p[h] + f_vc[g(h)] - F."""
        if f"pv@{li}" in self.exp:
            return self.get("pv", li, self.H * self.HD)
        return pv_exp(self.heads("p", li, self.H), self.v_cache(li), self.KV, self.HD)

    @classmethod
    def per_tensor(cls, e: Dict[str, int], *, L: int, H: int, KV: int, HD: int,
                   policy: str = "per-tensor") -> "LlamaFormats":
        """A table with one exponent per tensor class, the same in every layer:
        ``e`` maps the classes above (res, xf and logits at layer L) to ints."""
        per_layer = [k for k in e if k not in ("res", "xf", "logits")]
        exps = {f"{k}@{li}": int(e[k]) for li in range(L) for k in per_layer}
        for k in ("res", "xf", "logits"):
            if k in e:
                exps[f"{k}@{L}"] = int(e[k])
        return cls({"exponents": exps, "policy": policy}, L=L, H=H, KV=KV, HD=HD)


def _etype(lo: int, hi: int):
    return next(t for t in (np.int8, np.int16, np.int32, np.int64) if np.iinfo(t).min <= lo and hi <= np.iinfo(t).max)


def encode_matmul_weight(w: np.ndarray, f_in, f_out, f: int = F, lo: int = RAW_LO,
                         hi: int = RAW_HI) -> Tuple[np.ndarray, np.ndarray, int]:
    """A MatMul's constant B ([..., K, M] float) at wexp[i][j] = f_out[j] + f -
    f_in[i] (src/numeric.py:199-255).  ``f_in`` ([K] or a scalar) is A's
    exponent per input channel, ``f_out`` ([M] or a scalar) C's per output
    channel.  Returns (data = raw / 2^f as float32 in w's shape, wexp [K][M]
    in the narrowest integer type that holds it, the count of saturated
    elements); raw = RNE(w 2^wexp) clipped to [lo, hi].  Row blocks of about
    2^20 elements keep the float64 temporaries small; element-wise the
    arithmetic is the same."""
    w = np.asarray(w)
    if w.ndim < 2:
        raise NumericError("encode_matmul_weight: B needs at least 2 dims")
    K, M = int(w.shape[-2]), int(w.shape[-1])
    fa = np.broadcast_to(np.asarray(f_in, np.int64), (K,))
    fo = np.broadcast_to(np.asarray(f_out, np.int64), (M,))
    rows, cols = f - fa, fo
    wexp = np.empty((K, M), _etype(int(rows.min() + cols.min()), int(rows.max() + cols.max())))
    w3 = w.reshape(-1, K, M)
    out = np.empty(w3.shape, np.float32)
    n_sat = 0
    step = max(1, _ENCODE_BLOCK // max(1, w3.shape[0] * M))
    for r0 in range(0, K, step):
        e = np.add.outer(rows[r0:r0 + step], cols)
        wexp[r0:r0 + step] = e
        r = np.round(w3[:, r0:r0 + step].astype(np.float64) * np.power(2.0, e.astype(np.float64))[None])
        n_sat += int(((r < lo) | (r > hi)).sum())
        r = np.clip(r, lo, hi)
        out[:, r0:r0 + step] = (r / float(1 << f)).astype(np.float32)
    return out.reshape(w.shape), wexp, n_sat


def matmul_weight_raw(data: np.ndarray, f: int = F) -> np.ndarray:
    """The int16 raw words of an encoded weight's ``data`` (raw / 2^f)."""
    return np.round(np.asarray(data, np.float64) * (1 << f)).astype(np.int16)


def encode_conv_weight(w: np.ndarray, b: Optional[np.ndarray], fx, fy, *, depthwise: bool = False,
                       f: int = F, lo: int = RAW_LO, hi: int = RAW_HI):
    """A Conv's weight [M][C or 1][kh][kw] and bias [M] (src/numeric.py:258-307).
    ``fx`` / ``fy``: the input's / output's exponent, a scalar or per channel
    ([C] / [M]).  Per-tensor: the weight at f_y + f - f_x, the bias at f_y;
    per channel: f_w[m][c] = f_y[m] + f - f_x[c] (depthwise f_y[m] + f -
    f_x[m]), the bias at f_y[m].  Returns ((w data, w exponent, w saturated),
    (b data, b exponent, b saturated) or None); data = raw / 2^f as float32,
    raw = RNE(v 2^e) clipped."""
    w = np.asarray(w)
    M, C = int(w.shape[0]), int(w.shape[1])
    per_tensor = np.ndim(fx) == 0 and np.ndim(fy) == 0
    if per_tensor:
        fw = int(fy) + f - int(fx)
        fb = int(fy)
    else:
        in_ch = M if depthwise else C
        fxv = np.broadcast_to(np.asarray(fx, np.int64), (in_ch,))
        fyv = np.broadcast_to(np.asarray(fy, np.int64), (M,))
        fw = ((fyv + f - fxv)[:, None] if depthwise else np.add.outer(fyv + f, -fxv))
        fw = fw.reshape(fw.shape + (1, 1))
        fb = fyv

    def enc(v, e):
        ea = np.asarray(e, np.int64)
        r = np.round(np.asarray(v, np.float64) * np.power(2.0, ea))
        sat = int(((r < lo) | (r > hi)).sum())
        data = (np.clip(r, lo, hi) / float(1 << f)).astype(np.float32)
        if ea.ndim == 0:
            wexp = np.asarray(ea, np.int8 if -128 <= int(ea) <= 127 else np.int64)
        else:
            wexp = ea.astype(np.int8)
        return data, wexp, sat

    wres = enc(w, fw)
    bres = enc(np.asarray(b), fb) if b is not None else None
    return wres, bres
