"""The float host operations of the LLM entries restated on the CPU — TEST
INFRASTRUCTURE: the checker for ``corm_llm_*`` (csrc/llm_host.cu) and the
GpuSimulator's host-op branches.  Restates phoenix367/cormorant
inference-scheduler/src/llm_nodes.py (cited per function, LN) and the
write-back rule of src/dtype.py:278-285 (``quantize_exp``); pinned to the
reference's own outputs by tests/golden/sim_llm_host.npz.

Values are float64 (raw / 2^f of their tensors); float32 tensors as float64.
"""
from __future__ import annotations

import math

import numpy as np


def st(v, f):
    """dtype.quantize_exp as raw words: RNE(v 2^f), NaN -> 0, saturated (D:278-285)."""
    v = np.asarray(v, np.float64)
    r = np.round(np.where(np.isnan(v), 0.0, v) * np.power(2.0, np.asarray(f, np.float64)))
    return np.clip(r, -32768, 32767).astype(np.int64)


def f32(v):
    return np.asarray(v, np.float64).astype(np.float32).astype(np.float64)


def embed(ids, table, res32_f=None, scale=1.0):
    """LN:546-569 without image rows: rows of the float32 table at the clamped
    ids (times a float32 scale); ``res32_f``: the int32 residual's raw words."""
    tab = np.asarray(table, np.float32)
    k = np.clip(np.asarray(ids, np.int64).reshape(-1), 0, tab.shape[0] - 1)
    out = (tab[k] * np.float32(scale)).astype(np.float64) if scale != 1.0 else tab[k].astype(np.float64)
    if res32_f is None:
        return out
    return np.clip(np.rint(out * 2.0 ** res32_f), -2147483648.0, 2147483647.0).astype(np.int64)


def dequant(xraw, fx):
    """LN:1748-1749: float32(raw 2^-f[c])."""
    return f32(np.asarray(xraw, np.float64) / np.power(2.0, np.asarray(fx, np.float64))[None, :])


def resadd(h, draw, fd):
    """LN:600-603: float32((double) h + d)."""
    return f32(np.asarray(h, np.float64) + np.asarray(draw, np.float64) / np.power(2.0, np.asarray(fd, np.float64)))


def rmsnorm(h, n, gamma, eps, fy, W=None):
    """LN:678-694: per row of n, ss = cumsum of the squares (left to right),
    r = 1 / sqrt(ss / n + eps), y = (h r) gamma at fy per channel of W."""
    W = n if W is None else W
    hv = np.asarray(h, np.float64).reshape(-1, n)
    ss = np.cumsum(hv * hv, axis=-1)[:, -1]
    r = 1.0 / np.sqrt(ss / float(n) + eps)
    y = ((hv * r[:, None]) * np.asarray(gamma, np.float32).astype(np.float64)[None, :]).reshape(-1, W)
    return st(y, np.asarray(fy)[None, :])


def _act_table(kind, f):
    d = 2.0 ** f
    t = np.empty(65536)
    for i in range(65536):
        g = (i - 32768 + 0.0) / d
        if kind == "silu":                                     # LN:325-333
            t[i] = g / (1.0 + math.exp(-g)) if g > -700 else 0.0
        else:                                                  # LN:336-349
            z = -1.5957691216057308 * (g + 0.044715 * g * g * g)
            t[i] = g / (1.0 + math.exp(z)) if z < 700.0 else 0.0
    return t


def act_mul(kind, graw, uraw, fg, fu, fy):
    """LN:735-746 / 776-791: the table at g's raw word per gate exponent, times
    u, written back at fy."""
    graw = np.asarray(graw, np.int64)
    fg = np.asarray(fg)
    a = np.empty(graw.shape)
    for f in np.unique(fg):
        cols = fg == f
        a[:, cols] = _act_table(kind, int(f))[graw[:, cols] + 32768]
    u = np.asarray(uraw, np.float64) / np.power(2.0, np.asarray(fu, np.float64))[None, :]
    return st(a * u, np.asarray(fy)[None, :])


def rope(x, cos, sin):
    """LN:315-322: x c + rot s with the float32 table rows as double."""
    half = x.shape[-1] // 2
    c = np.concatenate([cos, cos]).astype(np.float64)
    s = np.concatenate([sin, sin]).astype(np.float64)
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * c + rot * s


def attn_prep(q0raw, k0raw, vraw, ckraw, cvraw, pos, n_in, *, T, H, KV, HD, C, Q, fq0, fk0, fv, fkc, fvc, fq, cos,
              sin):
    """LN:1146-1169 for one sequence on raw words: returns (qx [KV][HD][G T],
    the caches' raw words after the rows pos + t, t < n)."""
    from . import attn as A
    G = H // KV
    p2 = lambda e: np.power(2.0, np.asarray(e, np.float64))[None, :]  # noqa: E731
    q0 = (np.asarray(q0raw, np.float64) / p2(fq0)).reshape(T, H, HD)
    k0 = (np.asarray(k0raw, np.float64) / p2(fk0)).reshape(T, KV, HD)
    v = np.asarray(vraw, np.float64) / p2(fv)
    n, _k = A.attn_keys(pos, n_in, T, C, Q)
    ck = np.array(ckraw, np.int64)
    cv = np.array(cvraw, np.int64)
    for t in range(n):
        p = pos + t
        ck[p] = st(rope(k0[t], cos[p], sin[p]).reshape(-1), fkc)
        cv[p] = st(v[t], fvc)
    qx = np.zeros((KV, HD, G * T), np.int64)
    s = np.power(2.0, np.asarray(fq, np.float64))
    for t in range(n):
        qr = rope(q0[t], cos[pos + t], sin[pos + t])
        raw = np.clip(np.round(qr * s[:, None]), -32768, 32767).astype(np.int64)
        for h in range(H):
            g, hh = divmod(h, G)
            qx[g, :, hh * T + t] = raw[h]
    return qx, ck, cv
