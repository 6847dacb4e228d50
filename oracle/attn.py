"""CPU restatement of the prefill attention on the kernels — TEST
INFRASTRUCTURE: the checker for GpuSimulator's AttnPrepRoNode /
LlmAttnConvNode / LlmAttnSoftmaxVopNode / LlmAttnMergeNode.

Raw-integer arrays in their logical layouts: q0 [T][H HD], k0 / v [T][KV HD]
at their per-channel exponents, the caches [C][KV HD] (updated in place), the
q image qx [KV][HD][G T], scores s_g [C][G T], P_g [G T][C], o_g [G T][HD].

Reference files (phoenix367/cormorant inference-scheduler/src):
  LN = llm_nodes.py   RO = rowops_nodes.py   RS = rowops_spec.py
  SN = smx_nodes.py   VS = vectorop_smx.py
"""
from __future__ import annotations

import numpy as np

from . import spec

ROPE_BITS = 23


def attn_keys(pos: int, n: int, T: int, C: int, q: int = 16):
    """(valid rows n, keys = roundup(pos + n, q) in [q, C]) (LN:960-967)."""
    n = max(0, min(int(n), T, C - int(pos))) if int(pos) < C else 0
    k = -(-(int(pos) + n) // q) * q
    return n, max(q, min(k, C))


def kernel_out(acc: np.ndarray) -> np.ndarray:
    """ConvKernel / MatmulKernel output of exact sums: wrap to int32, floor
    / 2^8, saturate (LN:995-1001)."""
    return spec.sat16(spec.floor_shr(spec.wrap32(acc), 8))


def _dot(a, b) -> np.ndarray:
    """Exact integer product (float64 BLAS: every partial sum below 2^53 for
    int16 operands and up to 8192 terms)."""
    return np.matmul(np.asarray(a, np.float64), np.asarray(b, np.float64)).astype(np.int64)


def rope_tables(cos: np.ndarray, sin: np.ndarray):
    """int24 at 2^-23 of the float32 [C][HD/2] tables over both halves (RS:286-289)."""
    c = np.asarray(cos, np.float32).astype(np.float64)
    s = np.asarray(sin, np.float32).astype(np.float64)
    return (np.rint(np.concatenate([c, c], 1) * 2.0 ** ROPE_BITS).astype(np.int64),
            np.rint(np.concatenate([s, s], 1) * 2.0 ** ROPE_BITS).astype(np.int64))


def rope(x_raw: np.ndarray, f_x, c_raw: np.ndarray, s_raw: np.ndarray, f_out) -> np.ndarray:
    """Rotate-half RoPE of x [n][nh][HD] at per-channel f_x [nh][HD] to f_out
    (per head or channel): x c + rot(x) s exactly, both products at the finer
    exponent of the pair, one RNE, sat16 (RS:303-322)."""
    x_raw = np.asarray(x_raw, np.int64)
    n, nh, HD = x_raw.shape
    half = HD // 2
    f_x = np.broadcast_to(np.asarray(f_x, np.int64).reshape(nh, -1), (nh, HD))
    f_out = np.broadcast_to(np.asarray(f_out, np.int64).reshape(nh, -1), (nh, HD))
    f_rot = np.concatenate([f_x[:, half:], f_x[:, :half]], axis=1)
    fp = np.maximum(f_x, f_rot)
    rot = np.concatenate([-x_raw[..., half:], x_raw[..., :half]], axis=-1)
    num = ((x_raw * c_raw[:, None, :]) << (fp - f_x)[None]) + ((rot * s_raw[:, None, :]) << (fp - f_rot)[None])
    return spec.sat16(spec.rne_shr(num, (fp + ROPE_BITS - f_out)[None]))


def attn_prep(q0, k0, v, pos, n_in, *, T, H, KV, HD, C, fq0, fk0, fv, fq, fkc, fvc, cos, sin, ck, cv, Q=16):
    """LlmAttnPrep (RO:1112-1143): the rows t < n — RoPE(q0) at fq[h] into the
    q image qx[g][d][h' T + t] (h = g G + h'), RoPE(k0) at the K cache's
    exponent into ck[pos + t], v re-rounded (up by fvc - fv, RNE down by fv -
    fvc) into cv[pos + t]; qx elsewhere 0.  Returns qx."""
    G = H // KV
    n, _keys = attn_keys(pos, n_in, T, C, Q)
    qx = np.zeros((KV, HD, G * T), np.int64)
    if n == 0:
        return qx
    cr, sr = rope_tables(cos, sin)
    fq0, fk0, fv, fkc, fvc = (np.asarray(a, np.int64) for a in (fq0, fk0, fv, fkc, fvc))
    xq = np.asarray(q0, np.int64).reshape(T, H, HD)[:n]
    xk = np.asarray(k0, np.int64).reshape(T, KV, HD)[:n]
    yq = rope(xq, fq0.reshape(H, HD), cr[pos:pos + n], sr[pos:pos + n], np.asarray(fq, np.int64))
    yk = rope(xk, fk0.reshape(KV, HD), cr[pos:pos + n], sr[pos:pos + n],
              np.broadcast_to(fkc, (KV * HD,)).reshape(KV, HD))
    ck[pos:pos + n] = yk.reshape(n, -1)
    vr = np.asarray(v, np.int64).reshape(T, KV * HD)[:n]
    sa, sc = np.maximum(fvc - fv, 0), np.maximum(fv - fvc, 0)
    cv[pos:pos + n] = spec.sat16(spec.rne_shr(vr << np.broadcast_to(sa, (KV * HD,))[None, :],
                                              np.broadcast_to(sc, (KV * HD,))[None, :]))
    for h in range(H):
        g, hh = divmod(h, G)
        qx[g, :, hh * T:hh * T + n] = yq[:, h, :].T
    return qx


def attn_scores(ck, qx, g: int, *, HD: int, C: int, keys: int, r0: int = 0, nr: int = 0) -> np.ndarray:
    """q.K^T of group g (LN:1412-1420): the cache rows [:keys] (or r0 .. r0 +
    nr) of the group's columns @ qx[g]; rows keys .. C of the scores 0."""
    ck = np.asarray(ck, np.int64)
    x = np.asarray(qx, np.int64)[g]
    if nr:
        return kernel_out(_dot(ck[r0:r0 + nr, g * HD:(g + 1) * HD], x))
    out = np.zeros((C, x.shape[1]), np.int64)
    out[:keys] = kernel_out(_dot(ck[:keys, g * HD:(g + 1) * HD], x))
    return out


def attn_pv(P, cv, g: int, *, HD: int, keys: int) -> np.ndarray:
    """P.V of group g (LN:1421-1423): P[:, :keys] @ the V cache rows [:keys]."""
    return kernel_out(_dot(np.asarray(P, np.int64)[:, :keys], np.asarray(cv, np.int64)[:keys, g * HD:(g + 1) * HD]))


def attn_softmax(s, *, T: int, G: int, C: int, keys: int, pos: int, n: int, causal: bool, prefix_lm: bool,
                 cm, cfg) -> np.ndarray:
    """The column softmax of every head of a group (SN:320-338): P[h' T + t]
    [:keys] over the scores' columns h' T + t, row t valid over j < min(keys,
    pos + 1 + t) (causal) or j < max(min(keys, pos + n) - prefix_lm, 1)."""
    s = np.asarray(s, np.int64)
    if causal:
        valid = np.minimum(keys, pos + 1 + np.arange(T))
    else:
        valid = np.full(T, max(min(keys, pos + n) - int(prefix_lm), 1), np.int64)
    P = np.zeros((G * T, C), np.int64)
    for h in range(G):
        cs, fp = int(cfg[h]) & 63, (int(cfg[h]) >> 8) & 31
        P[h * T:(h + 1) * T, :keys] = spec.softmax_rows(s[:keys, h * T:(h + 1) * T].T, valid, int(cm[h]), cs, fp)
    return P


def attn_merge(o, *, T: int, H: int, KV: int, HD: int) -> np.ndarray:
    """pv[t][(g G + h') HD + d] = o_g[h' T + t][d] (LN:1645-1657)."""
    G = H // KV
    out = np.zeros((T, H, HD), np.int64)
    for g in range(KV):
        og = np.asarray(o[g], np.int64).reshape(G, T, HD)
        for hh in range(G):
            out[:, g * G + hh] = og[hh]
    return out.reshape(T, H * HD)


def prefill_layer(q0, k0, v, pos, n_in, *, T, H, KV, HD, C, fq0, fk0, fv, fq, fkc, fvc, cos, sin, ck, cv, cm, cfg,
                  causal=True, prefix_lm=False, Q=16):
    """One layer's chain: prep, per group scores / softmax / P.V, merge.
    Returns a dict of every intermediate (qx, s<g>, p<g>, o<g>, pv); the
    caches are updated in place.  cm / cfg: per query head."""
    G = H // KV
    out = {"qx": attn_prep(q0, k0, v, pos, n_in, T=T, H=H, KV=KV, HD=HD, C=C, fq0=fq0, fk0=fk0, fv=fv, fq=fq,
                           fkc=fkc, fvc=fvc, cos=cos, sin=sin, ck=ck, cv=cv, Q=Q)}
    n, keys = attn_keys(pos, n_in, T, C, Q)
    o = []
    for g in range(KV):
        s = attn_scores(ck, out["qx"], g, HD=HD, C=C, keys=keys)
        p = attn_softmax(s, T=T, G=G, C=C, keys=keys, pos=pos, n=n, causal=causal, prefix_lm=prefix_lm,
                         cm=cm[g * G:(g + 1) * G], cfg=cfg[g * G:(g + 1) * G])
        o.append(attn_pv(p, cv, g, HD=HD, keys=keys))
        out[f"s{g}"], out[f"p{g}"], out[f"o{g}"] = s, p, o[-1]
    out["pv"] = attn_merge(o, T=T, H=H, KV=KV, HD=HD)
    return out


_SEXP = {}


def sexp_table(f: int, scale: float) -> np.ndarray:
    """e[k] = exp(-k 2^-f scale) for k in [0, 65536), libm exp in this
    operation order (LN:357-364)."""
    import math
    key = (int(f), float(scale))
    if key not in _SEXP:
        d = 2.0 ** int(f)
        _SEXP[key] = np.array([math.exp(-k / d * scale) for k in range(65536)])
    return _SEXP[key]


def attn_softmax_host(s, *, T: int, G: int, C: int, pos: int, n_in: int, fs, fp, scale: float, window: int = 0,
                      Q: int = 16) -> np.ndarray:
    """The host's p12 softmax of one KV group (LN:1532-1557): for rows t < n
    of head h', keys j <= pos + t (and j > pos + t - W with a window): m =
    max, e = sexp_table(f_s[h'])[m - raw], the sum left to right in float64,
    P = RNE(fl(e / sum) 2^f_p[h']) saturated; every other entry 0."""
    n, _keys = attn_keys(pos, n_in, T, C, Q)
    s = np.asarray(s, np.int64)
    P = np.zeros((G * T, C), np.int64)
    if n == 0:
        return P
    S = pos + n
    j = np.arange(S)[None, :]
    t = np.arange(n)[:, None]
    mask = j <= pos + t
    if window:
        mask &= j > pos + t - window
    for hh in range(G):
        raw = s[:S, hh * T:hh * T + n].T
        m = np.where(mask, raw, -(1 << 20)).max(-1, keepdims=True)
        k = np.where(mask, m - raw, 0)
        e = np.where(mask, sexp_table(int(fs[hh]), scale)[k], 0.0)
        p = e / np.cumsum(e, -1)[..., -1:]
        P[hh * T:hh * T + n, :S] = np.clip(np.round(p * 2.0 ** int(fp[hh])), -32768, 32767).astype(np.int64)
    return P
