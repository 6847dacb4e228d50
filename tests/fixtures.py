"""Case builders shared by the oracle tests and the GPU parity tests: each
reference register-level fixture (tests/golden/hw_*.npz) becomes the input
buffers, register values and expected output that a job of the kernel sees."""
from __future__ import annotations

import numpy as np

from oracle import spec


def _pad(v, n, fill=0):
    out = np.full(max(n, len(v), 1), fill, np.int16)
    out[:len(v)] = v
    return out


def vecop_cases(z):
    """(label, regs dict, a, b, c_len, check(c) -> list of mismatches)."""
    P = z["params"]
    for row, label in zip(P, z["labels"]):
        idx, size, op, outer, a_inc, b_inc, act, alpha, cm, cfg, mask = (int(v) for v in row)
        a, b, cv = z[f"c{idx}_a"], z[f"c{idx}_b"], z[f"c{idx}_c"]
        softmax = op in (10, 11)
        c_inc = b_inc if softmax else a_inc + b_inc
        rows = (outer & ~15) if op == 11 else outer
        W = (size + 7) // 8 * 8
        if op == 11:
            a_need = (size - 1) * a_inc + outer + 8
        else:
            a_need = (outer - 1) * a_inc + W + 8
        b_need = (outer - 1) * b_inc + W + 8
        c_len = spec.vectorop_out_elems(size, op, outer, a_inc, b_inc)
        regs = dict(size=size, op=op, outer=outer, a_inc=a_inc, b_inc=b_inc, act=act, alpha=alpha,
                    smx_cm=cm, smx_cfg=cfg, smx_mask=mask)

        def check(c, size=size, rows=rows, c_inc=c_inc, W=W, cv=cv):
            bad = []
            for o in range(rows):
                e0 = o * c_inc
                seg = c[e0:e0 + W].astype(np.int64)
                exp = cv[e0:e0 + size].astype(np.int64) if e0 < len(cv) else None
                if exp is not None and len(exp):
                    n = len(exp)
                    d = np.nonzero(seg[:n] != exp)[0]
                    bad += [(o, int(i), int(seg[i]), int(exp[i])) for i in d[:4]]
                if o + 1 == rows and np.any(seg[size:W] != 0):
                    bad.append((o, "tail"))
            return bad
        yield f"{idx}_{label}", regs, _pad(a, a_need), _pad(b, b_need), c_len, check


def matmul_cases(z):
    for row, label in zip(z["params"], z["labels"]):
        idx, n, k, m, batch, as_, bs, packed, kw = (int(v) for v in row)
        a, b, cv = z[f"c{idx}_a"], z[f"c{idx}_b"], z[f"c{idx}_c"]
        regs = dict(n=n, k=k, m=m, batch=batch, a_batch_stride=as_, b_batch_stride=bs, c_batch_stride=n * m,
                    b_packed=packed, gemv_kw=kw)
        yield f"{idx}_{label}", regs, a, b, cv


def conv_cases(z):
    names = ["batch", "in_ch", "in_h", "in_w", "out_ch", "out_h", "out_w", "kh", "kw", "stride_h", "stride_w",
             "dilation_h", "dilation_w", "pad_top", "pad_left", "has_bias", "is_depthwise", "y_cs", "y_cn", "y_gs"]
    for row, label in zip(z["params"], z["labels"]):
        idx = int(row[0])
        regs = {k: int(v) for k, v in zip(names, row[1:])}
        yield f"{idx}_{label}", regs, z[f"c{idx}_x"], z[f"c{idx}_w"], z[f"c{idx}_b"], z[f"c{idx}_y"]


def pool_cases(z):
    names = ["batch", "channels", "in_h", "in_w", "out_h", "out_w", "pool_h", "pool_w", "stride_h", "stride_w",
             "pad_top", "pad_left", "dil_h", "dil_w", "pool_type", "lp_order", "count_include_pad"]
    for row, label in zip(z["params"], z["labels"]):
        idx = int(row[0])
        regs = {k: int(v) for k, v in zip(names, row[1:])}
        yield f"{idx}_{label}", regs, z[f"c{idx}_x"], z[f"c{idx}_y"]


def rowops_cases(z):
    names = ["op", "n", "c1", "c2", "a_s1", "a_s2", "b_s1", "b_s2", "c_s1", "c_s2", "eps", "aux", "bq_sh",
             "win_lo", "win_hi"]
    for row, label in zip(z["params"], z["labels"]):
        idx = int(row[0])
        regs = {k: int(v) for k, v in zip(names, row[1:])}
        yield (f"{idx}_{label}", regs, z[f"c{idx}_a"], z[f"c{idx}_b"], z[f"c{idx}_p"], z[f"c{idx}_c"])


def rowops_memory(a, b, p, c_len, poison=0xDE):
    """One flat image: a, b, p and a poisoned c region, each 256-byte aligned;
    returns (mem, offsets)."""
    offs, cur = {}, 0
    parts = [("a", a), ("b", b), ("p", p), ("c", np.full(c_len, poison, np.uint8))]
    for name, arr in parts:
        offs[name] = cur
        cur += (len(arr) + 255) // 256 * 256 + 256
    mem = np.zeros(cur, np.uint8)
    for name, arr in parts:
        mem[offs[name]:offs[name] + len(arr)] = arr
    return mem, offs
