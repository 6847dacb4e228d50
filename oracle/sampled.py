"""Sampled exact checks of large MatMul jobs — TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU legs
and its after-the-timed-region verification) may import this module; the
product path never does.

A MatMul job (phoenix367/cormorant inference-scheduler/src/codegen/
_simulate.py:620-633: ``C = sat16(floor(A B / 2^8))`` per batch slice, or
wrapped to int32 first on the exponent path :814-835) is checked exactly at a
seeded grid of outputs: a few batch slices, a few rows of A and a few columns
of B.  Every sampled output depends only on its row of A and its column of B,
so the caller gathers just those (on the device) and the oracle recomputes the
grid exactly with ``spec.matmul_raw``.  Small jobs are checked in full.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from . import spec

SAMPLE_OUTPUTS = 4096      # outputs checked per job when it is not checked in full
FULL_MACS = 1 << 30        # jobs up to this many MACs are checked in full by default


def plan(batch: int, m: int, k: int, n: int, seed: int = 0,
         full_macs: Optional[int] = FULL_MACS) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(batch indices, row indices, column indices), sorted, of the grid to
    check for a [batch][m][k] x [batch][k][n] job: everything when the job has
    at most ``full_macs`` MACs (None: never) or at most SAMPLE_OUTPUTS
    outputs, else at least SAMPLE_OUTPUTS outputs on min(batch, 4) slices."""
    if batch * m * n <= SAMPLE_OUTPUTS or (full_macs is not None and batch * m * k * n <= full_macs):
        return np.arange(batch), np.arange(m), np.arange(n)
    rng = np.random.default_rng([seed, batch, m, k, n])
    nb = min(batch, 4)
    per = -(-SAMPLE_OUTPUTS // nb)
    side = int(np.ceil(np.sqrt(per)))
    nr = min(m, side)
    nc = min(n, -(-per // nr))
    nr = min(m, -(-per // nc))
    pick = lambda total, cnt: np.sort(rng.choice(total, size=cnt, replace=False))  # noqa: E731
    return pick(batch, nb), pick(m, nr), pick(n, nc)


def check(a_sub: np.ndarray, b_sub: np.ndarray, c_sub: np.ndarray, wrap: bool = False) -> Tuple[int, int]:
    """(outputs checked, mismatches) of a gathered grid: a_sub [nb][nr][k]
    (the sampled rows of A per sampled slice), b_sub [nb][k][nc] (the sampled
    columns of B), c_sub [nb][nr][nc] (the job's outputs at the grid)."""
    want = spec.matmul_raw(np.asarray(a_sub, np.int64), np.asarray(b_sub, np.int64), wrap)
    got = np.asarray(c_sub, np.int64).reshape(want.shape)
    return int(want.size), int((want != got).sum())


def gather_t(A, B, C, batch: int, m: int, k: int, n: int, idx, a_bs: Optional[int] = None,
             b_bs: Optional[int] = None, c_bs: Optional[int] = None):
    """The grid's rows of A, columns of B and outputs of C as tensors on the
    operands' device, from flat torch tensors holding the job's [batch][m][k],
    [batch][k][n] and [batch][m][n] operands at the given batch strides
    (defaults: dense; 0: one slice for every batch)."""
    import torch
    bi, ri, ci = (torch.as_tensor(np.asarray(v, np.int64), device=A.device) for v in idx)
    a_bs = m * k if a_bs is None else a_bs
    b_bs = k * n if b_bs is None else b_bs
    c_bs = m * n if c_bs is None else c_bs
    a3 = A.as_strided((batch, m, k), (a_bs, k, 1))
    b3 = B.as_strided((batch, k, n), (b_bs, n, 1))
    c3 = C.as_strided((batch, m, n), (c_bs, n, 1))
    return a3[bi][:, ri, :], b3[bi][:, :, ci], c3[bi][:, ri][:, :, ci]


def gather(A, B, C, batch: int, m: int, k: int, n: int, idx, **strides):
    """``gather_t`` as host arrays for ``check``."""
    return tuple(t.cpu().numpy() for t in gather_t(A, B, C, batch, m, k, n, idx, **strides))
