"""CPU restatement of the Cormorant fixed-point kernels — TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (cpu baseline)
may import this module; the product path never does.

Conventions.  ``raw`` arrays are signed integers (numpy int64 unless stated)
holding the storage integer of a Q8.8 value (value = raw / 2^8) or of a tensor
at a power-of-two exponent f (value = raw / 2^f).  ``floor`` of a division by
2^s is the arithmetic right shift; ``sat16`` clamps to [-32768, 32767];
``rne`` is round half to even.

Reference files (phoenix367/cormorant), cited per function:
  S  = inference-scheduler/src/codegen/_simulate.py
  D  = inference-scheduler/src/dtype.py
  VA = inference-scheduler/src/vectorop_act.py
  VS = inference-scheduler/src/vectorop_smx.py
  RS = inference-scheduler/src/rowops_spec.py
  HE = inference-scheduler/test/host_emu.py
  RR = kernels/rowops_rtl/tb/verilator/rowops_ref.h
"""
from __future__ import annotations

import math
from functools import lru_cache
from typing import Optional, Tuple

import numpy as np

I16_LO, I16_HI = -32768, 32767
I32_LO, I32_HI = -(1 << 31), (1 << 31) - 1


# --------------------------------------------------------------------------- helpers
def sat16(v):
    """Clamp to int16 (D:367-375 AP_SAT; HE:170 emu_sat)."""
    return np.clip(v, I16_LO, I16_HI)


def sat32(v):
    return np.clip(v, I32_LO, I32_HI)


def floor_shr(v, s: int):
    """floor(v / 2^s) for int64 v (HE:171 emu_floor_shift; numpy >> is floor)."""
    return np.asarray(v, np.int64) >> s


def rne_shr(v, k):
    """round half to even of v / 2^k, k >= 0 scalar or array (RS:48-56, RS:292-300)."""
    v = np.asarray(v, np.int64)
    k = np.broadcast_to(np.asarray(k, np.int64), v.shape)
    kk = np.maximum(k, 1)
    q = v >> kk
    r = v - (q << kk)
    half = np.int64(1) << (kk - 1)
    up = (r > half) | ((r == half) & ((q & 1) == 1))
    return np.where(k > 0, q + up, v << np.maximum(-k, 0))


def wrap32(v):
    """two's-complement wrap of an exact sum to int32 (S:808-810, S:828-830)."""
    v = np.asarray(v, np.int64)
    return ((v + (1 << 31)) & 0xFFFFFFFF) - (1 << 31)


def rne_int(x: np.ndarray) -> np.ndarray:
    """round half to even of float64 x to an integer-valued float (np.round)."""
    return np.round(np.asarray(x, np.float64))


# --------------------------------------------------------------------------- activation unit
ACT_NONE, ACT_RELU, ACT_RELU6, ACT_LEAKY_RELU, ACT_SILU, ACT_GELU, ACT_GELU_TANH = range(7)
UNIT_ACTS = (ACT_LEAKY_RELU, ACT_SILU, ACT_GELU, ACT_GELU_TANH)
OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_RELU, OP_RELU6 = range(6)
OP_LEAKY_RELU, OP_SILU, OP_GELU, OP_GELU_TANH, OP_SOFTMAX, OP_SOFTMAX_T = range(6, 12)


def _vec(fn):
    return np.vectorize(fn, otypes=[np.float64])


def act_real(act: int, x: np.ndarray, alpha: int = 0) -> np.ndarray:
    """The unrounded activation of float64 values x, in double with the C
    library's exp / erf / tanh, formulas of VA:60-73 (VectorOP.cpp act_fn)."""
    x = np.asarray(x, np.float64)
    if act == ACT_LEAKY_RELU:
        return np.where(x >= 0.0, x, x * ((alpha & 0xFFFF) / 65536.0))
    if act == ACT_SILU:
        return x / (1.0 + _vec(math.exp)(-x))
    if act == ACT_GELU:
        return x * (0.5 * (1.0 + _vec(math.erf)(x / math.sqrt(2.0))))
    if act == ACT_GELU_TANH:
        inner = math.sqrt(2.0 / math.pi) * (x + 0.044715 * (x * x * x))
        return x * (0.5 * (1.0 + _vec(math.tanh)(inner)))
    raise ValueError(f"act {act} is not an activation of the unit")


def host_quantize_raw(v: np.ndarray) -> np.ndarray:
    """raw of D:214-219 host_quantize at Q8.8: clip, RNE, NaN -> 0."""
    v = np.asarray(v, np.float64)
    v = np.where(np.isnan(v), 0.0, v)
    return rne_int(np.clip(v, -128.0, 127.99609375) * 256.0).astype(np.int64)


@lru_cache(maxsize=None)
def act_table(act: int, alpha: int = 0) -> np.ndarray:
    """The unit's output for every Q8.8 input, indexed by raw + 32768
    (VA:92-95 kernel_table; LeakyReLU depends on alpha[15:0])."""
    x = np.arange(-32768, 32768, dtype=np.float64) / 256.0
    t = host_quantize_raw(act_real(act, x, alpha)).astype(np.int16)
    t.setflags(write=False)
    return t


def apply_act_raw(r: np.ndarray, act: int, alpha: int = 0) -> np.ndarray:
    """The ALU act (ReLU / ReLU6) or the unit act on saturated raw results
    (HE:250-252 emu_act after the relu clamps, HE:282-285)."""
    r = np.asarray(r, np.int64)
    if act == ACT_RELU:
        return np.maximum(r, 0)
    if act == ACT_RELU6:
        return np.clip(r, 0, 1536)
    if act in UNIT_ACTS:
        return act_table(act, alpha & 0xFFFF if act == ACT_LEAKY_RELU else 0)[r + 32768].astype(np.int64)
    return r


# --------------------------------------------------------------------------- softmax unit
SMX_F, SMX_E, SMX_RB = 12, 16, 40
SMX_TAB = np.round(np.power(2.0, SMX_E) * np.power(2.0, -np.arange(1 << SMX_F) / (1 << SMX_F))).astype(np.int64)


def smx_scale_regs(f_s: float, sigma: float = 1.0) -> Tuple[int, int]:
    """(Cm, Cs): Cm * 2^-Cs = log2(e) * sigma * 2^-f_s * 2^12 on a 24-bit
    mantissa (VS:37-47)."""
    c = math.log2(math.e) * float(sigma) * 2.0 ** (-float(f_s)) * (1 << SMX_F)
    cs = 23 - math.floor(math.log2(c))
    cm = int(round(c * 2.0 ** cs))
    if cm >= 1 << 24:
        cm, cs = cm >> 1, cs - 1
    if not 0 <= cs <= 63:
        raise ValueError("softmax scale out of range")
    return cm, cs


def smx_valid(rows: int, n: int, mask: int) -> np.ndarray:
    """valid length per vector from the mask register: min(n, valid0 + q mod
    period) (VS:75-78, HE:232-236)."""
    valid0, period = mask & 0xFFFF, (mask >> 16) & 0xFFFF
    q = np.arange(rows, dtype=np.int64)
    return np.minimum(n, valid0 + (q % period if period else 0))


def softmax_rows(x: np.ndarray, valid, cm: int, cs: int, f_p: int) -> np.ndarray:
    """The integer softmax of each row of raw scores x [rows][n] (VS:50-66):
    m = max, y = ((m - x) * Cm) >> Cs, e = TAB[y mod 4096] >> (y div 4096)
    (0 for a shift >= 63), R = floor(2^40 / S), P = min((e R + 2^(39-f_p))
    >> (40 - f_p), 32767); 0 past the valid length."""
    x = np.asarray(x, np.int64)
    rows, n = x.shape
    v = np.broadcast_to(np.minimum(np.asarray(valid, np.int64), n), (rows,))
    mask = np.arange(n)[None, :] < v[:, None]
    m = np.where(mask, x, np.iinfo(np.int64).min).max(axis=1, keepdims=True) if n else np.zeros((rows, 1), np.int64)
    d = np.where(mask, m - x, 0)
    y = (d * int(cm & 0xFFFFFF)) >> int(cs)
    sh = y >> SMX_F
    e = np.where(mask & (sh < 63), SMX_TAB[y & ((1 << SMX_F) - 1)] >> np.minimum(sh, 63), 0)
    S = e.sum(axis=1, keepdims=True)
    R = np.where(S > 0, (1 << SMX_RB) // np.maximum(S, 1), 0)
    P = (e * R + (1 << (SMX_RB - f_p - 1))) >> (SMX_RB - f_p)
    return np.where(mask, np.minimum(P, 32767), 0)


# --------------------------------------------------------------------------- VectorOP
def _words8(size: int) -> int:
    return (size + 7) // 8 * 8


def vectorop_out_elems(size: int, op: int, outer: int, a_inc: int, b_inc: int) -> int:
    """Elements of c a job writes from its base (HE:259-270)."""
    if size == 0 or outer == 0:
        return 0
    if op in (OP_SOFTMAX, OP_SOFTMAX_T):
        rows = outer & ~15 if op == OP_SOFTMAX_T else outer
        return (rows - 1) * b_inc + _words8(size) if rows else 0
    return (outer - 1) * (a_inc + b_inc) + _words8(size)


def vectorop_job(a: np.ndarray, b: Optional[np.ndarray], c: np.ndarray, size: int, op: int, outer: int,
                 a_inc: int, b_inc: int, act: int = 0, alpha: int = 0, smx_cm: int = 0, smx_cfg: int = 0,
                 smx_mask: int = 0) -> None:
    """One VectorOPKernel job on int16 buffers a, b, c (element offsets from
    the bases), written into c in place: the register semantics of HE:244-293
    (VectorOP.h:279-333).  c[o*(a_inc+b_inc)+i] = act(op(a[o*a_inc+i],
    b[o*b_inc+i])); the last 8-lane word of every row is written whole with
    zero tail lanes.  Softmax ops 10 / 11 write rows at stride b_inc."""
    if size == 0 or outer == 0:
        return
    W = _words8(size)
    a = np.asarray(a).astype(np.int64)
    if op in (OP_SOFTMAX, OP_SOFTMAX_T):
        cs, fp = smx_cfg & 63, (smx_cfg >> 8) & 31
        col = op == OP_SOFTMAX_T
        rows = outer & ~15 if col else outer
        if rows == 0:
            return
        if col:
            idx = np.arange(rows)[:, None] + np.arange(size)[None, :] * a_inc
        else:
            idx = np.arange(rows)[:, None] * a_inc + np.arange(size)[None, :]
        P = softmax_rows(a[idx], smx_valid(rows, size, smx_mask), smx_cm, cs, fp)
        out = np.zeros((rows, W), np.int64)
        out[:, :size] = P
        for o in range(rows):                       # sequential: later rows win on overlap
            c[o * b_inc: o * b_inc + W] = out[o].astype(np.int16)
        return
    o = np.arange(outer)[:, None]
    i = np.arange(size)[None, :]
    x = a[o * a_inc + i]
    if op <= OP_DIV:
        y = np.asarray(b).astype(np.int64)[o * b_inc + i]
    else:
        y = np.zeros_like(x)
    if op == OP_ADD:
        r = x + y
    elif op == OP_SUB:
        r = x - y
    elif op == OP_MUL:
        r = floor_shr(x * y, 8)
    elif op == OP_DIV:                            # C division truncates; b == 0 gives 0 (HE:280)
        num = x * 256
        q = np.abs(num) // np.maximum(np.abs(y), 1)
        r = np.where(y == 0, 0, np.where((num < 0) ^ (y < 0), -q, q))
    elif op == OP_RELU:
        r = np.maximum(x, 0)
    elif op == OP_RELU6:
        r = np.clip(x, 0, 1536)
    else:
        r = x
    r = sat16(r)
    jact = op - 3 if OP_LEAKY_RELU <= op <= OP_GELU_TANH else act
    r = apply_act_raw(r, jact, alpha)
    c_inc = a_inc + b_inc
    out = np.zeros((outer, W), np.int64)
    out[:, :size] = r
    if outer == 1 or c_inc >= W:
        idx = (np.arange(outer)[:, None] * c_inc + np.arange(W)[None, :]).reshape(-1)
        c[idx] = out.reshape(-1).astype(np.int16)
    else:
        for oo in range(outer):
            c[oo * c_inc: oo * c_inc + W] = out[oo].astype(np.int16)


# --------------------------------------------------------------------------- MatMul
MATMUL_TILE_M = 32          # platforms/kv260.json kernels.matmul.tile_m (packed-B tile width)


def gemv_index(kk: np.ndarray, j: np.ndarray, m: int, kw: int) -> np.ndarray:
    """Element offset of B[kk][j] in the GEMV image of width kw (HE:325-332,
    MatmulKernel.h matmul_gemv_index)."""
    if kw <= 1:
        return kk * m + j
    c = (kk // (16 * kw)) * 16 + kk % 16
    return (c * m + j) * kw + (kk // 16) % kw


def b_index(k: int, m: int, b_packed: int, gemv_kw: int, tile_m: int = MATMUL_TILE_M) -> np.ndarray:
    """[k][m] element offsets of B for the row-major, packed tile-major
    [ceil(m/T)][k][T] or GEMV layouts (HE:352-356)."""
    kk = np.arange(k, dtype=np.int64)[:, None]
    j = np.arange(m, dtype=np.int64)[None, :]
    if gemv_kw:
        return gemv_index(kk, j, m, gemv_kw)
    if b_packed:
        return ((j // tile_m) * k + kk) * tile_m + j % tile_m
    return kk * m + j


def matmul_raw(A: np.ndarray, B: np.ndarray, wrap: bool = False) -> np.ndarray:
    """sat16(floor(sum_k A B / 2^8)) of raw int matrices (any leading batch
    dims).  The sum is formed exactly (float64 BLAS on integers below 2^53,
    as S:631 does on values); ``wrap`` first wraps it to int32 (the exponent
    path S:828-832 and the hardware accumulator)."""
    acc = np.matmul(np.asarray(A, np.float64), np.asarray(B, np.float64)).astype(np.int64)
    if wrap:
        acc = wrap32(acc)
    return sat16(floor_shr(acc, 8))


def matmul_job(a: np.ndarray, b: np.ndarray, c: np.ndarray, n: int, k: int, m: int, batch: int,
               a_batch_stride: int, b_batch_stride: int, c_batch_stride: int, b_packed: int = 0,
               gemv_kw: int = 0, wrap: bool = False, tile_m: int = MATMUL_TILE_M) -> None:
    """One MatmulKernel job on flat int16 buffers (HE:338-362): per batch slice
    C[r][j] = sat16(floor(sum_kk A[r][kk] B[kk][j] / 2^8)), C rows at stride m."""
    bi = b_index(k, m, b_packed, gemv_kw, tile_m)
    for bt in range(batch):
        A = np.asarray(a[bt * a_batch_stride: bt * a_batch_stride + n * k]).astype(np.int64).reshape(n, k)
        B = np.asarray(b).astype(np.int64)[bt * b_batch_stride + bi]
        c[bt * c_batch_stride: bt * c_batch_stride + n * m] = matmul_raw(A, B, wrap).reshape(-1).astype(np.int16)


# --------------------------------------------------------------------------- Conv
CONV_TILE_IC = 16           # platforms/kv260.json kernels.conv.tile_ic


def conv_raw(x: np.ndarray, w: np.ndarray, bias: Optional[np.ndarray], stride_h: int, stride_w: int,
             pad_top: int, pad_left: int, dil_h: int, dil_w: int, out_h: int, out_w: int,
             depthwise: bool, wrap: bool = False) -> np.ndarray:
    """y = sat16(floor((bias << 8 + sum x w) / 2^8)) on raw NCHW x and raw
    weights w [M][C][kh][kw] ([C][1][kh][kw] depthwise), zero padding — the
    exact sum of S:121-197 (Q8.8) / S:198-220 + S:784-812 (exponents, with
    ``wrap``) and HE:393-455."""
    x = np.asarray(x, np.int64)
    w = np.asarray(w, np.int64)
    N, C, H, W = x.shape
    M, _, kh, kw = w.shape
    need_h = (out_h - 1) * stride_h + (kh - 1) * dil_h + 1
    need_w = (out_w - 1) * stride_w + (kw - 1) * dil_w + 1
    xp = np.zeros((N, C, max(need_h, pad_top + H), max(need_w, pad_left + W)), np.float64)
    xp[:, :, pad_top:pad_top + H, pad_left:pad_left + W] = x
    acc = np.zeros((N, M, out_h, out_w), np.float64)
    wf = w.astype(np.float64)
    for i in range(kh):
        for j in range(kw):
            xs = xp[:, :, i * dil_h: i * dil_h + (out_h - 1) * stride_h + 1: stride_h,
                    j * dil_w: j * dil_w + (out_w - 1) * stride_w + 1: stride_w]
            if depthwise:
                acc += xs * wf[:, 0, i, j][None, :, None, None]
            else:
                acc += np.einsum("nchw,mc->nmhw", xs, wf[:, :, i, j], optimize=True)
    acc = acc.astype(np.int64)
    if bias is not None:
        acc = acc + (np.asarray(bias, np.int64).reshape(1, -1, 1, 1) << 8)
    if wrap:
        acc = wrap32(acc)
    return sat16(floor_shr(acc, 8))


def conv_weight_index(out_ch: int, in_ch: int, kh: int, kw: int, depthwise: bool,
                      tile_ic: int = CONV_TILE_IC) -> np.ndarray:
    """Offsets of logical w[m][c][i][j] in the board's packed image (HE:398-426,
    nodes.py:1112-1151): standard [M][ceil(C/T)][kh][kw][lanes] with lanes = T
    (the last IC tile 8 wide when it holds <= 8 channels); depthwise
    [M][roundup(kh kw, 8)]."""
    KK = kh * kw
    if depthwise:
        per_m = (KK + 7) // 8 * 8
        m = np.arange(out_ch)[:, None, None, None]
        t = np.arange(kh)[None, None, :, None] * kw + np.arange(kw)[None, None, None, :]
        return m * per_m + t + np.zeros((1, 1, 1, 1), np.int64)
    T = tile_ic
    tiles = (in_ch + T - 1) // T
    last = 8 if in_ch - (tiles - 1) * T <= 8 else T
    per_m = KK * ((tiles - 1) * T + last)
    m = np.arange(out_ch)[:, None, None, None]
    c = np.arange(in_ch)[None, :, None, None]
    ict = c // T
    lanes = np.where(ict + 1 == tiles, last, T)
    tap = np.arange(kh)[None, None, :, None] * kw + np.arange(kw)[None, None, None, :]
    return m * per_m + ict * KK * T + tap * lanes + c % T


def conv_job(x: np.ndarray, wimg: np.ndarray, bimg: Optional[np.ndarray], y: np.ndarray, *, batch, in_ch, in_h,
             in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left,
             has_bias, is_depthwise, y_cs=0, y_cn=0, y_gs=0, wrap=False) -> None:
    """One ConvKernel job from board images (HE:393-455): packed weights,
    word-padded bias, NCHW x; output channel m placed at the y channel
    pattern (m mod y_cn) * y_cs + (m div y_cn) * y_gs (dense when 0)."""
    if (y_cn % 16) != 0 or y_cn > 1280 or ((y_cs or y_cn) and batch != 1):
        return
    wi = conv_weight_index(out_ch, in_ch, kh, kw, bool(is_depthwise))
    w = np.asarray(wimg, np.int64)[wi]
    xx = np.asarray(x[: batch * in_ch * in_h * in_w], np.int64).reshape(batch, in_ch, in_h, in_w)
    b = np.asarray(bimg[:out_ch], np.int64) if has_bias else None
    yy = conv_raw(xx, w, b, stride_h, stride_w, pad_top, pad_left, dilation_h, dilation_w, out_h, out_w,
                  bool(is_depthwise), wrap)
    P = out_h * out_w
    CS = y_cs if y_cs else P
    for n in range(batch):
        for m in range(out_ch):
            yb = n * out_ch * P + ((m % y_cn) * CS + (m // y_cn) * y_gs if y_cn else m * CS)
            y[yb: yb + P] = yy[n, m].reshape(-1).astype(np.int16)


# --------------------------------------------------------------------------- Pool
POOL_MAX, POOL_AVG, POOL_LP = 0, 1, 2


def _trn(v: float, bits: int) -> int:
    """raw of floor(v * 2^bits) (S:223-227 _quantize_trn)."""
    return int(math.floor(v * (1 << bits)))


# The kernel's poly_sqrt coefficients at ap_fixed<16,1> (S:257-261), as raw 2^-15.
POLY_C = (_trn(0.4434, 15), _trn(0.6432, 15), _trn(-0.0943, 15), _trn(0.0077, 15))


def poly_sqrt_q16(A: np.ndarray) -> np.ndarray:
    """S:230-272 restated on integers: A = sum x^2 in 2^-16 units (>= 0); the
    result in 2^-16 units.  Range reduction a = m 4^k with m in [1, 4) taken
    at 16 fractional bits (floor), Horner with floors at 20 bits, 2^k, floor
    at 16 bits."""
    A = np.asarray(A, np.int64)
    out = np.zeros_like(A)
    pos = A > 0
    if not pos.any():
        return out
    a = A[pos]
    b = np.floor(np.log2(a.astype(np.float64))).astype(np.int64)
    # exact bit length correction (log2 of large ints may round up)
    b = np.where((np.int64(1) << b) > a, b - 1, b)
    b = np.where((np.int64(1) << (b + 1)) <= a, b + 1, b)
    k = (b - 16) // 2                                   # floor
    Mq = np.where(k <= 0, a << np.maximum(-2 * k, 0), a >> np.maximum(2 * k, 0))
    c0, c1, c2, c3 = POLY_C
    T1 = (c3 * Mq + (c2 << 16)) >> 11                   # 2^-20
    T2 = (T1 * Mq + (c1 << 21)) >> 16
    S = (T2 * Mq + (c0 << 21)) >> 16                    # sqrt(m) at 2^-20
    out[pos] = np.where(k >= 4, S << np.maximum(k - 4, 0), S >> np.maximum(4 - k, 0))
    return out


def pool_raw(x: np.ndarray, pool_h: int, pool_w: int, stride_h: int, stride_w: int, pad_top: int, pad_left: int,
             dil_h: int, dil_w: int, out_h: int, out_w: int, pool_type: int, lp_order: int,
             count_include_pad: int) -> np.ndarray:
    """PoolingKernel on raw NCHW int16 x (S:275-358): MAX (an all-padding
    window gives -32768), AVG as sum * round(2^23 / d) >> 23 (floor), LP1
    sum |x|, LP2 poly_sqrt(sum x^2); then floor + sat16."""
    x = np.asarray(x, np.int64)
    N, C, H, W = x.shape
    y = np.zeros((N, C, out_h, out_w), np.int64)
    for oh in range(out_h):
        for ow in range(out_w):
            taps = []
            for i in range(pool_h):
                for j in range(pool_w):
                    ih = oh * stride_h + i * dil_h - pad_top
                    iw = ow * stride_w + j * dil_w - pad_left
                    if 0 <= ih < H and 0 <= iw < W:
                        taps.append(x[:, :, ih, iw])
            if pool_type == POOL_MAX:
                y[:, :, oh, ow] = np.max(np.stack(taps), axis=0) if taps else I16_LO
                continue
            d = max(pool_h * pool_w if count_include_pad else len(taps), 1)
            if pool_type == POOL_AVG:
                s = np.sum(np.stack(taps), axis=0) if taps else np.zeros((N, C), np.int64)
                inv = ((1 << 23) + d // 2) // d
                y[:, :, oh, ow] = (s * inv) >> 23
            elif lp_order == 1:
                y[:, :, oh, ow] = np.sum(np.abs(np.stack(taps)), axis=0) if taps else 0
            else:
                s2 = np.sum(np.stack(taps) ** 2, axis=0) if taps else np.zeros((N, C), np.int64)
                y[:, :, oh, ow] = poly_sqrt_q16(s2) >> 8
    return sat16(y)


# --------------------------------------------------------------------------- RowOps
RO_COPY, RO_ADDX, RO_DEQUANT, RO_MULACT, RO_NORM, RO_ROPE, RO_XPOSE, RO_TLOAD, RO_FOLD, RO_GATE = range(1, 11)
K_I16, K_I32, K_F32 = 0, 1, 2
F_B_EN, F_P_BCAST, F_P_KEEP, F_RELU, F_NORM_LN, F_SCALE = 1 << 12, 1 << 13, 1 << 14, 1 << 15, 1 << 16, 1 << 17
P1_BITS, RM_BITS, G_BITS, SIG_BITS, SIG_STEP, SIG_N, SILU_BITS = 24, 47, 14, 24, 8, 4096, 20


@lru_cache(maxsize=None)
def rsqrt_table() -> np.ndarray:
    """y0[i] = rint(2^47 / sqrt((i + 0.5) 2^19)) for i in [2048, 8192), 0 below
    (RS:91-101, RR:122-133)."""
    idx = np.arange(8192, dtype=np.float64)
    with np.errstate(divide="ignore"):
        y = np.rint(2.0 ** RM_BITS / np.sqrt((idx + 0.5) * 2.0 ** 19))
    y[:2048] = 0
    return np.minimum(y, 2.0 ** 32 - 1).astype(np.int64)


@lru_cache(maxsize=None)
def sigmoid_table() -> np.ndarray:
    """T[i] = round(2^24 / (1 + exp(-i / 256))), i = 0 .. 4096 (RS:337-342)."""
    return np.array([round(2.0 ** SIG_BITS / (1.0 + math.exp(-i / 2.0 ** SIG_STEP))) for i in range(SIG_N + 1)],
                    dtype=np.int64)


def table_image() -> bytes:
    """The 64 KiB OP_TLOAD image (RS:603-616): 4096 sigmoid entries
    {(T[i+1]-T[i]) << 25 | T[i]} as u64, then 8192 rsqrt entries as u32."""
    T = sigmoid_table()
    R = rsqrt_table()
    img = np.zeros(65536, np.uint8)
    d = (T[1:] - T[:-1]) & 0xFFFFFF
    words = ((d.astype(np.uint64) << np.uint64(25)) | (T[:-1].astype(np.uint64) & np.uint64(0x1FFFFFF)))
    img[:32768] = words.astype("<u8").view(np.uint8)
    img[32768:] = (R & 0xFFFFFFFF).astype("<u4").view(np.uint8)
    return img.tobytes()


def rsqrt_bf(D: int) -> Tuple[int, int]:
    """1/sqrt(D) ~ Rm 2^-sh: table on the leading 13 bits of the
    block-floated D, one Newton step in 32-bit integers (RS:104-121)."""
    D = int(D)
    e = D.bit_length()
    d = e - 32
    if d & 1:
        d += 1
    Dm = D >> d if d >= 0 else D << (-d)
    y0 = int(rsqrt_table()[Dm >> 19])
    t = (Dm * y0) >> 32
    u = (t * y0) >> 32
    y1 = y0 + ((y0 * ((1 << 30) - u)) >> 31)
    return min(max(y1, 1 << 31), (1 << 32) - 1), RM_BITS + d // 2


def sig_q(gv: int) -> int:
    """sigma(g) at 2^-24 for g = gv 2^-14, interpolated table (RS:345-358)."""
    T = sigmoid_table()
    a = abs(gv)
    big = a >= (16 << G_BITS)
    ai = min(a, (16 << G_BITS) - 1)
    idx, frac = ai >> (G_BITS - SIG_STEP), ai & ((1 << (G_BITS - SIG_STEP)) - 1)
    s = int(T[idx]) + (((int(T[idx + 1]) - int(T[idx])) * frac) >> (G_BITS - SIG_STEP))
    if big:
        s = 1 << SIG_BITS
    return (1 << SIG_BITS) - s if gv < 0 else s


def _rne(v: int, k: int) -> int:
    if k <= 0:
        return v << (-k)
    q = v >> k
    r = v - (q << k)
    h = 1 << (k - 1)
    return q + (1 if (r > h or (r == h and (q & 1))) else 0)


def silu_q(gv: int) -> int:
    """silu(g) at 2^-20 (RS:361-364)."""
    return _rne(gv * sig_q(gv), G_BITS + SIG_BITS - SILU_BITS)


def float_bits(v: int, sh_c: int) -> int:
    """IEEE float32 bits of v 2^-sh_c, round to nearest even (RR:190-203)."""
    if v == 0:
        return 0
    neg = v < 0
    mag = -v if neg else v
    lz = mag.bit_length() - 1
    norm = mag >> (lz - 31) if lz >= 31 else mag << (31 - lz)
    m24 = norm >> 8
    if (norm & 0x80) and ((norm & 0x7F) or (norm & 0x100)):
        m24 += 1
    exp = 127 + lz - sh_c + ((m24 >> 24) & 1)
    return ((1 if neg else 0) << 31) | ((exp & 0xFF) << 23) | (m24 & 0x7FFFFF)


def _s32(u: int) -> int:
    u &= 0xFFFFFFFF
    return u - (1 << 32) if u & 0x80000000 else u


class RowOpsMem:
    """A flat little-endian byte memory for row-ops jobs (addresses are byte
    offsets into ``buf``)."""

    def __init__(self, buf: np.ndarray):
        self.buf = buf

    def rd8(self, a):
        return int(self.buf[a])

    def rd16(self, a):
        v = int(self.buf[a]) | (int(self.buf[a + 1]) << 8)
        return v - 65536 if v & 0x8000 else v

    def rd32(self, a):
        return _s32(int(self.buf[a]) | (int(self.buf[a + 1]) << 8) | (int(self.buf[a + 2]) << 16)
                    | (int(self.buf[a + 3]) << 24))

    def elem(self, a, kind):
        return self.rd16(a) if kind == K_I16 else self.rd32(a)

    def wr(self, a, data: bytes):
        self.buf[a:a + len(data)] = np.frombuffer(data, np.uint8)


def _param(mem: RowOpsMem, p: int, c: int, bcast: bool):
    """One column's parameter entry (RR:207-217): int32 G, int22 Bq', u8 shifts."""
    a = p + 16 * (0 if bcast else c)
    g = mem.rd32(a)
    bq = _s32((mem.rd32(a + 4) << 10) & 0xFFFFFFFF) >> 10
    return g, bq, mem.rd8(a + 8) & 63, mem.rd8(a + 9) & 63, mem.rd8(a + 10) & 63


def _row_bytes(vals, kind) -> bytes:
    nb = 2 if kind == K_I16 else 4
    out = bytearray()
    for v in vals:
        out += (int(v) & ((1 << (8 * nb)) - 1)).to_bytes(nb, "little")
    while len(out) % 16:
        out.append(0)
    return bytes(out)


def _fold_elem(x: int, m: int, s: int) -> int:
    u = -x if x < 0 else x
    den = (m if x < 0 else 1) << s
    q, r = divmod(u, den)
    q += 1 if (2 * r > den or (2 * r == den and (q & 1))) else 0
    return -q if x < 0 else q


class ParamRAM:
    """The unit's parameter RAM between jobs (RR:86-95): column c's entry at
    ram[c], or with a broadcast load every column reads entry 0 (the load
    writes index 0 of all four banks); ``valid`` once a job has loaded."""

    def __init__(self):
        self.ram = [(0, 0, 0, 0, 0)] * 4096
        self.valid = False
        self.bcast = False

    def at(self, c: int):
        return self.ram[(c & 3) if self.bcast else c]


def rowops_job(mem: RowOpsMem, op: int, n: int, c1: int, c2: int, a: int, a_s1: int, a_s2: int, b: int,
               b_s1: int, b_s2: int, c: int, c_s1: int, c_s2: int, p: int, eps: int = 0, aux: int = 0,
               bq_sh: int = 0, win_lo: int = 0, win_hi: int = 0xFFFFFFFF, ps: Optional[ParamRAM] = None) -> None:
    """One RowOpsKernel job on ``mem`` (RR:259-427, HE:611-730).  ``ps``: the
    parameter RAM carried between the jobs of a chain (RR:262-276) — a job
    with work loads it from p unless it is P_KEEP (and the RAM holds a load),
    and a P_KEEP job reads it; without ``ps`` a P_KEEP job reads p."""
    code = op & 15
    if code == RO_TLOAD:
        return
    ak, bk, ck = (op >> 4) & 3, (op >> 6) & 3, (op >> 8) & 3
    ben, bcast, relu, ln, scale = op & F_B_EN, op & F_P_BCAST, op & F_RELU, op & F_NORM_LN, op & F_SCALE
    eps = eps - (1 << 64) if eps & (1 << 63) else eps
    if code == RO_FOLD:
        sh, dv = aux & 15, (aux >> 4) & 127
        if n == 0 or c1 == 0 or c2 == 0 or dv == 0:
            return
        vals = []
        for k in range(c2):
            for r in range(c1):
                for cc in range(n):
                    col = _s32(b_s2) + r * b_s1 + cc
                    y = 0
                    if win_lo <= col < win_hi:
                        y = _fold_elem(mem.rd16(a + k * _s32(a_s2) + 2 * col), dv, sh)
                    vals.append(y)
        mem.wr(c, _row_bytes(vals, K_I16))
        return
    if n == 0 or c1 == 0 or c2 == 0 or n > 4096:
        return
    nb = lambda kd: 2 if kd == K_I16 else 4  # noqa: E731
    keep = bool(op & F_P_KEEP) and ps is not None and ps.valid
    if code in (RO_COPY, RO_ADDX, RO_DEQUANT, RO_MULACT, RO_GATE, RO_NORM, RO_ROPE) and keep:
        prm = ps.at
    else:
        P = [_param(mem, p, cc, bool(bcast)) for cc in range(1 if bcast else n)]
        prm = (lambda cc: P[0]) if bcast else (lambda cc: P[cc])
        if ps is not None and code in (RO_COPY, RO_ADDX, RO_DEQUANT, RO_MULACT, RO_GATE, RO_NORM, RO_ROPE):
            ram = list(ps.ram)
            if bcast:
                ram[0:4] = [P[0]] * 4
            else:
                ram[0:n] = P
            ps.ram, ps.valid, ps.bcast = ram, True, bool(bcast)
    for i2 in range(c2):
        for i1 in range(c1):
            ra, rb, rc = a + i2 * a_s2 + i1 * a_s1, b + i2 * b_s2 + i1 * b_s1, c + i2 * c_s2 + i1 * c_s1
            if code in (RO_COPY, RO_ADDX, RO_DEQUANT, RO_MULACT, RO_GATE):
                zero_a = code in (RO_COPY, RO_ADDX) and (i1 < win_lo or i1 >= win_hi)
                vals = []
                for cc in range(n):
                    g, bq, sa, sb, sc = prm(cc)
                    x = 0 if zero_a else mem.elem(ra + nb(ak) * cc, ak)
                    y = mem.elem(rb + nb(bk) * cc, bk) if (ben and code != RO_DEQUANT) else 0
                    if code in (RO_COPY, RO_ADDX):
                        s = (x << sa) + (y << sb) + (bq << bq_sh)
                        v = _rne(s * g if scale else s, sc)
                        r = max(min(v, I16_HI), I16_LO) if ck == K_I16 else max(min(v, I32_HI), I32_LO)
                        if relu and r < 0:
                            r = 0
                    elif code == RO_DEQUANT:
                        r = float_bits(x, sc)
                    elif code == RO_GATE:
                        th = 2 * sig_q(x << sa) - (1 << SIG_BITS)
                        r = max(min(_rne(th * sig_q(y << sb), sc), I16_HI), I16_LO)
                    else:
                        r = max(min(_rne(silu_q(x << sa) * y, sc), I16_HI), I16_LO)
                    vals.append(r)
                mem.wr(rc, _row_bytes(vals, ck))
            elif code == RO_NORM:
                xs = [mem.elem(ra + nb(ak) * cc, ak) for cc in range(n)]
                S1 = sum(xs)
                S2 = sum(v * v for v in xs)
                D = (n * S2 - S1 * S1 + eps) if ln else (S2 + eps)
                if D <= 0:
                    D = 1
                Rm, sh = rsqrt_bf(D)
                vals = []
                for cc in range(n):
                    g, bq, sa, sb, sc = prm(cc)
                    A = (n * xs[cc] - S1) if ln else xs[cc]
                    P1 = (A * Rm) >> (sh - P1_BITS)
                    vals.append(max(min(_rne(P1 * g + (bq << bq_sh), sc), I16_HI), I16_LO))
                mem.wr(rc, _row_bytes(vals, K_I16))
            elif code == RO_ROPE:
                HD = aux & 0xFFF
                half = HD // 2
                if HD == 0 or (HD & 15) or HD > 128 or n % HD:
                    return
                xs = [mem.rd16(ra + 2 * cc) for cc in range(n)]
                vals = []
                for cc in range(n):
                    g, bq, sa, sb, sc = prm(cc)
                    d = cc % HD
                    cs_, sn = mem.rd32(rb + 4 * d), mem.rd32(rb + 4 * (HD + d))
                    rot = -xs[cc + half] if d < half else xs[cc - half]
                    s = ((xs[cc] * cs_) << sa) + ((rot * sn) << sb)
                    vals.append(max(min(_rne(s, sc), I16_HI), I16_LO))
                mem.wr(rc, _row_bytes(vals, K_I16))
            elif code == RO_XPOSE:
                R, L = aux & 15, n
                if R == 0 or R > 8:
                    return
                if b_s2 == 2 * R:
                    vals = [mem.rd16(ra + r * b_s1 + 2 * d) for d in range(L) for r in range(R)]
                    mem.wr(rc, _row_bytes(vals, K_I16))
                else:
                    for d in range(L):
                        vals = [mem.rd16(ra + r * b_s1 + 2 * d) for r in range(R)]
                        mem.wr(rc + d * b_s2, b"".join((v & 0xFFFF).to_bytes(2, "little") for v in vals))


# --------------------------------------------------------------------------- LayerNorm rows (BERT)
def ln_gamma_scale(gamma: np.ndarray) -> int:
    """g with max |round(gamma 2^g)| < 2^31: 30 - floor(log2 max|gamma|) (RS:125-130)."""
    m = float(np.abs(np.asarray(gamma, np.float64)).max())
    return 0 if m == 0.0 else 30 - int(math.floor(math.log2(m)))


def ln_beta_bits(beta: np.ndarray) -> int:
    """bb <= 20 with |round(beta 2^bb)| < 2^21 (RS:133-143)."""
    m = float(np.abs(np.asarray(beta, np.float64)).max()) if np.size(beta) else 0.0
    bb = 20
    while bb > 0 and abs(round(m * 2.0 ** bb)) >= (1 << 21):
        bb -= 1
    return bb


def layer_norm_rows(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float, f_x: int = 8,
                    f_out: int = 8) -> np.ndarray:
    """LayerNorm of int rows [rows][n] at 2^-f_x to int16 at 2^-f_out, the
    unit's integer datapath (RS:206-223 norm_params, RS:259-282 layer_norm;
    RR NORM): exact S1, S2; D = n S2 - S1^2 + E (1 if <= 0); rsqrt_bf(D) =
    Rm 2^-sh; P1 = floor((n x - S1) Rm / 2^(sh-24)); out = sat16(rne((P1 G +
    Bq) / 2^(24+g-f_out))) with G = rint(gamma 2^g), Bq = rint(beta 2^bb) <<
    (24+g-bb), E = rint(eps n^2 2^(2 f_x)).  int64 throughout where the
    bounds allow, Python integers per row where they do not."""
    x = np.asarray(x, np.int64)
    rows, n = x.shape
    gamma = np.asarray(gamma, np.float64)
    beta = np.asarray(beta, np.float64)
    g = ln_gamma_scale(gamma)
    G = np.rint(gamma * 2.0 ** g).astype(np.int64)
    bb = ln_beta_bits(beta)
    Bq = np.rint(beta * 2.0 ** bb).astype(np.int64) << (P1_BITS + g - bb)
    E = int(round(eps * n * n * 2.0 ** (2 * f_x)))
    S1 = x.sum(axis=1)
    S2 = (x * x).sum(axis=1)
    out = np.empty((rows, n), np.int64)
    sc = P1_BITS + g - f_out
    gmax = int(np.abs(G).max()) if n else 0
    bmax = int(np.abs(Bq).max()) if n else 0
    for r in range(rows):
        s1, s2 = int(S1[r]), int(S2[r])
        D = n * s2 - s1 * s1 + E
        if D <= 0:
            D = 1
        Rm, sh = rsqrt_bf(D)
        A = n * x[r] - s1
        amax = int(np.abs(A).max())
        if amax * Rm < (1 << 62) and ((amax * Rm) >> (sh - P1_BITS)) * gmax + bmax < (1 << 62):
            P1 = (A * np.int64(Rm)) >> (sh - P1_BITS)
            out[r] = sat16(rne_shr(P1 * G + Bq, sc))
        else:
            vals = [((int(a) * Rm) >> (sh - P1_BITS)) * int(gg) + int(bq) for a, gg, bq in zip(A, G, Bq)]
            out[r] = [max(min(_rne(v, sc), I16_HI), I16_LO) for v in vals]
    return out
