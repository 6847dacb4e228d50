"""Per-op host API over the C ABI: one function per kernel, taking torch CUDA
tensors (the buffers) and the register values, launched on the current torch
stream.  These are the calls the reference's generated ``run_op`` /
``run_matmul`` / ``run_conv`` / ``run_pool`` / ``run_softmax`` /
``run_rowops`` make (phoenix367/cormorant inference-scheduler/src/codegen/
_source.py:1112-1580), with device tensors in place of DMA buffers.

Errors: a descriptor the kernel's contract rejects raises ``CormError``
(nothing launched), as the reference raises ``SchedulerError`` /
``ValueError`` before emitting a call.
"""
from __future__ import annotations

import ctypes as C
import threading

import torch

from . import _lib
from ._lib import CormError, check, lib  # noqa: F401

_tls = threading.local()


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise CormError(_lib.CORM_EINVAL, "operand is not a CUDA tensor (the library has no CPU path)")
    return t.data_ptr()


def _ready() -> int:
    """Bind the library's runtime to torch's current device (once per thread
    and device) and return the current stream handle."""
    dev = torch.cuda.current_device()
    if getattr(_tls, "dev", None) != dev:
        check(lib().corm_bind_device(dev))
        _tls.dev = dev
    return torch.cuda.current_stream().cuda_stream


def _i16(t, name):
    if t is not None and t.dtype != torch.int16:
        raise CormError(_lib.CORM_EINVAL, f"{name} must be int16, got {t.dtype}")


def vectorop(a, b, c, *, size, op, outer=1, a_inc=0, b_inc=0, act=0, alpha=0, smx_cm=0, smx_cfg=0, smx_mask=0):
    """One VectorOPKernel job (host_emu.py:244-293): element offsets from the
    tensors' data pointers."""
    for t, n in ((a, "a"), (b, "b"), (c, "c")):
        _i16(t, n)
    st = _ready()
    d = _lib.VectorOpDesc(_ptr(a), _ptr(b), _ptr(c), size, op, outer, a_inc, b_inc, act, alpha & 0xFFFFFFFF,
                          smx_cm, smx_cfg, smx_mask)
    check(lib().corm_vectorop(C.byref(d), st))


def _post(post):
    """corm_postop from dict(b=tensor, op, act=0, alpha=0, b_mode=0, b_is_first=0)."""
    if post is None:
        return None
    _i16(post["b"], "post b")
    return _lib.PostOp(_ptr(post["b"]), post["op"], post.get("act", 0), post.get("alpha", 0) & 0xFFFFFFFF,
                       post.get("b_mode", 0), int(bool(post.get("b_is_first", 0))))


def matmul(a, b, c, *, n, k, m, batch=1, a_batch_stride=0, b_batch_stride=0, c_batch_stride=0, b_packed=0,
           gemv_kw=0, flags=0, workspace=None, post=None):
    """One MatmulKernel job (host_emu.py:338-362).  ``workspace``: a uint8
    CUDA tensor, or None to take one from torch's allocator.  ``post``: a
    VectorOP job fused onto the result (corm_matmul_post), a dict with keys b
    (int16 tensor), op, act, alpha, b_mode, b_is_first."""
    for t, nm in ((a, "a"), (b, "b"), (c, "c")):
        _i16(t, nm)
    st = _ready()
    d = _lib.MatmulDesc(_ptr(a), _ptr(b), _ptr(c), n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride,
                        b_packed, gemv_kw, flags, None, 0)
    need = C.c_size_t(0)
    check(lib().corm_matmul_workspace_size(C.byref(d), C.byref(need)))
    if need.value:
        if workspace is None:
            workspace = torch.empty(need.value, dtype=torch.uint8, device=a.device)
        d.workspace, d.workspace_bytes = _ptr(workspace), workspace.numel() * workspace.element_size()
    q = _post(post)
    if q is None:
        check(lib().corm_matmul(C.byref(d), st))
    else:
        check(lib().corm_matmul_post(C.byref(d), C.byref(q), st))
    return workspace


def _groups(outs, widths, mulact):
    g = _lib.OutGroups(len(outs), (C.c_uint32 * 4)(*(list(widths) + [0] * (4 - len(widths)))),
                       (C.c_void_p * 4)(*([_ptr(t) for t in outs] + [None] * (4 - len(outs)))))
    if mulact is not None:
        g.mulact, g.ma_sa, g.ma_sc = 1, int(mulact[0]), int(mulact[1])
    return g


def matmul_groups(a, b, outs, widths, *, n, k, batch=1, a_batch_stride=0, b_batch_stride=0, flags=0,
                  workspace=None, mulact=None):
    """One MatMul job over B = [k][sum(widths)] whose output columns go to
    several buffers (corm_matmul_groups): outs[g] receives the widths[g]
    columns of group g, row-major [batch][n][widths[g]].  Sibling projections
    that read the same A run as one launch; n > 2, all widths but the last
    multiples of 32.  ``mulact`` = (sa, sc): B's columns are gate / up pairs
    of 16-column blocks and outs[0] (one output, widths[0] = m / 2) receives
    their row-ops MULACT (SiLU(g << sa) u rounded at sc)."""
    for t, nm in ((a, "a"), (b, "b")):
        _i16(t, nm)
    if not 1 <= len(outs) == len(widths) <= 4:
        raise CormError(_lib.CORM_EINVAL, "matmul_groups: 1..4 outputs, one width each")
    for t in outs:
        _i16(t, "out")
    st = _ready()
    m = int(sum(widths)) * (2 if mulact is not None else 1)
    d = _lib.MatmulDesc(_ptr(a), _ptr(b), _ptr(outs[0]), n, k, m, batch, a_batch_stride, b_batch_stride,
                        n * widths[0], 0, 0, flags, None, 0)
    need = C.c_size_t(0)
    check(lib().corm_matmul_workspace_size(C.byref(d), C.byref(need)))
    if need.value:
        if workspace is None:
            workspace = torch.empty(need.value, dtype=torch.uint8, device=a.device)
        d.workspace, d.workspace_bytes = _ptr(workspace), workspace.numel() * workspace.element_size()
    g = _groups(outs, widths, mulact)
    check(lib().corm_matmul_groups(C.byref(d), C.byref(g), st))
    return workspace


def split_b_planes(b, *, k, m):
    """corm_split_b_planes: the int8 hi / lo planes (MN-major [k][mp], mp = m
    rounded up to 16) of a constant row-major int16 weight [k][m], for
    matmul_bplanes."""
    _i16(b, "b")
    st = _ready()
    mp = (m + 15) // 16 * 16
    hi = torch.empty(k * mp, dtype=torch.int8, device=b.device)
    lo = torch.empty(k * mp, dtype=torch.uint8, device=b.device)
    check(lib().corm_split_b_planes(_ptr(b), k, m, _ptr(hi), _ptr(lo), st))
    return hi, lo


def matmul_bplanes(a, planes, c, *, n, k, m, batch=1, a_batch_stride=0, c_batch_stride=0, flags=0, workspace=None,
                   outs=None, widths=None, mulact=None):
    """A MatMul job against a weight given as its planes (split_b_planes):
    the GEMM splits only A.  ``outs`` / ``widths``: output column groups
    instead of c (as matmul_groups); ``mulact``: gate / up pairs (as
    matmul_groups)."""
    _i16(a, "a")
    st = _ready()
    d = _lib.MatmulDesc(_ptr(a), None, _ptr(c) if c is not None else None, n, k, m, batch, a_batch_stride, 0,
                        c_batch_stride, 0, 0, flags, None, 0)
    need = C.c_size_t(0)
    check(lib().corm_matmul_workspace_size(C.byref(d), C.byref(need)))
    if need.value:
        if workspace is None:
            workspace = torch.empty(need.value, dtype=torch.uint8, device=a.device)
        d.workspace, d.workspace_bytes = _ptr(workspace), workspace.numel() * workspace.element_size()
    g = None
    if outs is not None:
        g = _groups(outs, widths, mulact)
    check(lib().corm_matmul_bplanes(C.byref(d), _ptr(planes[0]), _ptr(planes[1]), C.byref(g) if g is not None else None,
                                    st))
    return workspace


def gemm_strided(a, b, c, *, n, k, m, batch=1, lda=None, ldb=None, ldc=None, b_trans=False, a_batch_stride=0,
                 b_batch_stride=0, c_batch_stride=0, flags=0, workspace=None):
    """A strided batch of MatMul jobs (corm_gemm_strided): element row strides
    lda / ldb / ldc (default dense), batch strides (0 shares the operand), B
    transposed ([m][k]) with ``b_trans``."""
    for t, nm in ((a, "a"), (b, "b"), (c, "c")):
        _i16(t, nm)
    st = _ready()
    lda = k if lda is None else lda
    ldb = (k if b_trans else m) if ldb is None else ldb
    ldc = m if ldc is None else ldc
    d = _lib.GemmDesc(_ptr(a), _ptr(b), _ptr(c), n, k, m, batch, lda, ldb, ldc, int(bool(b_trans)), a_batch_stride,
                      b_batch_stride, c_batch_stride, flags, None, 0)
    need = C.c_size_t(0)
    check(lib().corm_gemm_strided_workspace_size(C.byref(d), C.byref(need)))
    if need.value:
        if workspace is None or workspace.numel() * workspace.element_size() < need.value:
            workspace = torch.empty(need.value, dtype=torch.uint8, device=a.device)
        d.workspace, d.workspace_bytes = _ptr(workspace), workspace.numel() * workspace.element_size()
    check(lib().corm_gemm_strided(C.byref(d), st))
    return workspace


def copy_nd(src, dst, dims, src_strides, dst_strides, *, src_off=0, dst_off=0):
    """dst[dst_off + sum x_i dst_strides[i]] = src[src_off + sum x_i
    src_strides[i]] over the index box ``dims`` (<= 6 dims, element strides)."""
    _i16(src, "src")
    _i16(dst, "dst")
    nd = len(dims)
    if not 1 <= nd <= 6 or len(src_strides) != nd or len(dst_strides) != nd:
        raise ValueError("copy_nd: 1..6 dims with one stride each")
    st = _ready()
    pad = lambda v, f: list(v) + [f] * (6 - nd)  # noqa: E731
    d = _lib.CopyDesc(_ptr(src) + 2 * src_off, _ptr(dst) + 2 * dst_off, nd, (C.c_uint32 * 6)(*pad(dims, 1)),
                      (C.c_int64 * 6)(*pad(src_strides, 0)), (C.c_int64 * 6)(*pad(dst_strides, 0)))
    check(lib().corm_copy_nd(C.byref(d), st))


def llm_attn_softmax(s, p, tab, ip, *, pos, n, T, G, rows, Q=16, window=0, batch=1, s_stride=None, p_stride=None):
    """The host's p12 softmax of one KV group (corm_llm_attn_softmax): scores
    s [rows][s_stride] int16 (rows = the cache rows C), P rows of ``rows``
    entries at p_stride, tab float64 [G][65536], ip float64 [G] (2^f_p per
    head)."""
    _i16(s, "s")
    _i16(p, "p")
    if tab.dtype != torch.float64 or ip.dtype != torch.float64:
        raise CormError(_lib.CORM_EINVAL, "tab / ip must be float64")
    st = _ready()
    d = _lib.LlmSmxDesc(_ptr(s), _ptr(p), _ptr(tab), _ptr(ip), pos, n, T, G, rows, Q, window, batch,
                        batch * G * T if s_stride is None else s_stride, rows if p_stride is None else p_stride)
    check(lib().corm_llm_attn_softmax(C.byref(d), st))


def _dtype(t, dt, name):
    if t.dtype != dt or not t.is_cuda:
        raise CormError(_lib.CORM_EINVAL, f"{name}: a CUDA {dt} tensor expected, got {t.dtype} on {t.device}")


def llm_embed(ids, table, out, *, n, rows, d, res32=False, f=0, scale=1.0):
    """LlmEmbed (corm_llm_embed): out [n][d] float32 rows, or the int32
    residual at 2^-f (res32), of table [rows][d] float32 at ids (int32)."""
    _dtype(ids, torch.int32, "ids")
    _dtype(table, torch.float32, "table")
    _dtype(out, torch.int32 if res32 else torch.float32, "out")
    st = _ready()
    check(lib().corm_llm_embed(C.byref(_lib.LlmEmbedDesc(_ptr(ids), _ptr(table), _ptr(out), n, rows, d, int(res32), f,
                                                        float(scale))), st))


def llm_dequant(x, y, f, *, count, n):
    """LlmDequant (corm_llm_dequant): y float32 = x 2^-f[c], f int8 [n]."""
    _i16(x, "x")
    _dtype(y, torch.float32, "y")
    _dtype(f, torch.int8, "f")
    st = _ready()
    check(lib().corm_llm_dequant(C.byref(_lib.LlmDequantDesc(_ptr(x), _ptr(y), _ptr(f), count, n)), st))


def llm_resadd(h, d, y, fd, *, rows, n):
    """LlmResAdd on the float32 residual (corm_llm_resadd)."""
    _dtype(h, torch.float32, "h")
    _i16(d, "d")
    _dtype(y, torch.float32, "y")
    _dtype(fd, torch.int8, "fd")
    st = _ready()
    check(lib().corm_llm_resadd(C.byref(_lib.LlmResAddDesc(_ptr(h), _ptr(d), _ptr(y), _ptr(fd), rows, n)), st))


def llm_rmsnorm(h, y, gamma, fy, *, rows, n, W, eps, fh=None):
    """LlmRMSNorm (corm_llm_rmsnorm): h float32 rows of n, or int16 rows of W
    at fh (int8 [W]); y int16 at fy (int8 [W]); rows = rows of n."""
    _i16(y, "y")
    _dtype(gamma, torch.float32, "gamma")
    _dtype(fy, torch.int8, "fy")
    if h.dtype == torch.float32:
        h32, h16, fhp = _ptr(h), None, None
    else:
        _i16(h, "h")
        _dtype(fh, torch.int8, "fh")
        h32, h16, fhp = None, _ptr(h), _ptr(fh)
    st = _ready()
    check(lib().corm_llm_rmsnorm(C.byref(_lib.LlmRMSNormDesc(h32, h16, fhp, _ptr(y), _ptr(gamma), _ptr(fy), float(eps),
                                                            rows, n, W)), st))


def llm_act_mul(g, u, y, tab, tab_of, fu, fy, *, rows, n):
    """LlmSiluMul / LlmGeluMul (corm_llm_act_mul): tab float64 [tables][65536],
    tab_of uint8 [n], fu / fy int8 [n]."""
    for t, nm in ((g, "g"), (u, "u"), (y, "y")):
        _i16(t, nm)
    _dtype(tab, torch.float64, "tab")
    _dtype(tab_of, torch.uint8, "tab_of")
    _dtype(fu, torch.int8, "fu")
    _dtype(fy, torch.int8, "fy")
    st = _ready()
    check(lib().corm_llm_act_mul(C.byref(_lib.LlmActMulDesc(_ptr(g), _ptr(u), _ptr(y), _ptr(tab), _ptr(tab_of),
                                                           _ptr(fu), _ptr(fy), rows, n)), st))


def llm_attn_prep_host(q0, k0, v, kc, vc, qx, cos, sin, fq0, fk0, fv, fkc, fvc, fq, *, pos, n, T, H, KV, HD, C_,
                       Q=16, batch=1, ldq=None, ldk=None, ldv=None):
    """LlmAttnPrep's host form (corm_llm_attn_prep_host) for ``batch``
    sequences: caches group-major [KV][batch][C_][HD], qx [KV][batch][HD][G T]."""
    for t, nm in ((q0, "q0"), (k0, "k0"), (v, "v"), (kc, "kc"), (vc, "vc"), (qx, "qx")):
        _i16(t, nm)
    _dtype(cos, torch.float32, "cos")
    _dtype(sin, torch.float32, "sin")
    for t, nm in ((fq0, "fq0"), (fk0, "fk0"), (fv, "fv"), (fkc, "fkc"), (fvc, "fvc"), (fq, "fq")):
        _dtype(t, torch.int8, nm)
    st = _ready()
    d = _lib.LlmPrepDesc(*[_ptr(t) for t in (q0, k0, v, kc, vc, qx, cos, sin, fq0, fk0, fv, fkc, fvc, fq)], pos, n, T,
                         H, KV, HD, C_, Q, batch, H * HD if ldq is None else ldq, KV * HD if ldk is None else ldk,
                         KV * HD if ldv is None else ldv)
    check(lib().corm_llm_attn_prep_host(C.byref(d), st))


def llm_decode_attn(qx, kc, vc, tab, ip, o, *, pos, B, KV, G, HD, rows, Q=16, window=0, o_stride=None, prep=None):
    """corm_llm_decode_attn: a decode step's q.K^T, host softmax, P.V and head
    merge of every KV group and sequence (caches of ``rows`` rows).
    ``prep``: the step's AttnPrep fused in — a dict with q0, k0, v0 (int16
    rows), ldq, ldk, ldv, rope (the int32 cos / sin table as int16 words), pq,
    pk, pv (parameter entries), pq_bc, pk_bc, pv_bc, v_direct; qx unused."""
    for t, nm in ((qx, "qx"), (kc, "kc"), (vc, "vc"), (o, "o")):
        _i16(t, nm)
    if tab.dtype != torch.float64 or ip.dtype != torch.float64:
        raise CormError(_lib.CORM_EINVAL, "tab / ip must be float64")
    st = _ready()
    d = _lib.DecodeAttnDesc(_ptr(qx), _ptr(kc), _ptr(vc), _ptr(tab), _ptr(ip), _ptr(o), pos, B, KV, G, HD, rows, Q,
                            window, KV * G * HD if o_stride is None else o_stride)
    if prep is not None:
        d.q0, d.k0, d.v0 = _ptr(prep["q0"]), _ptr(prep["k0"]), _ptr(prep["v0"])
        d.ldq, d.ldk, d.ldv = prep["ldq"], prep["ldk"], prep["ldv"]
        d.rope, d.pq, d.pk = _ptr(prep["rope"]), _ptr(prep["pq"]), _ptr(prep["pk"])
        d.pv = _ptr(prep.get("pv"))
        d.prep = 1 | (2 if prep.get("pq_bc") else 0) | (4 if prep.get("pk_bc") else 0) | \
            (8 if prep.get("pv_bc") else 0) | (16 if prep.get("v_direct") else 0)
    check(lib().corm_llm_decode_attn(C.byref(d), st))


def greedy_embed(logits, table, out, ids=None, *, batch, vocab, dim, ld=None):
    """corm_greedy_embed: ids = first argmax of each int16 logits row; out
    (int32) = those rows of the int32 table."""
    _i16(logits, "logits")
    if table.dtype != torch.int32 or out.dtype != torch.int32 or (ids is not None and ids.dtype != torch.int32):
        raise CormError(_lib.CORM_EINVAL, "table / out / ids must be int32")
    st = _ready()
    d = _lib.GreedyDesc(_ptr(logits), _ptr(table), _ptr(out), _ptr(ids), batch, vocab, dim,
                        vocab if ld is None else ld)
    check(lib().corm_greedy_embed(C.byref(d), st))


def conv(x, weight, bias, y, *, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h=1, stride_w=1,
         dilation_h=1, dilation_w=1, pad_top=0, pad_left=0, has_bias=0, is_depthwise=0, y_cs=0, y_cn=0, y_gs=0,
         flags=0, workspace=None, post=None):
    """One ConvKernel job (host_emu.py:393-455); CORM_F_WEIGHT_LOGICAL in
    ``flags`` for [M][C][kh][kw] weights instead of the board image.
    ``post``: a fused VectorOP job as for ``matmul``."""
    for t, nm in ((x, "x"), (weight, "weight"), (bias, "bias"), (y, "y")):
        _i16(t, nm)
    st = _ready()
    d = _lib.ConvDesc(_ptr(x), _ptr(weight), _ptr(bias), _ptr(y), batch, in_ch, in_h, in_w, out_ch, out_h, out_w,
                      kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, int(bool(has_bias)),
                      int(bool(is_depthwise)), y_cs, y_cn, y_gs, flags, None, 0)
    need = C.c_size_t(0)
    check(lib().corm_conv_workspace_size(C.byref(d), C.byref(need)))
    if need.value:
        if workspace is None:
            workspace = torch.empty(need.value, dtype=torch.uint8, device=x.device)
        d.workspace, d.workspace_bytes = _ptr(workspace), workspace.numel() * workspace.element_size()
    q = _post(post)
    if q is None:
        check(lib().corm_conv(C.byref(d), st))
    else:
        check(lib().corm_conv_post(C.byref(d), C.byref(q), st))
    return workspace


def pool(x, y, *, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h=1, stride_w=1, pad_top=0,
         pad_left=0, dil_h=1, dil_w=1, pool_type=0, lp_order=0, count_include_pad=0):
    """One PoolingKernel job (_simulate.py:275-358 semantics)."""
    _i16(x, "x")
    _i16(y, "y")
    st = _ready()
    d = _lib.PoolDesc(_ptr(x), _ptr(y), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h,
                      stride_w, pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad)
    check(lib().corm_pool(C.byref(d), st))


def rowops(a, b, c, p, *, op, n, rows=1, blocks=1, a_s1=0, a_s2=0, b_s1=0, b_s2=0, c_s1=0, c_s2=0, eps=0, aux=0,
           bq_sh=0, win_lo=0, win_hi=0xFFFFFFFF, a_off=0, b_off=0, c_off=0, p_off=0):
    """One RowOpsKernel job (rowops_ref.h:259-427): byte strides; a / b / c /
    p are tensors (any dtype) or raw device addresses, plus byte offsets."""
    st = _ready()

    def addr(t, off):
        return (_ptr(t) + off) if t is not None else 0
    d = _lib.RowOpsDesc(op, n, rows, blocks, addr(a, a_off), a_s1 & 0xFFFFFFFF, a_s2 & 0xFFFFFFFF, addr(b, b_off),
                        b_s1 & 0xFFFFFFFF, b_s2 & 0xFFFFFFFF, addr(c, c_off), c_s1 & 0xFFFFFFFF, c_s2 & 0xFFFFFFFF,
                        addr(p, p_off), eps & 0xFFFFFFFFFFFFFFFF, aux, bq_sh, win_lo & 0xFFFFFFFF,
                        win_hi & 0xFFFFFFFF)
    check(lib().corm_rowops(C.byref(d), st))


def rowops_chain(jobs):
    """A descriptor chain (corm_rowops_chain): ``jobs`` a list of dicts with
    the keys of ``rowops`` (a, b, c, p as tensors or raw addresses, plus byte
    offsets), run in order, at most 16."""
    st = _ready()

    def addr(t, off):
        return (_ptr(t) + off) if t is not None else 0
    arr = (_lib.RowOpsDesc * max(1, len(jobs)))()
    for k, j in enumerate(jobs):
        g = lambda key, dflt=0: j.get(key, dflt)  # noqa: E731
        arr[k] = _lib.RowOpsDesc(j["op"], j["n"], g("rows", 1), g("blocks", 1), addr(g("a", None), g("a_off")),
                                 g("a_s1") & 0xFFFFFFFF, g("a_s2") & 0xFFFFFFFF, addr(g("b", None), g("b_off")),
                                 g("b_s1") & 0xFFFFFFFF, g("b_s2") & 0xFFFFFFFF, addr(g("c", None), g("c_off")),
                                 g("c_s1") & 0xFFFFFFFF, g("c_s2") & 0xFFFFFFFF, addr(g("p", None), g("p_off")),
                                 g("eps") & 0xFFFFFFFFFFFFFFFF, g("aux"), g("bq_sh"), g("win_lo") & 0xFFFFFFFF,
                                 g("win_hi", 0xFFFFFFFF) & 0xFFFFFFFF)
    check(lib().corm_rowops_chain(arr, len(jobs), st))


def device_status() -> int:
    """Synchronise and return (and clear) the kernels' timeout status word."""
    _ready()
    code = C.c_int(0)
    check(lib().corm_device_status(C.byref(code)))
    return code.value


def launch_count() -> int:
    """Kernel launches the library has made in this process."""
    return int(lib().corm_launch_count())


def profile_enable(on: bool = True) -> None:
    check(lib().corm_profile_enable(1 if on else 0))


def profile_read() -> dict:
    """{kernel: (launches, total_ms, max_ms)} of the launches recorded since the
    last read (synchronises)."""
    buf = (_lib.ProfileEntry * 64)()
    n = C.c_int(0)
    check(lib().corm_profile_read(buf, 64, C.byref(n)))
    return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms), float(buf[i].max_ms))
            for i in range(n.value)}


# ---------------------------------------------------------------- host-side tables (no GPU needed)
def act_table(act: int, alpha: int = 0):
    import numpy as np
    out = np.zeros(65536, np.int16)
    check(lib().corm_act_table(act, alpha & 0xFFFFFFFF, out.ctypes.data))
    return out


def smx_table():
    import numpy as np
    out = np.zeros(4096, np.int32)
    check(lib().corm_smx_table(out.ctypes.data))
    return out


def rowops_table_image():
    import numpy as np
    out = np.zeros(65536, np.uint8)
    check(lib().corm_rowops_table_image(out.ctypes.data))
    return out
