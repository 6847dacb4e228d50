"""ctypes binding of libcorm_b200.so (include/cormorant_b200.h).

The structures mirror the C descriptors field for field; ``check`` turns a
negative status into ``CormError`` with the library's message.  Nothing here
computes: without the built library (or without a GPU, for the job entry
points) calls fail loudly — there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libcorm_b200.so")

CORM_OK, CORM_EINVAL, CORM_ELIMIT, CORM_ECUDA, CORM_ENOMEM, CORM_EDEVICE = 0, -1, -2, -3, -4, -5
F_WRAP32, F_WEIGHT_LOGICAL, F_ACT_RELU, F_ACT_RELU6 = 0x1, 0x2, 0x4, 0x8

# every symbol include/cormorant_b200.h declares
EXPORTS = ("corm_vectorop", "corm_matmul_workspace_size", "corm_matmul", "corm_matmul_noalloc", "corm_matmul_noalloc_status", "corm_conv_workspace_size", "corm_conv",
           "corm_matmul_post", "corm_matmul_groups", "corm_split_b_planes", "corm_matmul_bplanes", "corm_conv_post", "corm_gemm_strided_workspace_size", "corm_gemm_strided",
           "corm_copy_nd", "corm_llm_attn_softmax", "corm_greedy_embed", "corm_llm_embed", "corm_llm_dequant",
           "corm_llm_resadd", "corm_llm_rmsnorm", "corm_llm_act_mul", "corm_llm_attn_prep_host",
           "corm_llm_decode_attn", "corm_rowops_chain", "corm_rowops_chain_dev",
           "corm_stream_done",
           "corm_pool", "corm_rowops", "corm_act_table", "corm_smx_table", "corm_rowops_table_image",
           "corm_bind_device", "corm_device_status", "corm_set_wait_limit", "corm_launch_count", "corm_profile_enable",
           "corm_profile_read", "corm_version", "corm_last_error")


class CormError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libcorm_b200 error {code}: {msg}")
        self.code = code


def _u32_fields(names):
    return [(n, C.c_uint32) for n in names]


class VectorOpDesc(C.Structure):
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p)] + _u32_fields(
        ["size", "op", "outer", "a_inc", "b_inc", "act", "alpha", "smx_cm", "smx_cfg", "smx_mask"])


class MatmulDesc(C.Structure):
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p)] + _u32_fields(
        ["n", "k", "m", "batch", "a_batch_stride", "b_batch_stride", "c_batch_stride", "b_packed", "gemv_kw",
         "flags"]) + [("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class OutGroups(C.Structure):
    _fields_ = [("count", C.c_uint32), ("width", C.c_uint32 * 4), ("out", C.c_void_p * 4), ("mulact", C.c_uint32),
                ("ma_sa", C.c_int32), ("ma_sc", C.c_int32)]


class ConvDesc(C.Structure):
    _fields_ = [("x", C.c_void_p), ("weight", C.c_void_p), ("bias", C.c_void_p), ("y", C.c_void_p)] + _u32_fields(
        ["batch", "in_ch", "in_h", "in_w", "out_ch", "out_h", "out_w", "kh", "kw", "stride_h", "stride_w",
         "dilation_h", "dilation_w", "pad_top", "pad_left", "has_bias", "is_depthwise", "y_cs", "y_cn", "y_gs",
         "flags"]) + [("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class PostOp(C.Structure):
    """corm_postop: the VectorOP job fused into a MatMul / Conv epilogue."""
    _fields_ = [("b", C.c_void_p)] + _u32_fields(["op", "act", "alpha", "b_mode", "b_is_first"])


POST_B_COL, POST_B_SAME, POST_B_SCALAR = 0, 1, 2


class GemmDesc(C.Structure):
    """corm_gemm_desc: a strided batch of MatMul jobs (row and batch strides)."""
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p)] + _u32_fields(
        ["n", "k", "m", "batch", "lda", "ldb", "ldc", "b_trans"]) + [
        ("a_batch_stride", C.c_uint64), ("b_batch_stride", C.c_uint64), ("c_batch_stride", C.c_uint64),
        ("flags", C.c_uint32), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class CopyDesc(C.Structure):
    """corm_copy_desc: an int16 copy between two strided views of <= 6 dims."""
    _fields_ = [("src", C.c_void_p), ("dst", C.c_void_p), ("ndim", C.c_uint32), ("dims", C.c_uint32 * 6),
                ("src_strides", C.c_int64 * 6), ("dst_strides", C.c_int64 * 6)]


class LlmSmxDesc(C.Structure):
    """corm_llm_smx_desc: the host's p12 softmax of one KV group."""
    _fields_ = [("s", C.c_void_p), ("p", C.c_void_p), ("tab", C.c_void_p), ("ip", C.c_void_p)] + _u32_fields(
        ["pos", "n", "T", "G", "C", "Q", "window", "batch"]) + [("s_stride", C.c_uint64), ("p_stride", C.c_uint64)]


class LlmEmbedDesc(C.Structure):
    """corm_llm_embed_desc: LlmEmbed rows (float32, or the int32 residual)."""
    _fields_ = [("ids", C.c_void_p), ("table", C.c_void_p), ("out", C.c_void_p)] + _u32_fields(
        ["n", "rows", "d", "res32"]) + [("f", C.c_int32), ("scale", C.c_float)]


class LlmDequantDesc(C.Structure):
    _fields_ = [("x", C.c_void_p), ("y", C.c_void_p), ("f", C.c_void_p), ("count", C.c_uint64), ("n", C.c_uint32)]


class LlmResAddDesc(C.Structure):
    _fields_ = [("h", C.c_void_p), ("d", C.c_void_p), ("y", C.c_void_p), ("fd", C.c_void_p)] + _u32_fields(
        ["rows", "n"])


class LlmRMSNormDesc(C.Structure):
    _fields_ = [("h32", C.c_void_p), ("h16", C.c_void_p), ("fh", C.c_void_p), ("y", C.c_void_p),
                ("gamma", C.c_void_p), ("fy", C.c_void_p), ("eps", C.c_double), ("rows", C.c_uint64)] + _u32_fields(
        ["n", "W"])


class LlmActMulDesc(C.Structure):
    _fields_ = [("g", C.c_void_p), ("u", C.c_void_p), ("y", C.c_void_p), ("tab", C.c_void_p), ("tab_of", C.c_void_p),
                ("fu", C.c_void_p), ("fy", C.c_void_p)] + _u32_fields(["rows", "n"])


class LlmPrepDesc(C.Structure):
    _fields_ = [(nm, C.c_void_p) for nm in ("q0", "k0", "v", "kc", "vc", "qx", "cos", "sin", "fq0", "fk0", "fv", "fkc",
                                            "fvc", "fq")] + _u32_fields(
        ["pos", "n", "T", "H", "KV", "HD", "C", "Q", "batch"]) + [("ldq", C.c_uint64), ("ldk", C.c_uint64),
                                                                  ("ldv", C.c_uint64)]


class GreedyDesc(C.Structure):
    """corm_greedy_desc: argmax of each logits row and its embedding row."""
    _fields_ = [("logits", C.c_void_p), ("table", C.c_void_p), ("out", C.c_void_p), ("ids", C.c_void_p)] + \
        _u32_fields(["batch", "vocab", "dim"]) + [("ld", C.c_uint64)]


class DecodeAttnDesc(C.Structure):
    """corm_llm_decode_attn_desc: a decode step's attention of every group."""
    _fields_ = [("qx", C.c_void_p), ("kc", C.c_void_p), ("vc", C.c_void_p), ("tab", C.c_void_p), ("ip", C.c_void_p),
                ("o", C.c_void_p)] + _u32_fields(["pos", "B", "KV", "G", "HD", "C", "Q", "window"]) + [
                ("o_stride", C.c_uint64), ("q0", C.c_void_p), ("k0", C.c_void_p), ("v0", C.c_void_p),
                ("ldq", C.c_uint64), ("ldk", C.c_uint64), ("ldv", C.c_uint64), ("rope", C.c_void_p),
                ("pq", C.c_void_p), ("pk", C.c_void_p), ("pv", C.c_void_p), ("prep", C.c_uint32)]


class PoolDesc(C.Structure):
    _fields_ = [("x", C.c_void_p), ("y", C.c_void_p)] + _u32_fields(
        ["batch", "channels", "in_h", "in_w", "out_h", "out_w", "pool_h", "pool_w", "stride_h", "stride_w",
         "pad_top", "pad_left", "dil_h", "dil_w", "pool_type", "lp_order", "count_include_pad"])


class RowOpsDesc(C.Structure):
    _fields_ = _u32_fields(["op", "n", "rows", "blocks"]) + [
        ("a", C.c_void_p), ("a_s1", C.c_uint32), ("a_s2", C.c_uint32),
        ("b", C.c_void_p), ("b_s1", C.c_uint32), ("b_s2", C.c_uint32),
        ("c", C.c_void_p), ("c_s1", C.c_uint32), ("c_s2", C.c_uint32),
        ("p", C.c_void_p), ("eps", C.c_uint64)] + _u32_fields(["aux", "bq_sh", "win_lo", "win_hi"])


class ProfileEntry(C.Structure):
    _fields_ = [("name", C.c_char * 48), ("launches", C.c_uint64), ("total_ms", C.c_double), ("max_ms", C.c_double)]


_lib = None


def lib() -> C.CDLL:
    """The loaded library (built on first use when nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        try:
            from . import build as _build
            _build.build()
        except Exception as e:  # pragma: no cover - surfaced to the caller
            raise CormError(CORM_ECUDA, f"libcorm_b200.so is not built and the build failed: {e}") from e
    L = C.CDLL(LIB_PATH)
    for name, argt in (("corm_vectorop", [C.POINTER(VectorOpDesc), C.c_void_p]),
                       ("corm_matmul", [C.POINTER(MatmulDesc), C.c_void_p]),
                       ("corm_matmul_noalloc", [C.POINTER(MatmulDesc), C.c_void_p]),
                       ("corm_matmul_noalloc_status", [C.POINTER(C.c_int), C.c_void_p]),
                       ("corm_set_wait_limit", [C.c_longlong]),
                       ("corm_matmul_groups", [C.POINTER(MatmulDesc), C.POINTER(OutGroups), C.c_void_p]),
                       ("corm_split_b_planes", [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p,
                                                C.c_void_p]),
                       ("corm_matmul_bplanes", [C.POINTER(MatmulDesc), C.c_void_p, C.c_void_p, C.POINTER(OutGroups),
                                                C.c_void_p]),
                       ("corm_matmul_workspace_size", [C.POINTER(MatmulDesc), C.POINTER(C.c_size_t)]),
                       ("corm_conv", [C.POINTER(ConvDesc), C.c_void_p]),
                       ("corm_conv_workspace_size", [C.POINTER(ConvDesc), C.POINTER(C.c_size_t)]),
                       ("corm_gemm_strided", [C.POINTER(GemmDesc), C.c_void_p]),
                       ("corm_gemm_strided_workspace_size", [C.POINTER(GemmDesc), C.POINTER(C.c_size_t)]),
                       ("corm_copy_nd", [C.POINTER(CopyDesc), C.c_void_p]),
                       ("corm_llm_attn_softmax", [C.POINTER(LlmSmxDesc), C.c_void_p]),
                       ("corm_greedy_embed", [C.POINTER(GreedyDesc), C.c_void_p]),
                       ("corm_llm_embed", [C.POINTER(LlmEmbedDesc), C.c_void_p]),
                       ("corm_llm_dequant", [C.POINTER(LlmDequantDesc), C.c_void_p]),
                       ("corm_llm_resadd", [C.POINTER(LlmResAddDesc), C.c_void_p]),
                       ("corm_llm_rmsnorm", [C.POINTER(LlmRMSNormDesc), C.c_void_p]),
                       ("corm_llm_act_mul", [C.POINTER(LlmActMulDesc), C.c_void_p]),
                       ("corm_llm_attn_prep_host", [C.POINTER(LlmPrepDesc), C.c_void_p]),
                       ("corm_llm_decode_attn", [C.POINTER(DecodeAttnDesc), C.c_void_p]),
                       ("corm_pool", [C.POINTER(PoolDesc), C.c_void_p]),
                       ("corm_rowops", [C.POINTER(RowOpsDesc), C.c_void_p]),
                       ("corm_rowops_chain", [C.POINTER(RowOpsDesc), C.c_uint32, C.c_void_p]),
                       ("corm_act_table", [C.c_uint32, C.c_uint32, C.c_void_p]),
                       ("corm_smx_table", [C.c_void_p]),
                       ("corm_rowops_table_image", [C.c_void_p]),
                       ("corm_bind_device", [C.c_int]),
                       ("corm_device_status", [C.POINTER(C.c_int)]),
                       ("corm_profile_enable", [C.c_int]),
                       ("corm_profile_read", [C.POINTER(ProfileEntry), C.c_int, C.POINTER(C.c_int)])):
        f = getattr(L, name)
        f.argtypes = argt
        f.restype = C.c_int
    L.corm_launch_count.restype = C.c_uint64
    L.corm_launch_count.argtypes = []
    L.corm_version.restype = C.c_char_p
    L.corm_last_error.restype = C.c_char_p
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != CORM_OK:
        raise CormError(rc, lib().corm_last_error().decode(errors="replace"))
