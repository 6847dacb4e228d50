"""The C-ABI library without a GPU: it loads, exports every entry point the
header declares, rejects bad descriptors before touching a device, and its
host-side table builders equal the reference's tables."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from cormorant_b200 import _lib, ops
from oracle import spec

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "cormorant_b200.h")


def test_exports_match_header():
    text = open(HEADER).read()
    declared = set(re.findall(r"^(?:int|uint64_t|const char\*)\s+(corm_\w+)\(", text, re.M))
    assert declared == set(_lib.EXPORTS)
    L = _lib.lib()
    for name in declared:
        assert hasattr(L, name), name
    assert L.corm_version().startswith(b"cormorant_b200")


def test_struct_sizes():
    # the ctypes mirrors must match the C layout (natural alignment, 64-bit)
    assert C.sizeof(_lib.VectorOpDesc) == 3 * 8 + 10 * 4 + 0 * 4
    assert C.sizeof(_lib.MatmulDesc) == 3 * 8 + 10 * 4 + 8 + 8
    assert C.sizeof(_lib.PoolDesc) == 2 * 8 + 17 * 4 + 4
    assert C.sizeof(_lib.PostOp) == 8 + 5 * 4 + 4
    assert C.sizeof(_lib.RowOpsDesc) == 4 * 4 + 8 + 8 + 8 + 8 + 8 + 8 + 8 + 8 + 4 * 4


@pytest.mark.parametrize("act", [4, 5, 6])
def test_act_tables(golden, act):
    z = golden("sim_act.npz")
    assert np.array_equal(ops.act_table(act), z[f"act{act}"])


@pytest.mark.parametrize("alpha", [0, 655, 6554, 16384, 32768, 65535])
def test_leaky_table(golden, alpha):
    z = golden("sim_act.npz")
    assert np.array_equal(ops.act_table(3, alpha), z[f"leaky{alpha}"])


def test_smx_and_rowops_tables(golden):
    assert np.array_equal(ops.smx_table().astype(np.int64), spec.SMX_TAB)
    assert np.array_equal(ops.rowops_table_image(), golden("hw_rowops.npz")["tables"])


def test_host_rejects_without_launch():
    """Descriptor validation happens before any device work."""
    L = _lib.lib()
    d = _lib.MatmulDesc(0, 0, 0, 4, 5000, 4, 1, 0, 0, 0, 0, 0, 0, None, 0)
    sz = C.c_size_t(0)
    assert L.corm_matmul_workspace_size(C.byref(d), C.byref(sz)) == _lib.CORM_EINVAL
    assert b"max_k" in L.corm_last_error()
    cv = _lib.ConvDesc()
    cv.kh = cv.kw = 9
    cv.stride_h = cv.stride_w = cv.dilation_h = cv.dilation_w = 1
    assert L.corm_conv_workspace_size(C.byref(cv), C.byref(sz)) == _lib.CORM_EINVAL
