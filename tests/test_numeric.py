"""The exponent planner (cormorant_b200.numeric) against the reference's own
weight encodings and formats lookups (tests/golden/sim_numeric.npz, made by
make_golden.py from src/numeric.py encode_matmul_weights / encode_conv_weights
and src/llama.py Formats): raw words, exponent arrays and their integer type,
saturation counts; and the table semantics the reference fixes (broadcast,
per-head repeat, a missing class is an error)."""
import json
import os
import zlib

import numpy as np
import pytest

from cormorant_b200 import numeric as NU

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "sim_numeric.npz"))


@pytest.mark.parametrize("tag", ["mm_t", "mm_ch", "mm_wide", "mm_sat"])
def test_matmul_weight_vs_reference(tag):
    data, wexp, sat = NU.encode_matmul_weight(G[f"{tag}_w"], G[f"{tag}_fin"], G[f"{tag}_fout"])
    assert np.array_equal(np.round(data.astype(np.float64) * 256).astype(np.int64), G[f"{tag}_raw"])
    assert np.array_equal(wexp, G[f"{tag}_wexp"])
    assert wexp.dtype.itemsize == int(G[f"{tag}_wexp_dtype"][0])
    assert sat == int(G[f"{tag}_sat"][0])


def test_matmul_weight_row_blocks_vs_reference():
    """2^21 elements: the encoding runs in two row blocks, element-wise the same."""
    K, M = 2048, 1024
    brng = np.random.default_rng(int(G["mm_big_seed"][0]))
    w = (brng.standard_normal((K, M)) * 0.03).astype(np.float32)
    assert zlib.crc32(w.tobytes()) == int(G["mm_big_w_crc"][0])
    fi, fo = brng.integers(9, 13, K), brng.integers(9, 12, M)
    assert np.array_equal(fi, G["mm_big_fin"]) and np.array_equal(fo, G["mm_big_fout"])
    data, wexp, sat = NU.encode_matmul_weight(w, fi, fo)
    raw = NU.matmul_weight_raw(data)
    crc_raw, crc_exp, n_sat, isz = (int(v) for v in G["mm_big_crc"])
    assert zlib.crc32(raw.tobytes()) == crc_raw
    assert zlib.crc32(np.ascontiguousarray(wexp).tobytes()) == crc_exp
    assert sat == n_sat and wexp.dtype.itemsize == isz


@pytest.mark.parametrize("tag,dw", [("cv_t", False), ("cv_tdw", True), ("cv_ch", False), ("cv_chdw", True),
                                    ("cv_sat", False)])
def test_conv_weight_vs_reference(tag, dw):
    fx, fy = G[f"{tag}_fx"], G[f"{tag}_fy"]
    fx = int(fx) if fx.ndim == 0 else fx
    fy = int(fy) if fy.ndim == 0 else fy
    (wd, we, ws), (bd, be, bs) = NU.encode_conv_weight(G[f"{tag}_w"], G[f"{tag}_b"], fx, fy, depthwise=dw)
    assert np.array_equal(np.round(wd.astype(np.float64) * 256).astype(np.int64), G[f"{tag}_wraw"])
    assert np.array_equal(np.round(bd.astype(np.float64) * 256).astype(np.int64), G[f"{tag}_braw"])
    assert np.array_equal(we, G[f"{tag}_wexp"]) and we.dtype == G[f"{tag}_wexp"].dtype
    assert np.array_equal(be, G[f"{tag}_bexp"])
    assert [ws, bs] == [int(v) for v in G[f"{tag}_sat"]]


def test_llama_formats_vs_reference():
    exps = json.loads(bytes(G["fm_exps"]).decode())
    fm = NU.LlamaFormats({"exponents": exps, "policy": "test"}, L=2, H=6, KV=2, HD=4)
    for li in range(2):
        assert np.array_equal(fm.k_cache(li), G[f"fm_k{li}"])
        assert np.array_equal(fm.v_cache(li), G[f"fm_v{li}"])
        assert np.array_equal(fm.pv(li), G[f"fm_pv{li}"])
        assert np.array_equal(fm.scores(li), G[f"fm_s{li}"])
    assert fm.res_bits == int(G["fm_res"][0])


def test_expand_exp_and_table_rules():
    assert np.array_equal(NU.expand_exp(7, 4), [7, 7, 7, 7])
    assert np.array_equal(NU.expand_exp([1, 2], 6), [1, 1, 1, 2, 2, 2])
    assert np.array_equal(NU.expand_exp([1, 2, 3], 3), [1, 2, 3])
    with pytest.raises(NU.NumericError):
        NU.expand_exp([1, 2, 3], 4)
    t = NU.ExponentTable({"exponents": {"x@0": 12}, "policy": "p"})
    assert t.has("x@0") and not t.has("x@1")
    with pytest.raises(KeyError):
        t.lookup("x@1", 4)  # a class the calibration did not write is an error, not a default
    fm = NU.LlamaFormats({"exponents": {}}, L=1, H=2, KV=1, HD=2)
    assert fm.res_bits == NU.RES_BITS


def test_per_tensor_table_matches_uniform_lookups():
    e = dict(x=12, q0=13, k0=13, v=13, q=10, k=10, vc=9, p=12, o=13, x2=12, g=13, u=13, a=13, d=13, xf=12,
             logits=11, res=15)
    fm = NU.LlamaFormats.per_tensor(e, L=3, H=6, KV=2, HD=4)
    assert np.array_equal(fm.get("o", 2, 5), [13] * 5)
    assert np.array_equal(fm.get("logits", 3, 2), [11, 11])
    assert np.array_equal(fm.v_cache(1), [9] * 8)
    assert np.array_equal(fm.pv(0), [12 + 9 - 8] * 24)
    assert fm.res_bits == 15
