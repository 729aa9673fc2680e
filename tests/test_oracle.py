"""The CPU oracle, pinned against the reference's own outputs.

Golden fixtures (tests/golden/golden.npz) were produced by the reference's
quantise()/quantise_nf4() compiled in place (tests/golden/make_golden.py).
When oracle/_ref/libref.so is present the oracle is also compared with the
reference on fresh random inputs.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

from oracle_py import REF_LIB, rel_err


def same_bits(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and a.view(np.uint8).tobytes() == b.view(np.uint8).tobytes()


def test_kat_words(golden):
    """Known-answer words of the reference benchmark's generator on glibc."""
    g = golden["kat_glibc"]
    assert [int(v) for v in g["int4_packed"].ravel()[:4]] == [0xc64ecc7d, 0xee86a895, 0xc341a3ba, 0xd84f3373]
    assert [int(v) for v in g["nf4_packed"].ravel()[:4]] == [0xd42edd5e, 0xef74a783, 0xd120a1ca, 0xe72f1151]
    assert g["int4_scales"].ravel()[:2].view(np.float16).astype(np.float32).tolist() == [
        float.fromhex("0x1.75cp-9"), float.fromhex("0x1.768p-9")]
    assert g["nf4_absmax"].ravel()[:2].tolist() == [float.fromhex("0x1.46f9a4p-6"), float.fromhex("0x1.3dafd4p-6")]


def test_kat_double_y(golden, oracle):
    g = golden["kat_glibc"]
    y4 = oracle.gemv_f64(False, g["int4_packed"], g["int4_scales"], g["x"])[0]
    yn = oracle.gemv_f64(True, g["nf4_packed"], g["nf4_absmax"], g["x"])[0]
    np.testing.assert_allclose(y4, [-0.0642109701, -0.0480383335], rtol=0, atol=5e-10)
    np.testing.assert_allclose(yn, [-0.0709378856, -0.0447724419], rtol=0, atol=5e-10)


@pytest.mark.parametrize("case", ["kat_glibc", "gauss_7x128", "gauss_33x384", "gauss_8x1024", "gauss_1x128",
                                  "gauss_5x640", "gauss_16x256", "edge"])
def test_oracle_quantisers_match_reference_fixtures(golden, oracle, case):
    g = golden[case]
    p, s, d = oracle.quantise(g["W"])
    assert same_bits(p, g["int4_packed"]) and same_bits(s, g["int4_scales"]) and same_bits(d, g["int4_deq"])
    pn, a, dn = oracle.quantise_nf4(g["W"])
    assert same_bits(pn, g["nf4_packed"]) and same_bits(a, g["nf4_absmax"]) and same_bits(dn, g["nf4_deq"])


@pytest.mark.parametrize("case", ["gauss_33x384", "edge"])
def test_oracle_dequant_is_the_reference_deq(golden, oracle, case):
    g = golden[case]
    assert same_bits(oracle.dequant_int4(g["int4_packed"], g["int4_scales"]), g["int4_deq"])
    assert same_bits(oracle.dequant_nf4(g["nf4_packed"], g["nf4_absmax"]), g["nf4_deq"])


def test_unpack_codes(golden, oracle):
    g = golden["gauss_5x640"]
    codes = oracle.unpack(g["int4_packed"], 640)
    p = g["int4_packed"]
    expect = np.stack([(p >> (4 * k)) & 0xF for k in range(8)], axis=-1).reshape(5, 640)
    assert np.array_equal(codes, expect.astype(np.uint8))
    # INT4 dequant reconstructs from the codes: (c - 8) * scale
    s = g["int4_scales"].view(np.float16).astype(np.float32)
    deq = (codes.astype(np.float32) - 8.0) * np.repeat(s, 128, axis=1)
    assert same_bits(deq, g["int4_deq"])


def test_edge_semantics(golden):
    """Pins the reference's handling of degenerate groups on glibc x86-64."""
    g = golden["edge"]
    s = g["int4_scales"].view(np.float16)
    assert s[0, 0] == 1.0 and s[0, 1] == 0.0 and np.isinf(s[0, 2])
    codes = np.stack([(g["int4_packed"] >> (4 * k)) & 0xF for k in range(8)], axis=-1).reshape(4, 512)
    assert np.all(codes[0, 128:384] == 8)          # scale 0 or inf: every code is 8
    assert np.all(np.isnan(g["int4_deq"][0, 256:384]))  # 0 * inf
    assert codes[1, 3] == 8                         # NaN weight
    # ties round half away from zero: 0.5 -> 1, -0.5 -> -1, 6.5 -> 7, -6.5 -> -7
    assert codes[3, 1:9].tolist() == [9, 7, 10, 6, 11, 5, 15, 1]
    nf = np.stack([(g["nf4_packed"] >> (4 * k)) & 0xF for k in range(8)], axis=-1).reshape(4, 512)
    assert nf[1, 3] == 0                            # NaN -> no strict improvement -> code 0


def test_half_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    v = np.concatenate([v, np.array([65504, 65519.99, 65520, 65536, 2 ** -24, 2 ** -25, 2 ** -25 * 1.0001,
                                     3 * 2 ** -26, 6.1e-5, 0, -0.0, np.inf, -np.inf], np.float32)])
    mine = np.array([oracle.lib.b4o_half_from_float(float(x)) for x in v], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(mine, v.astype(np.float16).view(np.uint16))
    h = np.arange(0, 65536, 7, dtype=np.uint32).astype(np.uint16)
    back = np.array([oracle.lib.b4o_float_from_half(int(x)) for x in h], np.float32)
    ref = h.view(np.float16).astype(np.float32)
    assert np.array_equal(np.isnan(back), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(back[ok].view(np.uint32), ref[ok].view(np.uint32))


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="oracle/_ref not built (needs the reference sources)")
def test_oracle_matches_compiled_reference_random(oracle):
    ref = ctypes.CDLL(REF_LIB)
    P = lambda a: ctypes.c_void_p(a.ctypes.data)
    rng = np.random.default_rng(1)
    for t in range(12):
        o, n = int(rng.integers(1, 9)), 128 * int(rng.integers(1, 6))
        W = (rng.standard_normal((o, n)) * 10 ** rng.uniform(-9, 6)).astype(np.float32)
        k = rng.integers(0, W.size, 4)
        W.flat[k[0]] = np.nan
        W.flat[k[1]] = np.inf
        W.flat[k[2]] = -np.inf
        W.flat[k[3]] = 1e-30
        p, s, d = oracle.quantise(W)
        rp = np.zeros_like(p); rs = np.zeros_like(s); rd = np.zeros_like(d)
        ref.ref_quantise(P(W), o, n, P(rp), P(rs), P(rd))
        assert same_bits(p, rp) and same_bits(s, rs) and same_bits(d, rd)
        pn, a, dn = oracle.quantise_nf4(W)
        rpn = np.zeros_like(pn); ra = np.zeros_like(a); rdn = np.zeros_like(dn)
        ref.ref_quantise_nf4(P(W), o, n, P(rpn), P(ra), P(rdn))
        assert same_bits(pn, rpn) and same_bits(a, ra) and same_bits(dn, rdn)


def test_fused_cpu_gemv_within_tolerance(golden, oracle):
    for case in ["gauss_33x384", "gauss_8x1024", "kat_glibc"]:
        g = golden[case]
        for nf4, p, s in [(False, g["int4_packed"], g["int4_scales"]), (True, g["nf4_packed"], g["nf4_absmax"])]:
            y64 = oracle.gemv_f64(nf4, p, s, g["x"])
            y, _ = oracle.gemv_fused(nf4, p, s, g["x"], nthreads=3)
            assert rel_err(y, y64) < 1e-5
            assert abs(oracle.rel_err(y, y64) - rel_err(y, y64)) < 1e-12


def test_reference_cpu_loop_matches_f64(golden, oracle):
    """int4_gemv.cu:33-38 (fp32 over deq) agrees with the double GEMV."""
    g = golden["gauss_16x256"]
    x = g["x"].astype(np.float32)
    y32 = oracle.gemv_deq_f32(g["int4_deq"], x)
    y64 = oracle.gemv_f64(False, g["int4_packed"], g["int4_scales"], g["x"])[0]
    assert rel_err(y32, y64) < 1e-5


def test_bnb_packing_helper_puts_the_lower_column_in_the_high_nibble():
    from oracle_py import bnb_pack_nf4
    codes = np.array([[1, 2, 3, 4, 15, 0, 7, 8]], np.uint8)
    assert bnb_pack_nf4(codes).tolist() == [[0x12, 0x34, 0xF0, 0x78]]
