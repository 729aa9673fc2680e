"""The C ABI library on a machine without a GPU: it loads, exports every
symbol include/b4gemv.h declares, and its host-only logic (shape checks, the
dispatch rule, the host quantisers) works."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

import b4gemv
from b4gemv import _lib
from b4gemv.diag import LEAN_VARIANTS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
QWEN = [(3584, 3584), (512, 3584), (18944, 3584), (3584, 18944)]
LLAMA_TP = [(8192, 8192), (1024, 8192), (28672, 8192), (8192, 28672), (1024, 1024), (128, 8192), (8192, 3584),
            (3584, 8192)]


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "b4gemv.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(b4_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = b4gemv.load()
    syms = declared_symbols()
    assert len(syms) >= 14
    for s in syms:
        assert hasattr(lib, s), s
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    assert lib.b4_abi_version() == 8


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("out_f,in_f", QWEN + LLAMA_TP)
@pytest.mark.parametrize("m", [1, 2, 3, 4, 8, 16])
def test_default_config_is_valid(fmt, out_f, in_f, m):
    c = b4gemv.default_config(fmt, in_f, out_f, m)
    e = c["engine"]
    assert c["vec_words"] in (1, 2, 4) and (in_f // 8) % c["vec_words"] == 0
    assert 1 <= c["warps_k"] * c["row_groups"] <= 8 or (e == 0 and c["warps_k"] * c["row_groups"] <= 16)
    if e in (1, 2):      # tensor pipe, register-fed or bulk-copy ring
        assert fmt == 0 and c["vec_words"] == 4
        assert c["rows_per_warp"] in (16, 32) and c["batch_tile"] in (8, 16)
        if e == 2:
            assert m <= c["batch_tile"] and c["rows_per_warp"] == 16
    elif e == 4:         # lean batch-1 INT4, register pipeline
        assert fmt == 0 and m == 1 and c["rows_per_warp"] == 16 and c["stages"] in (2, 3, 4, 6)
    elif e == 5:         # lean INT4 (m <= 16: batch rows in the MMA's N), cp.async ring of `stage_groups` groups
        assert fmt == 0 and m <= 16 and c["rows_per_warp"] == 16
        assert (c["stages"], c["stage_groups"]) in LEAN_VARIANTS and (in_f // 128) % c["stage_groups"] == 0
    elif e == 7:         # NF4 tensor pipe (m <= 16: batch rows in the MMA's N)
        assert fmt == 1 and m <= 16 and in_f % 128 == 0 and c["rows_per_warp"] == 16 and c["stages"] in (2, 3, 4)
    elif e == 6:         # lean batch-1 NF4
        assert fmt == 1 and m == 1 and c["rows_per_warp"] in (4, 8) and c["nf4_lut"] in (0, 2)
    else:
        assert e == 0
        assert c["rows_per_warp"] in (1, 2, 4, 8)
        assert c["batch_tile"] in (1, 2, 4)
        assert 1 <= c["warps_k"] * c["row_groups"] <= (16 if c["rows_per_warp"] * c["batch_tile"] == 1 else 8)


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("shapes,in_f", [((3584, 512, 512), 3584), ((18944, 18944), 3584), ((8192, 1024, 1024), 8192),
                                         ((1024, 128, 128), 8192), ((28672, 28672), 8192), ((100,), 1024)])
def test_multi_default_config_is_one_lean_launch_at_batch_1(fmt, shapes, in_f):
    segs = (_lib.GemvSegment * len(shapes))(*[_lib.GemvSegment(256 * (i + 1), 256, None, o)
                                              for i, o in enumerate(shapes)])
    c = _lib.GemvConfig()
    assert b4gemv.load().b4_gemv_multi_default_config(fmt, segs, len(shapes), in_f, 1, ctypes.byref(c)) == 0
    assert c.engine in ((4, 5) if fmt == 0 else (6, 7))
    # the rule sees the total rows: the fused q/k/v gets the config of a 4608-row matrix
    assert c.as_dict() == b4gemv.default_config(fmt, in_f, sum(shapes), 1)


def test_multi_rejects_bad_segments_before_any_launch():
    lib = b4gemv.load()
    inv = 1
    segs = (_lib.GemvSegment * 5)(*[_lib.GemvSegment(4096, 4096, 4096, 64) for _ in range(5)])
    x = ctypes.c_void_p(4096)
    assert lib.b4_gemv_multi(0, segs, 0, x, 1024, 1, None, None) == inv      # no segment
    assert lib.b4_gemv_multi(0, segs, 5, x, 1024, 1, None, None) == inv      # more than B4_MAX_SEGMENTS
    assert lib.b4_gemv_multi(0, segs, 2, x, 1000, 1, None, None) == inv      # in_f % 128
    assert lib.b4_gemv_multi(1, segs, 2, x, 96, 1, None, None) == inv        # in_f % 64
    assert lib.b4_gemv_multi(0, None, 2, x, 1024, 1, None, None) == inv
    segs[1].out_f = 0
    assert lib.b4_gemv_multi(0, segs, 2, x, 1024, 1, None, None) == inv      # empty segment
    segs[1].out_f = 64
    segs[1].y = None
    assert lib.b4_gemv_multi(0, segs, 2, x, 1024, 1, None, None) == inv      # null y
    c = _lib.GemvConfig()
    assert lib.b4_gemv_multi_default_config(0, segs, 2, 1024, 1, ctypes.byref(c)) == 0   # y not read
    segs[1].qw = 4098
    assert lib.b4_gemv_multi_default_config(0, segs, 2, 1024, 1, ctypes.byref(c)) == inv  # misaligned codes
    # a lean config whose stage does not tile the row: 9 groups, 2 per stage
    segs[1].qw, segs[1].y = 4096, 4096
    cfg = _lib.GemvConfig(vec_words=4, rows_per_warp=16, warps_k=8, row_groups=1, batch_tile=1, engine=5, stages=4,
                          stage_groups=2)
    assert lib.b4_gemv_multi(0, segs, 2, x, 1152, 1, ctypes.byref(cfg), None) == inv


def test_tile_rows_out_of_range_is_rejected():
    lib = b4gemv.load()
    bogus = ctypes.c_void_p(4096)
    for e, fmt, st, sg in [(4, 0, 4, 1), (5, 0, 2, 4), (7, 1, 3, 0)]:
        for tr in (-1, 17):
            cfg = _lib.GemvConfig(vec_words=4, rows_per_warp=16, warps_k=8, row_groups=1, batch_tile=1, engine=e,
                                  stages=st, stage_groups=sg, tile_rows=tr)
            assert lib.b4_gemv_ex(fmt, bogus, bogus, bogus, bogus, 1024, 64, 1, ctypes.byref(cfg), None) == 1


def test_invalid_shapes_are_rejected_before_any_launch():
    lib = b4gemv.load()
    bogus = ctypes.c_void_p(4096)
    inv = 1  # cudaErrorInvalidValue
    # in_f not a multiple of the group / block
    assert lib.b4_gemv_int4_g128(bogus, bogus, bogus, bogus, 100, 8, 1, None) == inv
    assert lib.b4_gemv_int4_g128(bogus, bogus, bogus, bogus, 64, 8, 1, None) == inv
    assert lib.b4_gemv_nf4_b64(bogus, bogus, bogus, bogus, 96, 8, 1, None) == inv
    # empty / negative sizes, null pointers
    assert lib.b4_gemv_nf4_b64(bogus, bogus, bogus, bogus, 64, 0, 1, None) == inv
    assert lib.b4_gemv_nf4_b64(bogus, bogus, bogus, bogus, 64, 8, 0, None) == inv
    assert lib.b4_gemv_nf4_b64(None, bogus, bogus, bogus, 64, 8, 1, None) == inv
    # misaligned packed words (the reference assumes 4-byte alignment)
    assert lib.b4_gemv_nf4_b64(ctypes.c_void_p(4098), bogus, bogus, bogus, 64, 8, 1, None) == inv
    # a config the kernel set does not contain
    cfg = _lib.GemvConfig(vec_words=3, rows_per_warp=1, warps_k=1, row_groups=1, batch_tile=1)
    assert lib.b4_gemv_ex(1, bogus, bogus, bogus, bogus, 64, 8, 1, ctypes.byref(cfg), None) == inv
    # the tensor-pipe engine is INT4 only
    cfg = _lib.GemvConfig(vec_words=4, rows_per_warp=16, warps_k=1, row_groups=1, batch_tile=8, engine=1)
    assert lib.b4_gemv_ex(1, bogus, bogus, bogus, bogus, 128, 8, 1, ctypes.byref(cfg), None) == inv
    assert lib.b4_dequant_int4_g128(bogus, bogus, bogus, 96, 8, None) == inv
    assert lib.b4_unpack_codes(bogus, bogus, 12, 8, None) == inv
    assert lib.b4_quantise_nf4_b64_device(bogus, 8, 100, bogus, bogus, None, None) == inv
    assert lib.b4_status_string(1).decode() != ""


def test_host_quantisers_match_reference_fixtures(golden):
    for name, g in golden.items():
        for nthreads in (1, 3):
            p, s, d = b4gemv.quantise(g["W"], nthreads=nthreads)
            assert p.tobytes() == g["int4_packed"].tobytes(), name
            assert s.view(np.uint16).tobytes() == g["int4_scales"].tobytes(), name
            assert d.tobytes() == g["int4_deq"].tobytes(), name
            pn, a, dn = b4gemv.quantise_nf4(g["W"], nthreads=nthreads)
            assert pn.tobytes() == g["nf4_packed"].tobytes(), name
            assert a.tobytes() == g["nf4_absmax"].tobytes(), name
            assert dn.tobytes() == g["nf4_deq"].tobytes(), name


def test_host_quantisers_match_oracle_random(oracle):
    rng = np.random.default_rng(3)
    for t in range(6):
        o, n = int(rng.integers(1, 40)), 128 * int(rng.integers(1, 9))
        W = (rng.standard_normal((o, n)) * 10 ** rng.uniform(-8, 5)).astype(np.float32)
        W.flat[rng.integers(0, W.size, 3)] = [np.nan, np.inf, 0.0]
        p, s, d = b4gemv.quantise(W)
        op, os_, od = oracle.quantise(W)
        assert p.tobytes() == op.tobytes() and s.view(np.uint16).tobytes() == os_.tobytes()
        assert d.tobytes() == od.tobytes()
        pn, a, dn = b4gemv.quantise_nf4(W)
        opn, oa, odn = oracle.quantise_nf4(W)
        assert pn.tobytes() == opn.tobytes() and a.tobytes() == oa.tobytes() and dn.tobytes() == odn.tobytes()


def test_median_is_the_reference_upper_median():
    assert b4gemv.median([3.0, 1.0, 2.0, 4.0]) == 3.0
    assert b4gemv.median([5.0]) == 5.0


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("out_f,in_f", QWEN + LLAMA_TP)
@pytest.mark.parametrize("m", [1, 2, 16])
def test_workspace_rule(fmt, out_f, in_f, m):
    """b4_gemv_default_config_ws: the x-pair table kernel for NF4 at batch 1
    with in_f % 256 == 0 and at least 17.5 MB of weights (5 MB for rows of 8192
    columns or more; it needs the workspace), else b4_gemv_default_config's
    choice (no measured shape ran faster split: split only when asked)."""
    c = b4gemv.default_config_ws(fmt, in_f, out_f, m)
    assert not c["flags"] & b4gemv.FLAG_SPLIT
    weight_bytes = out_f * in_f // 2 + out_f * (in_f // 64) * 4
    pays = weight_bytes >= 17_500_000 or (in_f >= 8192 and weight_bytes >= 5_000_000)
    if fmt == 1 and m == 1 and in_f % 256 == 0 and pays:
        assert c["engine"] == b4gemv.ENGINE_NF4_XTAB
        big = weight_bytes >= 9_000_000
        assert (c["row_groups"], c["stages"]) == ((16, 2) if big else (12, 3))
        assert b4gemv.workspace_size(fmt, in_f, out_f, m, device=0) == b4gemv.XTAB_WORKSPACE_BYTES
    elif c["flags"] & b4gemv.FLAG_KSLICE:
        # a batch whose x does not fit beside the small-batch kernel: the fewest
        # column slices whose x does, each run by that kernel
        plain = b4gemv.default_config(fmt, in_f, out_f, m)
        assert m >= 2 and plain["engine"] not in (5, 7)
        sw = c["x_tile"]
        slices = in_f // sw
        assert in_f % sw == 0 and 2 <= slices <= 4 and sw % 128 == 0
        for fewer in range(2, slices):
            if (in_f // 128) % fewer == 0:
                assert b4gemv.default_config(fmt, in_f // fewer, out_f, m)["engine"] not in (5, 7)
        one = b4gemv.default_config(fmt, sw, out_f, m)
        assert c["engine"] == one["engine"] in (5, 7) and c["row_groups"] == one["row_groups"]
        # past the x-pair table kernel's counters, which every b4_gemv_ws workspace keeps
        assert (b4gemv.workspace_size(fmt, in_f, out_f, m, device=0)
                == b4gemv.XTAB_WORKSPACE_BYTES + slices * m * out_f * 4)
    else:
        assert c == b4gemv.default_config(fmt, in_f, out_f, m)


def test_xtab_config_needs_the_workspace_entry_points():
    """b4_gemv_ex and b4_gemv_multi have no workspace: an x-pair table config is
    rejected before any device call; other in_f fall back to the plain rule."""
    lib = b4gemv.load()
    c = _lib.GemvConfig.from_dict({"engine": b4gemv.ENGINE_NF4_XTAB, "stages": 3})
    p = ctypes.c_void_p(4096)
    assert lib.b4_gemv_ex(1, p, p, p, p, 3584, 3584, 1, ctypes.byref(c), None) == 1
    assert b4gemv.default_config_ws(1, 1088, 512, 1) == b4gemv.default_config(1, 1088, 512, 1)


@pytest.mark.parametrize("out_f,in_f", QWEN + LLAMA_TP)
def test_batch1_int4_rule_gives_one_resident_tile_per_cta(out_f, in_f):
    """Batch-1 INT4: the cp.async-ring engine with 8-warp CTAs and the fewest
    power-of-two row groups whose tiles fit the 2 x 148 resident CTAs."""
    c = b4gemv.default_config(0, in_f, out_f, 1)
    blocks = (out_f + 15) // 16
    assert c["engine"] == 5 and c["warps_k"] * c["row_groups"] == 8 and c["row_groups"] in (1, 2, 4, 8)
    rg = c["row_groups"]
    tiles = -(-blocks // rg)
    assert tiles <= 296 or rg == 8
    assert rg == 1 or -(-blocks // (rg // 2)) > 296


def test_split_flag_needs_the_workspace_entry_point():
    """b4_gemv_ex has no workspace: a split config is rejected before any device call."""
    lib = b4gemv.load()
    c = _lib.GemvConfig.from_dict(dict(b4gemv.default_config(0, 8192, 8192, 1), flags=b4gemv.FLAG_SPLIT))
    p = ctypes.c_void_p(4096)
    assert lib.b4_gemv_ex(0, p, p, p, p, 8192, 8192, 1, ctypes.byref(c), None) == 1
