"""GPU parity of the split batch-1 GEMV (b4_gemv_ws, B4_FLAG_SPLIT) against the
CPU oracle, through the C ABI.

The split kernels cut a matrix into equal runs of (16-row block, k-step) units
per warp and add a block's pieces through a workspace; these tests check y
against the double-precision GEMV over the same dequantised weights (TOL, the
north-star bar), against the unsplit kernels, bit-identical repeats, the
arrival counters (after the workspace's first 256 bytes) left zero after
every call, and the argument checks.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import b4gemv
from b4gemv._lib import GemvConfig, load
from oracle_py import rel_err
from test_gemv_gpu import QWEN, f64_ref, quantised, rand_problem, to_dev

TOL = 1e-3
pytestmark = pytest.mark.gpu

# (stages, stage_groups) of the INT4 split kernel, depth of the NF4 one
INT4_VARIANTS = [(4, 1), (6, 1), (3, 2), (4, 2), (2, 4), (3, 4)]
NF4_VARIANTS = [2, 3, 4]


def split_config(fmt, stages, groups=1, flags=0):
    cfg = {"vec_words": 4, "rows_per_warp": 16, "batch_tile": 1, "warps_k": 1, "row_groups": 8,
           "stages": stages, "stage_groups": groups, "flags": b4gemv.FLAG_SPLIT | flags}
    cfg["engine"] = b4gemv._lib.ENGINE_MMA_LEAN_ASYNC if fmt == 0 else b4gemv._lib.ENGINE_MMA_NF4
    return cfg


def fresh_ws(cuda, fmt, in_f, out_f, cfg=None):
    import torch
    n = b4gemv.workspace_size(fmt, in_f, out_f, 1, cfg)
    assert n > 0
    return torch.zeros(n, dtype=torch.uint8, device=cuda)


@pytest.mark.parametrize("fmt,out_f,in_f", [(0, 8192, 8192), (0, 3584, 3584), (1, 3584, 18944)])
def test_explicit_split_matches_the_rule_and_oracle(cuda, oracle, fmt, out_f, in_f):
    rng = np.random.default_rng(300 + fmt + out_f)
    W, X = rand_problem(rng, out_f, in_f)
    qw, sc = quantised(fmt, W, cuda)
    cfg = split_config(fmt, 2 if fmt == 0 else 3, 4 if fmt == 0 else 1)
    ws = fresh_ws(cuda, fmt, in_f, out_f, cfg)
    y = b4gemv.gemv_ws(fmt, qw, sc, to_dev(X, cuda), config=cfg, ws=ws).cpu().numpy()
    ref = f64_ref(oracle, fmt, qw, sc, X)
    assert rel_err(y, ref) < TOL
    y0 = (b4gemv.gemv_int4 if fmt == 0 else b4gemv.gemv_nf4)(qw, sc, to_dev(X, cuda), use_ws=False).cpu().numpy()
    assert rel_err(y, y0) < TOL
    # the counters (past the x-pair table kernel's 256 bytes) are zero again after the call
    assert int(ws[256: 256 + ((out_f + 15) // 16) * 4].count_nonzero()) == 0


@pytest.mark.parametrize("name", list(QWEN))
def test_rule_does_not_split_where_it_does_not_pay(cuda, name):
    """No batch-1 shape measured faster split once every CTA has one resident tile:
    the workspace rule never sets B4_FLAG_SPLIT, and the only workspace it asks
    for is the x-pair table kernel's two counters (NF4, >= 24 MB of weights)."""
    out_f, in_f = QWEN[name]
    for fmt in (0, 1):
        for o, i in ((out_f, in_f), (8192, 8192), (28672, 8192)):
            cfg = b4gemv.default_config_ws(fmt, i, o, 1)
            assert not cfg["flags"] & b4gemv.FLAG_SPLIT
            xtab = cfg["engine"] == b4gemv.ENGINE_NF4_XTAB
            wb = o * i // 2 + o * (i // 64) * 4
            assert xtab == (fmt == 1 and (wb >= 17_500_000 or (i >= 8192 and wb >= 5_000_000)))
            assert b4gemv.workspace_size(fmt, i, o) == (b4gemv.XTAB_WORKSPACE_BYTES if xtab else 0)


@pytest.mark.parametrize("stages,groups", INT4_VARIANTS)
@pytest.mark.parametrize("shape", [(3584, 3584), (2049, 1024), (16, 4096), (300, 18944)])
def test_int4_split_every_variant(cuda, oracle, stages, groups, shape):
    out_f, in_f = shape
    if (in_f // 128) % groups:
        pytest.skip("stage groups must divide in_f/128")
    rng = np.random.default_rng(out_f + in_f + stages * 10 + groups)
    W, X = rand_problem(rng, out_f, in_f)
    qw, sc = quantised(0, W, cuda)
    cfg = split_config(0, stages, groups)
    ws = fresh_ws(cuda, 0, in_f, out_f, cfg)
    y = b4gemv.gemv_ws(0, qw, sc, to_dev(X, cuda), config=cfg, ws=ws).cpu().numpy()
    assert rel_err(y, f64_ref(oracle, 0, qw, sc, X)) < TOL, (stages, groups, shape)


@pytest.mark.parametrize("stages", NF4_VARIANTS)
@pytest.mark.parametrize("shape", [(3584, 3584), (2049, 1024), (16, 4096), (300, 18944)])
def test_nf4_split_every_variant(cuda, oracle, stages, shape):
    out_f, in_f = shape
    rng = np.random.default_rng(out_f + in_f + stages)
    W, X = rand_problem(rng, out_f, in_f)
    qw, sc = quantised(1, W, cuda)
    cfg = split_config(1, stages)
    ws = fresh_ws(cuda, 1, in_f, out_f, cfg)
    y = b4gemv.gemv_ws(1, qw, sc, to_dev(X, cuda), config=cfg, ws=ws).cpu().numpy()
    assert rel_err(y, f64_ref(oracle, 1, qw, sc, X)) < TOL, (stages, shape)


@pytest.mark.parametrize("fmt", [0, 1])
def test_split_repeats_bit_identical_and_leaves_counters_zero(cuda, fmt):
    import torch
    out_f, in_f = 3584, 18944
    rng = np.random.default_rng(77 + fmt)
    W, X = rand_problem(rng, out_f, in_f)
    qw, sc = quantised(fmt, W, cuda)
    cfg = split_config(fmt, 4 if fmt == 0 else 3, 2 if fmt == 0 else 1)
    ws = fresh_ws(cuda, fmt, in_f, out_f, cfg)
    Xd = to_dev(X, cuda)
    ys = [b4gemv.gemv_ws(fmt, qw, sc, Xd, config=cfg, ws=ws).clone() for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    nblocks = (out_f + 15) // 16
    assert int(ws[256: 256 + nblocks * 4].count_nonzero()) == 0


@pytest.mark.parametrize("fmt", [0, 1])
def test_split_as_programmatic_dependent_and_in_a_graph(cuda, oracle, fmt):
    import torch
    out_f, in_f = 3584, 3584
    rng = np.random.default_rng(91 + fmt)
    W, X = rand_problem(rng, out_f, in_f)
    qw, sc = quantised(fmt, W, cuda)
    cfg = split_config(fmt, 4 if fmt == 0 else 3, 2 if fmt == 0 else 1, flags=b4gemv.FLAG_PDL)
    ws = fresh_ws(cuda, fmt, in_f, out_f, cfg)
    xsrc = to_dev(X, cuda)
    x = torch.zeros_like(xsrc)
    y = torch.zeros((1, out_f), dtype=torch.float32, device=cuda)
    ref = f64_ref(oracle, fmt, qw, sc, X)
    for _ in range(3):
        x.zero_()
        x.copy_(xsrc)                      # the producer kernel
        b4gemv.gemv_ws(fmt, qw, sc, x, y=y, config=cfg, ws=ws)
    assert rel_err(y.cpu().numpy(), ref) < TOL
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(4):
            b4gemv.gemv_ws(fmt, qw, sc, x, y=y, config=cfg, ws=ws, stream=s)
    y.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), ref) < TOL
    assert int(ws[256: 256 + ((out_f + 15) // 16) * 4].count_nonzero()) == 0


def test_split_argument_checks(cuda):
    import torch
    out_f, in_f = 8192, 8192
    rng = np.random.default_rng(5)
    W, X = rand_problem(rng, out_f, in_f)
    qw, sc = quantised(0, W, cuda)
    Xd = to_dev(X, cuda)
    y = torch.empty((1, out_f), dtype=torch.float32, device=cuda)
    lib = load()
    cfg_d = split_config(0, 2, 4)
    cfg = GemvConfig.from_dict(cfg_d)
    need = b4gemv.workspace_size(0, in_f, out_f, 1, cfg_d)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    p = ctypes.c_void_p
    args = (0, p(qw.data_ptr()), p(sc.data_ptr()), p(Xd.data_ptr()), p(y.data_ptr()), in_f, out_f, 1)
    st = p(torch.cuda.current_stream().cuda_stream)
    # too small, missing or misaligned workspace: rejected before any launch
    assert lib.b4_gemv_ws(*args, ctypes.byref(cfg), p(ws.data_ptr()), need - 1, st) == 1
    assert lib.b4_gemv_ws(*args, ctypes.byref(cfg), None, 0, st) == 1
    assert lib.b4_gemv_ws(*args, ctypes.byref(cfg), p(ws.data_ptr() + 4), need - 4, st) == 1
    # the split flag needs the workspace entry point
    assert lib.b4_gemv_ex(*args, ctypes.byref(cfg), st) == 1
    # batch > 1 never splits, nor does the rule: no workspace needed
    assert b4gemv.workspace_size(0, in_f, out_f, 2) == 0
    assert lib.b4_gemv_ws(*args, None, None, 0, st) == 0
    assert lib.b4_gemv_ws(*args, ctypes.byref(cfg), p(ws.data_ptr()), need, st) == 0
    torch.cuda.synchronize()
