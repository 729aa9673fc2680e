"""GPU parity of the x-pair table NF4 kernel (B4_ENGINE_NF4_XTAB), through the C ABI.

The kernel covers in_f in 256-column slices, one CTA per SM; the slices' shares
of y meet through fp32 atomic adds after every CTA has zeroed its rows and
counted itself in on the workspace.  These tests check y against the oracle's
double GEMV (max relative error below TOL, the metric of int4_gemv.cu:74-81)
on the shapes that exercise each part of that scheme: one slice, slices shared
by 10-11 CTAs, more slices than CTAs (each CTA loops over slices), rows not a
multiple of the 16-row batch, several segments in one launch, y pre-filled with
NaN (every row must be zeroed), back-to-back calls (the workspace's two
running counters, arrivals and base, must be equal between calls and advance
by the grid each call), and the NaN rows of the reference's edge fixture.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import b4gemv
from b4gemv._lib import GemvConfig, GemvSegment, load
from oracle_py import rel_err
from test_gemv_gpu import QWEN, f64_ref, quantised, rand_problem, to_dev

TOL = 1e-3
pytestmark = pytest.mark.gpu
XTAB = b4gemv.ENGINE_NF4_XTAB


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


VARIANTS = [(8, 4), (12, 2), (12, 3), (16, 2), (20, 1), (24, 1)]   # (warps per CTA, batches in flight per warp)


def xtab_cfg(warps=12, stages=3, flags=0):
    return dict(engine=XTAB, row_groups=warps, stages=stages, flags=flags)


def run_xtab(qw, am, x, out_f, in_f, cfg, ws, prefill=float("nan")):
    import torch
    y = torch.full((1, out_f), prefill, dtype=torch.float32, device=qw.device)
    c = GemvConfig.from_dict(cfg)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = load().b4_gemv_ws(1, _p(qw), _p(am), _p(x), _p(y), in_f, out_f, 1, ctypes.byref(c), _p(ws), ws.numel(), st)
    assert rc == 0, rc
    return y


@pytest.mark.parametrize("out_f,in_f", [(9, 512), (70, 3584), (300, 256), (5, 18944), (1000, 2048), (3, 40960),
                                        (2053, 1024), (1, 256)])
def test_xtab_every_variant_and_launch_kind(cuda, oracle, out_f, in_f):
    import torch
    rng = np.random.default_rng(out_f * 7 + in_f)
    W, X = rand_problem(rng, out_f, in_f)
    qw, am = quantised(1, W, cuda)
    ref = f64_ref(oracle, 1, qw, am, X)
    x = to_dev(X, cuda)
    ws = torch.zeros(b4gemv.XTAB_WORKSPACE_BYTES, dtype=torch.uint8, device=cuda)
    grid = torch.cuda.get_device_properties(cuda).multi_processor_count   # one CTA per SM
    calls = 0
    for warps, stages in VARIANTS:
        for flags in (0, b4gemv.FLAG_PDL):
            y = run_xtab(qw, am, x, out_f, in_f, xtab_cfg(warps, stages, flags), ws).cpu().numpy()
            calls += 1
            assert np.isfinite(y).all(), (out_f, in_f, warps, stages, flags)
            assert rel_err(y, ref) < TOL, (out_f, in_f, warps, stages, flags)
            counters = ws[:8].view(torch.int32).cpu().tolist()
            assert counters == [calls * grid] * 2, (counters, calls, grid)
    torch.cuda.synchronize()
    assert not ws[8:].any().item()
    assert load().b4_device_error(1) == 0


@pytest.mark.parametrize("name", list(QWEN))
def test_xtab_in_the_ws_rule_on_qwen_shapes(cuda, oracle, name):
    """The rule of b4_gemv_ws takes the x-pair table kernel for the large
    projections (gate/up/down) and the other NF4 kernels for q/k/v/o; either
    way the public GEMV is within tolerance."""
    out_f, in_f = QWEN[name]
    cfg = b4gemv.default_config_ws(1, in_f, out_f, 1)
    big = name in ("gate_proj", "up_proj", "down_proj")
    assert (cfg["engine"] == XTAB) == big
    assert b4gemv.workspace_size(1, in_f, out_f, 1) == (b4gemv.XTAB_WORKSPACE_BYTES if big else 0)
    rng = np.random.default_rng(len(name) * 31 + out_f)
    W, X = rand_problem(rng, out_f, in_f)
    qw, am = quantised(1, W, cuda)
    ref = f64_ref(oracle, 1, qw, am, X)
    for pdl in (False, True):
        y = b4gemv.gemv_nf4(qw, am, to_dev(X, cuda), pdl=pdl).cpu().numpy()
        assert rel_err(y, ref) < TOL


def test_xtab_back_to_back_calls_new_inputs(cuda, oracle):
    """Two calls in a row with different x and the same y and workspace: the
    second must not see the first's sums or counters."""
    import torch
    rng = np.random.default_rng(5)
    out_f, in_f = 4096, 3584
    W, X1 = rand_problem(rng, out_f, in_f)
    X2 = rng.standard_normal((1, in_f)).astype(np.float16)
    qw, am = quantised(1, W, cuda)
    ws = torch.zeros(b4gemv.XTAB_WORKSPACE_BYTES, dtype=torch.uint8, device=cuda)
    y = torch.empty((1, out_f), dtype=torch.float32, device=cuda)
    outs = []
    for X in (X1, X2, X1):
        b4gemv.gemv_ws(1, qw, am, to_dev(X, cuda), y, ws=ws, pdl=True)
        outs.append(y.cpu().numpy().copy())
    assert rel_err(outs[0], f64_ref(oracle, 1, qw, am, X1)) < TOL
    assert rel_err(outs[1], f64_ref(oracle, 1, qw, am, X2)) < TOL
    assert rel_err(outs[2], outs[0]) < 1e-6


def test_one_workspace_serves_every_path_in_any_order(cuda, oracle):
    """A b4_gemv_ws workspace keeps the x-pair table kernel's running counters
    in its first 256 bytes and hands the rest to the split and k-slice paths
    (the split's arrival counters first, zero after each call; the k-slice
    partials, cleared once summed): x-pair table, k-slice and split calls
    alternating on one workspace all stay within tolerance, and no arrival
    wait times out."""
    import torch
    from test_gemv_gpu import ksliced_config
    from test_split_gpu import split_config
    rng = np.random.default_rng(21)
    W1, X1 = rand_problem(rng, 2048, 3584)
    qw1, am1 = quantised(1, W1, cuda)
    W2, X2 = rand_problem(rng, 300, 4096, 3)
    qw2, am2 = quantised(1, W2, cuda)
    W3, X3 = rand_problem(rng, 3584, 3584)
    qw3, sc3 = quantised(0, W3, cuda)
    c1 = xtab_cfg(16, 2, b4gemv.FLAG_PDL)
    c2 = ksliced_config(1, 4096, 300, 3, 2, pdl=True)
    c3 = split_config(0, 2, 4)
    need = max(b4gemv.workspace_size(1, 3584, 2048, 1, c1), b4gemv.workspace_size(1, 4096, 300, 3, c2),
               b4gemv.workspace_size(0, 3584, 3584, 1, c3))
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    refs = {"xtab": f64_ref(oracle, 1, qw1, am1, X1), "kslice": f64_ref(oracle, 1, qw2, am2, X2),
            "split": f64_ref(oracle, 0, qw3, sc3, X3)}
    runs = {"xtab": lambda: b4gemv.gemv_ws(1, qw1, am1, to_dev(X1, cuda), config=c1, ws=ws),
            "kslice": lambda: b4gemv.gemv_ws(1, qw2, am2, to_dev(X2, cuda), config=c2, ws=ws),
            "split": lambda: b4gemv.gemv_ws(0, qw3, sc3, to_dev(X3, cuda), config=c3, ws=ws)}
    load().b4_device_error(1)
    for name in ("xtab", "kslice", "xtab", "split", "xtab", "kslice", "split", "kslice", "xtab"):
        y = runs[name]().cpu().numpy()
        assert rel_err(y, refs[name]) < TOL, name
        counters = ws[:8].view(torch.int32).cpu().tolist()
        assert counters[0] == counters[1], (name, counters)
        assert int(ws[256: 256 + 224 * 4].count_nonzero()) == 0, name   # the split's 224 row-block counters
        if name == "kslice":   # its 2 slices x 3 rows x 300 partials, cleared
            assert int(ws[256: 256 + 2 * 3 * 300 * 4].count_nonzero()) == 0
    assert load().b4_device_error(1) == 0


def _tail_split(S, nb, G, item_cost=45):
    """The host's choice of tail batches per slice (xtab_tail in b4_gemv.cu),
    restated to pick test shapes that take the main + tail split."""
    if S > G or G % S == 0 or nb < 2:
        return 0
    k, E = G // S, G - (G // S) * S
    even = -(-nb // k)
    best, best_r = even, 0
    for r in range(1, nb - k + 1):
        worst = -(-(nb - r) // k)
        T = S * r
        for e in range(E):
            lo, hi = e * T // E, (e + 1) * T // E
            if hi > lo:
                worst = max(worst, hi - lo + item_cost * ((hi - 1) // r - lo // r))
            if worst >= best:
                break
        if worst < best:
            best, best_r = worst, r
    return best_r if 100 * best < 97 * even else 0


@pytest.mark.parametrize("outs,in_f", [([8192], 14336), ([7168, 7168], 8192)])
def test_xtab_main_and_tail_ctas(cuda, oracle, outs, in_f):
    """Shapes whose slices divide unevenly over the SMs (56 and 32 slices on
    148 SMs) run on main CTAs per slice plus tail CTAs whose runs cross slice
    boundaries (several table builds per CTA, the next item's loads issued
    before the barrier): every row within tolerance of the oracle, one and
    two segments."""
    import torch
    G = torch.cuda.get_device_properties(cuda).multi_processor_count
    nb = sum((o + 15) // 16 for o in outs)
    if _tail_split(in_f // 256, nb, G) == 0:
        pytest.skip(f"the even split is taken on {G} SMs")
    rng = np.random.default_rng(sum(outs) + in_f)
    X = rng.standard_normal((1, in_f)).astype(np.float16)
    pairs, refs = [], []
    for o in outs:
        W = (rng.standard_normal((o, in_f)) * 0.02).astype(np.float32)
        qw, am = quantised(1, W, cuda)
        pairs.append((qw, am))
        refs.append(f64_ref(oracle, 1, qw, am, X))
    ws = torch.zeros(b4gemv.XTAB_WORKSPACE_BYTES, dtype=torch.uint8, device=cuda)
    load().b4_device_error(1)
    for _ in range(2):
        ys = b4gemv.gemv_multi(1, pairs, to_dev(X, cuda), ws=ws, pdl=True)
        for y, ref in zip(ys, refs):
            assert rel_err(y.cpu().numpy(), ref) < TOL
    assert load().b4_device_error(1) == 0


def test_xtab_multi_segment_one_launch(cuda, oracle):
    """q/k/v-like and ragged segments in one launch through b4_gemv_multi_ws."""
    import torch
    rng = np.random.default_rng(17)
    for shapes, in_f in [([3584, 512, 512], 3584), ([37, 9, 100, 1], 1024), ([18944, 18944], 3584)]:
        X = rng.standard_normal((1, in_f)).astype(np.float16)
        pairs, refs = [], []
        for out_f in shapes:
            W = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float32)
            qw, am = quantised(1, W, cuda)
            pairs.append((qw, am))
            refs.append(f64_ref(oracle, 1, qw, am, X))
        rule = b4gemv.multi_default_config_ws(1, pairs, to_dev(X, cuda))
        assert (rule["engine"] == XTAB) == (sum(shapes) == 2 * 18944)   # only gate+up is large enough
        ys = [torch.full((1, o), float("nan"), dtype=torch.float32, device=cuda) for o in shapes]
        for cfg in (None, xtab_cfg(), xtab_cfg(24, 1, b4gemv.FLAG_PDL), xtab_cfg(16, 2, b4gemv.FLAG_PDL)):
            for y in ys:
                y.fill_(float("nan"))
            out = b4gemv.gemv_multi(1, pairs, to_dev(X, cuda), ys=ys, config=cfg, pdl=cfg is None)
            for y, ref in zip(out, refs):
                assert rel_err(y.cpu().numpy(), ref) < TOL, (shapes, cfg)
    assert load().b4_device_error(1) == 0


def test_xtab_edge_fixture_nan_rows(cuda, golden, oracle):
    """The reference's edge case (NaN/inf weights, fp16 scale overflow): rows
    whose dequantised weights hold NaN or inf give NaN as the oracle does; the
    other rows stay within tolerance."""
    import torch
    g = golden["edge"]
    qw, am = to_dev(g["nf4_packed"], cuda), to_dev(g["nf4_absmax"], cuda)
    in_f = g["W"].shape[1]
    ws = torch.zeros(b4gemv.XTAB_WORKSPACE_BYTES, dtype=torch.uint8, device=cuda)
    ref = f64_ref(oracle, 1, qw, am, g["x"])[0]
    ok = np.isfinite(ref)
    for warps, stages in ((12, 3), (24, 1)):
        y = run_xtab(qw, am, to_dev(g["x"], cuda), qw.shape[0], in_f, xtab_cfg(warps, stages), ws).cpu().numpy()[0]
        assert np.array_equal(np.isfinite(y), np.isfinite(ref)), warps
        assert rel_err(y[ok], ref[ok]) < TOL, warps


def test_xtab_refusals(cuda):
    """The kernel needs a workspace and in_f % 256 == 0: the entry points
    without one, a short workspace and other shapes are refused before any
    launch."""
    import torch
    out_f, in_f = 64, 1024
    qw = torch.zeros((out_f, in_f // 8), dtype=torch.int32, device=cuda)
    am = torch.ones((out_f, in_f // 64), dtype=torch.float32, device=cuda)
    x = torch.zeros((1, in_f), dtype=torch.float16, device=cuda)
    y = torch.zeros((1, out_f), dtype=torch.float32, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    c = GemvConfig.from_dict(xtab_cfg())
    lib = load()
    assert lib.b4_gemv_ex(1, _p(qw), _p(am), _p(x), _p(y), in_f, out_f, 1, ctypes.byref(c), st) == 1
    ws = torch.zeros(64, dtype=torch.uint8, device=cuda)
    assert lib.b4_gemv_ws(1, _p(qw), _p(am), _p(x), _p(y), in_f, out_f, 1, ctypes.byref(c), _p(ws), 64, st) == 1
    ws = torch.zeros(256, dtype=torch.uint8, device=cuda)
    qw2 = torch.zeros((out_f, 1088 // 8), dtype=torch.int32, device=cuda)
    am2 = torch.ones((out_f, 1088 // 64), dtype=torch.float32, device=cuda)
    x2 = torch.zeros((1, 1088), dtype=torch.float16, device=cuda)
    assert lib.b4_gemv_ws(1, _p(qw2), _p(am2), _p(x2), _p(y), 1088, out_f, 1, ctypes.byref(c), _p(ws), 256, st) == 1
    seg = (GemvSegment * 1)(GemvSegment(qw.data_ptr(), am.data_ptr(), y.data_ptr(), out_f))
    assert lib.b4_gemv_multi(1, seg, 1, _p(x), in_f, 1, ctypes.byref(c), st) == 1
    for bad_cfg in (xtab_cfg(32, 3), xtab_cfg(16, 5), xtab_cfg(24, 2)):   # no such (warps, stages) kernel
        bad = GemvConfig.from_dict(bad_cfg)
        assert lib.b4_gemv_ws(1, _p(qw), _p(am), _p(x), _p(y), in_f, out_f, 1, ctypes.byref(bad), _p(ws), 256, st) == 1
    torch.cuda.synchronize()
