"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bars: packed codes, dequantised values and the W_dequant reconstruction are
bit-exact; y is within TOL max relative error (max|y-ref| / max|ref|, the
metric of int4_gemv.cu:74-81) of a double-precision GEMV over the same
dequantised weights and fp16 x.
"""
from __future__ import annotations

import itertools

import numpy as np
import pytest

import b4gemv
from b4gemv.diag import LEAN_VARIANTS
from oracle_py import rel_err

TOL = 1e-3
pytestmark = pytest.mark.gpu

QWEN = {"q_proj": (3584, 3584), "k_proj": (512, 3584), "v_proj": (512, 3584), "o_proj": (3584, 3584),
        "gate_proj": (18944, 3584), "up_proj": (18944, 3584), "down_proj": (3584, 18944)}


def to_dev(a, dev):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    if a.dtype == np.uint16:
        a = a.view(np.float16)
    return torch.from_numpy(a).to(dev)


def quantised(fmt, W, dev):
    """Host-quantised weights on the device: (qw, scale)."""
    if fmt == 0:
        p, s, _ = b4gemv.quantise(W)
        return to_dev(p, dev), to_dev(s, dev)
    p, a, _ = b4gemv.quantise_nf4(W)
    return to_dev(p, dev), to_dev(a, dev)


def f64_ref(oracle, fmt, qw, scale, X):
    p = qw.cpu().numpy().view(np.uint32)
    s = scale.cpu().numpy()
    return oracle.gemv_f64(fmt == 1, p, s.view(np.uint16) if fmt == 0 else s, X)


def rand_problem(rng, out_f, in_f, m=1):
    W = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float32)
    X = rng.standard_normal((m, in_f)).astype(np.float16)
    return W, X


# ---- bit-exact format kernels ---------------------------------------------------

@pytest.mark.parametrize("case", ["kat_glibc", "gauss_33x384", "gauss_5x640", "edge"])
def test_device_quantiser_dequant_and_codes_bit_exact(cuda, golden, oracle, case):
    import torch
    g = golden[case]
    W = torch.from_numpy(g["W"]).to(cuda)
    p, s, d = b4gemv.quantise_device(W, with_deq=True)
    pn, a, dn = b4gemv.quantise_nf4_device(W, with_deq=True)
    torch.cuda.synchronize()
    assert p.cpu().numpy().view(np.uint32).tobytes() == g["int4_packed"].tobytes()
    assert s.cpu().numpy().view(np.uint16).tobytes() == g["int4_scales"].tobytes()
    assert d.cpu().numpy().tobytes() == g["int4_deq"].tobytes()
    assert pn.cpu().numpy().view(np.uint32).tobytes() == g["nf4_packed"].tobytes()
    assert a.cpu().numpy().tobytes() == g["nf4_absmax"].tobytes()
    assert dn.cpu().numpy().tobytes() == g["nf4_deq"].tobytes()
    # W_dequant reconstruction and unpacked codes from the reference's buffers
    qw = to_dev(g["int4_packed"], cuda)
    assert b4gemv.dequant_int4(qw, to_dev(g["int4_scales"], cuda)).cpu().numpy().tobytes() == g["int4_deq"].tobytes()
    qn = to_dev(g["nf4_packed"], cuda)
    assert b4gemv.dequant_nf4(qn, to_dev(g["nf4_absmax"], cuda)).cpu().numpy().tobytes() == g["nf4_deq"].tobytes()
    in_f = g["W"].shape[1]
    assert np.array_equal(b4gemv.unpack_codes(qw).cpu().numpy(), oracle.unpack(g["int4_packed"], in_f))


def test_device_quantiser_bit_exact_at_qwen_size(cuda):
    import torch
    rng = np.random.default_rng(11)
    for out_f, in_f in [(512, 3584), (256, 18944)]:
        W = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float32)
        p, s, d = b4gemv.quantise(W)
        pn, a, dn = b4gemv.quantise_nf4(W)
        Wd = torch.from_numpy(W).to(cuda)
        gp, gs, gd = b4gemv.quantise_device(Wd, with_deq=True)
        gpn, ga, gdn = b4gemv.quantise_nf4_device(Wd, with_deq=True)
        assert gp.cpu().numpy().view(np.uint32).tobytes() == p.tobytes()
        assert gs.cpu().numpy().tobytes() == s.tobytes() and gd.cpu().numpy().tobytes() == d.tobytes()
        assert gpn.cpu().numpy().view(np.uint32).tobytes() == pn.tobytes()
        assert ga.cpu().numpy().tobytes() == a.tobytes() and gdn.cpu().numpy().tobytes() == dn.tobytes()
        assert b4gemv.dequant_nf4(gpn, ga).cpu().numpy().tobytes() == dn.tobytes()
        assert b4gemv.dequant_int4(gp, gs).cpu().numpy().tobytes() == d.tobytes()


# ---- GEMV parity ------------------------------------------------------------------

@pytest.mark.parametrize("case", ["kat_glibc", "gauss_7x128", "gauss_33x384", "gauss_8x1024", "gauss_1x128",
                                  "gauss_5x640", "gauss_16x256"])
@pytest.mark.parametrize("fmt", [0, 1])
def test_gemv_golden_cases(cuda, golden, oracle, case, fmt):
    g = golden[case]
    if fmt == 0:
        qw, sc = to_dev(g["int4_packed"], cuda), to_dev(g["int4_scales"], cuda)
        y = b4gemv.gemv_int4(qw, sc, to_dev(g["x"], cuda))
    else:
        qw, sc = to_dev(g["nf4_packed"], cuda), to_dev(g["nf4_absmax"], cuda)
        y = b4gemv.gemv_nf4(qw, sc, to_dev(g["x"], cuda))
    ref = f64_ref(oracle, fmt, qw, sc, g["x"])
    assert rel_err(y.cpu().numpy(), ref) < TOL


def test_gemv_edge_case_nan_rows(cuda, golden, oracle):
    """Rows whose dequantised weights hold NaN (fp16 scale overflow) give NaN;
    the other rows stay within tolerance."""
    g = golden["edge"]
    for fmt, p, s in [(0, g["int4_packed"], g["int4_scales"]), (1, g["nf4_packed"], g["nf4_absmax"])]:
        qw, sc = to_dev(p, cuda), to_dev(s, cuda)
        y = b4gemv.gemv(fmt, qw, sc, to_dev(g["x"], cuda)).cpu().numpy()[0]
        ref = f64_ref(oracle, fmt, qw, sc, g["x"])[0]
        assert np.array_equal(np.isnan(y), np.isnan(ref))
        ok = ~np.isnan(ref)
        assert rel_err(y[ok], ref[ok]) < TOL


def kernel_configs():
    """Every instantiated kernel (vec_words, rows_per_warp, batch_tile, nf4_lut)."""
    out = [(0, 4, rw, mb, 0, 1) for rw in (16, 32) for mb in (8, 16)]  # tensor-pipe INT4
    out += [(0, 4, 16, mb, 0, 2) for mb in (8, 16)]                     # tensor pipe + bulk-copy ring
    out += [(0, 4, 16, 1, 0, 5)]                                                         # lean INT4, m = 1
    out += [(1, vw, rw, 1, lut, 6) for vw, rw, lut in [(2, 4, 0), (2, 8, 0), (4, 4, 0), (2, 4, 2), (2, 8, 2),
                                                       (4, 4, 2)]]                       # lean NF4, m = 1
    out += [(1, 4, 16, 1, 0, 7)]                                                         # NF4 tensor pipe, m = 1
    for fmt in (0, 1):
        for lut in ((0,) if fmt == 0 else (0, 1)):
            for vw, rw in [(1, 1), (1, 4)]:
                out.append((fmt, vw, rw, 1, lut, 0))
            for vw in (2, 4):
                for mb in (1, 2, 4):
                    for rw in (1, 2, 4, 8):
                        if not (mb == 4 and rw == 8):
                            out.append((fmt, vw, rw, mb, lut, 0))
    return out


@pytest.mark.parametrize("fmt,vw,rw,mb,lut,engine", kernel_configs())
def test_gemv_every_kernel(cuda, oracle, fmt, vw, rw, mb, lut, engine):
    rng = np.random.default_rng(1000 + fmt * 100 + vw * 10 + rw + mb * 7 + lut + engine)
    cases = [(37, 1152, 1), (9, 512, 3), (70, 3584, 5)]
    if engine in (1, 2):
        cases += [(100, 1024, 11 if mb == 16 else 7), (33, 2048, mb), (48, 640, 8), (16, 128, 1)]
    if engine == 6:   # m = 1, ragged last step included
        cases = [(37, 1152, 1), (9, 512, 1), (70, 3584, 1), (300, 64, 1), (5, 18944, 1), (3, 1088, 1)]
    if engine == 5:        # m = 1
        cases = [(37, 1152, 1), (9, 512, 1), (70, 3584, 1), (300, 128, 1), (5, 18944, 1)]
    if engine == 7:        # m = 1, in_f a multiple of 128
        cases = [(37, 1152, 1), (9, 512, 1), (70, 3584, 1), (300, 128, 1), (5, 18944, 1), (33, 896, 1)]
    for out_f, in_f, m in cases:
        W, X = rand_problem(rng, out_f, in_f, m)
        qw, sc = quantised(fmt, W, cuda)
        ref = f64_ref(oracle, fmt, qw, sc, X)
        Xd = to_dev(X, cuda)
        for kw, rg in [(1, 1), (2, 2), (4, 1), (1, 4)]:
            if (rw > 1 or mb > 1) and kw * rg > 8:
                continue
            cfg = dict(vec_words=vw, rows_per_warp=rw, warps_k=kw, row_groups=rg, batch_tile=mb, nf4_lut=lut,
                       engine=engine)
            if engine == 2:
                for st, kcg in [(4, 4), (3, 4), (6, 4), (4, 2), (4, 8), (8, 2)] if mb == 8 else [(4, 4)]:
                    cfg.update(stages=st, stage_groups=kcg)
                    y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
                    assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
                assert b4gemv.load().b4_device_error(1) == 0
                continue
            if engine == 6:
                sts = {(2, 4, 0): (4, 6), (2, 8, 0): (4,), (4, 4, 0): (4,), (2, 4, 2): (4, 6, 8), (2, 8, 2): (4,),
                       (4, 4, 2): (4,)}[(vw, rw, lut)]
                for st in sts:
                    for flags in (0, b4gemv.FLAG_PDL):
                        cfg.update(stages=st, flags=flags)
                        y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
                        assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
                continue
            if engine == 7:
                for st in (2, 3, 4):
                    for flags in (0, b4gemv.FLAG_PDL):
                        cfg.update(stages=st, flags=flags)
                        y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
                        assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
                for tr in (1, 5, 13):   # rows per 16-row MMA block that carry weights
                    cfg.update(stages=3, flags=0, tile_rows=tr)
                    y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
                    assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
                cfg.update(tile_rows=0)
                continue
            if engine == 5:
                variants = LEAN_VARIANTS
                for st, sg in variants:
                    cfg.update(stages=st, stage_groups=sg)
                    if (in_f // 128) % sg:   # a stage of sg groups must tile the row
                        with pytest.raises(b4gemv.B4Error):
                            b4gemv.gemv(fmt, qw, sc, Xd, config=cfg)
                        continue
                    for flags in (0, b4gemv.FLAG_PDL):
                        cfg.update(flags=flags)
                        y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
                        assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
                for tr in (1, 5, 13):   # rows per 16-row MMA block that carry weights
                    cfg.update(stages=variants[0][0], stage_groups=variants[0][1], flags=0, tile_rows=tr)
                    y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
                    assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
                cfg.update(tile_rows=0)
                continue
            y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
            assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
        if engine >= 2:
            continue   # x is staged whole: no x tiles
        # several x tiles in shared memory
        cfg = dict(vec_words=vw, rows_per_warp=rw, warps_k=2, row_groups=1, batch_tile=mb, nf4_lut=lut,
                   x_tile=(128 if engine == 1 else 8 * vw * 32), engine=engine)
        y = b4gemv.gemv(fmt, qw, sc, Xd, config=cfg).cpu().numpy()
        assert rel_err(y, ref) < TOL, ("x_tile", out_f, in_f, m, cfg)


@pytest.mark.parametrize("name", list(QWEN))
@pytest.mark.parametrize("fmt", [0, 1])
def test_gemv_qwen_shapes(cuda, oracle, name, fmt):
    out_f, in_f = QWEN[name]
    rng = np.random.default_rng(hash(name) % 1000 + fmt)
    W, X = rand_problem(rng, out_f, in_f)
    qw, sc = quantised(fmt, W, cuda)
    y = (b4gemv.gemv_int4 if fmt == 0 else b4gemv.gemv_nf4)(qw, sc, to_dev(X, cuda)).cpu().numpy()
    ref = f64_ref(oracle, fmt, qw, sc, X)
    assert rel_err(y, ref) < TOL


@pytest.mark.parametrize("m", [2, 3, 4, 8, 16])
@pytest.mark.parametrize("fmt", [0, 1])
def test_gemv_small_batch(cuda, oracle, m, fmt):
    rng = np.random.default_rng(50 + m)
    W, X = rand_problem(rng, 1000, 2048, m)
    qw, sc = quantised(fmt, W, cuda)
    y = b4gemv.gemv(fmt, qw, sc, to_dev(X, cuda)).cpu().numpy()
    assert rel_err(y, f64_ref(oracle, fmt, qw, sc, X)) < TOL


def test_gemv_misaligned_buffers_use_narrow_loads(cuda, oracle):
    """Codes at a 4-byte (not 16-byte) offset and x at a 2-byte offset: the
    4-byte load path runs and the result is unchanged."""
    import torch
    rng = np.random.default_rng(5)
    W, X = rand_problem(rng, 64, 1024)
    for fmt in (0, 1):
        qw, sc = quantised(fmt, W, cuda)
        big = torch.zeros(qw.numel() + 1, dtype=torch.int32, device=cuda)
        big[1:] = qw.reshape(-1)
        qw_off = big[1:].view(qw.shape)
        xb = torch.zeros(1024 + 1, dtype=torch.float16, device=cuda)
        xb[1:] = to_dev(X[0], cuda)
        x_off = xb[1:]
        assert qw_off.data_ptr() % 16 == 4 and x_off.data_ptr() % 4 == 2
        cfg = b4gemv.default_config(fmt, 1024, 64, 1)
        y = b4gemv.gemv(fmt, qw_off, sc, x_off.view(1, 1024)).cpu().numpy()
        assert rel_err(y, f64_ref(oracle, fmt, qw, sc, X)) < TOL
        assert cfg["vec_words"] >= 2  # the rule itself prefers vector loads


@pytest.mark.parametrize("wpb", [1, 2, 4, 8, 16])
def test_nf4_block_per_row_entry(cuda, oracle, wpb):
    rng = np.random.default_rng(wpb)
    W, X = rand_problem(rng, 96, 18944 // 4)
    qw, sc = quantised(1, W, cuda)
    y = b4gemv.gemv_nf4_block_per_row(qw, sc, to_dev(X, cuda), wpb).cpu().numpy()
    assert rel_err(y, f64_ref(oracle, 1, qw, sc, X)) < TOL


def test_pdl_launch_after_producer(cuda, oracle):
    """With the PDL flag the GEMV starts before the kernel that writes x has
    finished, and still reads the final x."""
    import torch
    rng = np.random.default_rng(9)
    W, X = rand_problem(rng, 3584, 3584)
    for fmt in (0, 1):
        qw, sc = quantised(fmt, W, cuda)
        cfg = b4gemv.default_config(fmt, 3584, 3584, 1)
        cfg["flags"] = b4gemv.FLAG_PDL
        xsrc = to_dev(X, cuda)
        x = torch.zeros_like(xsrc)
        for _ in range(3):
            x.zero_()
            x.copy_(xsrc)          # the producer kernel
            y = b4gemv.gemv(fmt, qw, sc, x, config=cfg)
        assert rel_err(y.cpu().numpy(), f64_ref(oracle, fmt, qw, sc, X)) < TOL


def test_results_are_deterministic(cuda):
    rng = np.random.default_rng(12)
    W, X = rand_problem(rng, 3584, 18944)
    for fmt in (0, 1):
        qw, sc = quantised(fmt, W, cuda)
        Xd = to_dev(X, cuda)
        a = b4gemv.gemv(fmt, qw, sc, Xd).cpu().numpy()
        b = b4gemv.gemv(fmt, qw, sc, Xd).cpu().numpy()
        assert a.tobytes() == b.tobytes()


@pytest.mark.parametrize("fmt", [0, 1])
def test_gemv_multi_segments_one_launch(cuda, oracle, fmt):
    """b4_gemv_multi: q/k/v-like segments (ragged row counts) over one x, each
    y_s within tolerance of its double GEMV, for the default config, every
    lean variant and the one-launch-per-segment engines; m = 2 takes the
    per-segment path."""
    rng = np.random.default_rng(77 + fmt)
    in_f = 1024
    shapes = [100, 37, 16, 250]
    Ws = [rand_problem(rng, o, in_f)[0] for o in shapes]
    X = rand_problem(rng, 1, in_f, 2)[1]
    pairs = [quantised(fmt, W, cuda) for W in Ws]
    refs = [[f64_ref(oracle, fmt, qw, sc, X[b:b + 1]) for qw, sc in pairs] for b in range(2)]
    x1 = to_dev(X[:1], cuda)
    for nseg in (1, 2, 3, 4):
        cfgs = [None]
        if fmt == 0:
            cfgs += [dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, engine=5,
                          stages=st, stage_groups=sg) for kw, rg in [(8, 1), (2, 4), (1, 2)]
                     for st, sg in LEAN_VARIANTS]
            cfgs += [dict(vec_words=4, rows_per_warp=16, warps_k=2, row_groups=2, batch_tile=8, engine=1)]
            cfgs += [dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, engine=e, stages=st,
                          stage_groups=sg, tile_rows=tr) for kw, rg in [(8, 1), (2, 2)] for tr in (3, 13)
                     for e, st, sg in [(5, 4, 1), (5, 2, 4)]]
        else:
            cfgs += [dict(vec_words=vw, rows_per_warp=rw, warps_k=kw, row_groups=rg, batch_tile=1, nf4_lut=lut,
                          engine=6, stages=4) for vw, rw, lut in [(2, 4, 0), (4, 4, 0), (2, 8, 2)]
                     for kw, rg in [(1, 8), (4, 2)]]
            cfgs += [dict(vec_words=2, rows_per_warp=2, warps_k=2, row_groups=2, batch_tile=1, engine=0)]
            cfgs += [dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, engine=7, stages=st)
                     for kw, rg in [(8, 1), (2, 4), (1, 2)] for st in (2, 3, 4)]
            cfgs += [dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, engine=7, stages=3,
                          tile_rows=tr) for kw, rg in [(8, 1), (2, 2)] for tr in (3, 13)]
        for cfg in cfgs:
            ys = b4gemv.gemv_multi(fmt, pairs[:nseg], x1, config=cfg)
            for s in range(nseg):
                assert rel_err(ys[s].cpu().numpy(), refs[0][s]) < TOL, (nseg, s, cfg)
    ys = b4gemv.gemv_multi(fmt, pairs, to_dev(X, cuda))
    for s in range(len(pairs)):
        for b in range(2):
            assert rel_err(ys[s][b:b + 1].cpu().numpy(), refs[b][s]) < TOL
    # the one-launch default agrees with separate launches within the fp32 accumulation order
    sep = [b4gemv.gemv(fmt, qw, sc, x1) for qw, sc in pairs]
    ys = b4gemv.gemv_multi(fmt, pairs, x1)
    for a, b in zip(ys, sep):
        assert rel_err(a.cpu().numpy(), b.cpu().numpy().astype(np.float64)) < 1e-5


def test_gemv_multi_rejects_bad_segments(cuda):
    import torch
    rng = np.random.default_rng(3)
    W, X = rand_problem(rng, 64, 1024)
    qw, sc = quantised(0, W, cuda)
    x = to_dev(X, cuda)
    with pytest.raises(AssertionError):
        b4gemv.gemv_multi(0, [(qw, sc)] * 5, x)           # more than B4_MAX_SEGMENTS
    qw2, sc2 = quantised(0, rand_problem(rng, 64, 512)[0], cuda)
    with pytest.raises(AssertionError):
        b4gemv.gemv_multi(0, [(qw, sc), (qw2, sc2)], x)   # in_f differs: x is shared
    segs = (b4gemv.GemvSegment * 2)(b4gemv.GemvSegment(qw.data_ptr(), sc.data_ptr(), None, 64),
                                    b4gemv.GemvSegment(qw.data_ptr(), sc.data_ptr(), None, 64))
    y = torch.empty(64, device=cuda)
    lib = b4gemv.load()
    assert lib.b4_gemv_multi(0, segs, 2, x.data_ptr(), 1024, 1, None, None) == 1   # null y
    segs[0].y = segs[1].y = y.data_ptr()
    assert lib.b4_gemv_multi(0, segs, 0, x.data_ptr(), 1024, 1, None, None) == 1   # no segment
    assert lib.b4_gemv_multi(0, segs, 2, x.data_ptr(), 1000, 1, None, None) == 1   # in_f % 128
    assert lib.b4_gemv_multi(0, segs, 2, x.data_ptr(), 1024, 1, None, None) == 0
    torch.cuda.synchronize()


def test_repack_bnb_nf4_matches_reference_packing(cuda, oracle):
    """bitsandbytes-layout bytes (lower column in the high nibble) of the
    reference quantiser's codes, repacked on the GPU, equal the reference's
    packed words bit for bit; repacking twice is the identity; the GEMV over
    repacked codes equals the GEMV over the reference-packed ones."""
    import torch
    from oracle_py import bnb_pack_nf4
    rng = np.random.default_rng(11)
    for out_f, in_f in [(7, 64), (33, 384), (256, 3584), (5, 18944)]:
        W = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float32)
        p, a, _ = oracle.quantise_nf4(W)
        codes = oracle.unpack(p, in_f)
        bnb = torch.from_numpy(bnb_pack_nf4(codes).reshape(out_f, in_f // 2)).to(cuda)
        qw = b4gemv.repack_bnb_nf4(bnb)
        assert qw.cpu().numpy().view(np.uint32).tobytes() == p.tobytes()
        back = b4gemv.repack_bnb_nf4(qw.view(torch.uint8).reshape(out_f, in_f // 2))
        assert back.cpu().numpy().view(np.uint8).tobytes() == bnb.cpu().numpy().tobytes()
        am = torch.from_numpy(a).to(cuda)
        x = torch.from_numpy(rng.standard_normal((1, in_f)).astype(np.float16)).to(cuda)
        y1 = b4gemv.gemv_nf4(qw, am, x).cpu().numpy()
        y2 = b4gemv.gemv_nf4(torch.from_numpy(p.view(np.int32)).to(cuda), am, x).cpu().numpy()
        assert y1.tobytes() == y2.tobytes()


@pytest.mark.parametrize("m", [2, 3, 5, 8, 9, 16])
def test_int4_small_batch_lean_kernel(cuda, oracle, m):
    """The lean INT4 kernel with batch rows in the MMA's N columns (engine 5,
    m = 2..16): every (stages, groups) variant, several warp splits and
    weight-carrying rows per MMA block, against the double GEMV per batch row."""
    rng = np.random.default_rng(300 + m)
    for out_f, in_f in [(70, 1024), (37, 3584), (300, 512)]:
        W, X = rand_problem(rng, out_f, in_f, m)
        qw, sc = quantised(0, W, cuda)
        ref = f64_ref(oracle, 0, qw, sc, X)
        Xd = to_dev(X, cuda)
        for (st, sg), (kw, rg), tr in itertools.product([(2, 4), (3, 2), (4, 1)], [(8, 1), (2, 2), (1, 4)], (0, 5)):
            if (in_f // 128) % sg:
                continue
            cfg = dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, engine=5, stages=st,
                       stage_groups=sg, tile_rows=tr)
            y = b4gemv.gemv(0, qw, sc, Xd, config=cfg).cpu().numpy()
            assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
    assert b4gemv.default_config(0, 3584, 18944, m)["engine"] == 5


@pytest.mark.parametrize("m", [2, 3, 5, 8, 9, 16])
def test_nf4_small_batch_tensor_pipe_kernel(cuda, oracle, m):
    """The NF4 tensor-pipe kernel with four batch rows per 8-column MMA block
    (engine 7, m = 2..16): both pipeline depths, several warp splits and
    weight-carrying rows per MMA block, against the double GEMV per batch row."""
    rng = np.random.default_rng(400 + m)
    for out_f, in_f in [(70, 1024), (37, 3584), (300, 512)]:
        W, X = rand_problem(rng, out_f, in_f, m)
        qw, sc = quantised(1, W, cuda)
        ref = f64_ref(oracle, 1, qw, sc, X)
        Xd = to_dev(X, cuda)
        for st, (kw, rg), tr in itertools.product((2, 3), [(8, 1), (2, 2), (1, 4)], (0, 5)):
            cfg = dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, engine=7, stages=st,
                       tile_rows=tr)
            y = b4gemv.gemv(1, qw, sc, Xd, config=cfg).cpu().numpy()
            assert rel_err(y, ref) < TOL, (out_f, in_f, m, cfg)
    assert b4gemv.default_config(1, 3584, 18944, m)["engine"] == 7


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("m", [8, 9, 16])
def test_long_rows_large_batch_run_as_tensor_pipe_chunks(cuda, oracle, fmt, m):
    """x for 8+ rows of 18944 columns does not fit next to the tensor-pipe
    engines' buffers: with the dispatch rule (cfg NULL, or B4_ENGINE_AUTO with
    the PDL flag) the plain entry points run batch chunks through them, and
    b4_gemv_ws (the Python default) runs column slices (B4_FLAG_KSLICE)."""
    import ctypes
    import torch
    out_f, in_f = 640, 18944
    rng = np.random.default_rng(70 + m + fmt)
    W, X = rand_problem(rng, out_f, in_f, m)
    qw, sc = quantised(fmt, W, cuda)
    assert b4gemv.default_config(fmt, in_f, out_f, m)["engine"] not in (5, 7)
    ref = f64_ref(oracle, fmt, qw, sc, X)
    Xd = to_dev(X, cuda)
    y = (b4gemv.gemv_int4 if fmt == 0 else b4gemv.gemv_nf4)(qw, sc, Xd).cpu().numpy()
    assert rel_err(y, ref) < TOL
    y2 = torch.full((m, out_f), float("nan"), dtype=torch.float32, device=cuda)
    cfg = b4gemv.GemvConfig.from_dict({"engine": b4gemv._lib.ENGINE_AUTO, "flags": b4gemv.FLAG_PDL})
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = ctypes.c_void_p
    assert b4gemv.load().b4_gemv_ex(fmt, p(qw.data_ptr()), p(sc.data_ptr()), p(Xd.data_ptr()), p(y2.data_ptr()),
                                    in_f, out_f, m, ctypes.byref(cfg), st) == 0
    torch.cuda.synchronize()
    assert rel_err(y2.cpu().numpy(), ref) < TOL


def ksliced_config(fmt, in_f, out_f, m, slices, pdl=False):
    """The k-sliced small-batch config: the rule's small-batch geometry for
    one slice, B4_FLAG_KSLICE, x_tile = the slice width."""
    sw = in_f // slices
    c = b4gemv.default_config(fmt, sw, out_f, m)
    assert c["engine"] in (5, 7), c
    if fmt == 0:
        while (sw // 128) % c["stage_groups"]:
            c["stage_groups"] //= 2
    c["flags"] = b4gemv.FLAG_KSLICE | (b4gemv.FLAG_PDL if pdl else 0)
    c["x_tile"] = sw
    return c


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("m", [2, 3, 8, 9, 16])
@pytest.mark.parametrize("out_f,in_f,slices", [(640, 18944, 4), (300, 4096, 2), (37, 2048, 4), (1200, 9472, 2)])
def test_ksliced_small_batch(cuda, oracle, fmt, m, out_f, in_f, slices):
    """B4_FLAG_KSLICE: the batch's GEMV as column slices (segments of one
    small-batch launch, x staged per slice, CTAs on contiguous tile runs) and
    an ordered sum of the slices' partial y; within tolerance of the oracle,
    the workspace size as b4_gemv_workspace_size reports it, and refused
    without one or with slices that do not tile the rows."""
    import ctypes
    import torch
    rng = np.random.default_rng(400 + m + fmt + in_f + out_f)
    W, X = rand_problem(rng, out_f, in_f, m)
    qw, sc = quantised(fmt, W, cuda)
    ref = f64_ref(oracle, fmt, qw, sc, X)
    Xd = to_dev(X, cuda)
    for pdl in (False, True):
        cfg = ksliced_config(fmt, in_f, out_f, m, slices, pdl)
        n = b4gemv.workspace_size(fmt, in_f, out_f, m, cfg)
        assert n == b4gemv.XTAB_WORKSPACE_BYTES + slices * m * out_f * 4
        ws = torch.zeros(n, dtype=torch.uint8, device=cuda)
        y = b4gemv.gemv_ws(fmt, qw, sc, Xd, torch.full((m, out_f), float("nan"), device=cuda), config=cfg,
                           ws=ws).cpu().numpy()
        assert rel_err(y, ref) < TOL, (pdl, cfg)
        assert int(ws.count_nonzero()) == 0   # the partials are cleared once summed
    lib, p = b4gemv.load(), ctypes.c_void_p
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    y = torch.empty((m, out_f), device=cuda)
    c = b4gemv.GemvConfig.from_dict(cfg)
    args = (fmt, p(qw.data_ptr()), p(sc.data_ptr()), p(Xd.data_ptr()), p(y.data_ptr()), in_f, out_f, m, ctypes.byref(c))
    assert lib.b4_gemv_ws(*args, p(ws.data_ptr()), n - 4, st) == 1
    assert lib.b4_gemv_ex(*args, st) == 1
    bad = b4gemv.GemvConfig.from_dict(dict(cfg, x_tile=in_f // slices + 64))
    assert lib.b4_gemv_ws(*args[:-1], ctypes.byref(bad), p(ws.data_ptr()), n, st) == 1
    torch.cuda.synchronize()


@pytest.mark.parametrize("fmt", [0, 1])
def test_python_api_pdl_matches_oracle(cuda, oracle, fmt):
    """gemv_int4 / gemv_nf4 with pdl=True: the dispatch rule's launch as a
    programmatic dependent (B4_ENGINE_AUTO + B4_FLAG_PDL) after a producer of x."""
    import torch
    rng = np.random.default_rng(808 + fmt)
    W, X = rand_problem(rng, 3584, 3584)
    qw, sc = quantised(fmt, W, cuda)
    xsrc = to_dev(X, cuda)
    x = torch.zeros_like(xsrc)
    fn = b4gemv.gemv_int4 if fmt == 0 else b4gemv.gemv_nf4
    for _ in range(3):
        x.zero_()
        x.copy_(xsrc)
        y = fn(qw, sc, x, pdl=True)
    assert rel_err(y.cpu().numpy(), f64_ref(oracle, fmt, qw, sc, X)) < TOL


@pytest.mark.parametrize("m", [9, 12, 16])
def test_int4_small_batch_sixteen_warp_ctas(cuda, oracle, m):
    """Batches of 9..16 rows on CTAs of 16 warps sharing one copy of x (engine 5,
    4 stages of 1 group; an explicit config): several warp splits, against the
    double GEMV."""
    rng = np.random.default_rng(900 + m)
    for out_f, in_f in [(70, 1024), (300, 3584), (2049, 512)]:
        W, X = rand_problem(rng, out_f, in_f, m)
        qw, sc = quantised(0, W, cuda)
        ref = f64_ref(oracle, 0, qw, sc, X)
        Xd = to_dev(X, cuda)
        for kw, rg in [(16, 1), (8, 2), (2, 8)]:
            cfg = dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, engine=5, stages=4,
                       stage_groups=1)
            y = b4gemv.gemv(0, qw, sc, Xd, config=cfg).cpu().numpy()
            assert rel_err(y, ref) < TOL, (out_f, in_f, m, kw, rg)


def test_int4_sixteen_warp_ctas_need_nine_rows(cuda):
    import torch
    qw = torch.zeros((64, 128), dtype=torch.int32, device=cuda)
    sc = torch.zeros((64, 8), dtype=torch.float16, device=cuda)
    x = torch.zeros((8, 1024), dtype=torch.float16, device=cuda)
    cfg = dict(vec_words=4, rows_per_warp=16, warps_k=16, row_groups=1, batch_tile=1, engine=5, stages=4,
               stage_groups=1)
    with pytest.raises(b4gemv.B4Error):
        b4gemv.gemv(0, qw, sc, x, config=cfg)


# ---- full-size properties (Llama-3-70B shapes, too large for a full CPU reference) ----

L70 = {"qo": (8192, 8192), "gate_up": (28672, 8192), "down": (8192, 28672)}
ORDER_TOL = 1e-6   # fp32 rounding of a different order of at most ~112 slice partials


def device_quantised(fmt, out_f, in_f, seed, cuda):
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    W = torch.randn((out_f, in_f), generator=g, device=cuda) * 0.02
    qw, sc, _ = (b4gemv.quantise_device if fmt == 0 else b4gemv.quantise_nf4_device)(W)
    del W
    return qw, sc


@pytest.mark.parametrize("name", list(L70))
@pytest.mark.parametrize("fmt", [0, 1])
def test_full_size_doubling_row_permutation_and_sampled_rows(cuda, oracle, name, fmt):
    """At the full Llama-3-70B shapes: y(2x) == 2 y(x) bit for bit (scaling x by
    2 is exact in fp16 and doubles every product and partial sum exactly);
    permuting the weight rows permutes y bit for bit (rows are independent);
    64 sampled rows within TOL of the double GEMV over their dequantised
    weights.  Where the rule picks the x-pair table kernel (NF4 here), whose
    256-column slices meet in y through atomic adds in run-dependent order,
    both properties hold to fp32 summation-order rounding instead: within
    ORDER_TOL of max |y|."""
    import torch
    out_f, in_f = L70[name]
    qw, sc = device_quantised(fmt, out_f, in_f, 40 + fmt, cuda)
    rng = np.random.default_rng(41 + fmt)
    X = rng.standard_normal((1, in_f)).astype(np.float16)
    x = to_dev(X, cuda)
    fn = b4gemv.gemv_int4 if fmt == 0 else b4gemv.gemv_nf4
    y1 = fn(qw, sc, x)
    y2 = fn(qw, sc, x * 2)
    torch.cuda.synchronize()
    assert torch.isfinite(y1).all()
    order_free = b4gemv.default_config_ws(fmt, in_f, out_f, 1)["engine"] == b4gemv.ENGINE_NF4_XTAB

    def same(a, b):
        if not order_free:
            return torch.equal(a, b)
        return float((a.double() - b.double()).abs().max()) <= ORDER_TOL * float(b.double().abs().max())

    assert same(y2, y1 * 2)
    perm = torch.randperm(out_f, generator=torch.Generator().manual_seed(7)).to(cuda)
    yp = fn(qw[perm].contiguous(), sc[perm].contiguous(), x)
    assert same(yp, y1[:, perm])
    rows = np.sort(rng.choice(out_f, 64, replace=False))
    ref = f64_ref(oracle, fmt, qw[rows].contiguous(), sc[rows].contiguous(), X)
    assert rel_err(y1.cpu().numpy()[:, rows], ref) < TOL
