"""Launch-geometry sweeps and profiling drivers (the role of the reference's
src/diag_aspect.cu on B200): the measurements the dispatch rule is fitted to.

  python -m b4gemv.diag sweep   [--fmt nf4|int4|both] [--shapes q_proj,...] [--json out.json]
      every kernel configuration in a grid, per shape: us per GEMV over 100
      graph-chained launches rotating over weight copies larger than L2.
  python -m b4gemv.diag aspect  [--fmt nf4|int4]
      the three sweeps of diag_aspect.cu:346-358 (aspect ratio at constant
      weight count, rows at fixed x, x size at fixed rows) with the dispatch
      rule's config.
  python -m b4gemv.diag run     --fmt nf4 --shape gate_proj [--m 1] [--launches 4] [--config k=v,...]
      a few launches of one GEMV (the command profiled by ncu).
  python -m b4gemv.diag step    [--steps 10]
      the benchmark's NF4 decode step, eagerly (the launch list's command).
  python -m b4gemv.diag glue    [--n 28672] [--launches 3]
      the decode layer's elementwise kernels.
Run from int4-gemv_b200/ (or with it on sys.path).
"""
from __future__ import annotations

import argparse
import ctypes
import itertools
import json
import sys

from . import FLAG_PDL, FLAG_SPLIT, FMT_INT4_G128, FMT_NF4_B64, GemvConfig, check, load, quantise_nf4_device

SHAPES = {"q_proj": (3584, 3584), "k_proj": (512, 3584), "v_proj": (512, 3584), "o_proj": (3584, 3584),
          "gate_proj": (18944, 3584), "up_proj": (18944, 3584), "down_proj": (3584, 18944),
          # Llama-3-70B layer and its tensor-parallel shards (column-parallel rows, row-parallel columns)
          "l70_qo": (8192, 8192), "l70_kv": (1024, 8192), "l70_gu": (28672, 8192), "l70_down": (8192, 28672),
          "tp2_q": (4096, 8192), "tp2_kv": (512, 8192), "tp2_gu": (14336, 8192), "tp2_o": (8192, 4096),
          "tp2_down": (8192, 14336), "tp4_q": (2048, 8192), "tp4_gu": (7168, 8192), "tp4_o": (8192, 2048),
          "tp4_down": (8192, 7168), "tp8_q": (1024, 8192), "tp8_gu": (3584, 8192), "tp8_o": (8192, 1024),
          "tp8_down": (8192, 3584)}
L2_BYTES = 126 * 1024 * 1024
WS_BYTES = 8 << 20   # workspace for the split configs (the largest shape here needs < 1 MiB)


def alg_bytes(fmt, out_f, in_f, m=1):
    scale = out_f * (in_f // 64) * 4 if fmt == FMT_NF4_B64 else out_f * (in_f // 128) * 2
    return out_f * in_f // 2 + scale + m * in_f * 2


class Problem:
    """Device buffers for one shape: enough weight copies that together exceed
    4x L2 (so a launch that rotates over them reads its weights from HBM, not
    from the 126 MB L2, even when the copies are reused)."""

    def __init__(self, torch, fmt, out_f, in_f, m=1, seed=0, copies=None):
        from . import quantise_device, quantise_nf4_device
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        W = torch.randn((out_f, in_f), generator=g, device=dev) * 0.02
        qw, sc, _ = (quantise_nf4_device if fmt == FMT_NF4_B64 else quantise_device)(W)
        del W
        nb = alg_bytes(fmt, out_f, in_f)
        n = copies or max(2, min(4096, -(-4 * L2_BYTES // nb)))
        self.copies = [(qw, sc)] + [(qw.clone(), sc.clone()) for _ in range(n - 1)]
        self.x = torch.randn((m, in_f), generator=g, device=dev).half()
        self.y = torch.empty((m, out_f), device=dev)
        self.fmt, self.out_f, self.in_f, self.m = fmt, out_f, in_f, m
        self.ptrs = [(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(s.data_ptr())) for q, s in self.copies]
        # one zero-filled workspace for every config (each call leaves it ready for the next)
        self.ws = torch.zeros(WS_BYTES, dtype=torch.uint8, device=dev)

    def launch(self, k, cfg, stream):
        """One GEMV through b4_gemv_ws (cfg None: the rule of b4_gemv_ws)."""
        q, s = self.ptrs[k % len(self.ptrs)]
        return load().b4_gemv_ws(self.fmt, q, s, ctypes.c_void_p(self.x.data_ptr()),
                                 ctypes.c_void_p(self.y.data_ptr()), self.in_f, self.out_f, self.m,
                                 ctypes.byref(cfg) if cfg is not None else None,
                                 ctypes.c_void_p(self.ws.data_ptr()), self.ws.numel(), stream)


def time_chained(torch, prob, cfg, reps=None):
    """us per GEMV over `reps` launches captured in one CUDA graph (default:
    at least 100 and at least one per weight copy, so every copy is read once
    per replay and the copies between two reads of one exceed 4x L2); None if
    the config is rejected."""
    if reps is None:
        reps = max(100, len(prob.copies))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if prob.launch(0, cfg, stream) != 0:
        return None
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=cs, capture_error_mode="relaxed"):
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for k in range(reps):
            prob.launch(k, cfg, st)
    torch.cuda.current_stream().wait_stream(cs)
    g.replay()
    torch.cuda.synchronize()
    best = None
    for _ in range(3):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / reps
        best = us if best is None else min(best, us)
    del g
    return best


TMA_VARIANTS = [(4, 4), (3, 4), (6, 4), (4, 2), (4, 8), (8, 2)]   # (stages, stage_groups) instantiated
LEAN_VARIANTS = [(4, 1), (6, 1), (8, 1), (3, 2), (4, 2), (6, 2), (2, 4), (3, 4)]   # engine 5 (stages, stage_groups)
XTAB_VARIANTS = [(8, 4), (12, 2), (12, 3), (16, 2), (20, 1), (24, 1)]   # engine 8 (warps per CTA, batches in flight)
NF4_LEAN_VARIANTS = [(4, 4, 2, 0), (4, 8, 2, 0), (6, 4, 2, 0), (4, 4, 4, 0), (4, 4, 2, 2), (4, 8, 2, 2),
                     (6, 4, 2, 2), (8, 4, 2, 2), (4, 4, 4, 2)]   # (stages, rw, vw, lut) instantiated


SPLIT_INT4_VARIANTS = [(4, 1), (6, 1), (3, 2), (4, 2), (2, 4), (3, 4)]   # split INT4 (stages, stage_groups)


def split_grid(fmt):
    """The split configs (B4_FLAG_SPLIT, batch 1)."""
    base = dict(vec_words=4, rows_per_warp=16, warps_k=1, row_groups=8, batch_tile=1, nf4_lut=0, x_tile=0,
                flags=FLAG_SPLIT)
    if fmt == FMT_INT4_G128:
        for st, sg in SPLIT_INT4_VARIANTS:
            yield dict(base, engine=5, stages=st, stage_groups=sg)
    else:
        for st in (2, 3, 4):
            yield dict(base, engine=7, stages=st, stage_groups=0)


def config_grid(fmt, m=1):
    if m == 1:
        yield from split_grid(fmt)
    if fmt == FMT_INT4_G128 and m == 1:
        for kw, rg, (st, sg) in itertools.product((1, 2, 4, 8), (1, 2, 4, 8), LEAN_VARIANTS):
            if kw * rg <= 8:
                yield dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, nf4_lut=0,
                           x_tile=0, flags=0, engine=5, stages=st, stage_groups=sg)
    if fmt == FMT_INT4_G128 and 2 <= m <= 16:   # lean kernel with the batch rows in the MMA's N
        for kw, rg, (st, sg) in itertools.product((1, 2, 4, 8), (1, 2, 4, 8), [(2, 4), (3, 2), (4, 1)]):
            if kw * rg <= 8:
                yield dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, nf4_lut=0,
                           x_tile=0, flags=0, engine=5, stages=st, stage_groups=sg)
    if fmt == FMT_INT4_G128 and m <= 16:
        nt = 8 if m <= 8 else 16
        for kw, rg, (st, kcg) in itertools.product((1, 2, 4, 8), (1, 2, 4, 8), TMA_VARIANTS):
            if kw * rg <= 8 and (nt == 8 or (st, kcg) == (4, 4)):
                yield dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=nt, nf4_lut=0,
                           x_tile=0, flags=0, engine=2, stages=st, stage_groups=kcg)
    if fmt == FMT_INT4_G128:
        for rw, kw, rg, nt in itertools.product((16, 32), (1, 2, 4, 8), (1, 2, 4, 8), (8, 16)):
            if kw * rg <= 8 and (nt == 8 or m > 8):
                yield dict(vec_words=4, rows_per_warp=rw, warps_k=kw, row_groups=rg, batch_tile=nt, nf4_lut=0,
                           x_tile=0, flags=0, engine=1)
    if fmt == FMT_NF4_B64 and m == 1:   # x-pair table kernel: (warps per CTA, batches in flight per warp)
        for nw, st in XTAB_VARIANTS:
            yield dict(vec_words=1, rows_per_warp=8, warps_k=1, row_groups=nw, batch_tile=1, nf4_lut=0,
                       x_tile=0, flags=0, engine=8, stages=st, stage_groups=0)
    if fmt == FMT_NF4_B64 and m <= 16:
        for kw, rg, st in itertools.product((1, 2, 4, 8), (1, 2, 4, 8), (2, 3, 4) if m == 1 else (2, 3)):
            if kw * rg <= 8:
                yield dict(vec_words=4, rows_per_warp=16, warps_k=kw, row_groups=rg, batch_tile=1, nf4_lut=0,
                           x_tile=0, flags=0, engine=7, stages=st, stage_groups=0)
        for kw, rg, (st, rw, vw, lut) in itertools.product((1, 2, 4, 8), (1, 2, 4, 8), NF4_LEAN_VARIANTS):
            if kw * rg <= 8:
                yield dict(vec_words=vw, rows_per_warp=rw, warps_k=kw, row_groups=rg, batch_tile=1, nf4_lut=lut,
                           x_tile=0, flags=0, engine=6, stages=st, stage_groups=0)
    luts = (0,) if fmt == FMT_INT4_G128 else (0, 1)
    mbs = (1,) if m == 1 else ((2,) if m == 2 else (4,))
    for vw, rw, kw, rg, mb, lut in itertools.product((2, 4), (1, 2, 4, 8), (1, 2, 4, 8), (1, 2, 4, 8), mbs, luts):
        if mb == 4 and rw == 8:
            continue
        if kw * rg > 8 or kw * rg < 2:
            continue
        yield dict(vec_words=vw, rows_per_warp=rw, warps_k=kw, row_groups=rg, batch_tile=mb, nf4_lut=lut,
                   x_tile=0, flags=0, engine=0)


def cmd_sweep(args, torch):
    fmts = {"nf4": [FMT_NF4_B64], "int4": [FMT_INT4_G128], "both": [FMT_INT4_G128, FMT_NF4_B64]}[args.fmt]
    names = args.shapes.split(",") if args.shapes else list(SHAPES)[:7]
    out = []
    for fmt in fmts:
        for name in names:
            out_f, in_f = SHAPES[name]
            prob = Problem(torch, fmt, out_f, in_f, m=args.m)
            nb = alg_bytes(fmt, out_f, in_f, args.m)
            dflt = GemvConfig()
            check("default_config", load().b4_gemv_default_config_ws(fmt, in_f, out_f, args.m, ctypes.byref(dflt)))
            tile = GemvConfig()
            check("default_config", load().b4_gemv_default_config(fmt, in_f, out_f, args.m, ctypes.byref(tile)))
            rows = []
            if args.pdl:
                dflt.flags |= FLAG_PDL
                tile.flags |= FLAG_PDL
            us_d = time_chained(torch, prob, dflt)
            rows.append(("default", dflt.as_dict(), us_d))
            us_t = time_chained(torch, prob, tile)
            rows.append(("default_unsplit", tile.as_dict(), us_t))
            print(f"  rule (b4_gemv_ws) {us_d:.3f} us, unsplit rule (b4_gemv_default_config) {us_t:.3f} us", flush=True)
            engines = {int(e) for e in args.engines.split(",")} if args.engines else None
            grid = split_grid(fmt) if args.split_only else config_grid(fmt, args.m)
            for c in grid:
                if engines is not None and c.get("engine", 0) not in engines:
                    continue
                if args.pdl:
                    c = dict(c, flags=c.get("flags", 0) | FLAG_PDL)
                us = time_chained(torch, prob, GemvConfig.from_dict(c))
                if us is not None:
                    rows.append(("grid", c, us))
            rows.sort(key=lambda r: r[2])
            best = rows[0]
            print(f"{'nf4' if fmt else 'int4'} {name:10s} {out_f}x{in_f} m={args.m}: default {us_d:.3f} us "
                  f"({nb / us_d / 1e3:.0f} GB/s)  best {best[2]:.3f} us ({nb / best[2] / 1e3:.0f} GB/s) {best[1]}",
                  flush=True)
            out.append({"fmt": "nf4" if fmt else "int4", "shape": name, "out_f": out_f, "in_f": in_f, "m": args.m,
                        "bytes": nb, "default": {"cfg": dflt.as_dict(), "us": us_d},
                        "top": [{"cfg": c, "us": us} for _, c, us in rows[:12]],
                        "all": [[c.get("engine", 0), c["vec_words"], c["rows_per_warp"], c["warps_k"], c["row_groups"],
                                 c["batch_tile"], c["nf4_lut"], c.get("flags", 0), c.get("stages", 0),
                                 c.get("stage_groups", 0), round(us, 3)] for _, c, us in rows]})
            del prob
            torch.cuda.empty_cache()
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f)


def cmd_aspect(args, torch):
    fmt = FMT_NF4_B64 if args.fmt == "nf4" else FMT_INT4_G128
    sweeps = {
        "aspect": [(18944, 3584), (9472, 7168), (4736, 14336), (3584, 18944), (2368, 28672), (1184, 57344)],
        "rows": [(1184, 3584), (2368, 3584), (4736, 3584), (9472, 3584), (18944, 3584), (37888, 3584)],
        "x": [(3584, 3584), (3584, 7168), (3584, 14336), (3584, 18944), (3584, 28672), (3584, 57344)],
    }
    for title, cases in sweeps.items():
        print(f"sweep {title}")
        for out_f, in_f in cases:
            prob = Problem(torch, fmt, out_f, in_f)
            us = time_chained(torch, prob, None)
            nb = alg_bytes(fmt, out_f, in_f)
            print(f"  {out_f:6d}x{in_f:<6d} {us:8.3f} us {nb / us / 1e3:8.0f} GB/s "
                  f"{out_f * in_f / us / 1e3:8.0f} MW/ms", flush=True)
            del prob
            torch.cuda.empty_cache()


def cmd_run(args, torch):
    fmt = FMT_NF4_B64 if args.fmt == "nf4" else FMT_INT4_G128
    out_f, in_f = SHAPES[args.shape]
    prob = Problem(torch, fmt, out_f, in_f, m=args.m, copies=args.copies)
    cfg = None
    if args.config:
        d = GemvConfig()
        check("default_config", load().b4_gemv_default_config_ws(fmt, in_f, out_f, args.m, ctypes.byref(d)))
        c = d.as_dict()
        for kv in args.config.split(","):
            k, v = kv.split("=")
            c[k] = int(v)
        cfg = GemvConfig.from_dict(c)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for k in range(args.launches):
        check("b4_gemv_ws", prob.launch(k, cfg, stream))
    torch.cuda.synchronize()
    print(f"ran {args.launches} launches of {args.fmt} {args.shape} {out_f}x{in_f} m={args.m}")


def cmd_step(args, torch):
    """The benchmark's NF4 decode step (q/k/v and gate/up as one launch each, o
    and down alone, programmatic dependents, the package's workspace) run
    `steps` times eagerly: the command whose launch list is profiled."""
    from . import gemv_multi, gemv_ws
    dev = torch.device("cuda", torch.cuda.current_device())
    shapes = [SHAPES[n] for n in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")]
    mats = []
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    for out_f, in_f in shapes:
        W = torch.randn((out_f, in_f), generator=g, device=dev) * 0.02
        qw, sc, _ = quantise_nf4_device(W)
        mats.append((qw, sc))
        del W
    xa = torch.randn((1, 3584), generator=g, device=dev).half()
    xo = torch.randn((1, 3584), generator=g, device=dev).half()
    xm = torch.randn((1, 3584), generator=g, device=dev).half()
    xd = torch.randn((1, 18944), generator=g, device=dev).half()
    for _ in range(args.steps):
        gemv_multi(FMT_NF4_B64, mats[0:3], xa, pdl=True)
        gemv_ws(FMT_NF4_B64, *mats[3], xo, pdl=True)
        gemv_multi(FMT_NF4_B64, mats[4:6], xm, pdl=True)
        gemv_ws(FMT_NF4_B64, *mats[6], xd, pdl=True)
    torch.cuda.synchronize()
    print(f"ran {args.steps} NF4 decode steps (4 launches each)")


def cmd_glue(args, torch):
    """The decode layer's elementwise kernels (b4_swiglu_f16, b4_cast_f16) on
    `n` elements, `launches` times each."""
    dev = torch.device("cuda", torch.cuda.current_device())
    lib = load()
    g = torch.randn((args.n,), device=dev)
    u = torch.randn((args.n,), device=dev)
    out = torch.empty((args.n,), dtype=torch.float16, device=dev)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    for _ in range(args.launches):
        check("b4_swiglu_f16", lib.b4_swiglu_f16(P(g), P(u), P(out), args.n, st))
        check("b4_cast_f16", lib.b4_cast_f16(P(g), P(out), args.n, st))
    torch.cuda.synchronize()
    print(f"ran {args.launches} x (swiglu, cast) on {args.n} elements")


def cmd_p2p(args, torch):
    """The row-parallel GEMV with the peer-memory all-reduce in its epilogue
    (b4_tp_gemv_p2p_ex) in a world of one rank (its own slots, no peer, no
    collective: one process, so the kernel can be profiled alone), on a
    row-parallel shard's shape; --swiglu: x computed from fp32 [gate | up]
    while it is staged, and y also written in fp16."""
    from . import quantise_device
    from ._lib import FLAG_PDL, FLAG_X_SWIGLU
    fmt = FMT_NF4_B64 if args.fmt == "nf4" else FMT_INT4_G128
    out_f, in_f = SHAPES[args.shape]
    dev = torch.device("cuda", torch.cuda.current_device())
    lib = load()
    h = ctypes.c_void_p()
    check("b4_p2p_create", lib.b4_p2p_create(0, 1, out_f, ctypes.byref(h)))
    try:
        g = torch.Generator(device=dev)
        g.manual_seed(2)
        W = torch.randn((out_f, in_f), generator=g, device=dev) * 0.02
        qw, sc, _ = (quantise_nf4_device if fmt == FMT_NF4_B64 else quantise_device)(W)
        del W
        x = (torch.randn((2 * in_f,), generator=g, device=dev) if args.swiglu else
             torch.randn((in_f,), generator=g, device=dev).half())
        y = torch.empty((out_f,), device=dev)
        y16 = torch.empty((out_f,), dtype=torch.float16, device=dev)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        flags = FLAG_PDL | (FLAG_X_SWIGLU if args.swiglu else 0)
        for _ in range(args.launches):
            check("b4_tp_gemv_p2p_ex", lib.b4_tp_gemv_p2p_ex(fmt, P(qw), P(sc), P(x), P(y), P(y16) if args.swiglu else None,
                                                             in_f, out_f, h, flags, st))
        torch.cuda.synchronize()
        check("b4_p2p_status", lib.b4_p2p_status(h, 1))
    finally:
        lib.b4_p2p_destroy(h)
    print(f"ran {args.launches} peer-memory row-parallel GEMVs of {args.fmt} {args.shape} {out_f}x{in_f} (world 1)")


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m b4gemv.diag")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("sweep")
    s.add_argument("--fmt", default="both", choices=["nf4", "int4", "both"])
    s.add_argument("--shapes", default="")
    s.add_argument("--m", type=int, default=1)
    s.add_argument("--json", default="")
    s.add_argument("--engines", default="", help="comma-separated engine numbers to sweep (default: all)")
    s.add_argument("--pdl", action="store_true", help="launch every config as a programmatic dependent")
    s.add_argument("--split-only", action="store_true", help="sweep only the split configs (B4_FLAG_SPLIT)")
    a = sub.add_parser("aspect")
    a.add_argument("--fmt", default="nf4", choices=["nf4", "int4"])
    r = sub.add_parser("run")
    r.add_argument("--fmt", default="nf4", choices=["nf4", "int4"])
    r.add_argument("--shape", default="gate_proj", choices=list(SHAPES))
    r.add_argument("--m", type=int, default=1)
    r.add_argument("--launches", type=int, default=4)
    r.add_argument("--copies", type=int, default=4)
    r.add_argument("--config", default="")
    t = sub.add_parser("step")
    t.add_argument("--steps", type=int, default=10)
    gl = sub.add_parser("glue")
    gl.add_argument("--n", type=int, default=28672)
    gl.add_argument("--launches", type=int, default=3)
    pp = sub.add_parser("p2p")
    pp.add_argument("--fmt", default="nf4", choices=["nf4", "int4"])
    pp.add_argument("--shape", default="tp2_down", choices=list(SHAPES))
    pp.add_argument("--launches", type=int, default=3)
    pp.add_argument("--swiglu", action="store_true")
    args = ap.parse_args(argv)
    import torch
    torch.cuda.init()
    {"sweep": cmd_sweep, "aspect": cmd_aspect, "run": cmd_run, "step": cmd_step, "glue": cmd_glue,
     "p2p": cmd_p2p}[args.cmd](args, torch)


if __name__ == "__main__":
    sys.exit(main())
