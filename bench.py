#!/usr/bin/env python3
"""Benchmark of the B200 fused 4-bit dequantisation GEMV (one JSON line).

Metric: us/GEMV and achieved HBM GB/s, batch-1 INT4/NF4 GEMV.

One GPU (--gpus 1): the workload is BASELINE.json configs[1], the NF4 b64
GEMV at batch 1 over the seven Qwen2.5-7B projections q/k/v/o (3584x3584,
512x3584 x2, 3584x3584), gate/up (18944x3584) and down (3584x18944).  A step is
one GEMV of each, issued through the C ABI as decode issues them: q/k/v read
one x and gate/up another (as in the model), and each of those groups is one
b4_gemv_multi_ws launch; o and down are b4_gemv_ws launches (4 launches per
step, programmatic dependents).  value = algorithmic bytes of the step
(packed codes + absmax + x) x steps / device time.  Beside it: every
projection in both formats (configs[0] is INT4 q_proj) with the reference's
own kernels rebuilt for sm_100a timed on the same buffers, the configs[4]
small-batch sweep, the configs[2] 28-layer chain, the configs[3] layer on
one GPU, and the CPU baseline.

N GPUs (torchrun, --gpus N): the workload is configs[3], the Llama-3-70B
decode layer tensor-parallel over the N ranks (NF4; o/down all-reduced inside
the GEMV over peer memory); value = the layer's algorithmic bytes x steps /
max-over-ranks time (strong scaling), and the layer's y is checked against
the same layer on one GPU (tp_rel_err).  The configs[1] step run as N
independent replicas is reported as `replicas`.

Timing: W warm-up steps, then exactly K steps bracketed by a barrier and
torch.cuda.synchronize on both sides, timed with CUDA events on the launching
stream and maxed over ranks.  The steps are replays of a CUDA graph holding
100 steps; consecutive configs[1] steps rotate over 4 independent weight
copies (524 MB, more than 4x the 126 MB L2), so every GEMV streams its
weights from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's CPU implementation of the path (the
fp32 loop over the dequantised matrix of int4_gemv.cu:33-38, ported in
oracle/, rows spread over all host cores) on the same workload and metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os

# NCCL prints its version banner on stdout unless told otherwise; the contract
# line must be the only line this script prints (a caller's setting wins).
os.environ.setdefault("NCCL_DEBUG", "WARN")
import re
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "int4-gemv_b200"))

SHAPES = [("q_proj", 3584, 3584), ("k_proj", 512, 3584), ("v_proj", 512, 3584), ("o_proj", 3584, 3584),
          ("gate_proj", 18944, 3584), ("up_proj", 18944, 3584), ("down_proj", 3584, 18944)]
N_SETS = 4            # rotating weight copies
GRAPH_STEPS = 100     # steps per captured graph
METRIC = "us/GEMV and achieved HBM GB/s (% of B200 peak), batch-1 INT4/NF4 GEMV"
WORKLOAD = "NF4 b64 GEMV, batch 1, Qwen2.5-7B q/k/v/o/gate/up/down (configs[1])"


def nf4_bytes(out_f, in_f, m=1):
    """Algorithmic bytes: packed codes + fp32 absmax + fp16 x."""
    return out_f * in_f // 2 + out_f * (in_f // 64) * 4 + m * in_f * 2


def int4_bytes(out_f, in_f, m=1):
    return out_f * in_f // 2 + out_f * (in_f // 128) * 2 + m * in_f * 2


STEP_BYTES = sum(nf4_bytes(o, i) for _, o, i in SHAPES)


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


ENGINE_KERNELS = {0: "b4_gemv_kernel", 1: "b4_gemv_mma_kernel", 2: "b4_gemv_tma_kernel",
                  5: "b4_gemv_lean_kernel (cp.async ring)", 6: "b4_gemv_lean_nf4_kernel",
                  7: "b4_gemv_nf4_mma_kernel", 8: "b4_gemv_xtab_kernel"}


def engine_kernel(b4, fmt, in_f, out_f):
    """Name of the kernel the dispatch rule (of b4_gemv_ws) picks for one batch-1 shape."""
    cfg = b4.default_config_ws(fmt, in_f, out_f, 1)
    if cfg["flags"] & b4.FLAG_SPLIT:
        return "b4_gemv_split_int4_kernel" if fmt == 0 else "b4_gemv_split_nf4_kernel"
    return ENGINE_KERNELS.get(cfg["engine"], f"engine {cfg['engine']}")


def profiled_traffic(kernel_tag):
    """dram bytes per launch recorded by an ncu capture summary in profiles/."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if not name.endswith(".md"):
            continue
        text = open(os.path.join(pdir, name)).read()
        m = re.search(r"traffic_bytes_per_launch\[" + re.escape(kernel_tag) + r"\]:\s*([0-9.eE+]+)", text)
        if m:
            return float(m.group(1))
    return None


# ---- distributed plumbing ---------------------------------------------------------

class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend):
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v, device=None):
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---- clocks ----------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        sms, maxes, reasons, power = [], [], set(), []
        for ts, line in self.lines:
            if ts < t0 or ts > t1:
                continue
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"],
                                 f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "power_w_max": max(power), "samples": len(sms)}


# ---- the measured arm -----------------------------------------------------------

# the input each projection reads, as in the model: q/k/v share the attention
# block's input, gate/up the MLP's
X_GROUP = {"q_proj": 0, "k_proj": 0, "v_proj": 0, "o_proj": 3, "gate_proj": 4, "up_proj": 4, "down_proj": 6}
# the step's launches: (projections, one b4_gemv_multi launch if several)
FUSED_STEP = [(0, 1, 2), (3,), (4, 5), (6,)]


def build_weights(b4, torch, dev, fmt):
    """Per shape: N_SETS copies of (qw, scale) quantised on the device from
    W ~ N(0, 0.02) (seed = shape index) and one y; x ~ N(0, 1) fp16 per input
    (q/k/v share one, gate/up another, X_GROUP)."""
    sets = [[] for _ in range(N_SETS)]
    xs, ys = [], []
    for idx, (name, out_f, in_f) in enumerate(SHAPES):
        g = torch.Generator(device=dev)
        g.manual_seed(idx)
        W = torch.randn((out_f, in_f), generator=g, device=dev, dtype=torch.float32) * 0.02
        if fmt == 1:
            qw, sc, _ = b4.quantise_nf4_device(W)
        else:
            qw, sc, _ = b4.quantise_device(W)
        del W
        for s in range(N_SETS):
            sets[s].append((qw.clone(), sc.clone()) if s else (qw, sc))
        src = X_GROUP[name]
        if src == idx:
            gx = torch.Generator(device=dev)
            gx.manual_seed(1000 + idx)
            xs.append(torch.randn((1, in_f), generator=gx, device=dev, dtype=torch.float32).half())
        else:
            xs.append(xs[src])
        ys.append(torch.empty((1, out_f), dtype=torch.float32, device=dev))
    torch.cuda.synchronize()
    return sets, xs, ys


class Launcher:
    """Pre-bound C ABI calls: one ctypes call per GEMV, nothing else.  Every
    GEMV goes through b4_gemv_ws with one zero-filled workspace (the split
    kernels of the few-row shapes use it; the GEMVs run one after another on
    one stream, so they may share it).  With pdl, the config is the dispatch
    rule's (b4_gemv_default_config_ws) plus B4_FLAG_PDL (programmatic dependent
    launch: the next GEMV's weight stream starts while the previous kernel
    drains); without, the rule's own (cfg NULL)."""

    def __init__(self, b4, torch, sets, xs, ys, fmt, pdl=False, fused=False):
        lib = b4.load()
        self.lib, self.fmt, self.pdl, self.fused = lib, fmt, pdl, fused
        self.cfg_objs = []
        need = 0
        for name, out_f, in_f in SHAPES:
            c = b4.GemvConfig.from_dict(b4.default_config_ws(fmt, in_f, out_f, 1))
            c.flags |= b4.FLAG_PDL
            self.cfg_objs.append(c)
            need = max(need, b4.workspace_size(fmt, in_f, out_f, 1, c.as_dict()))
        self.cfgs = [ctypes.byref(c) for c in self.cfg_objs]
        self.ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=xs[0].device)
        self.ws_ptr, self.ws_len = ctypes.c_void_p(self.ws.data_ptr()), self.ws.numel()
        self.calls = []
        for s in range(len(sets)):
            row = []
            for i, (name, out_f, in_f) in enumerate(SHAPES):
                qw, sc = sets[s][i]
                row.append((ctypes.c_void_p(qw.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                            ctypes.c_void_p(xs[i].data_ptr()), ctypes.c_void_p(ys[i].data_ptr()), in_f, out_f))
            self.calls.append(row)
        # fused step: q/k/v and gate/up as one b4_gemv_multi launch each (they share x)
        self.multi = []
        for s in range(len(sets)):
            row = []
            for group in FUSED_STEP:
                if len(group) == 1:
                    row.append(("single", group[0]))
                    continue
                segs = (b4.GemvSegment * len(group))(*[
                    b4.GemvSegment(sets[s][i][0].data_ptr(), sets[s][i][1].data_ptr(), ys[i].data_ptr(), SHAPES[i][1])
                    for i in group])
                in_f = SHAPES[group[0]][2]
                c = b4.GemvConfig()
                st = lib.b4_gemv_multi_default_config_ws(fmt, segs, len(group), in_f, 1, ctypes.byref(c))
                if st:
                    raise RuntimeError(f"multi config failed with status {st}")
                c.flags |= b4.FLAG_PDL if pdl else 0
                row.append(("multi", (segs, len(group), ctypes.c_void_p(xs[group[0]].data_ptr()), in_f, c)))
            self.multi.append(row)

    def call(self, i, q, sc, x, y, in_f, out_f, stream):
        st = self.lib.b4_gemv_ws(self.fmt, q, sc, x, y, in_f, out_f, 1, self.cfgs[i] if self.pdl else None,
                                 self.ws_ptr, self.ws_len, stream)
        if st:
            raise RuntimeError(f"GEMV launch failed with status {st}")

    def launches_per_step(self):
        return len(FUSED_STEP) if self.fused else len(SHAPES)

    def step(self, s, stream, events=None):
        if self.fused:
            calls = self.calls[s % len(self.calls)]
            for j, (kind, a) in enumerate(self.multi[s % len(self.multi)]):
                if kind == "single":
                    self.call(a, *calls[a], stream)
                else:
                    segs, n, x, in_f, c = a
                    st = self.lib.b4_gemv_multi_ws(self.fmt, segs, n, x, in_f, 1, ctypes.byref(c), self.ws_ptr,
                                                   self.ws_len, stream)
                    if st:
                        raise RuntimeError(f"GEMV launch failed with status {st}")
                if events is not None:
                    events[j].record()
            return
        for i, (q, sc, x, y, in_f, out_f) in enumerate(self.calls[s % len(self.calls)]):
            self.call(i, q, sc, x, y, in_f, out_f, stream)
            if events is not None:
                events[i].record()


def capture(torch, launcher, n_steps, first_step, with_events):
    """A CUDA graph of n_steps steps; with_events adds external timing events
    before the first and after every GEMV."""
    g = torch.cuda.CUDAGraph()
    evs = []
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=s, capture_error_mode="relaxed"):
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        if with_events:
            e0 = torch.cuda.Event(enable_timing=True, external=True)
            e0.record()
            evs.append(e0)
        for k in range(n_steps):
            step_evs = None
            if with_events:
                step_evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in SHAPES]
                evs.extend(step_evs)
            launcher.step(first_step + k, stream, step_evs)
    torch.cuda.current_stream().wait_stream(s)
    return g, evs


def correctness_gate(b4, torch, sets, xs, ys, fmt):
    """Correctness first (as int4_gemv.cu:70-86): y against a float64 GEMV over
    the bit-exact dequantised weights, max relative error below 1e-3."""
    worst = 0.0
    for i, (name, out_f, in_f) in enumerate(SHAPES):
        qw, sc = sets[0][i]
        y = b4.gemv_ws(fmt, qw, sc, xs[i])
        deq = b4.dequant_nf4(qw, sc) if fmt == 1 else b4.dequant_int4(qw, sc)
        ref = (deq.double() @ xs[i].double().t()).t()
        err = float((y.double() - ref).abs().max() / ref.abs().max())
        worst = max(worst, err)
        del deq
        if not err < 1e-3:
            raise SystemExit(f"FAILED correctness ({name}): rel max err {err:.3e}")
    return worst


def step_graph_ms(torch, launcher, n_steps):
    """ms for n_steps steps of `launcher` captured in one CUDA graph (best of 3
    replays after 2 untimed ones), events on the launching stream."""
    g, _ = capture(torch, launcher, n_steps, 0, with_events=False)
    for _ in range(2):
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
        best = a.elapsed_time(b) if best is None else min(best, a.elapsed_time(b))
    del g
    return best


def empty_launch_floor(b4, torch, reps=200):
    lib = b4.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t = []
    for _ in range(reps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        lib.b4_empty_launch(stream)
        b.record()
        b.synchronize()
        t.append(a.elapsed_time(b) * 1e3)
    return round(sorted(t)[len(t) // 2], 3)


def e2e_steps(b4, torch, sets, xs, ys, n_steps, graph=True, depth=1):
    """End to end through the public API with host buffers: every step copies
    its x (all seven projections, pinned host) to the device, runs the seven
    GEMVs through b4gemv.gemv_nf4 (the C ABI), copies y back and reads it.
    With `graph`, the seven b4gemv.gemv_nf4 calls of each weight set are
    captured once in a CUDA graph (as a decode loop runs them) and every step
    replays one between its copies; without, every step calls the Python API
    seven times (its host cost included).  depth 2: the host queues step s + 1
    before it waits for step s and reads its y (two pinned y buffers; the
    device work stays in one stream, in step order), so the GPU does not
    idle while the host synchronises; depth 1: the host waits for every step
    before it queues the next."""
    inputs = sorted(set(X_GROUP.values()))                # one x per input group
    in_sizes = [SHAPES[i][2] for i in inputs]
    out_sizes = [out_f for _, out_f, _ in SHAPES]
    hx = torch.empty(sum(in_sizes), dtype=torch.float16).pin_memory()
    hx.copy_(torch.cat([xs[i].reshape(-1).cpu() for i in inputs]))
    hys = [torch.empty(sum(out_sizes), dtype=torch.float32).pin_memory() for _ in range(depth)]
    hy = hys[0]
    done = [torch.cuda.Event() for _ in range(depth)]
    dx = torch.empty_like(hx, device=xs[0].device)
    dy = torch.empty_like(hy, device=xs[0].device)
    xg, yv, o = {}, [], 0
    for i, n in zip(inputs, in_sizes):
        xg[i] = dx[o:o + n].view(1, n)
        o += n
    xv = [xg[X_GROUP[name]] for name, _, _ in SHAPES]
    o = 0
    for n in out_sizes:
        yv.append(dy[o:o + n].view(1, n))
        o += n
    checksum = 0.0

    def gemvs(s, stream=None):
        # as decode runs them: q/k/v and gate/up (one x each) as one launch each
        for group in FUSED_STEP:
            if len(group) == 1:
                i = group[0]
                qw, sc = sets[s % N_SETS][i]
                b4.gemv_nf4(qw, sc, xv[i], yv[i], stream=stream, pdl=True)
            else:
                b4.gemv_multi(1, [sets[s % N_SETS][i] for i in group], xv[group[0]], [yv[i] for i in group],
                              stream=stream, pdl=True)

    graphs = []
    if graph:
        for k in range(N_SETS):
            gemvs(k)                      # eager first: configs and caches settle outside capture
        torch.cuda.synchronize()
        for k in range(N_SETS):
            g = torch.cuda.CUDAGraph()
            cs = torch.cuda.Stream()
            cs.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(g, stream=cs):
                gemvs(k, cs)
            torch.cuda.current_stream().wait_stream(cs)
            graphs.append(g)

    def queue(s):
        dx.copy_(hx, non_blocking=True)
        if graph:
            graphs[s % N_SETS].replay()
        else:
            gemvs(s)
        hys[s % depth].copy_(dy, non_blocking=True)
        done[s % depth].record()

    def read(s):
        nonlocal checksum
        done[s % depth].synchronize()
        checksum += float(hys[s % depth][0])

    def run(n):
        for s in range(n):
            queue(s)
            if s >= depth - 1:
                read(s - depth + 1)
        for s in range(max(0, n - depth + 1), n):
            read(s)

    run(3)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    run(n_steps)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    return ms, hx.numel() * 2, hy.numel() * 4


def e2e_overlap(b4, torch, sets, xs, n_steps):
    """End to end as a serving loop over independent steps runs it: the same
    public-API calls (b4gemv.gemv_nf4 / gemv_multi, captured once per weight
    set and buffer in a CUDA graph), every step's x copied in from pinned
    host memory and its y copied out and read on the host, with two device
    buffers so that step s + 1's x goes in on one copy stream and step s - 1's
    y comes out on another while step s computes.  Every wait is an event:
    step s's GEMVs wait for its x; its x copy waits until step s - 2's GEMVs
    are done with that buffer, and step s's GEMVs until step s - 2's y has been
    copied out; the host reads step s - 1's y after it has queued step s.
    Returns ms for n_steps, h2d and d2h bytes per step."""
    inputs = sorted(set(X_GROUP.values()))
    in_sizes = [SHAPES[i][2] for i in inputs]
    out_sizes = [out_f for _, out_f, _ in SHAPES]
    dev = xs[0].device
    hx = torch.empty(sum(in_sizes), dtype=torch.float16).pin_memory()
    hx.copy_(torch.cat([xs[i].reshape(-1).cpu() for i in inputs]))
    hys = [torch.empty(sum(out_sizes), dtype=torch.float32).pin_memory() for _ in range(2)]
    dxs = [torch.empty_like(hx, device=dev) for _ in range(2)]
    dys = [torch.empty_like(hys[0], device=dev) for _ in range(2)]
    views = []
    for b in range(2):
        xg, o = {}, 0
        for i, n in zip(inputs, in_sizes):
            xg[i] = dxs[b][o:o + n].view(1, n)
            o += n
        yv, o = [], 0
        for n in out_sizes:
            yv.append(dys[b][o:o + n].view(1, n))
            o += n
        views.append(([xg[X_GROUP[name]] for name, _, _ in SHAPES], yv))

    def gemvs(k, b, stream=None):
        xv, yv = views[b]
        for group in FUSED_STEP:
            if len(group) == 1:
                i = group[0]
                qw, sc = sets[k][i]
                b4.gemv_nf4(qw, sc, xv[i], yv[i], stream=stream, pdl=True)
            else:
                b4.gemv_multi(1, [sets[k][i] for i in group], xv[group[0]], [yv[i] for i in group],
                              stream=stream, pdl=True)

    for k in range(N_SETS):
        for b in range(2):
            gemvs(k, b)
    torch.cuda.synchronize()
    graphs = {}
    for k in range(N_SETS):
        for b in range(2):
            g = torch.cuda.CUDAGraph()
            cs = torch.cuda.Stream()
            cs.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(g, stream=cs):
                gemvs(k, b, cs)
            torch.cuda.current_stream().wait_stream(cs)
            graphs[(k, b)] = g
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("x_in", "computed", "y_out")}
    checksum = 0.0

    def queue(s):
        b = s % 2
        with torch.cuda.stream(h2d):
            if s >= 2:
                h2d.wait_event(ev["computed"][b])
            dxs[b].copy_(hx, non_blocking=True)
            ev["x_in"][b].record(h2d)
        comp.wait_event(ev["x_in"][b])
        if s >= 2:
            comp.wait_event(ev["y_out"][b])
        graphs[(s % N_SETS, b)].replay()
        ev["computed"][b].record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev["computed"][b])
            hys[b].copy_(dys[b], non_blocking=True)
            ev["y_out"][b].record(d2h)

    def read(s):
        nonlocal checksum
        ev["y_out"][s % 2].synchronize()
        checksum += float(hys[s % 2][0])

    def run(n):
        for s in range(n):
            queue(s)
            if s >= 1:
                read(s - 1)
        read(n - 1)
        comp.wait_event(ev["y_out"][(n - 1) % 2])

    run(4)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    run(n_steps)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b), hx.numel() * 2, hys[0].numel() * 4


def cpu_fused_baseline(sets, xs, budget_s=10.0):
    """The oracle's fused CPU GEMV (the reference kernels' per-lane arithmetic,
    oracle/b4_oracle.c) over the seven NF4 projections, rows spread over all
    host cores; steps repeated until budget_s elapses (at least one)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle_py import Oracle
    o = Oracle()
    host = []
    for i, (name, out_f, in_f) in enumerate(SHAPES):
        qw, sc = sets[0][i]
        host.append((qw.cpu().numpy().view(np.uint32), sc.cpu().numpy(), xs[i].cpu().numpy()))
    steps, t0, threads = 0, time.perf_counter(), 0
    while True:
        for p, a, x in host:
            _, threads = o.gemv_fused(True, p, a, x)
        steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": round(STEP_BYTES * steps / el / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{steps} full steps (all 7 NF4 projections) of the fused CPU GEMV, "
                      f"{el:.1f} s, {threads} threads on {os.cpu_count()} host cores"}


def load_ref_kernels():
    """The reference's CUDA kernels (kernels.cuh:26-266) with their benchmark's
    launch rule (int4_gemv.cu:52-68), compiled in place for sm_100a into
    oracle/_ref/libref.so by oracle/ref/Makefile: the second baseline, timed
    beside ours on the same device buffers.  None when it was not built."""
    path = os.path.join(ROOT, "oracle", "_ref", "libref.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    fn = lib.ref_launch_dispatch
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p]
    return lib


def graph_us(torch, launch, reps):
    """us per launch over `reps` calls of launch(k, stream) captured in one CUDA
    graph (best of 3 replays after one untimed), events on the launching
    stream; None if the first eager call fails."""
    if launch(0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) != 0:
        return None
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=cs, capture_error_mode="relaxed"):
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for k in range(reps):
            launch(k, st)
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


def isolated_us(torch, launch, reps=100):
    """The reference's protocol (int4_gemv.cu:88-108): event-bracketed single
    launches, each followed by a synchronize; median us."""
    st_obj = torch.cuda.current_stream()
    st = ctypes.c_void_p(st_obj.cuda_stream)
    t = []
    for k in range(reps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        launch(k, st)
        b.record()
        b.synchronize()
        t.append(a.elapsed_time(b) * 1e3)
    return sorted(t)[len(t) // 2]


def shape_table(b4, torch, ref):
    """Both formats x the seven Qwen2.5-7B projections at batch 1 (configs[0]
    is INT4 q_proj, configs[1] the NF4 rows): us per GEMV of ours (the rule of
    b4_gemv_ws, as programmatic dependents and as plain launches) and of the
    reference's kernels rebuilt for sm_100a (its own launch rule), each as
    back-to-back launches in one CUDA graph and as isolated event-bracketed
    launches; every timing rotates over weight copies that together exceed
    4x L2, so each launch streams its weights from HBM."""
    from b4gemv.diag import Problem, alg_bytes
    peak, _ = measured_peak()
    out = []
    auto_pdl = b4.GemvConfig.from_dict({"engine": -1, "flags": b4.FLAG_PDL})
    for fmt in (0, 1):
        for name, out_f, in_f in SHAPES:
            prob = Problem(torch, fmt, out_f, in_f, seed=11)
            reps = max(100, len(prob.copies))
            nb = alg_bytes(fmt, out_f, in_f)
            ours = lambda k, st, cfg=auto_pdl: prob.launch(k, cfg, st)
            ours_plain = lambda k, st: prob.launch(k, None, st)
            row = {"format": "int4_g128" if fmt == 0 else "nf4_b64", "shape": name, "out_f": out_f, "in_f": in_f,
                   "bytes": nb, "copies": len(prob.copies),
                   "kernel": engine_kernel(b4, fmt, in_f, out_f)}
            us = graph_us(torch, ours, reps)
            row["us"] = round(us, 3)
            row["gbs"] = round(nb / us / 1e3, 1)
            row["frac"] = round(nb / us / 1e3 / peak, 4)
            row["us_plain_launch"] = round(graph_us(torch, ours_plain, reps), 3)
            row["us_isolated"] = round(isolated_us(torch, ours_plain), 3)
            if ref is not None:
                def ref_launch(k, st):
                    q, sc = prob.ptrs[k % len(prob.ptrs)]
                    return ref.ref_launch_dispatch(fmt, q, sc, ctypes.c_void_p(prob.x.data_ptr()),
                                                   ctypes.c_void_p(prob.y.data_ptr()), in_f, out_f, st)
                rus = graph_us(torch, ref_launch, reps)
                row["ref_kernel_us"] = round(rus, 3) if rus is not None else None
                row["ref_kernel_us_isolated"] = round(isolated_us(torch, ref_launch), 3)
                if rus:
                    row["ref_kernel_gbs"] = round(nb / rus / 1e3, 1)
                    row["speedup_vs_ref_kernel"] = round(rus / us, 2)
            out.append(row)
            del prob
            torch.cuda.empty_cache()
    return out


def small_batch_bench(b4, torch):
    """batch M in {1, 2, 4, 8, 16} on gate_proj and
    down_proj, INT4 and NF4, the dispatch rule's engine per (shape, M); us per
    GEMV as 100 back-to-back programmatic-dependent launches in one graph
    (b4gemv.diag's chained timing, 4+ weight copies > 4x L2)."""
    from b4gemv.diag import Problem, alg_bytes, time_chained
    out = []
    for fmt in (0, 1):
        for name, out_f, in_f in (("gate_proj", 18944, 3584), ("down_proj", 3584, 18944)):
            for m in (1, 2, 4, 8, 16):
                prob = Problem(torch, fmt, out_f, in_f, m=m)
                rule = b4.default_config_ws(fmt, in_f, out_f, m)   # the rule the timed launches (b4_gemv_ws) use
                # the rule as the entry points run it (B4_ENGINE_AUTO: batch chunks where x
                # does not fit the tensor-pipe engines), each launch a programmatic dependent
                cfg = b4.GemvConfig.from_dict(dict(rule, engine=-1, flags=b4.FLAG_PDL))
                us = time_chained(torch, prob, cfg)
                engine, launches = rule["engine"], 1
                if rule["flags"] & b4.FLAG_KSLICE:   # column slices in one launch + their sum
                    launches = 2
                elif m > 1 and engine not in (5, 7):   # the entry points' batch chunks
                    for mc in (8, 4, 2):
                        e = b4.default_config(fmt, in_f, out_f, mc)["engine"] if mc < m else -1
                        if e in (5, 7):
                            engine, launches = e, -(-m // mc)
                            break
                nb = alg_bytes(fmt, out_f, in_f, m)
                row = {"format": "int4_g128" if fmt == 0 else "nf4_b64", "shape": name, "m": m,
                       "engine": engine, "launches": launches}
                if rule["flags"] & b4.FLAG_KSLICE:
                    row["column_slices"] = in_f // rule["x_tile"]
                out.append({**row, "us": round(us, 3),
                            "gbs": round(nb / us / 1e3, 1), "tflops": round(2.0 * m * out_f * in_f / us / 1e6, 2)})
                del prob
                torch.cuda.empty_cache()
    return out


def chain_bench(b4, torch, dev):
    """28 Qwen2.5-7B layers x 7 INT4 projections in one
    CUDA graph, one token; us per token with and without programmatic
    dependent launch."""
    from b4gemv.chain import DecodeChain
    ch = DecodeChain(torch, dev, fmt=0, layers=28)
    peak, _ = measured_peak()
    out = {"config": "configs[2]: 28 layers x q/k/v/o/gate/up/down INT4 g128, batch 1, one CUDA graph",
           "bytes_per_token": ch.bytes, "gemvs_per_token": ch.launch_count(False)}
    for key, pdl, fused in (("plain", False, False), ("pdl", True, False), ("fused_pdl", True, True)):
        us = ch.time_token(pdl, fused)
        out[key] = {"us_per_token": round(us, 2), "gbs": round(ch.bytes / us / 1e3, 1),
                    "frac": round(ch.bytes / us / 1e3 / peak, 4), "launches_per_token": ch.launch_count(fused)}
    out["fused_pdl"]["how"] = "q/k/v and gate/up as one b4_gemv_multi launch each, programmatic dependent launch"
    del ch
    torch.cuda.empty_cache()
    return out


L70 = [("q", 8192, 8192), ("k", 1024, 8192), ("v", 1024, 8192), ("o", 8192, 8192), ("gate", 28672, 8192),
       ("up", 28672, 8192), ("down", 8192, 28672)]
L70_WORKLOAD = ("Llama-3-70B decode layer (configs[3]): q/o 8192x8192, k/v 1024x8192, gate/up 28672x8192, "
                "down 8192x28672, batch 1, tensor-parallel over the run's ranks")


def l70_bytes(fmt):
    """Algorithmic bytes of one Llama-3-70B layer's seven projections (codes +
    scales + the fp16 input each reads); the shards of a tensor-parallel layer
    partition the weights, so this is also the sum over ranks."""
    f = nf4_bytes if fmt == 1 else int4_bytes
    return sum(f(o, i) for _, o, i in L70)


class TPBench:
    """the Llama-3-70B decode layer's projections sharded
    over the N ranks of this run (column-parallel q/k/v/gate/up, row-parallel
    o/down whose fp32 y is all-reduced, either by NCCL after the GEMV or inside
    the GEMV over peer memory).  x is replicated and the attention output is a
    seeded full vector of which each rank feeds its own heads to o, so the
    sharded layer computes exactly what one GPU computes for the same layer."""

    def __init__(self, b4, torch, dev, d, fmt, comm):
        from b4gemv.tp import TPDecodeLayer
        self.torch, self.dev, self.d, self.fmt = torch, dev, d, fmt
        self.layer = TPDecodeLayer(fmt, d.rank, d.world, comm, dev, seed=5, fused=True, pdl=True)
        g = torch.Generator(device=dev)
        g.manual_seed(9)
        self.x = torch.randn((1, 8192), generator=g, device=dev).half()
        self.attn_full = torch.randn((1, 8192), generator=g, device=dev).half()
        c0, c1 = self.layer.ranges["o"]
        self.attn = self.attn_full[:, c0:c1].contiguous()
        self.bytes = l70_bytes(fmt)
        self.glue_fused = False

    def graph(self, p2p, reps):
        torch = self.torch
        self.layer.p2p = p2p
        if p2p is not None:
            self.glue_fused = self.layer.glue_fused()   # 4 launches per layer, else 6
        self.layer.forward(self.x, self.attn)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=cs, capture_error_mode="relaxed"):
            for _ in range(reps):
                self.layer.forward(self.x, self.attn)
        torch.cuda.current_stream().wait_stream(cs)
        return g

    def us_per_layer(self, p2p, steps=200, reps=20):
        """us per layer, max over ranks: a graph of `reps` layers replayed."""
        torch, d = self.torch, self.d
        g = self.graph(p2p, reps)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        d.barrier()
        n = max(1, steps // reps)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        d.barrier()
        del g
        torch.cuda.synchronize()
        self.layer.p2p = None
        return d.max(a.elapsed_time(b) * 1e3 / (n * reps), self.dev)

    def breakdown(self, p2p, reps=20, rounds=5):
        """us per launch of each of the layer's four launch groups on the
        glue-free peer-memory path, each timed alone (a graph of `reps`
        back-to-back launches of that group, programmatic dependents), max
        over ranks; the layer's own time is less than their sum by the overlap
        of consecutive launches."""
        torch, d = self.torch, self.d
        self.layer.p2p = p2p
        out = {}
        if not self.layer.glue_fused():
            self.layer.p2p = None
            return out
        for name in self.layer.STAGES:
            self.layer.stage(name, self.x, self.attn)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            cs = torch.cuda.Stream()
            cs.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(g, stream=cs, capture_error_mode="relaxed"):
                for _ in range(reps):
                    self.layer.stage(name, self.x, self.attn)
            torch.cuda.current_stream().wait_stream(cs)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            d.barrier()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(rounds):
                g.replay()
            b.record()
            torch.cuda.synchronize()
            d.barrier()
            del g
            out[name] = round(d.max(a.elapsed_time(b) * 1e3 / (rounds * reps), self.dev), 2)
        torch.cuda.synchronize()
        self.layer.p2p = None
        return out

    def rel_err(self, p2p, y_ref):
        """max |y - y_ref| / max |y_ref| over every rank's y (gathered to rank
        0), y_ref the same layer on one GPU; None on the other ranks."""
        torch, d = self.torch, self.d
        self.layer.p2p = p2p
        y = self.layer.forward(self.x, self.attn).clone()
        torch.cuda.synchronize()
        self.layer.p2p = None
        ys = [torch.empty_like(y) for _ in range(d.world)]
        if d.pg:
            d.pg.all_gather(ys, y)
        else:
            ys = [y]
        if d.rank != 0:
            return None
        ref = y_ref.double()
        return max(float((t.double() - ref).abs().max() / ref.abs().max()) for t in ys)

    def reference_y(self):
        """Rank 0: the same seeded layer at tp = 1 on this GPU, y for the full
        attention vector (the parity reference of the sharded layers)."""
        from b4gemv.tp import TPDecodeLayer
        one = TPDecodeLayer(self.fmt, 0, 1, None, self.dev, seed=5, fused=True, pdl=True)
        y = one.forward(self.x, self.attn_full).clone()
        self.torch.cuda.synchronize()
        del one
        self.torch.cuda.empty_cache()
        return y

    def close(self):
        del self.layer
        self.torch.cuda.empty_cache()


def tp_layer_detail(b4, torch, dev, d, fmt, comm, p2p, skip_p2p_time=False):
    """One format's TP layer: us per layer with NCCL and with the fused
    peer-memory all-reduce (max over ranks), and both paths' y against the
    same layer on one GPU (tp_rel_err)."""
    tb = TPBench(b4, torch, dev, d, fmt, comm)
    peak, _ = measured_peak()
    res = {"format": "int4_g128" if fmt == 0 else "nf4_b64", "tp": d.world, "layer_bytes": tb.bytes,
           "weight_bytes_per_rank": tb.layer.weight_bytes()}
    us_nccl = tb.us_per_layer(None)
    res["us_per_layer_nccl" if d.world > 1 else "us_per_layer"] = round(us_nccl, 2)
    if d.world > 1:
        us_p2p = tb.us_per_layer(p2p)
        res["us_per_layer_p2p"] = round(us_p2p, 2)
        res["p2p_us_per_launch_alone"] = tb.breakdown(p2p)
        res["p2p_status"] = p2p.status()
        best = min(us_p2p, us_nccl)
    else:
        best = us_nccl
    res["gbs"] = round(tb.bytes / best / 1e3, 1)
    res["gbs_per_rank"] = round(tb.bytes / d.world / best / 1e3, 1)
    res["frac_per_rank"] = round(tb.bytes / d.world / best / 1e3 / peak, 4)
    if d.world > 1:
        y_ref = tb.reference_y() if d.rank == 0 else None
        e_nccl = tb.rel_err(None, y_ref)
        e_p2p = tb.rel_err(p2p, y_ref)
        if d.rank == 0:
            res["tp_rel_err"] = {"nccl": e_nccl, "p2p": e_p2p,
                                 "vs": "the same seeded layer at tp = 1 on rank 0's GPU, every rank's y"}
    glue = tb.glue_fused
    tb.close()
    res["launches"] = ("q/k/v and gate/up fused (b4_gemv_multi_ws), GEMVs as programmatic dependents; "
                       "o/down + NCCL all-reduce with the cast and SwiGLU glue launches (us_per_layer_nccl), or "
                       "with the all-reduce fused into the GEMV over peer memory (us_per_layer_p2p" +
                       (": the cast and SwiGLU folded into o and down, 4 launches)" if glue else ")"))
    return res


def clock_sampler(d):
    return ClockSampler(d.local if "CUDA_VISIBLE_DEVICES" not in os.environ else
                        os.environ["CUDA_VISIBLE_DEVICES"].split(",")[d.local])


def qwen_step_main(args, b4, torch, dev, d):
    """The configs[1] step (NF4, the seven Qwen2.5-7B projections, 4 launches)
    timed by the contract's rules: W warm-up steps, then K steps bracketed by
    a barrier and a synchronize on both sides, CUDA events on the launching
    stream, max over ranks.  Returns the timing and the objects the other legs
    reuse."""
    sets, xs, ys = build_weights(b4, torch, dev, 1)
    gate_err = correctness_gate(b4, torch, sets, xs, ys, 1)
    # the timed step as decode runs it: q/k/v and gate/up (one x each) as one
    # launch each; `separate`: the seven GEMVs as seven launches
    launcher = Launcher(b4, torch, sets, xs, ys, 1, pdl=not args.no_pdl, fused=True)
    separate = Launcher(b4, torch, sets, xs, ys, 1, pdl=not args.no_pdl)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for s in range(N_SETS):
        launcher.step(s, stream)  # eager first launches (attribute set-up) before capture
        separate.step(s, stream)
    torch.cuda.synchronize()
    K, W = args.steps, args.warmup
    gsteps = min(GRAPH_STEPS, K)
    g_main, _ = capture(torch, launcher, gsteps, 0, with_events=False)
    rem = K % gsteps
    g_rem = capture(torch, launcher, rem, 0, with_events=False)[0] if rem else None
    sampler = clock_sampler(d)
    sampler.start()
    time.sleep(0.5)
    t_soak = time.time()
    for _ in range(max(1, -(-W // gsteps))):
        g_main.replay()
    torch.cuda.synchronize()
    soak_until = time.time() + args.soak_seconds
    while time.time() < soak_until:
        g_main.replay()
        torch.cuda.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(K // gsteps):
        g_main.replay()
    if g_rem is not None:
        g_rem.replay()
    end.record()
    torch.cuda.synchronize()
    d.barrier()
    t_clock1 = time.time()
    time.sleep(0.3)
    sampler.stop()
    ms_max = d.max(start.elapsed_time(end), dev)
    sep_ms = d.max(step_graph_ms(torch, separate, min(K, 500)), dev)
    clocks = sampler.summary(t_soak, t_clock1)
    clocks["window"] = "warm-up soak and timed region"
    del g_main, g_rem, separate
    torch.cuda.synchronize()
    return {"ms_max": ms_max, "sep_ms": sep_ms, "gsteps": gsteps, "clocks": clocks, "gate_err": gate_err,
            "launches_per_step": launcher.launches_per_step(), "sets": sets, "xs": xs, "ys": ys}


def run_single(args, b4, torch, dev, d):
    K, W = args.steps, args.warmup
    q = qwen_step_main(args, b4, torch, dev, d)
    sets, xs, ys = q["sets"], q["xs"], q["ys"]
    ms_max = q["ms_max"]
    peak, peak_kind = measured_peak()

    # per projection and format, ours and the reference kernel, HBM-fed
    ref = load_ref_kernels()
    table = shape_table(b4, torch, ref)
    nf4_rows = {r["shape"]: r for r in table if r["format"] == "nf4_b64"}
    dom = nf4_rows["gate_proj"]
    traffic = profiled_traffic("nf4_xtab_gate_proj_18944x3584")

    # end to end through the public API with host buffers
    e2e_n = max(3, min(K, 200))
    e2e_ms, h2d, d2h = e2e_overlap(b4, torch, sets, xs, e2e_n)
    e2e_queued_ms, _, _ = e2e_steps(b4, torch, sets, xs, ys, e2e_n, depth=2)
    e2e_serial_ms, _, _ = e2e_steps(b4, torch, sets, xs, ys, e2e_n)
    e2e_eager_ms, _, _ = e2e_steps(b4, torch, sets, xs, ys, e2e_n, graph=False)
    floor = empty_launch_floor(b4, torch)

    result = {
        "metric": METRIC,
        "value": round(K * STEP_BYTES / (ms_max / 1e3) / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_max / K, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u4 codes, fp32 accumulate (fp16 x, fp32 y)",
        "data": "synthetic: W ~ N(0, 0.02) seeded per projection, quantised on the device; x ~ N(0, 1) fp16",
        "config": {"workload": WORKLOAD, "format": "nf4_b64", "batch": 1,
                   "shapes": {nm: [o, i] for nm, o, i in SHAPES},
                   "bytes_per_step": STEP_BYTES,
                   "l2": f"{N_SETS} rotating weight copies, {N_SETS * STEP_BYTES / 1e6:.0f} MB (> 4x the 126 MB L2)",
                   "timing": f"CUDA graphs of {q['gsteps']} steps, events on the launching stream",
                   "launches": "q/k/v read one x and gate/up another (as in the model) and run as one "
                               "b4_gemv_multi_ws launch each: 4 launches per step, programmatic dependents",
                   "parallelism": "1 GPU"},
        "us_per_gemv": {nm: r["us"] for nm, r in nf4_rows.items()},
        "gbs_per_gemv": {nm: r["gbs"] for nm, r in nf4_rows.items()},
        "us_per_gemv_how": "per projection: back-to-back launches in one CUDA graph as programmatic dependents, "
                           "rotating over weight copies > 4x L2 (shape_table)",
        "roofline": {"bound": "hbm", "kernel": f"{dom['kernel']} (NF4, gate_proj 18944x3584)",
                     "achieved": dom["gbs"], "peak": peak, "unit": "GB/s", "frac": dom["frac"],
                     "peak_source": peak_kind, "bytes_per_launch": dom["bytes"], "us_per_launch": dom["us"],
                     "traffic": traffic},
        "step_roofline_frac": round(STEP_BYTES / (ms_max / K * 1e-3) / 1e9 / peak, 4),
        "e2e": {"value": round(e2e_n * STEP_BYTES / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "how": "public API b4gemv.gemv_nf4 / gemv_multi (pdl=True) -> C ABI, the step's calls captured "
                       "once per weight set and buffer in a CUDA graph and replayed; every step's x copied in "
                       "from pinned host memory and its y copied out and read on the host, on two copy streams "
                       "and two device buffers so that step s + 1's x and step s - 1's y move while step s "
                       "computes (independent steps, as a serving loop over requests)", "steps": e2e_n,
                "queued_value": round(e2e_n * STEP_BYTES / (e2e_queued_ms / 1e3) / 1e9, 2),
                "queued_how": "one stream, one device buffer: copy in, GEMVs, copy out in step order, the host "
                              "queueing step s + 1 before it waits for and reads step s's y",
                "serial_value": round(e2e_n * STEP_BYTES / (e2e_serial_ms / 1e3) / 1e9, 2),
                "serial_how": "one stream, the host waiting for each step before it queues the next (a decode "
                              "loop whose next x depends on this step's y)",
                "eager_value": round(e2e_n * STEP_BYTES / (e2e_eager_ms / 1e3) / 1e9, 2),
                "eager_how": "the same with the step's Python API calls made every step (serial)"},
        "shape_table": table,
        "empty_launch_floor_us": floor,
        "gpu_launches": K * q["launches_per_step"],
        "separate_launches": {"value": round(min(K, 500) * STEP_BYTES / (q["sep_ms"] / 1e3) / 1e9, 2),
                              "unit": "GB/s", "ms_per_step": round(q["sep_ms"] / min(K, 500), 5),
                              "launches_per_step": len(SHAPES),
                              "how": "the same step as seven launches, one per projection (programmatic "
                                     "dependents)"},
        "correctness_rel_err": q["gate_err"],
        "clocks": q["clocks"],
    }
    if ref is None:
        result["ref_kernel_note"] = "oracle/_ref/libref.so not built: no reference-kernel timings"
    if not args.no_small_batch:
        result["small_batch"] = small_batch_bench(b4, torch)
    if not args.no_chain:
        result["qwen28_int4_chain"] = chain_bench(b4, torch, dev)
    if not args.no_tp:
        result["l70_tp_layer"] = [tp_layer_detail(b4, torch, dev, d, fmt, None, None) for fmt in (0, 1)]
    if not args.no_cpu:
        result["cpu_baseline"] = cpu_fused_baseline(sets, xs, budget_s=args.cpu_seconds)
    print(json.dumps(result), flush=True)


def tp_e2e(torch, tb, p2p, n_steps, depth=2):
    """configs[3] end to end: every step copies x and this rank's attention
    shard from pinned host memory, replays the layer graph and copies y back
    and reads it; with depth 2 the host queues step s + 1 before it waits for
    and reads step s's y (two pinned y buffers, device work in one stream in
    step order).  ms, h2d and d2h bytes per step."""
    hx = tb.x.cpu().pin_memory()
    ha = tb.attn.cpu().pin_memory()
    hys = [torch.empty((1, 8192), dtype=torch.float32).pin_memory() for _ in range(depth)]
    hy = hys[0]
    done = [torch.cuda.Event() for _ in range(depth)]
    g = tb.graph(p2p, 1)
    y = tb.layer.buf["y"]

    def queue(s):
        tb.x.copy_(hx, non_blocking=True)
        tb.attn.copy_(ha, non_blocking=True)
        g.replay()
        hys[s % depth].copy_(y, non_blocking=True)
        done[s % depth].record()

    def read(s):
        done[s % depth].synchronize()
        return float(hys[s % depth][0, 0])

    def run(n):
        for s in range(n):
            queue(s)
            if s >= depth - 1:
                read(s - depth + 1)
        for s in range(max(0, n - depth + 1), n):
            read(s)

    run(3)
    tb.d.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    run(n_steps)
    b.record()
    torch.cuda.synchronize()
    tb.d.barrier()
    del g
    tb.layer.p2p = None
    return a.elapsed_time(b), hx.numel() * 2 + ha.numel() * 2, hy.numel() * 4


def run_multi(args, b4, torch, dev, d):
    """N > 1: the contract value is configs[3], the Llama-3-70B layer
    tensor-parallel over the N ranks (NF4, o/down with the all-reduce fused
    into the GEMV over peer memory): total layer bytes per step / max-over-
    ranks time, strong scaling (the layer is fixed as N grows).  The layer's
    y is checked against the same layer on one GPU (tp_rel_err); the
    independent-replica figure of the configs[1] step is kept as
    `replicas`."""
    from b4gemv.tp import NcclComm, P2pComm
    K, W = args.steps, args.warmup
    comm = NcclComm(d.rank, d.world)
    p2p = P2pComm(d.rank, d.world, max_rows=8192)
    peak, peak_kind = measured_peak()
    tb = TPBench(b4, torch, dev, d, 1, comm)
    gsteps = min(GRAPH_STEPS, K)
    g = tb.graph(p2p, gsteps)
    sampler = clock_sampler(d)
    sampler.start()
    time.sleep(0.5)
    t_soak = time.time()
    for _ in range(max(1, -(-W // gsteps))):
        g.replay()
    torch.cuda.synchronize()
    soak_until = time.time() + args.soak_seconds
    while time.time() < soak_until:
        g.replay()
        torch.cuda.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    n_rep = max(1, K // gsteps)
    steps = n_rep * gsteps
    start.record()
    for _ in range(n_rep):
        g.replay()
    end.record()
    torch.cuda.synchronize()
    d.barrier()
    t_clock1 = time.time()
    time.sleep(0.3)
    sampler.stop()
    del g
    tb.layer.p2p = None
    torch.cuda.synchronize()
    ms_max = d.max(start.elapsed_time(end), dev)
    clocks = sampler.summary(t_soak, t_clock1)
    clocks["window"] = "warm-up soak and timed region"
    status = p2p.status()
    e2e_n = max(3, min(K, 200))
    e2e_ms, h2d, d2h = tp_e2e(torch, tb, p2p, e2e_n)
    e2e_ms = d.max(e2e_ms, dev)
    y_ref = tb.reference_y() if d.rank == 0 else None
    err = {"p2p": tb.rel_err(p2p, y_ref), "nccl": tb.rel_err(None, y_ref)}
    us_nccl = tb.us_per_layer(None)
    per_launch = tb.breakdown(p2p)
    tb.close()
    del y_ref
    value = steps * tb.bytes / (ms_max / 1e3) / 1e9
    result = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": d.world,
        "steps": steps,
        "warmup": W,
        "ms_per_step": round(ms_max / steps, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "u4 codes, fp32 accumulate (fp16 x, fp32 y)",
        "data": "synthetic: W ~ N(0, 0.02) seeded per projection, quantised on the device; x and the attention "
                "output ~ N(0, 1) fp16",
        "config": {"workload": L70_WORKLOAD, "format": "nf4_b64", "batch": 1, "tp": d.world,
                   "layer_bytes": tb.bytes,
                   "l2": f"one layer streams {tb.bytes / d.world / 1e6:.0f} MB per rank per step (inputs larger "
                         f"than L2 where that is > 126 MB; the layer is replayed as decode replays it)",
                   "timing": f"CUDA graphs of {gsteps} layer steps, events on the launching stream, max over ranks",
                   "launches": ("per rank: q/k/v (one b4_gemv_multi_ws launch), o with the all-reduce over peer "
                                "memory and the fp16 cast folded in (b4_tp_gemv_p2p_ex), gate/up (one launch), "
                                "down with the SwiGLU of gate/up computed as it stages x and the all-reduce "
                                "folded in: 4 launches, programmatic dependents") if tb.glue_fused else
                               ("per rank: q/k/v (one b4_gemv_multi_ws launch), o with the fused all-reduce, fp16 "
                                "cast, gate/up (one launch), SwiGLU, down with the fused all-reduce: 6 launches"),
                   "parallelism": f"tp{d.world}"},
        "us_per_layer": round(ms_max * 1e3 / steps, 2),
        "us_per_layer_nccl": round(us_nccl, 2),
        "us_per_launch_alone": per_launch,
        "p2p_status": status,
        "gbs_per_rank": round(value / d.world, 1),
        "roofline": {"bound": "hbm", "kernel": "the layer's GEMVs (per rank)", "achieved": round(value / d.world, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(value / d.world / peak, 4),
                     "peak_source": peak_kind, "traffic": None},
        "tp_rel_err": err if d.rank == 0 else None,
        "e2e": {"value": round(e2e_n * tb.bytes / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_n,
                "how": "per step and rank: x and the rank's attention shard copied in from pinned host memory, "
                       "the layer (TPDecodeLayer, C ABI calls captured in a CUDA graph) replayed, y copied out "
                       "and read on the host, the host queueing step s + 1 before it waits for step s; max "
                       "over ranks"},
        "gpu_launches": steps * (4 if tb.glue_fused else 6),
        "clocks": clocks,
    }
    if not args.no_tp:
        result["l70_tp_layer_int4"] = tp_layer_detail(b4, torch, dev, d, 0, comm, p2p)
    # the configs[1] step on every rank at once, no data-path collective
    q = qwen_step_main(args, b4, torch, dev, d)
    result["replicas"] = {"value": round(d.world * K * STEP_BYTES / (q["ms_max"] / 1e3) / 1e9, 2), "unit": "GB/s",
                          "ms_per_step": round(q["ms_max"] / K, 5), "workload": WORKLOAD,
                          "how": f"{d.world} independent replicas of the configs[1] step (no collective), value = "
                                 "all ranks' bytes / max-over-ranks time"}
    del q
    torch.cuda.synchronize()
    d.barrier()
    p2p.destroy()
    comm.destroy()
    if d.rank == 0:
        print(json.dumps(result), flush=True)


def run_ours(args, d):
    import torch
    import b4gemv as b4
    torch.cuda.set_device(d.local)
    dev = torch.device("cuda", d.local)
    d.init("nccl")
    b4.load()
    if d.world == 1:
        run_single(args, b4, torch, dev, d)
    else:
        run_multi(args, b4, torch, dev, d)
    d.close()


# ---- the reference arm -----------------------------------------------------------

def run_reference(args, d):
    """The reference's CPU path (int4_gemv.cu:33-38: fp32 sum over the
    dequantised matrix, row by row) ported in oracle/, rows spread over all
    host cores, on a row sample of every projection sized so that the run
    stays within a few minutes.  Weights are quantised by the reference's own
    quantise_nf4 (oracle/_ref) when it was compiled, else by the oracle's port."""
    if d.world > 1 and d.rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle_py import REF_LIB, Oracle
    o = Oracle()
    ref = ctypes.CDLL(REF_LIB) if os.path.exists(REF_LIB) else None
    K, W = args.steps, args.warmup
    cores = os.cpu_count() or 1
    # rows per projection: ~60 s of timed CPU work at an assumed 10 GB/s of
    # fp32 dequantised weights, between 1/64 and 1/4 of each projection
    frac = min(0.25, max(1 / 64, 60.0 * 10e9 / max(1, K + W) / (sum(o_ * i_ for _, o_, i_ in SHAPES) * 4)))
    P = lambda a: ctypes.c_void_p(a.ctypes.data)
    data = []
    sample_bytes = 0
    rng = np.random.default_rng(0)
    for idx, (name, out_f, in_f) in enumerate(SHAPES):
        rows = max(8, int(out_f * frac))
        Wm = (rng.standard_normal((rows, in_f)) * 0.02).astype(np.float32)
        p = np.zeros((rows, in_f // 8), np.uint32)
        a = np.zeros((rows, in_f // 64), np.float32)
        deq = np.zeros((rows, in_f), np.float32)
        if ref is not None:
            ref.ref_quantise_nf4(P(Wm), rows, in_f, P(p), P(a), P(deq))
        else:
            p, a, deq = o.quantise_nf4(Wm)
        x = rng.standard_normal(in_f).astype(np.float16).astype(np.float32)
        data.append((deq, x, np.zeros(rows, np.float32), rows, in_f))
        sample_bytes += nf4_bytes(rows, in_f)
    fn = o.lib.b4o_gemv_deq_f32_mt

    def step():
        for deq, x, y, rows, in_f in data:
            fn(P(deq), P(x), rows, in_f, P(y), 0)

    for _ in range(max(W, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(K):
        step()
    el = time.perf_counter() - t0
    value = sample_bytes * K / el / 1e9
    result = {
        "impl": "reference",
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": d.world, "steps": K, "warmup": W,
        "ms_per_step": round(el * 1e3 / K, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (dequantised weights), fp16-rounded x",
        "data": "synthetic: W ~ N(0, 0.02), x ~ N(0, 1) fp16; NF4 b64 by the reference's quantise_nf4",
        "config": {"workload": WORKLOAD, "format": "nf4_b64", "batch": 1,
                   "shapes": {nm: [o_, i_] for nm, o_, i_ in SHAPES}, "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"every projection cut to {frac:.4f} of its rows ({sample_bytes} algorithmic "
                                   f"bytes per step); the int4_gemv.cu:33-38 loop ported in oracle/b4_oracle.c, "
                                   f"rows over {cores} threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-small-batch", action="store_true", help="skip the configs[4] small-batch sweep")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-chain", action="store_true", help="skip the 28-layer INT4 graph chain")
    ap.add_argument("--no-tp", action="store_true", help="skip the Llama-3-70B tensor-parallel layer")
    ap.add_argument("--no-pdl", action="store_true",
                    help="time the step and per-GEMV graphs with plain launches instead of programmatic dependents")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--soak-seconds", type=float, default=1.0,
                    help="untimed load before the timed region, for the clock samples")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    d = Dist()
    if args.impl == "reference":
        run_reference(args, d)
    else:
        run_ours(args, d)


if __name__ == "__main__":
    main()
