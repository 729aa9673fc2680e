"""Tensor-parallel decode layer over NVLink (one process per GPU).

A Llama-style decoder layer's seven projections at batch 1, sharded over a
tensor-parallel group of T ranks:

  column-parallel (rows split, no communication):  q, k, v, gate, up
  row-parallel (in_f split on group boundaries, then an all-reduce of fp32 y):
                                                     o, down

Data flow of one decode step on each rank (attention itself is out of scope:
its output shard is an input):

  x (fp16, replicated) -> q, k, v shards
  attn shard (fp16)    -> o partial -> all-reduce -> h (fp32) -> fp16
  h                    -> gate, up shards -> silu(gate) * up (fp16) -> down partial
                       -> all-reduce -> y (fp32, replicated)

On the peer-memory path the two elementwise steps are folded into the GEMVs
(b4_tp_gemv_p2p_ex): o's all-reduce also writes h in fp16, and down computes
silu(gate) * up while it stages its x, so a layer is four launches (q/k/v,
o, gate/up, down); with NCCL the glue kernels run between them.

The GEMVs, the sharding copies, the activation and the all-reduce are C ABI
calls (include/b4gemv.h); torch.distributed is only used to hand the NCCL
unique id from rank 0 to the others.  The reference has no multi-GPU code.
"""
from __future__ import annotations

import ctypes

from ._lib import (FLAG_PDL, FLAG_SPLIT, FLAG_X_SWIGLU, FMT_INT4_G128, FMT_NF4_B64, GROUP, NF4_BLOCK,
                   XTAB_WORKSPACE_BYTES, GemvConfig, GemvSegment, check, load)


def row_range(n: int, tp: int, rank: int):
    """Rows [r0, r1) of rank `rank` when n rows are split over tp ranks as
    evenly as possible (column-parallel projections)."""
    return n * rank // tp, n * (rank + 1) // tp


def col_range(in_f: int, unit: int, tp: int, rank: int):
    """Columns [c0, c1) of rank `rank` for a row-parallel projection: in_f is
    split on `unit` boundaries (128 for INT4 groups, 64 for NF4 blocks)."""
    if in_f % unit:
        raise ValueError(f"in_f={in_f} is not a multiple of {unit}")
    units = in_f // unit
    if units < tp:
        raise ValueError(f"{units} groups cannot be split over {tp} ranks")
    u0, u1 = units * rank // tp, units * (rank + 1) // tp
    return u0 * unit, u1 * unit


def fmt_unit(fmt: int) -> int:
    return GROUP if fmt == FMT_INT4_G128 else NF4_BLOCK


class NcclComm:
    """An NCCL communicator created through the C ABI; the unique id travels
    from rank 0 over torch.distributed (any backend)."""

    def __init__(self, rank: int, world: int, group=None):
        import torch.distributed as dist
        lib = load()
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            check("b4_nccl_get_unique_id", lib.b4_nccl_get_unique_id(uid))
        obj = [bytes(uid.raw) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        uid = ctypes.create_string_buffer(obj[0], 128)
        self.ptr = ctypes.c_void_p()
        check("b4_nccl_comm_init", lib.b4_nccl_comm_init(ctypes.byref(self.ptr), world, uid, rank))
        self.rank, self.world = rank, world

    def wait(self, stream, timeout_ms: int = 10000) -> int:
        """Host-side wait with a deadline; aborts the communicator on failure
        and returns the status (0 on success)."""
        return load().b4_nccl_wait(self.ptr, ctypes.c_void_p(stream.cuda_stream), timeout_ms)

    def destroy(self):
        if self.ptr:
            load().b4_nccl_comm_destroy(self.ptr)
            self.ptr = ctypes.c_void_p()


class P2pComm:
    """The peer-memory all-reduce of b4_tp_gemv_p2p: one device allocation per
    rank, its CUDA IPC handle sent to every peer over torch.distributed (any
    backend), every peer's allocation mapped here."""

    def __init__(self, rank: int, world: int, max_rows: int, group=None):
        import torch.distributed as dist
        lib = load()
        self.ptr = ctypes.c_void_p()
        check("b4_p2p_create", lib.b4_p2p_create(rank, world, max_rows, ctypes.byref(self.ptr)))
        h = ctypes.create_string_buffer(64)
        check("b4_p2p_ipc_handle", lib.b4_p2p_ipc_handle(self.ptr, h))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h.raw), group=group)
        for r in range(world):
            if r != rank:
                check("b4_p2p_open_peer", lib.b4_p2p_open_peer(self.ptr, r, ctypes.create_string_buffer(handles[r], 64)))
        self.rank, self.world, self.max_rows = rank, world, max_rows

    def status(self, clear: bool = False) -> int:
        """0, or B4_STATUS_TIMEOUT if a wait in a kernel gave up (a peer did not arrive)."""
        return load().b4_p2p_status(self.ptr, 1 if clear else 0)

    def destroy(self):
        if self.ptr:
            load().b4_p2p_destroy(self.ptr)
            self.ptr = ctypes.c_void_p()


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def quantise_full(fmt, out_f, in_f, seed, device):
    """W ~ N(0, 0.02) from a seeded device generator, quantised on the device:
    the same full matrix on every rank."""
    import torch
    from . import quantise_device, quantise_nf4_device
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    W = torch.randn((out_f, in_f), generator=g, device=device) * 0.02
    qw, sc, _ = (quantise_nf4_device if fmt == FMT_NF4_B64 else quantise_device)(W)
    del W
    return qw, sc


def shard_columns(fmt, qw, sc, c0, c1, stream=None):
    """Contiguous copy of columns [c0, c1) of a packed weight and its scales."""
    import torch
    out_f, words = qw.shape
    in_f = words * 8
    unit = fmt_unit(fmt)
    q_out = torch.empty((out_f, (c1 - c0) // 8), dtype=qw.dtype, device=qw.device)
    s_out = torch.empty((out_f, (c1 - c0) // unit), dtype=sc.dtype, device=sc.device)
    st = stream if stream is not None else torch.cuda.current_stream()
    check("b4_shard_columns", load().b4_shard_columns(fmt, _p(qw), _p(sc), in_f, out_f, c0, c1 - c0, _p(q_out),
                                                      _p(s_out), ctypes.c_void_p(st.cuda_stream)))
    return q_out, s_out


class TPDecodeLayer:
    """One decoder layer's projections sharded over `tp` ranks.

    Shapes (Llama-3-70B defaults): hidden 8192, intermediate 28672, q 8192
    rows (64 heads x 128), k/v 1024 rows (8 heads x 128).  With `fused`, this
    rank's q/k/v shards run as one launch and gate/up as another
    (b4_gemv_multi); with `pdl`, the GEMVs are programmatic dependents."""

    NAMES = ("q", "k", "v", "o", "gate", "up", "down")

    def __init__(self, fmt, rank, tp, comm, device, hidden=8192, inter=28672, q_out=8192, kv_out=1024, seed=0,
                 fused=True, pdl=False, p2p=None):
        import torch
        self.fmt, self.rank, self.tp, self.comm, self.device = fmt, rank, tp, comm, device
        self.fused, self.pdl = fused, pdl
        self.p2p = p2p   # a P2pComm: row-parallel INT4 GEMVs all-reduce over peer memory instead of NCCL
        self.hidden, self.inter, self.q_out, self.kv_out = hidden, inter, q_out, kv_out
        unit = fmt_unit(fmt)
        # (name, out_f, in_f, kind)
        self.specs = [("q", q_out, hidden, "col"), ("k", kv_out, hidden, "col"), ("v", kv_out, hidden, "col"),
                      ("o", hidden, q_out, "row"), ("gate", inter, hidden, "col"), ("up", inter, hidden, "col"),
                      ("down", hidden, inter, "row")]
        self.w = {}
        self.ranges = {}
        for i, (name, out_f, in_f, kind) in enumerate(self.specs):
            qw, sc = quantise_full(fmt, out_f, in_f, seed * 100 + i, device)
            if kind == "col":
                r0, r1 = row_range(out_f, tp, rank)
                self.w[name] = (qw[r0:r1].contiguous(), sc[r0:r1].contiguous())
                self.ranges[name] = (r0, r1)
            else:
                c0, c1 = col_range(in_f, unit, tp, rank)
                self.w[name] = shard_columns(fmt, qw, sc, c0, c1)
                self.ranges[name] = (c0, c1)
            del qw, sc
        # the attention output shard feeding o is this rank's q heads
        assert tp == 1 or self.ranges["o"] == self.ranges["q"], "q rows and o columns must shard alike"
        f32 = dict(dtype=torch.float32, device=device)
        f16 = dict(dtype=torch.float16, device=device)
        rq, rk, rg = (self.ranges[n][1] - self.ranges[n][0] for n in ("q", "k", "gate"))
        # gate and up rows side by side in one buffer: [gate | up] is the x of the
        # down projection's SwiGLU mode (b4_tp_gemv_p2p_ex, B4_FLAG_X_SWIGLU)
        assert tp == 1 or self.ranges["down"] == self.ranges["gate"], "gate rows and down columns must shard alike"
        gu = torch.empty((1, 2 * rg), **f32)
        self.buf = {"q": torch.empty((1, rq), **f32), "k": torch.empty((1, rk), **f32),
                    "v": torch.empty((1, rk), **f32), "h": torch.empty((1, hidden), **f32),
                    "h16": torch.empty((1, hidden), **f16), "gu": gu, "gate": gu[:, :rg], "up": gu[:, rg:],
                    "act": torch.empty((1, rg), **f16), "y": torch.empty((1, hidden), **f32)}
        torch.cuda.synchronize(device)
        # launch configs: q/k/v and gate/up as one launch each (b4_gemv_multi)
        # when fused, else one per projection; PDL on the GEMV launches if asked
        lib = load()
        self.cfg = {}
        self.segs = {}
        for group, names in (("qkv", ("q", "k", "v")), ("gateup", ("gate", "up"))):
            segs = (GemvSegment * len(names))(*[GemvSegment(self.w[n][0].data_ptr(), self.w[n][1].data_ptr(),
                                                            self.buf[n].data_ptr(), self.w[n][0].shape[0])
                                                for n in names])
            c = GemvConfig()
            in_f = self.w[names[0]][0].shape[1] * 8
            check("multi config", lib.b4_gemv_multi_default_config_ws(fmt, segs, len(names), in_f, 1,
                                                                      ctypes.byref(c)))
            c.flags = FLAG_PDL if pdl else 0
            self.segs[group] = (segs, len(names), in_f)
            self.cfg[group] = c
        # every GEMV through the workspace entry points (b4_gemv_ws,
        # b4_gemv_multi_ws) with this layer's workspace: NF4 runs on the x-pair
        # table kernel, whose count-in needs it (the layer's GEMVs run one after
        # another on one stream, so they share it)
        need = XTAB_WORKSPACE_BYTES
        for name in self.NAMES:
            qw = self.w[name][0]
            c = GemvConfig()
            check("config", lib.b4_gemv_default_config_ws(fmt, qw.shape[1] * 8, qw.shape[0], 1, ctypes.byref(c)))
            c.flags = (c.flags & FLAG_SPLIT) | (FLAG_PDL if pdl else 0)
            self.cfg[name] = c
            n = ctypes.c_size_t(0)
            check("workspace", lib.b4_gemv_workspace_size(fmt, qw.shape[1] * 8, qw.shape[0], 1, ctypes.byref(c),
                                                          ctypes.byref(n)))
            need = max(need, n.value)
        self.ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)

    def weight_bytes(self) -> int:
        """Algorithmic bytes this rank streams per step (codes + scales)."""
        return sum(q.numel() * 4 + s.numel() * s.element_size() for q, s in self.w.values())

    def _gemv(self, name, x, y, stream):
        qw, sc = self.w[name]
        check(f"gemv {name}", load().b4_gemv_ws(self.fmt, _p(qw), _p(sc), _p(x), _p(y), qw.shape[1] * 8,
                                                 qw.shape[0], 1, ctypes.byref(self.cfg[name]), _p(self.ws),
                                                 self.ws.numel(), stream))

    def _multi(self, group, x, stream):
        segs, n, in_f = self.segs[group]
        check(f"gemv {group}", load().b4_gemv_multi_ws(self.fmt, segs, n, _p(x), in_f, 1,
                                                       ctypes.byref(self.cfg[group]), _p(self.ws), self.ws.numel(),
                                                       stream))

    def _p2p_ok(self, name):
        # the fused peer-memory kernel takes NF4 shards of whole 128-column
        # steps (its MMA k-step); narrower NF4 shards keep the NCCL all-reduce
        qw = self.w[name][0]
        return self.tp > 1 and self.p2p is not None and (self.fmt == FMT_INT4_G128 or (qw.shape[1] * 8) % 128 == 0)

    def glue_fused(self) -> bool:
        """True when the layer runs without glue launches: o writes h in fp16 as
        well, and down computes silu(gate) * up while it stages x (both on the
        peer-memory path)."""
        return self._p2p_ok("o") and self._p2p_ok("down")

    def _p2p_ex(self, name, x, y, y16, flags, stream):
        qw, sc = self.w[name]
        check(f"tp p2p {name}", load().b4_tp_gemv_p2p_ex(self.fmt, _p(qw), _p(sc), _p(x), _p(y),
                                                         _p(y16) if y16 is not None else None, qw.shape[1] * 8,
                                                         qw.shape[0], self.p2p.ptr,
                                                         flags | (FLAG_PDL if self.pdl else 0), stream))

    def _rowpar(self, name, x, y, stream):
        qw, sc = self.w[name]
        if self.tp == 1:
            return self._gemv(name, x, y, stream)
        if self._p2p_ok(name):
            self._p2p_ex(name, x, y, None, 0, stream)
            return
        check(f"tp {name}", load().b4_tp_gemv_allreduce_ws(self.fmt, _p(qw), _p(sc), _p(x), _p(y), qw.shape[1] * 8,
                                                            qw.shape[0], 1, _p(self.ws), self.ws.numel(),
                                                            self.comm.ptr, stream))

    STAGES = ("qkv", "o", "gateup", "down")

    def stage(self, name, x, attn, stream=None):
        """One launch group of forward() alone ("qkv", "o", "gateup", "down"), on
        this layer's buffers, as forward() issues it on the glue-free
        peer-memory path (for timing each launch of a layer; every rank must
        call the same stages, the row-parallel ones exchange rows)."""
        import torch
        assert self.fused and self.glue_fused(), "stage() times the fused, glue-free layer"
        st = stream if stream is not None else torch.cuda.current_stream()
        s = ctypes.c_void_p(st.cuda_stream)
        b = self.buf
        if name == "qkv":
            self._multi("qkv", x, s)
        elif name == "o":
            self._p2p_ex("o", attn, b["h"], b["h16"], 0, s)
        elif name == "gateup":
            self._multi("gateup", b["h16"], s)
        elif name == "down":
            self._p2p_ex("down", b["gu"], b["y"], None, FLAG_X_SWIGLU, s)
        else:
            raise ValueError(name)

    def forward(self, x, attn, stream=None):
        """x: fp16 [1, hidden] (replicated); attn: fp16 [1, q shard] (this
        rank's heads of the attention output).  Returns y fp32 [1, hidden]."""
        import torch
        st = stream if stream is not None else torch.cuda.current_stream()
        s = ctypes.c_void_p(st.cuda_stream)
        b, lib = self.buf, load()
        if self.fused:
            self._multi("qkv", x, s)
        else:
            self._gemv("q", x, b["q"], s)
            self._gemv("k", x, b["k"], s)
            self._gemv("v", x, b["v"], s)
        glue = not self.glue_fused()
        if glue:
            self._rowpar("o", attn, b["h"], s)
            check("cast", lib.b4_cast_f16(_p(b["h"]), _p(b["h16"]), b["h"].numel(), s))
        else:   # o writes h and its fp16 copy (the cast folded into the all-reduce)
            self._p2p_ex("o", attn, b["h"], b["h16"], 0, s)
        if self.fused:
            self._multi("gateup", b["h16"], s)
        else:
            self._gemv("gate", b["h16"], b["gate"], s)
            self._gemv("up", b["h16"], b["up"], s)
        if glue:
            check("swiglu", lib.b4_swiglu_f16(_p(b["gate"]), _p(b["up"]), _p(b["act"]), b["act"].numel(), s))
            self._rowpar("down", b["act"], b["y"], s)
        else:   # down stages x = fp16(silu(gate) * up) from [gate | up] itself
            self._p2p_ex("down", b["gu"], b["y"], None, FLAG_X_SWIGLU, s)
        return b["y"]
