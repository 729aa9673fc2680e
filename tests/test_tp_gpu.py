"""Tensor-parallel decode layer on 2, 4 and 8 GPUs (one process per GPU, NCCL
created through the C ABI; gloo only hands over the NCCL unique id); each
world size runs where that many GPUs are visible.

* parity: the layer's y at tp = 2/4/8 against the same layer at tp=1 on one
  GPU (a small layer, and the Llama-3-70B-shaped layer with both all-reduce
  paths: NCCL and the fused peer-memory one), and each row-parallel
  projection's all-reduced y against a double GEMV of the full matrix (1e-3,
  the rel metric of int4_gemv.cu:74-81);
* failure detection without a GPU fault: b4_nccl_wait's host deadline on a
  stream that is merely busy (a finite sleep kernel), and a rank that leaves
  between steps, which the other learns of through the store before its next
  launch.  NVLS is off (NCCL_NVLS_ENABLE=0).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=1024, inter=2048, q_out=1024, kv_out=256)


def _n_gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fmt, results):
    import sys
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(os.path.dirname(here), "int4-gemv_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    import b4gemv
    from b4gemv.tp import NcclComm, TPDecodeLayer, col_range, fmt_unit
    from oracle_py import Oracle, rel_err

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = NcclComm(rank, world)
    out = {}
    try:
        layer = TPDecodeLayer(fmt, rank, world, comm, dev, seed=3, **SMALL)
        full = TPDecodeLayer(fmt, 0, 1, None, dev, seed=3, **SMALL)
        g = torch.Generator(device=dev)
        g.manual_seed(77)
        x = torch.randn((1, SMALL["hidden"]), generator=g, device=dev).half()
        attn = torch.randn((1, SMALL["q_out"]), generator=g, device=dev).half()
        c0, c1 = layer.ranges["o"]
        y_tp = layer.forward(x, attn[:, c0:c1].contiguous()).clone()
        torch.cuda.synchronize()
        y_full = full.forward(x, attn).clone()
        torch.cuda.synchronize()
        out["layer"] = rel_err(y_tp.cpu().numpy(), y_full.cpu().numpy().astype(np.float64))
        # o_proj alone: all-reduced partials against the double GEMV of the full matrix
        o = Oracle()
        qw, sc = full.w["o"]
        ref = o.gemv_f64(fmt == 1, qw.cpu().numpy().view(np.uint32),
                         sc.cpu().numpy().view(np.uint16) if fmt == 0 else sc.cpu().numpy(),
                         attn.cpu().numpy())
        out["o_proj"] = rel_err(layer.buf["h"].cpu().numpy(), ref)
        # column-parallel q: this rank's rows of the full q
        r0, r1 = layer.ranges["q"]
        out["q_rows"] = rel_err(layer.buf["q"].cpu().numpy(), full.buf["q"][:, r0:r1].cpu().numpy())
        results[rank] = out
    finally:
        dist.barrier()
        comm.destroy()
        dist.destroy_process_group()


def _run(world, fmt):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    res = mgr.dict()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, fmt, res)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    return dict(res)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fmt", [0, 1])
def test_tp_layer_matches_single_gpu(fmt, world):
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run(world, fmt)
    for r in range(world):
        assert res[r]["layer"] < 1e-3, res
        assert res[r]["o_proj"] < 1e-3, res
        assert res[r]["q_rows"] == 0.0, res


def _l70_worker(rank, world, port, fmt, results):
    """The Llama-3-70B-shaped layer at tp = world, row-parallel projections on
    NCCL and on the fused peer-memory all-reduce, every rank's y gathered to
    rank 0 and compared with the same seeded layer at tp = 1."""
    import sys
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(os.path.dirname(here), "int4-gemv_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    from b4gemv.tp import NcclComm, P2pComm, TPDecodeLayer
    from oracle_py import rel_err

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = NcclComm(rank, world)
    p2p = P2pComm(rank, world, max_rows=8192)
    out = {}
    try:
        layer = TPDecodeLayer(fmt, rank, world, comm, dev, seed=5, pdl=True)
        g = torch.Generator(device=dev)
        g.manual_seed(9)
        x = torch.randn((1, 8192), generator=g, device=dev).half()
        attn = torch.randn((1, 8192), generator=g, device=dev).half()
        c0, c1 = layer.ranges["o"]
        shard = attn[:, c0:c1].contiguous()
        y_nccl = layer.forward(x, shard).clone()
        layer.p2p = p2p
        y_p2p = layer.forward(x, shard).clone()
        torch.cuda.synchronize()
        out["p2p_status"] = p2p.status()
        mine = np.stack([y_nccl.cpu().numpy()[0], y_p2p.cpu().numpy()[0]])
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        if rank == 0:
            del layer
            torch.cuda.empty_cache()
            one = TPDecodeLayer(fmt, 0, 1, None, dev, seed=5, pdl=True)
            ref = one.forward(x, attn).cpu().numpy().astype(np.float64)
            out["err"] = max(rel_err(a[None, :], ref) for ys in gathered for a in ys)
        results[rank] = out
    finally:
        dist.barrier()
        p2p.destroy()
        comm.destroy()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fmt", [0, 1], ids=["int4", "nf4"])
def test_tp_llama70b_layer_both_allreduce_paths_match_single_gpu(fmt, world):
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    res = ctx.Manager().dict()
    port = _port()
    ps = [ctx.Process(target=_l70_worker, args=(r, world, port, fmt, res)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=600)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    res = dict(res)
    assert res[0]["err"] < 1e-3, res
    assert all(res[r]["p2p_status"] == 0 for r in range(world)), res


def _leaver(rank, world, port, results):
    import sys
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "int4-gemv_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    from b4gemv.tp import NcclComm, TPDecodeLayer

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    store = dist.distributed_c10d._get_default_store()
    comm = NcclComm(rank, world)
    layer = TPDecodeLayer(0, rank, world, comm, dev, seed=1, **SMALL)
    x = torch.zeros((1, SMALL["hidden"]), device=dev).half()
    attn = torch.zeros((1, SMALL["q_out"] // world), device=dev).half()
    steps = 0
    for step in range(5):
        # heartbeat check before every launch: a rank that left is seen here
        if store.add("left", 0) > 0:
            break
        layer.forward(x, attn)
        st = comm.wait(torch.cuda.current_stream(), 10000)
        assert st == 0, st
        steps += 1
        if rank == 1 and step == 1:
            store.add("left", 1)      # leaves between steps, nothing in flight
            break
        store.add(f"done{step}", 1)
        while store.add(f"done{step}", 0) < world and store.add("left", 0) == 0:
            pass
    results[rank] = steps
    comm.destroy()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
def test_rank_leaving_between_steps_is_seen_before_next_launch():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    res = ctx.Manager().dict()
    port = _port()
    ps = [ctx.Process(target=_leaver, args=(r, 2, port, res)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=240)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in ps)
    assert res[1] == 2 and res[0] == 2


def test_nccl_wait_host_deadline_on_a_busy_stream(cuda):
    """b4_nccl_wait returns B4_STATUS_TIMEOUT (and aborts the communicator)
    when the stream is still busy at the deadline; the busy work is a finite
    sleep kernel, so the GPU stays healthy and the stream drains afterwards."""
    import ctypes

    import torch

    import b4gemv
    lib = b4gemv.load()
    uid = ctypes.create_string_buffer(128)
    assert lib.b4_nccl_get_unique_id(uid) == 0
    comm = ctypes.c_void_p()
    assert lib.b4_nccl_comm_init(ctypes.byref(comm), 1, uid, 0) == 0
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        torch.cuda._sleep(int(2e9))   # about a second at B200 clocks
    st = lib.b4_nccl_wait(comm, ctypes.c_void_p(s.cuda_stream), 50)
    assert st == 10901, st            # B4_STATUS_TIMEOUT; the communicator is aborted (freed)
    s.synchronize()                   # the sleep ends by itself
    comm2 = ctypes.c_void_p()
    assert lib.b4_nccl_get_unique_id(uid) == 0
    assert lib.b4_nccl_comm_init(ctypes.byref(comm2), 1, uid, 0) == 0
    assert lib.b4_nccl_wait(comm2, ctypes.c_void_p(s.cuda_stream), 1000) == 0
    assert lib.b4_nccl_comm_destroy(comm2) == 0


@pytest.mark.parametrize("fmt", [0, 1])
def test_tp1_layer_fused_and_pdl_match_separate_launches(cuda, fmt):
    """One GPU, no collective: the layer with q/k/v and gate/up fused into one
    launch each, and with programmatic dependent launches, gives the same
    outputs (within the fp32 accumulation order) as seven separate plain
    launches."""
    import torch

    from b4gemv.tp import TPDecodeLayer
    from oracle_py import rel_err
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    x = torch.randn((1, SMALL["hidden"]), generator=g, device=cuda).half()
    attn = torch.randn((1, SMALL["q_out"]), generator=g, device=cuda).half()
    ref = TPDecodeLayer(fmt, 0, 1, None, cuda, seed=4, fused=False, pdl=False, **SMALL)
    y_ref = ref.forward(x, attn).clone()
    bufs = {n: ref.buf[n].clone() for n in ("q", "k", "v", "gate", "up")}
    for fused, pdl in ((True, False), (True, True), (False, True)):
        lay = TPDecodeLayer(fmt, 0, 1, None, cuda, seed=4, fused=fused, pdl=pdl, **SMALL)
        y = lay.forward(x, attn).clone()
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), y_ref.cpu().numpy().astype(np.float64)) < 1e-5, (fused, pdl)
        for n, b in bufs.items():
            assert rel_err(lay.buf[n].cpu().numpy(), b.cpu().numpy().astype(np.float64)) < 1e-5, (n, fused, pdl)


def _p2p_worker(rank, world, port, mode, results, fmt=0):
    import sys
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(os.path.dirname(here), "int4-gemv_b200"))
    import ctypes
    import datetime

    import torch
    import torch.distributed as dist

    import b4gemv
    from b4gemv.tp import NcclComm, P2pComm, TPDecodeLayer, col_range, quantise_full, shard_columns
    from oracle_py import Oracle, rel_err

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    # NF4: at least 2048 rows, where the dispatch rule picks the tensor-pipe
    # kernel that the fused path runs (ragged last block either way); fmt 2:
    # an NF4 shard large enough for the x-pair table kernel, whose all-reduce
    # is its own launch
    big = fmt == 2
    fmt = 1 if big else fmt
    out_f, in_f = (8192, 8192) if big else ((1000, 2048) if fmt == 0 else (2056, 2048))
    p2p = P2pComm(rank, world, max_rows=8192)
    lib = b4gemv.load()
    out = {}
    try:
        qw, sc = quantise_full(fmt, out_f, in_f, 7, dev)
        c0, c1 = col_range(in_f, 128, world, rank)
        qs, ss = shard_columns(fmt, qw, sc, c0, c1)
        g = torch.Generator(device=dev)
        g.manual_seed(3)
        x = torch.randn((1, in_f), generator=g, device=dev).half()
        xs = x[:, c0:c1].contiguous()
        y = torch.zeros((1, out_f), device=dev)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        flags = 0
        if mode == "timeout":
            if rank == 0:   # the peer never makes this call: every wait must give up by itself
                assert lib.b4_tp_gemv_p2p(fmt, P(qs), P(ss), P(xs), P(y), c1 - c0, out_f, p2p.ptr, flags, st) == 0
                torch.cuda.synchronize()
                out["status"] = p2p.status(clear=True)
                out["rows_nan"] = bool(torch.isnan(y).all().item())   # no partial sums pass as results
                y2 = b4gemv.gemv(fmt, qw, sc, x)      # the GPU is still usable
                torch.cuda.synchronize()
                out["after"] = bool(torch.isfinite(y2).all().item())
            dist.barrier()
            results[rank] = out
            return
        ys = []
        for i in range(4):   # successive calls: the call counter advances on the device
            flags = b4gemv.FLAG_PDL if i >= 2 else 0
            y.fill_(float("nan"))
            assert lib.b4_tp_gemv_p2p(fmt, P(qs), P(ss), P(xs), P(y), c1 - c0, out_f, p2p.ptr, flags, st) == 0
            torch.cuda.synchronize()
            ys.append(y.clone())
        # captured once, replayed: still a fresh epoch every replay
        graph = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(graph, stream=cs, capture_error_mode="relaxed"):
            s2 = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            lib.b4_tp_gemv_p2p(fmt, P(qs), P(ss), P(xs), P(y), c1 - c0, out_f, p2p.ptr, flags, s2)
        torch.cuda.current_stream().wait_stream(cs)
        for _ in range(3):
            y.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            ys.append(y.clone())
        del graph
        out["status"] = p2p.status()
        if big:   # the kernel's slices add in a varying order
            out["same_calls"] = all(rel_err(t.cpu().numpy(), ys[0].cpu().numpy().astype(np.float64)) < 1e-6 for t in ys)
        else:
            out["same_calls"] = all(torch.equal(ys[0], t) for t in ys)
        out["big"] = big
        ref = Oracle().gemv_f64(fmt == 1, qw.cpu().numpy().view(np.uint32),
                                sc.cpu().numpy().view(np.uint16) if fmt == 0 else sc.cpu().numpy(), x.cpu().numpy())
        out["err"] = rel_err(ys[0].cpu().numpy(), ref)
        comm = NcclComm(rank, world)
        yn = torch.zeros((1, out_f), device=dev)
        assert lib.b4_tp_gemv_allreduce(fmt, P(qs), P(ss), P(xs), P(yn), c1 - c0, out_f, 1, comm.ptr, st) == 0
        torch.cuda.synchronize()
        comm.destroy()
        out["vs_nccl"] = rel_err(ys[0].cpu().numpy(), yn.cpu().numpy().astype(np.float64))
        gathered = [None] * world
        dist.all_gather_object(gathered, ys[0].cpu().numpy().tobytes())
        out["same_ranks"] = all(b == gathered[0] for b in gathered)
        # the decode layer with both row-parallel projections on the P2P path
        # against the same layer on NCCL (world 2: a + b either way, bit for bit)
        comm = NcclComm(rank, world)
        lp = TPDecodeLayer(fmt, rank, world, comm, dev, seed=3, pdl=True, p2p=p2p, **SMALL)
        ln = TPDecodeLayer(fmt, rank, world, comm, dev, seed=3, pdl=True, **SMALL)
        xl = torch.randn((1, SMALL["hidden"]), generator=g, device=dev).half()
        a0, a1 = lp.ranges["o"]
        attn = torch.randn((1, SMALL["q_out"]), generator=g, device=dev).half()[:, a0:a1].contiguous()
        y_p = lp.forward(xl, attn).clone()
        y_n = ln.forward(xl, attn).clone()
        torch.cuda.synchronize()
        comm.destroy()
        out["layer_equal"] = torch.equal(y_p, y_n)
        out["layer_err"] = rel_err(y_p.cpu().numpy(), y_n.cpu().numpy().astype(np.float64))
        out["layer_status"] = p2p.status()
        results[rank] = out
    finally:
        dist.barrier()
        p2p.destroy()
        dist.destroy_process_group()


def _run_p2p(world, mode, fmt=0):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    res = ctx.Manager().dict()
    port = _port()
    ps = [ctx.Process(target=_p2p_worker, args=(r, world, port, mode, res, fmt)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    return dict(res)


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fmt", [0, 1, 2], ids=["int4", "nf4", "nf4_xtab"])
def test_p2p_rowparallel_gemv_matches_nccl_and_is_identical_on_every_rank(fmt):
    res = _run_p2p(2, "parity", fmt)
    for r in (0, 1):
        assert res[r]["status"] == 0, res
        assert res[r]["same_calls"], res       # 4 calls + 3 graph replays, bit for bit
        assert res[r]["err"] < 1e-3, res       # against the double GEMV of the full matrix
        assert res[r]["vs_nccl"] < 1e-5, res   # against the NCCL all-reduce of the same partials
        if fmt == 1:   # same kernel and geometry as the plain GEMV: the same partials, the same sum
            assert res[r]["vs_nccl"] == 0.0, res
        assert res[r]["same_ranks"], res       # every rank sums in rank order
        # TPDecodeLayer(p2p=...) against TPDecodeLayer on NCCL: bit for bit for
        # INT4; for NF4 the small layer's o/down (1024 rows) run the CUDA-core
        # NF4 kernel on the NCCL path and the tensor-pipe one fused: fp32 rounding
        if fmt == 0:
            assert res[r]["layer_equal"], res
        else:
            assert res[r]["layer_err"] < 1e-6, res
        assert res[r]["layer_status"] == 0, res


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fmt", [0, 1, 2], ids=["int4", "nf4", "nf4_xtab"])
def test_p2p_wait_for_a_peer_that_never_arrives_times_out_and_the_gpu_stays_usable(fmt):
    res = _run_p2p(2, "timeout", fmt)
    assert res[0]["status"] == 10901, res      # B4_STATUS_TIMEOUT
    assert res[0]["rows_nan"], res
    assert res[0]["after"], res


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("out_f,in_f", [(2048, 3584), (8192, 4096)])
def test_p2p_ex_folds_the_glue_bit_identically(cuda, fmt, out_f, in_f):
    """b4_tp_gemv_p2p_ex on one GPU (a world of one rank, its own slots): with
    B4_FLAG_X_SWIGLU the GEMV of [gate | up] equals b4_swiglu_f16 followed by
    b4_tp_gemv_p2p bit for bit (NF4 shards of >= 17.5 MB run on the x-pair
    table kernel, whose slices add in a varying order: within 1e-6 there), and
    y16 equals y rounded to fp16 (what b4_cast_f16 writes); bad flags and a
    misaligned gate/up buffer are refused before any launch."""
    from oracle_py import rel_err
    import ctypes

    import torch

    import b4gemv
    from b4gemv._lib import FLAG_PDL, FLAG_X_SWIGLU, load
    lib = load()
    h = ctypes.c_void_p()
    assert lib.b4_p2p_create(0, 1, 8192, ctypes.byref(h)) == 0
    xtab = fmt == 1 and out_f * in_f // 2 + out_f * (in_f // 64) * 4 >= 17_500_000
    same = (lambda a, b: rel_err(a.cpu().numpy(), b.cpu().numpy()) < 1e-6) if xtab else torch.equal
    try:
        g = torch.Generator(device=cuda)
        g.manual_seed(11 + fmt)
        W = torch.randn((out_f, in_f), generator=g, device=cuda) * 0.02
        qw, sc, _ = (b4gemv.quantise_nf4_device if fmt else b4gemv.quantise_device)(W)
        gu = torch.randn((2 * in_f,), generator=g, device=cuda) * 3.0
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        act = torch.empty((in_f,), dtype=torch.float16, device=cuda)
        assert lib.b4_swiglu_f16(P(gu), ctypes.c_void_p(gu.data_ptr() + 4 * in_f), P(act), in_f, st) == 0
        y_ref = torch.empty((out_f,), device=cuda)
        assert lib.b4_tp_gemv_p2p(fmt, P(qw), P(sc), P(act), P(y_ref), in_f, out_f, h, 0, st) == 0
        for flags in (0, FLAG_PDL):
            y = torch.full((out_f,), float("nan"), device=cuda)
            assert lib.b4_tp_gemv_p2p_ex(fmt, P(qw), P(sc), P(gu), P(y), None, in_f, out_f, h,
                                         FLAG_X_SWIGLU | flags, st) == 0
            assert same(y, y_ref)
            y2 = torch.full((out_f,), float("nan"), device=cuda)
            y16 = torch.empty((out_f,), dtype=torch.float16, device=cuda)
            assert lib.b4_tp_gemv_p2p_ex(fmt, P(qw), P(sc), P(act), P(y2), P(y16), in_f, out_f, h, flags, st) == 0
            assert same(y2, y_ref)
            assert torch.equal(y16, y2.half())
        assert lib.b4_tp_gemv_p2p_ex(fmt, P(qw), P(sc), P(gu), P(y), None, in_f, out_f, h, 64, st) == 1
        assert lib.b4_tp_gemv_p2p_ex(fmt, P(qw), P(sc), ctypes.c_void_p(gu.data_ptr() + 8), P(y), None, in_f, out_f,
                                     h, FLAG_X_SWIGLU, st) == 1
        assert lib.b4_tp_gemv_p2p(fmt, P(qw), P(sc), P(gu), P(y), in_f, out_f, h, FLAG_X_SWIGLU, st) == 1
        torch.cuda.synchronize()
        assert lib.b4_p2p_status(h, 1) == 0
    finally:
        lib.b4_p2p_destroy(h)


def test_swiglu_glue_is_within_one_fp16_step_of_silu(cuda):
    """b4_swiglu_f16 (the silu of the decode layer's MLP, the same code the
    GEMVs with B4_FLAG_X_SWIGLU run while staging x) against silu(g) * u in
    double precision, over g in [-100, 100]: every element within one fp16 step
    of the exact value (the device silu is the fast exponential and divide,
    its error far below fp16's), and g below -87 gives 0."""
    import ctypes

    import torch

    from b4gemv._lib import load
    lib = load()
    n = 1 << 16
    g = torch.Generator(device=cuda)
    g.manual_seed(4)
    gate = torch.cat([torch.linspace(-100.0, 100.0, n // 2, device=cuda),
                      torch.randn((n // 2,), generator=g, device=cuda) * 4.0])
    up = torch.randn((n,), generator=g, device=cuda) * 2.0
    out = torch.empty((n,), dtype=torch.float16, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    assert lib.b4_swiglu_f16(P(gate), P(up), P(out), n, st) == 0
    torch.cuda.synchronize()
    gd, ud = gate.double().cpu(), up.double().cpu()
    exact = gd / (1.0 + torch.exp(-gd)) * ud
    got = out.double().cpu()
    step = torch.clamp(exact.abs(), min=2.0 ** -14) * 2.0 ** -10
    assert ((got - exact).abs() <= step).all(), float(((got - exact).abs() / step).max())
    assert (got[gd < -87.5] == 0).all()
