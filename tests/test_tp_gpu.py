"""Tensor-parallel decode layer on 2 GPUs (one process per GPU, NCCL created
through the C ABI; gloo only hands over the NCCL unique id).

* parity: the layer's y at tp=2 against the same layer at tp=1 on one GPU,
  and each row-parallel projection's all-reduced y against a double GEMV of
  the full matrix (1e-3, the rel metric of int4_gemv.cu:74-81);
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


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fmt", [0, 1])
def test_tp2_layer_matches_single_gpu(fmt):
    res = _run(2, fmt)
    for r in (0, 1):
        assert res[r]["layer"] < 1e-3, res
        assert res[r]["o_proj"] < 1e-3, res
        assert res[r]["q_rows"] == 0.0, res


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
