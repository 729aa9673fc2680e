"""Host logic of the tensor-parallel layer on CPU: the shard partitions, the
column shards of packed buffers, and the shard math (sum of rank partials =
full GEMV) across two gloo ranks, with the oracle as the per-rank GEMV."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from b4gemv.tp import col_range, row_range


def test_row_and_col_ranges_partition():
    for n, tp in [(8192, 8), (1024, 8), (28672, 8), (512, 3), (7, 2)]:
        rs = [row_range(n, tp, r) for r in range(tp)]
        assert rs[0][0] == 0 and rs[-1][1] == n and all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
    for in_f, unit, tp in [(8192, 128, 8), (28672, 128, 8), (28672, 64, 8), (3584, 128, 4), (384, 64, 4)]:
        cs = [col_range(in_f, unit, tp, r) for r in range(tp)]
        assert cs[0][0] == 0 and cs[-1][1] == in_f
        assert all(c0 % unit == 0 and c1 % unit == 0 and c1 > c0 for c0, c1 in cs)
    with pytest.raises(ValueError):
        col_range(200, 128, 2, 0)
    with pytest.raises(ValueError):
        col_range(256, 128, 4, 0)


def numpy_shard_columns(packed, scales, unit, c0, c1):
    """Column shard of packed words and scales (what b4_shard_columns copies)."""
    return packed[:, c0 // 8:c1 // 8].copy(), scales[:, c0 // unit:c1 // unit].copy()


@pytest.mark.parametrize("nf4", [False, True])
def test_column_shard_equals_quantised_column_slice(oracle, nf4):
    rng = np.random.default_rng(4)
    W = (rng.standard_normal((16, 1024)) * 0.02).astype(np.float32)
    q = oracle.quantise_nf4 if nf4 else oracle.quantise
    unit = 64 if nf4 else 128
    p, s, _ = q(W)
    for tp in (2, 4, 8):
        for r in range(tp):
            c0, c1 = col_range(1024, unit, tp, r)
            ps, ss = numpy_shard_columns(p, s, unit, c0, c1)
            p2, s2, _ = q(W[:, c0:c1])
            assert ps.tobytes() == p2.tobytes() and ss.tobytes() == s2.tobytes()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import sys
    import torch
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(os.path.dirname(here), "int4-gemv_b200"))
    from oracle_py import Oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    o = Oracle()
    rng = np.random.default_rng(7)
    out_f, in_f = 24, 1536
    W = (rng.standard_normal((out_f, in_f)) * 0.02).astype(np.float32)
    x = rng.standard_normal((1, in_f)).astype(np.float16)
    ok = True
    for nf4 in (False, True):
        q = o.quantise_nf4 if nf4 else o.quantise
        unit = 64 if nf4 else 128
        p, s, _ = q(W)
        full = o.gemv_f64(nf4, p, s if nf4 else s.view(np.uint16), x)[0]
        # row-parallel: partial over this rank's columns, then all-reduce (sum)
        c0, c1 = col_range(in_f, unit, world, rank)
        ps, ss = numpy_shard_columns(p, s, unit, c0, c1)
        part = o.gemv_f64(nf4, ps, ss if nf4 else ss.view(np.uint16), x[:, c0:c1])[0]
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        ok &= bool(np.max(np.abs(t.numpy() - full)) <= 1e-12 * max(1.0, np.max(np.abs(full))))
        # column-parallel: each rank's rows, gathered
        r0, r1 = row_range(out_f, world, rank)
        mine = torch.from_numpy(o.gemv_f64(nf4, p[r0:r1], s[r0:r1] if nf4 else s[r0:r1].view(np.uint16), x)[0])
        gathered = [None] * world
        dist.all_gather_object(gathered, mine.numpy())
        ok &= bool(np.array_equal(np.concatenate(gathered), full))
    results[rank] = ok
    dist.destroy_process_group()


def test_shard_math_two_gloo_ranks():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert dict(results) == {0: True, 1: True}
