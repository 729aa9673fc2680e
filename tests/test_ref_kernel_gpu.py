"""The reference's own kernels, rebuilt for sm_100a from its sources
(oracle/_ref/libref.so), run on the same device buffers as this library.

Pins the oracle's fused CPU GEMV (the reference kernels' per-lane arithmetic)
bit-exactly against the real reference kernels, and checks that this
library's y agrees with the reference's y within tolerance.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

import b4gemv
from oracle_py import REF_LIB, rel_err
from test_gemv_gpu import TOL, quantised, rand_problem, to_dev

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(REF_LIB), reason="oracle/_ref not built")]


@pytest.fixture(scope="module")
def ref():
    lib = ctypes.CDLL(REF_LIB)
    for n in ["ref_launch_int4_warp_per_row", "ref_launch_nf4_warp_per_row", "ref_launch_nf4_block_per_row",
              "ref_launch_nf4_split_k", "ref_launch_dispatch"]:
        getattr(lib, n).restype = ctypes.c_int
    return lib


def P(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("out_f,in_f", [(8, 256), (33, 384), (512, 3584), (64, 18944)])
def test_reference_kernels_equal_oracle_emulation_bit_exact(cuda, oracle, ref, out_f, in_f):
    import torch
    rng = np.random.default_rng(out_f + in_f)
    W, X = rand_problem(rng, out_f, in_f)
    x = to_dev(X[0], cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for fmt in (0, 1):
        qw, sc = quantised(fmt, W, cuda)
        y = torch.full((out_f,), float("nan"), dtype=torch.float32, device=cuda)
        fn = ref.ref_launch_int4_warp_per_row if fmt == 0 else ref.ref_launch_nf4_warp_per_row
        assert fn(P(qw), P(sc), P(x), P(y), in_f, out_f, stream) == 0
        torch.cuda.synchronize()
        p = qw.cpu().numpy().view(np.uint32)
        s = sc.cpu().numpy()
        emu, _ = oracle.gemv_fused(fmt == 1, p, s.view(np.uint16) if fmt == 0 else s, X)
        assert y.cpu().numpy().tobytes() == emu[0].tobytes()


@pytest.mark.parametrize("out_f,in_f", [(3584, 3584), (512, 3584), (3584, 18944)])
def test_library_agrees_with_reference_kernels(cuda, oracle, ref, out_f, in_f):
    import torch
    rng = np.random.default_rng(out_f * 3 + in_f)
    W, X = rand_problem(rng, out_f, in_f)
    x = to_dev(X[0], cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for fmt in (0, 1):
        qw, sc = quantised(fmt, W, cuda)
        y_ref = torch.empty(out_f, dtype=torch.float32, device=cuda)
        assert ref.ref_launch_dispatch(fmt, P(qw), P(sc), P(x), P(y_ref), in_f, out_f, stream) == 0
        y = b4gemv.gemv(fmt, qw, sc, x.view(1, in_f))
        ref64 = oracle.gemv_f64(fmt == 1, qw.cpu().numpy().view(np.uint32),
                                sc.cpu().numpy().view(np.uint16) if fmt == 0 else sc.cpu().numpy(), X)
        assert rel_err(y_ref.cpu().numpy(), ref64) < TOL
        assert rel_err(y.cpu().numpy(), ref64) < TOL
