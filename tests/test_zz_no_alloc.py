"""The split GEMV without allocation (b4_gemv_split_noalloc), through the C ABI.

Some callers cannot allocate device memory: a plugin that a host framework
hands only its input and output buffers (the framework owns every
allocation), or code whose memory budget is fixed before its first call.  For
them the split GEMV keeps its scratch in the library's static device array
instead of a caller-owned workspace.  These tests check that entry point
against the existing one with a caller-owned workspace (b4_gemv_ws, same
config) on two calls in a row with different inputs -- the array keeps the
previous call's contents, so the second call must not depend on them -- and
that a shape needing more scratch than the array holds is refused before
anything is launched.  This file is collected last, so a run that stops at
the first failure has run every other test; it also passes on its own in a
fresh process (the first call on the device sets up the array).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import b4gemv
from b4gemv._lib import GemvConfig, load
from oracle_py import rel_err
from test_gemv_gpu import f64_ref, quantised, rand_problem, to_dev

TOL = 1e-3
pytestmark = pytest.mark.gpu

SCRATCH_TOO_SMALL = 10902   # B4_STATUS_SCRATCH_TOO_SMALL
STATIC_SCRATCH_BYTES = 1 << 20


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def split_cfg(fmt, in_f):
    """The config b4_gemv_split_noalloc uses with cfg NULL (aligned buffers)."""
    c = {"vec_words": 4, "rows_per_warp": 16, "batch_tile": 1, "warps_k": 1, "row_groups": 8,
         "flags": b4gemv.FLAG_SPLIT}
    if fmt == 0:
        ng = in_f // 128
        st, sg = (2, 4) if ng % 4 == 0 else ((3, 2) if ng % 2 == 0 else (6, 1))
        c.update(engine=5, stages=st, stage_groups=sg)
    else:
        c.update(engine=7, stages=3, stage_groups=0)
    return c


@pytest.mark.parametrize("fmt,out_f,in_f", [(0, 8192, 8192), (1, 3584, 18944), (0, 2049, 1152), (1, 300, 1024)])
def test_noalloc_matches_workspace_entry_on_two_calls(cuda, oracle, fmt, out_f, in_f):
    import torch
    lib = load()
    rng = np.random.default_rng(out_f + in_f + fmt)
    W, X1 = rand_problem(rng, out_f, in_f)
    X2 = rng.standard_normal((1, in_f)).astype(np.float16)
    qw, sc = quantised(fmt, W, cuda)
    cfg_d = split_cfg(fmt, in_f)
    cfg = GemvConfig.from_dict(cfg_d)
    need = b4gemv.workspace_size(fmt, in_f, out_f, 1, cfg_d)
    assert 0 < need <= STATIC_SCRATCH_BYTES
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for X in (X1, X2):
        x = to_dev(X, cuda)
        y_static = torch.full((1, out_f), float("nan"), dtype=torch.float32, device=cuda)
        y_ws = torch.full((1, out_f), float("nan"), dtype=torch.float32, device=cuda)
        # cfg NULL: the entry point's own split config
        assert lib.b4_gemv_split_noalloc(fmt, _p(qw), _p(sc), _p(x), _p(y_static), in_f, out_f, None, st) == 0
        assert lib.b4_gemv_ws(fmt, _p(qw), _p(sc), _p(x), _p(y_ws), in_f, out_f, 1, ctypes.byref(cfg), _p(ws),
                              need, st) == 0
        torch.cuda.synchronize()
        a, b = y_static.cpu().numpy(), y_ws.cpu().numpy()
        assert np.isfinite(a).all()
        assert rel_err(a, b) < TOL
        assert rel_err(a, f64_ref(oracle, fmt, qw, sc, X)) < TOL


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda):
    import torch
    lib = load()
    out_f, in_f = 131072, 128       # 8192 row blocks: the split needs > 1 MiB of scratch
    cfg_d = split_cfg(0, in_f)
    assert b4gemv.workspace_size(0, in_f, out_f, 1, cfg_d) > STATIC_SCRATCH_BYTES
    qw = torch.zeros((out_f, in_f // 8), dtype=torch.int32, device=cuda)
    sc = torch.zeros((out_f, 1), dtype=torch.float16, device=cuda)
    x = torch.zeros((1, in_f), dtype=torch.float16, device=cuda)
    y = torch.zeros((1, out_f), dtype=torch.float32, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.b4_gemv_split_noalloc(0, _p(qw), _p(sc), _p(x), _p(y), in_f, out_f, None, st) == SCRATCH_TOO_SMALL
    assert b"static array" in lib.b4_status_string(SCRATCH_TOO_SMALL)
    # a config without the split flag is not this entry point's
    plain = GemvConfig.from_dict(b4gemv.default_config(0, in_f, 4096, 1))
    assert lib.b4_gemv_split_noalloc(0, _p(qw), _p(sc), _p(x), _p(y), in_f, 4096, ctypes.byref(plain), st) == 1
    torch.cuda.synchronize()


def test_noalloc_refuses_nf4_rows_not_a_multiple_of_128(cuda):
    """The NF4 split takes 128-column steps: in_f = 1088 (a multiple of 64,
    not of 128) is refused before any launch, so a caller can fall back to
    b4_gemv_nf4_b64."""
    import torch
    lib = load()
    out_f, in_f = 64, 1088
    qw = torch.zeros((out_f, in_f // 8), dtype=torch.int32, device=cuda)
    am = torch.ones((out_f, in_f // 64), dtype=torch.float32, device=cuda)
    x = torch.zeros((1, in_f), dtype=torch.float16, device=cuda)
    y = torch.zeros((1, out_f), dtype=torch.float32, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.b4_gemv_split_noalloc(1, _p(qw), _p(am), _p(x), _p(y), in_f, out_f, None, st) == 1
    assert lib.b4_gemv_nf4_b64(_p(qw), _p(am), _p(x), _p(y), in_f, out_f, 1, st) == 0
    torch.cuda.synchronize()


_FRESH = r"""
import ctypes, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
import numpy as np, torch
import b4gemv
from b4gemv._lib import GemvConfig, load
from test_zz_no_alloc import split_cfg
from test_gemv_gpu import quantised, rand_problem, to_dev
dev = torch.device("cuda", 0)
lib = load()
out_f, in_f = 3584, 3584
rng = np.random.default_rng(9)
W, X = rand_problem(rng, out_f, in_f)
qw, sc = quantised(0, W, dev)
x = to_dev(X, dev)
P = lambda t: ctypes.c_void_p(t.data_ptr())
cfg_d = split_cfg(0, in_f)
need = b4gemv.workspace_size(0, in_f, out_f, 1, cfg_d)
ws = torch.zeros(need, dtype=torch.uint8, device=dev)
y_ws = torch.empty((1, out_f), device=dev)
assert lib.b4_gemv_ws(0, P(qw), P(sc), P(x), P(y_ws), in_f, out_f, 1, ctypes.byref(GemvConfig.from_dict(cfg_d)), P(ws),
                      need, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
torch.cuda.synchronize()
# the process's first no-allocation call, on a stream not ordered with the legacy stream
s = torch.cuda.Stream()
y = torch.full((1, out_f), float("nan"), device=dev)
with torch.cuda.stream(s):
    assert lib.b4_gemv_split_noalloc(0, P(qw), P(sc), P(x), P(y), in_f, out_f, None, ctypes.c_void_p(s.cuda_stream)) == 0
s.synchronize()
d = float((y - y_ws).abs().max() / y_ws.abs().max())
assert d < 1e-6, d
# after that first call the entry point may be captured in a CUDA graph
g = torch.cuda.CUDAGraph()
with torch.cuda.graph(g, stream=s):
    lib.b4_gemv_split_noalloc(0, P(qw), P(sc), P(x), P(y), in_f, out_f, None, ctypes.c_void_p(s.cuda_stream))
for _ in range(2):
    y.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    d = float((y - y_ws).abs().max() / y_ws.abs().max())
    assert d < 1e-6, d
print("ok")
"""


def test_noalloc_first_call_on_a_non_blocking_stream_then_captured(cuda):
    """In a fresh process: the first no-allocation call (which sets up the
    static array) on a torch stream, which is not ordered with the legacy
    stream, gives the workspace entry's y; after it the call can be captured
    in a CUDA graph and replayed."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    pkg = os.path.join(os.path.dirname(here), "int4-gemv_b200")
    r = subprocess.run([sys.executable, "-c", _FRESH, here, pkg], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.stdout[-2000:], r.stderr[-2000:])
