"""Python host side of the B200 fused 4-bit dequantisation GEMV.

Thin wrappers over the C ABI (include/b4gemv.h, libb4gemv.so) that take torch
tensors for device buffers and numpy arrays for host buffers.  Names and
argument meaning follow the reference's host API (QuantumDrizzy/int4-gemv,
src/kernels.cuh): ``quantise`` / ``quantise_nf4`` (kernels.cuh:270,308), the
``GROUP`` / ``NF4_BLOCK`` constants (kernels.cuh:12,85) and one GEMV per
format (kernels.cuh:26,87).  Every GPU call goes through the CUDA library;
there is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import (ENGINE_NF4_XTAB, FLAG_KSLICE, FLAG_PDL, FLAG_SPLIT, FMT_INT4_G128, FMT_NF4_B64, GROUP, MAX_SEGMENTS,
                   NF4_BLOCK, XTAB_WORKSPACE_BYTES, B4Error, GemvConfig, GemvSegment, check, load)

__all__ = [
    "GROUP", "NF4_BLOCK", "FMT_INT4_G128", "FMT_NF4_B64", "FLAG_PDL", "B4Error",
    "GemvConfig", "load", "quantise", "quantise_nf4", "gemv_int4", "gemv_nf4", "gemv",
    "gemv_nf4_block_per_row", "dequant_int4", "dequant_nf4", "unpack_codes",
    "quantise_device", "quantise_nf4_device", "default_config", "median", "gemv_multi",
    "multi_default_config", "MAX_SEGMENTS", "GemvSegment", "repack_bnb_nf4", "FLAG_SPLIT", "FLAG_KSLICE",
    "gemv_ws", "workspace_size", "workspace", "default_config_ws", "multi_default_config_ws",
    "ENGINE_NF4_XTAB", "XTAB_WORKSPACE_BYTES",
]


def _ptr(a) -> ctypes.c_void_p:
    if isinstance(a, np.ndarray):
        return ctypes.c_void_p(a.ctypes.data)
    return ctypes.c_void_p(a.data_ptr())


def _stream(stream=None) -> ctypes.c_void_p:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


# ---- host quantisers (kernels.cuh:268-339) ---------------------------------

def quantise(W: np.ndarray, nthreads: int = 0):
    """INT4 g128: returns (packed uint32 [out][in/8], scales fp16 [out][in/128],
    deq fp32 [out][in]) byte-identical to the reference's quantise()."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    out_f, in_f = W.shape
    packed = np.zeros((out_f, in_f // 8), np.uint32)
    scales = np.zeros((out_f, max(in_f // GROUP, 1)), np.float16)
    deq = np.zeros((out_f, in_f), np.float32)
    check("b4_quantise_int4_g128",
          load().b4_quantise_int4_g128(_ptr(W), out_f, in_f, _ptr(packed), _ptr(scales), _ptr(deq),
                                       nthreads))
    return packed, scales, deq


def quantise_nf4(W: np.ndarray, nthreads: int = 0):
    """NF4 b64: returns (packed uint32 [out][in/8], absmax fp32 [out][in/64],
    deq fp32 [out][in]) byte-identical to the reference's quantise_nf4()."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    out_f, in_f = W.shape
    packed = np.zeros((out_f, in_f // 8), np.uint32)
    absmax = np.zeros((out_f, max(in_f // NF4_BLOCK, 1)), np.float32)
    deq = np.zeros((out_f, in_f), np.float32)
    check("b4_quantise_nf4_b64",
          load().b4_quantise_nf4_b64(_ptr(W), out_f, in_f, _ptr(packed), _ptr(absmax), _ptr(deq),
                                     nthreads))
    return packed, absmax, deq


def median(v):
    """kernels.cuh:341-345: the upper median (element len/2 after sorting)."""
    s = sorted(v)
    return s[len(s) // 2]


# ---- device quantisers -------------------------------------------------------

def quantise_device(W, with_deq: bool = False, stream=None):
    """INT4 g128 on the GPU.  W: float32 CUDA tensor [out][in].  Returns
    (packed int32 [out][in/8], scales fp16 [out][in/128], deq or None)."""
    import torch
    assert W.is_cuda and W.dtype == torch.float32 and W.is_contiguous()
    out_f, in_f = W.shape
    packed = torch.empty((out_f, in_f // 8), dtype=torch.int32, device=W.device)
    scales = torch.empty((out_f, max(in_f // GROUP, 1)), dtype=torch.float16, device=W.device)
    deq = torch.empty_like(W) if with_deq else None
    check("b4_quantise_int4_g128_device",
          load().b4_quantise_int4_g128_device(_ptr(W), out_f, in_f, _ptr(packed), _ptr(scales),
                                              _ptr(deq) if deq is not None else None,
                                              _stream(stream)))
    return packed, scales, deq


def quantise_nf4_device(W, with_deq: bool = False, stream=None):
    """NF4 b64 on the GPU.  Returns (packed int32, absmax fp32, deq or None)."""
    import torch
    assert W.is_cuda and W.dtype == torch.float32 and W.is_contiguous()
    out_f, in_f = W.shape
    packed = torch.empty((out_f, in_f // 8), dtype=torch.int32, device=W.device)
    absmax = torch.empty((out_f, max(in_f // NF4_BLOCK, 1)), dtype=torch.float32, device=W.device)
    deq = torch.empty_like(W) if with_deq else None
    check("b4_quantise_nf4_b64_device",
          load().b4_quantise_nf4_b64_device(_ptr(W), out_f, in_f, _ptr(packed), _ptr(absmax),
                                            _ptr(deq) if deq is not None else None,
                                            _stream(stream)))
    return packed, absmax, deq


# ---- GEMV ----------------------------------------------------------------------

def default_config(fmt: int, in_f: int, out_f: int, m: int = 1) -> dict:
    c = GemvConfig()
    check("b4_gemv_default_config", load().b4_gemv_default_config(fmt, in_f, out_f, m, ctypes.byref(c)))
    return c.as_dict()


def default_config_ws(fmt: int, in_f: int, out_f: int, m: int = 1) -> dict:
    """b4_gemv_default_config_ws: the config b4_gemv_ws uses: the x-pair table
    kernel for NF4 at batch 1 on matrices of >= 17.5 MB of weights (5 MB for
    in_f >= 8192), b4_gemv_default_config's choice otherwise."""
    c = GemvConfig()
    check("b4_gemv_default_config_ws", load().b4_gemv_default_config_ws(fmt, in_f, out_f, m, ctypes.byref(c)))
    return c.as_dict()


def _gemv_args(qw, scale, x, y):
    import torch
    assert qw.is_cuda and qw.dtype in (torch.int32, torch.uint32) and qw.is_contiguous()
    out_f, words = qw.shape
    in_f = words * 8
    x2 = x.reshape(-1, in_f) if x.dim() != 2 else x
    assert x2.dtype == torch.float16 and x2.is_contiguous() and x2.shape[1] == in_f
    m = x2.shape[0]
    if y is None:
        y = torch.empty((m, out_f), dtype=torch.float32, device=qw.device)
    assert y.dtype == torch.float32 and y.is_contiguous() and y.numel() == m * out_f
    return out_f, in_f, m, x2, y


def gemv(fmt: int, qw, scale, x, y=None, config: dict | None = None, stream=None):
    """y[m][out] = dequant(qw, scale) @ x[m][in]^T through b4_gemv_ex."""
    out_f, in_f, m, x2, y = _gemv_args(qw, scale, x, y)
    cfg = ctypes.byref(GemvConfig.from_dict(config)) if config is not None else None
    check("b4_gemv_ex", load().b4_gemv_ex(fmt, _ptr(qw), _ptr(scale), _ptr(x2), _ptr(y), in_f, out_f, m,
                                          cfg, _stream(stream)))
    return y


_WS_SIZE = {}
_WS = {}


def workspace_size(fmt: int, in_f: int, out_f: int, m: int = 1, config: dict | None = None, device=None) -> int:
    """b4_gemv_workspace_size on the current device (or `device`, an index):
    bytes of workspace b4_gemv_ws needs for this shape (0 when the config needs
    none: neither the x-pair table kernel nor a split).  Rule answers are
    cached per (shape, device)."""
    import torch
    if config is None:
        key = (fmt, in_f, out_f, m, torch.cuda.current_device() if device is None else device)
        n = _WS_SIZE.get(key)
        if n is not None:
            return n
    else:
        key = None
    cfg = ctypes.byref(GemvConfig.from_dict(config)) if config is not None else None
    n = ctypes.c_size_t(0)
    check("b4_gemv_workspace_size", load().b4_gemv_workspace_size(fmt, in_f, out_f, m, cfg, ctypes.byref(n)))
    if key is not None:
        _WS_SIZE[key] = n.value
    return n.value


def workspace(device, nbytes: int):
    """The package's workspace for b4_gemv_ws on `device`: one zero-filled
    uint8 tensor per device, grown on demand (at least 1 MiB).  Every call
    leaves it ready for the next (the x-pair table kernel's running counters
    in the first 256 bytes, the split path's counters zero after them).
    Calls on different streams
    that may overlap must not share it: pass them their own
    (torch.zeros(n, dtype=torch.uint8))."""
    import torch
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=f"cuda:{idx}")
        _WS[idx] = ws
    return ws


_AUTO_PDL = {"engine": -1, "flags": FLAG_PDL}


def gemv_ws(fmt: int, qw, scale, x, y=None, config: dict | None = None, ws=None, stream=None, pdl: bool = False):
    """b4_gemv_ws: the GEMV with a workspace (config None = the rule of
    b4_gemv_ws: the x-pair table kernel for NF4 at batch 1 with in_f % 256 ==
    0, the plain dispatch rule otherwise; the split kernels when a split
    config is passed).
    ws: a zero-filled CUDA uint8 tensor of at least workspace_size() bytes, or
    None for the package's per-device workspace.  pdl (with config None): the
    dispatch rule's launch as a programmatic dependent of the previous kernel
    on the stream (B4_ENGINE_AUTO + B4_FLAG_PDL)."""
    if pdl and config is None:
        config = _AUTO_PDL
    out_f, in_f, m, x2, y = _gemv_args(qw, scale, x, y)
    need = workspace_size(fmt, in_f, out_f, m, config, qw.device.index)
    if ws is None and need:
        ws = workspace(qw.device, need)
    cfg = ctypes.byref(GemvConfig.from_dict(config)) if config is not None else None
    check("b4_gemv_ws", load().b4_gemv_ws(fmt, _ptr(qw), _ptr(scale), _ptr(x2), _ptr(y), in_f, out_f, m, cfg,
                                          _ptr(ws) if ws is not None else None,
                                          ws.numel() if ws is not None else 0, _stream(stream)))
    return y


def gemv_int4(qw, scales, x, y=None, stream=None, use_ws: bool = True, pdl: bool = False):
    """The INT4 g128 GEMV with the dispatch rule's config: b4_gemv_ws with the
    package's workspace (use_ws: True; pdl: as a programmatic dependent of the
    previous kernel), or b4_gemv_int4_g128 (use_ws: False)."""
    if use_ws:
        return gemv_ws(FMT_INT4_G128, qw, scales, x, y, stream=stream, pdl=pdl)
    out_f, in_f, m, x2, y = _gemv_args(qw, scales, x, y)
    check("b4_gemv_int4_g128", load().b4_gemv_int4_g128(_ptr(qw), _ptr(scales), _ptr(x2), _ptr(y), in_f,
                                                        out_f, m, _stream(stream)))
    return y


def gemv_nf4(qw, absmax, x, y=None, stream=None, use_ws: bool = True, pdl: bool = False):
    """The NF4 b64 GEMV with the dispatch rule's config: b4_gemv_ws with the
    package's workspace (use_ws: True, the x-pair table kernel where the rule
    picks it; pdl: as a programmatic dependent of the previous kernel), or
    b4_gemv_nf4_b64 (use_ws: False)."""
    if use_ws:
        return gemv_ws(FMT_NF4_B64, qw, absmax, x, y, stream=stream, pdl=pdl)
    out_f, in_f, m, x2, y = _gemv_args(qw, absmax, x, y)
    check("b4_gemv_nf4_b64", load().b4_gemv_nf4_b64(_ptr(qw), _ptr(absmax), _ptr(x2), _ptr(y), in_f,
                                                    out_f, m, _stream(stream)))
    return y


def _segments(pairs, x, ys, alloc=True):
    import torch
    assert 1 <= len(pairs) <= MAX_SEGMENTS
    in_f = pairs[0][0].shape[1] * 8
    x2 = x.reshape(-1, in_f) if x.dim() != 2 else x
    assert x2.dtype == torch.float16 and x2.is_contiguous() and x2.shape[1] == in_f
    m = x2.shape[0]
    segs = (GemvSegment * len(pairs))()
    out = []
    for i, (qw, scale) in enumerate(pairs):
        assert qw.is_cuda and qw.dtype in (torch.int32, torch.uint32) and qw.is_contiguous()
        assert qw.shape[1] * 8 == in_f, "every segment shares x, so in_f must match"
        out_f = qw.shape[0]
        if not alloc:
            segs[i] = GemvSegment(qw.data_ptr(), scale.data_ptr(), None, out_f)
            continue
        y = ys[i] if ys is not None else torch.empty((m, out_f), dtype=torch.float32, device=qw.device)
        assert y.dtype == torch.float32 and y.is_contiguous() and y.numel() == m * out_f
        segs[i] = GemvSegment(qw.data_ptr(), scale.data_ptr(), y.data_ptr(), out_f)
        out.append(y)
    return segs, x2, in_f, m, out


def multi_default_config(fmt: int, pairs, x) -> dict:
    """b4_gemv_multi_default_config: the dispatch rule over the segments' total rows."""
    segs, _, in_f, m, _ = _segments(pairs, x, None, alloc=False)
    c = GemvConfig()
    check("b4_gemv_multi_default_config",
          load().b4_gemv_multi_default_config(fmt, segs, len(pairs), in_f, m, ctypes.byref(c)))
    return c.as_dict()


def multi_default_config_ws(fmt: int, pairs, x) -> dict:
    """b4_gemv_multi_default_config_ws: the rule of b4_gemv_multi_ws."""
    segs, _, in_f, m, _ = _segments(pairs, x, None, alloc=False)
    c = GemvConfig()
    check("b4_gemv_multi_default_config_ws",
          load().b4_gemv_multi_default_config_ws(fmt, segs, len(pairs), in_f, m, ctypes.byref(c)))
    return c.as_dict()


def gemv_multi(fmt: int, pairs, x, ys=None, config: dict | None = None, stream=None, pdl: bool = False,
               ws=None, use_ws: bool = True):
    """y_s = dequant(qw_s, scale_s) @ x for every (qw_s, scale_s) in `pairs`
    (up to four matrices with the same in_f), one launch at batch 1.  With
    use_ws (the default): b4_gemv_multi_ws with `ws` or the package's
    per-device workspace (NF4 at batch 1 runs on the x-pair table kernel);
    else b4_gemv_multi.  pdl (with config None): the rule's launch as a
    programmatic dependent of the previous kernel.  Returns the list of y_s."""
    segs, x2, in_f, m, out = _segments(pairs, x, ys)
    if use_ws:
        if config is None and pdl:
            config = _AUTO_PDL
        if ws is None:
            ws = workspace(pairs[0][0].device, XTAB_WORKSPACE_BYTES)
        cfg = ctypes.byref(GemvConfig.from_dict(config)) if config is not None else None
        check("b4_gemv_multi_ws", load().b4_gemv_multi_ws(fmt, segs, len(pairs), _ptr(x2), in_f, m, cfg, _ptr(ws),
                                                          ws.numel(), _stream(stream)))
        return out
    if pdl and config is None:
        config = dict(multi_default_config(fmt, pairs, x), flags=FLAG_PDL)
    cfg = ctypes.byref(GemvConfig.from_dict(config)) if config is not None else None
    check("b4_gemv_multi", load().b4_gemv_multi(fmt, segs, len(pairs), _ptr(x2), in_f, m, cfg, _stream(stream)))
    return out


def gemv_nf4_block_per_row(qw, absmax, x, warps_per_block: int, y=None, stream=None):
    out_f, in_f, m, x2, y = _gemv_args(qw, absmax, x, y)
    assert m == 1
    check("b4_gemv_nf4_b64_block_per_row",
          load().b4_gemv_nf4_b64_block_per_row(_ptr(qw), _ptr(absmax), _ptr(x2), _ptr(y), in_f, out_f,
                                               warps_per_block, _stream(stream)))
    return y


# ---- bit-exact format helpers -------------------------------------------------

def dequant_int4(qw, scales, out=None, stream=None):
    import torch
    out_f, words = qw.shape
    in_f = words * 8
    if out is None:
        out = torch.empty((out_f, in_f), dtype=torch.float32, device=qw.device)
    check("b4_dequant_int4_g128", load().b4_dequant_int4_g128(_ptr(qw), _ptr(scales), _ptr(out), in_f, out_f,
                                                              _stream(stream)))
    return out


def dequant_nf4(qw, absmax, out=None, stream=None):
    import torch
    out_f, words = qw.shape
    in_f = words * 8
    if out is None:
        out = torch.empty((out_f, in_f), dtype=torch.float32, device=qw.device)
    check("b4_dequant_nf4_b64", load().b4_dequant_nf4_b64(_ptr(qw), _ptr(absmax), _ptr(out), in_f, out_f,
                                                          _stream(stream)))
    return out


def repack_bnb_nf4(bnb_packed, out=None, stream=None):
    """b4_repack_bnb_nf4: bitsandbytes-layout NF4 bytes [out_f][in_f/2] (lower
    column in the high nibble) -> packed words [out_f][in_f/8] of this library;
    applied to packed words it converts back."""
    import torch
    out_f = bnb_packed.shape[0]
    in_f = bnb_packed.numel() * 2 // out_f
    if out is None:
        out = torch.empty((out_f, in_f // 8), dtype=torch.int32, device=bnb_packed.device)
    check("b4_repack_bnb_nf4", load().b4_repack_bnb_nf4(_ptr(bnb_packed), _ptr(out), in_f, out_f, _stream(stream)))
    return out


def unpack_codes(qw, out=None, stream=None):
    import torch
    out_f, words = qw.shape
    in_f = words * 8
    if out is None:
        out = torch.empty((out_f, in_f), dtype=torch.uint8, device=qw.device)
    check("b4_unpack_codes", load().b4_unpack_codes(_ptr(qw), _ptr(out), in_f, out_f, _stream(stream)))
    return out
