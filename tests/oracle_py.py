"""ctypes binding of the C oracle (oracle/b4_oracle.c).  Test infrastructure:
only tests, the smoke check and the bench's CPU-baseline legs use it."""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_build", "libb4oracle.so")
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libref.so")


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


class Oracle:
    def __init__(self):
        if not os.path.exists(LIB):
            subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "_build/libb4oracle.so"],
                           check=True, capture_output=True)
        self.lib = ctypes.CDLL(LIB)
        self.lib.b4o_half_from_float.restype = ctypes.c_uint16
        self.lib.b4o_half_from_float.argtypes = [ctypes.c_float]
        self.lib.b4o_float_from_half.restype = ctypes.c_float
        self.lib.b4o_float_from_half.argtypes = [ctypes.c_uint16]
        self.lib.b4o_rel_err.restype = ctypes.c_double
        self.lib.b4o_gemv_int4_fused.restype = ctypes.c_int
        self.lib.b4o_gemv_nf4_fused.restype = ctypes.c_int
        self.nf4_table = np.ctypeslib.as_array((ctypes.c_float * 16).in_dll(self.lib, "b4o_nf4_table")).copy()

    # kernels.cuh:268-297
    def quantise(self, W):
        W = np.ascontiguousarray(W, np.float32)
        o, n = W.shape
        p = np.zeros((o, n // 8), np.uint32)
        s = np.zeros((o, n // 128), np.uint16)
        d = np.zeros((o, n), np.float32)
        self.lib.b4o_quantise_int4(_p(W), o, n, _p(p), _p(s), _p(d))
        return p, s, d

    # kernels.cuh:308-339
    def quantise_nf4(self, W):
        W = np.ascontiguousarray(W, np.float32)
        o, n = W.shape
        p = np.zeros((o, n // 8), np.uint32)
        a = np.zeros((o, n // 64), np.float32)
        d = np.zeros((o, n), np.float32)
        self.lib.b4o_quantise_nf4(_p(W), o, n, _p(p), _p(a), _p(d))
        return p, a, d

    def unpack(self, packed, in_f):
        packed = np.ascontiguousarray(packed, np.uint32)
        o = packed.shape[0]
        c = np.zeros((o, in_f), np.uint8)
        self.lib.b4o_unpack_codes(_p(packed), o, in_f, _p(c))
        return c

    def dequant_int4(self, packed, scales):
        packed = np.ascontiguousarray(packed, np.uint32)
        scales = np.ascontiguousarray(scales).view(np.uint16)
        o, w = packed.shape
        d = np.zeros((o, w * 8), np.float32)
        self.lib.b4o_dequant_int4(_p(packed), _p(scales), o, w * 8, _p(d))
        return d

    def dequant_nf4(self, packed, absmax):
        packed = np.ascontiguousarray(packed, np.uint32)
        absmax = np.ascontiguousarray(absmax, np.float32)
        o, w = packed.shape
        d = np.zeros((o, w * 8), np.float32)
        self.lib.b4o_dequant_nf4(_p(packed), _p(absmax), o, w * 8, _p(d))
        return d

    def gemv_f64(self, nf4, packed, scale, X):
        """Double GEMV over the dequantised weights; X fp16 [m][in] -> [m][out]."""
        packed = np.ascontiguousarray(packed, np.uint32)
        X = np.ascontiguousarray(np.atleast_2d(X).astype(np.float16)).view(np.uint16)
        o, w = packed.shape
        m = X.shape[0]
        Y = np.zeros((m, o), np.float64)
        if nf4:
            self.lib.b4o_gemv_nf4_f64(_p(packed), _p(np.ascontiguousarray(scale, np.float32)), _p(X), o, w * 8, m, _p(Y))
        else:
            sc = np.ascontiguousarray(scale).view(np.uint16)
            self.lib.b4o_gemv_int4_f64(_p(packed), _p(sc), _p(X), o, w * 8, m, _p(Y))
        return Y

    def gemv_fused(self, nf4, packed, scale, X, nthreads=0):
        """The reference kernels' per-lane fp32 arithmetic on the CPU."""
        packed = np.ascontiguousarray(packed, np.uint32)
        X = np.ascontiguousarray(np.atleast_2d(X).astype(np.float16)).view(np.uint16)
        o, w = packed.shape
        m = X.shape[0]
        Y = np.zeros((m, o), np.float32)
        if nf4:
            n = self.lib.b4o_gemv_nf4_fused(_p(packed), _p(np.ascontiguousarray(scale, np.float32)), _p(X), o,
                                            w * 8, m, _p(Y), nthreads)
        else:
            sc = np.ascontiguousarray(scale).view(np.uint16)
            n = self.lib.b4o_gemv_int4_fused(_p(packed), _p(sc), _p(X), o, w * 8, m, _p(Y), nthreads)
        return Y, n

    def gemv_deq_f32(self, deq, x):
        """int4_gemv.cu:33-38: fp32 loop over the dequantised matrix."""
        deq = np.ascontiguousarray(deq, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        o, n = deq.shape
        y = np.zeros(o, np.float32)
        self.lib.b4o_gemv_deq_f32(_p(deq), _p(x), o, n, _p(y))
        return y

    def rel_err(self, got, ref):
        got = np.ascontiguousarray(got, np.float32).ravel()
        ref = np.ascontiguousarray(ref, np.float64).ravel()
        return self.lib.b4o_rel_err(_p(got), _p(ref), got.size)


def rel_err(got, ref) -> float:
    """max|got-ref| / max|ref| (int4_gemv.cu:74-81), NaN-aware, in numpy."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.max(np.abs(got - ref)) if got.size else 0.0
    scale = np.max(np.abs(ref)) if ref.size else 0.0
    return float(err / scale) if scale > 0 else float(err)


def bnb_pack_nf4(codes):
    """bitsandbytes' 4-bit packing of a row-major code matrix [out][in]
    (uint8 values 0..15): byte j of a row = (code[2j] << 4) | code[2j+1], the
    lower column in the high nibble (bitsandbytes' blockwise 4-bit quantiser
    packs pairs this way; bitsandbytes itself is not installed here, so this
    restatement is unpinned).  Test helper for b4_repack_bnb_nf4."""
    import numpy as np
    c = np.asarray(codes, np.uint8)
    return ((c[:, 0::2] << 4) | c[:, 1::2]).astype(np.uint8)

