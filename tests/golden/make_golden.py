"""Generates tests/golden/golden.npz from the reference's own host code.

The reference (QuantumDrizzy/int4-gemv) ships no golden vectors, so these are
made by running its quantise() / quantise_nf4() (src/kernels.cuh:268-339),
compiled in place into oracle/_ref/libref.so by oracle/ref/Makefile, on seeded
inputs.  Run from the repository root after `make -C oracle`:

    python tests/golden/make_golden.py

Cases (W fp32 [out][in], x fp16 [in]):
  kat_glibc   the reference benchmark's own generator (int4_gemv.cu:139-142):
              srand(0), W = (rand()/RAND_MAX - .5) * .04, then x likewise
              without the .04 factor, out=2, in=256 (glibc rand()).
  gauss_*     W ~ N(0, 0.02), x ~ N(0, 1) rounded to fp16 (numpy PCG64 seeds).
  edge        groups of zeros, of magnitudes whose fp16 scale underflows to 0
              or overflows to inf, NaN/inf entries, subnormals and exact
              rounding ties.
Stored per case: W, x (fp16), the reference's INT4 packed/scales/deq and NF4
packed/absmax/deq.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, "oracle", "_ref", "libref.so")


def ref_quantise(lib, W):
    out_f, in_f = W.shape
    W = np.ascontiguousarray(W, np.float32)
    p = np.zeros((out_f, in_f // 8), np.uint32)
    s = np.zeros((out_f, in_f // 128), np.uint16)
    d = np.zeros((out_f, in_f), np.float32)
    P = lambda a: ctypes.c_void_p(a.ctypes.data)
    lib.ref_quantise(P(W), out_f, in_f, P(p), P(s), P(d))
    pn = np.zeros((out_f, in_f // 8), np.uint32)
    a = np.zeros((out_f, in_f // 64), np.float32)
    dn = np.zeros((out_f, in_f), np.float32)
    lib.ref_quantise_nf4(P(W), out_f, in_f, P(pn), P(a), P(dn))
    return p, s, d, pn, a, dn


def glibc_case():
    libc = ctypes.CDLL("libc.so.6")
    libc.srand(0)
    rmax = np.float32(2147483647)  # RAND_MAX on glibc, converted to float as in the reference
    W = np.array([(np.float32(libc.rand()) / rmax - np.float32(0.5)) * np.float32(0.04)
                  for _ in range(2 * 256)], np.float32).reshape(2, 256)
    x = np.array([np.float32(libc.rand()) / rmax - np.float32(0.5) for _ in range(256)], np.float32)
    return W, x.astype(np.float16)


def edge_case():
    rng = np.random.default_rng(7)
    W = (rng.standard_normal((4, 512)) * 0.02).astype(np.float32)
    W[0, 0:128] = 0.0                                    # zero group -> scale 1.0, amax 1.0
    W[0, 128:256] = (rng.standard_normal(128) * 1e-9).astype(np.float32)  # fp16 scale -> 0
    W[0, 256:384] = (rng.standard_normal(128) * 1e6).astype(np.float32)   # fp16 scale -> inf
    W[1, 3] = np.nan
    W[1, 200] = np.inf
    W[1, 300] = -np.inf
    W[2, 0:64] = np.float32(1e-40)                       # subnormal inputs
    W[2, 64:128] = -np.float32(3e-39)
    # exact ties for lround: w = (k + 0.5) * s with s = half(7/7) = 1.0
    W[3, 0:128] = 0.0
    W[3, 0] = 7.0
    W[3, 1:9] = np.array([0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 6.5, -6.5], np.float32)
    x = rng.standard_normal(512).astype(np.float16)
    x[5] = np.float16(0.0)
    return W, x


def main() -> int:
    if not os.path.exists(REF):
        print(f"{REF} missing: run `make -C oracle` (needs the reference sources)", file=sys.stderr)
        return 1
    lib = ctypes.CDLL(REF)
    cases = {"kat_glibc": glibc_case()}
    for i, (o, n) in enumerate([(7, 128), (33, 384), (8, 1024), (1, 128), (5, 640), (16, 256)]):
        rng = np.random.default_rng(100 + i)
        W = (rng.standard_normal((o, n)) * 0.02).astype(np.float32)
        x = rng.standard_normal(n).astype(np.float16)
        cases[f"gauss_{o}x{n}"] = (W, x)
    cases["edge"] = edge_case()
    out = {}
    for name, (W, x) in cases.items():
        p, s, d, pn, a, dn = ref_quantise(lib, W)
        out.update({f"{name}/W": W, f"{name}/x": x, f"{name}/int4_packed": p, f"{name}/int4_scales": s,
                    f"{name}/int4_deq": d, f"{name}/nf4_packed": pn, f"{name}/nf4_absmax": a,
                    f"{name}/nf4_deq": dn})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(cases)} cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
