"""The 28-layer decode chain: one token through the seven
projections of every Qwen2.5-7B layer (hidden 3584, intermediate 18944, 4 KV
heads x 128), INT4 g128 weights, random fp16 activations between projections,
all 196 GEMVs captured in one CUDA graph on one GPU.  It exposes the launch
overhead the isolated-launch numbers hide; with programmatic dependent launch
each GEMV streams its first weights while the previous one finishes.
"""
from __future__ import annotations

import ctypes

from ._lib import FLAG_PDL, FMT_INT4_G128, FMT_NF4_B64, GemvConfig, check, load

QWEN_LAYER = [("q", 3584, 3584), ("k", 512, 3584), ("v", 512, 3584), ("o", 3584, 3584),
              ("gate", 18944, 3584), ("up", 18944, 3584), ("down", 3584, 18944)]


def alg_bytes(fmt, out_f, in_f):
    scale = out_f * (in_f // 64) * 4 if fmt == FMT_NF4_B64 else out_f * (in_f // 128) * 2
    return out_f * in_f // 2 + scale + in_f * 2


class DecodeChain:
    def __init__(self, torch, device, fmt=FMT_INT4_G128, layers=28, seed=0):
        from . import quantise_device, quantise_nf4_device
        self.torch, self.fmt, self.layers = torch, fmt, layers
        quant = quantise_nf4_device if fmt == FMT_NF4_B64 else quantise_device
        self.calls = []   # (qw, sc, x, y, in_f, out_f)
        self.bytes = 0
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        for layer in range(layers):
            for i, (name, out_f, in_f) in enumerate(QWEN_LAYER):
                W = torch.randn((out_f, in_f), generator=g, device=device) * 0.02
                qw, sc, _ = quant(W)
                del W
                x = torch.randn((1, in_f), generator=g, device=device).half()
                y = torch.empty((1, out_f), device=device)
                self.calls.append((qw, sc, x, y, in_f, out_f))
                self.bytes += alg_bytes(fmt, out_f, in_f)
        torch.cuda.synchronize(device)
        lib = load()
        self.cfgs = {}
        for (qw, sc, x, y, in_f, out_f) in self.calls:
            key = (in_f, out_f)
            if key not in self.cfgs:
                c = GemvConfig()
                check("default_config", lib.b4_gemv_default_config(fmt, in_f, out_f, 1, ctypes.byref(c)))
                self.cfgs[key] = c

    def launch_all(self, stream, pdl: bool):
        lib = load()
        for (qw, sc, x, y, in_f, out_f) in self.calls:
            c = self.cfgs[(in_f, out_f)]
            c.flags = FLAG_PDL if pdl else 0
            check("b4_gemv_ex", lib.b4_gemv_ex(self.fmt, ctypes.c_void_p(qw.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                                               ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), in_f,
                                               out_f, 1, ctypes.byref(c), stream))

    def capture(self, pdl: bool):
        torch = self.torch
        self.launch_all(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), pdl)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(graph, stream=cs, capture_error_mode="relaxed"):
            self.launch_all(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), pdl)
        torch.cuda.current_stream().wait_stream(cs)
        return graph

    def time_token(self, pdl: bool, tokens: int = 20):
        """us per token: the graph (all layers) replayed `tokens` times."""
        torch = self.torch
        graph = self.capture(pdl)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(tokens):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / tokens
        del graph
        return us
