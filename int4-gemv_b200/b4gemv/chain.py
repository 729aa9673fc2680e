"""The 28-layer decode chain: one token through the seven
projections of every Qwen2.5-7B layer (hidden 3584, intermediate 18944, 4 KV
heads x 128), INT4 g128 weights, random fp16 activations between projections,
all 196 GEMVs captured in one CUDA graph on one GPU.  It exposes the launch
overhead the isolated-launch numbers hide; with programmatic dependent launch
each GEMV streams its first weights while the previous one finishes, and with
`fused` the q/k/v and gate/up projections of a layer run as one launch each
(b4_gemv_multi), 112 launches per token instead of 196.  The other GEMVs go
through b4_gemv_ws with the chain's workspace and the config of its rule
(b4_gemv_default_config_ws: for INT4 the plain tile rule, which never splits;
a split config passed in is kept); the GEMVs run one after another on one
stream, so they share the workspace.
"""
from __future__ import annotations

import ctypes

from ._lib import FLAG_PDL, FLAG_SPLIT, FMT_INT4_G128, FMT_NF4_B64, GemvConfig, GemvSegment, check, load

QWEN_LAYER = [("q", 3584, 3584), ("k", 512, 3584), ("v", 512, 3584), ("o", 3584, 3584),
              ("gate", 18944, 3584), ("up", 18944, 3584), ("down", 3584, 18944)]


def alg_bytes(fmt, out_f, in_f):
    scale = out_f * (in_f // 64) * 4 if fmt == FMT_NF4_B64 else out_f * (in_f // 128) * 2
    return out_f * in_f // 2 + scale + in_f * 2


class DecodeChain:
    """The weights and activations of `layers` layers; q/k/v read the same x,
    and so do gate/up (as in the model), so they can also run fused."""

    def __init__(self, torch, device, fmt=FMT_INT4_G128, layers=28, seed=0):
        from . import quantise_device, quantise_nf4_device
        self.torch, self.fmt, self.layers = torch, fmt, layers
        quant = quantise_nf4_device if fmt == FMT_NF4_B64 else quantise_device
        self.layer_w = []   # per layer: {name: (qw, sc, y)} and the x of each input
        self.bytes = 0
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        for layer in range(layers):
            w = {}
            for name, out_f, in_f in QWEN_LAYER:
                W = torch.randn((out_f, in_f), generator=g, device=device) * 0.02
                qw, sc, _ = quant(W)
                del W
                w[name] = (qw, sc, torch.empty((1, out_f), device=device))
                self.bytes += alg_bytes(fmt, out_f, in_f)
            xs = {k: torch.randn((1, n), generator=g, device=device).half()
                  for k, n in (("qkv", 3584), ("o", 3584), ("gateup", 3584), ("down", 18944))}
            self.layer_w.append((w, xs))
        torch.cuda.synchronize(device)
        self.cfg_single = {}
        self.cfg_multi = {}
        need = 0
        for name, out_f, in_f in QWEN_LAYER:
            n = ctypes.c_size_t(0)
            check("b4_gemv_workspace_size", load().b4_gemv_workspace_size(fmt, in_f, out_f, 1, None, ctypes.byref(n)))
            need = max(need, n.value)
        self.ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)

    def launches(self, fused: bool):
        """(kind, args) per launch of one token, configs resolved."""
        lib = load()
        out = []
        groups = [("qkv", ("q", "k", "v")), ("o", ("o",)), ("gateup", ("gate", "up")), ("down", ("down",))]
        for w, xs in self.layer_w:
            for xkey, names in groups:
                x = xs[xkey]
                if fused and len(names) > 1:
                    segs = (GemvSegment * len(names))(*[GemvSegment(w[n][0].data_ptr(), w[n][1].data_ptr(),
                                                                    w[n][2].data_ptr(), w[n][0].shape[0])
                                                        for n in names])
                    in_f = x.shape[1]
                    key = (in_f, tuple(w[n][0].shape[0] for n in names))
                    if key not in self.cfg_multi:
                        c = GemvConfig()
                        check("multi config", lib.b4_gemv_multi_default_config(self.fmt, segs, len(names), in_f, 1,
                                                                               ctypes.byref(c)))
                        self.cfg_multi[key] = c
                    out.append(("multi", (segs, len(names), x, in_f, self.cfg_multi[key])))
                    continue
                for n in names:
                    qw, sc, y = w[n]
                    in_f, out_f = qw.shape[1] * 8, qw.shape[0]
                    if (in_f, out_f) not in self.cfg_single:
                        c = GemvConfig()
                        check("default_config", lib.b4_gemv_default_config_ws(self.fmt, in_f, out_f, 1,
                                                                              ctypes.byref(c)))
                        self.cfg_single[(in_f, out_f)] = c
                    out.append(("single", (qw, sc, x, y, in_f, out_f, self.cfg_single[(in_f, out_f)])))
        return out

    def launch_all(self, stream, pdl: bool, fused: bool = False):
        lib = load()
        for kind, a in self.launches(fused):
            if kind == "multi":
                segs, n, x, in_f, c = a
                c.flags = FLAG_PDL if pdl else 0
                check("b4_gemv_multi", lib.b4_gemv_multi(self.fmt, segs, n, ctypes.c_void_p(x.data_ptr()), in_f, 1,
                                                         ctypes.byref(c), stream))
            else:
                qw, sc, x, y, in_f, out_f, c = a
                c.flags = (c.flags & FLAG_SPLIT) | (FLAG_PDL if pdl else 0)
                check("b4_gemv_ws", lib.b4_gemv_ws(self.fmt, ctypes.c_void_p(qw.data_ptr()),
                                                   ctypes.c_void_p(sc.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                                   ctypes.c_void_p(y.data_ptr()), in_f, out_f, 1, ctypes.byref(c),
                                                   ctypes.c_void_p(self.ws.data_ptr()), self.ws.numel(), stream))

    def launch_count(self, fused: bool) -> int:
        return len(self.launches(fused))

    def capture(self, pdl: bool, fused: bool = False):
        torch = self.torch
        self.launch_all(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), pdl, fused)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(graph, stream=cs, capture_error_mode="relaxed"):
            self.launch_all(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), pdl, fused)
        torch.cuda.current_stream().wait_stream(cs)
        return graph

    def time_token(self, pdl: bool, fused: bool = False, tokens: int = 20):
        """us per token: the graph (all layers) replayed `tokens` times."""
        torch = self.torch
        graph = self.capture(pdl, fused)
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
