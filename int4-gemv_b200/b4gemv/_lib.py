"""ctypes binding of libb4gemv.so, the C ABI declared in include/b4gemv.h.

The library is built in-tree (``make -C int4-gemv_b200``) and loaded from
``int4-gemv_b200/lib/libb4gemv.so``.  There is no fallback: if the library is
missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_ROOT, "lib", "libb4gemv.so")

FMT_INT4_G128 = 0
FMT_NF4_B64 = 1
GROUP = 128
NF4_BLOCK = 64
FLAG_PDL = 1
FLAG_SPLIT = 2
FLAG_X_SWIGLU = 4   # b4_tp_gemv_p2p_ex: x = fp16(silu(gate) * up) of fp32 [gate | up]
FLAG_KSLICE = 8     # b4_gemv_ws, batch 2..16: column slices of x_tile columns, summed by a second launch
ENGINE_AUTO = -1
ENGINE_FMA = 0
ENGINE_MMA = 1
ENGINE_MMA_TMA = 2
ENGINE_FMA_TMA = 3      # retired: rejected
ENGINE_MMA_LEAN = 4     # retired: rejected
ENGINE_MMA_LEAN_ASYNC = 5
ENGINE_FMA_LEAN = 6
ENGINE_MMA_NF4 = 7
ENGINE_NF4_XTAB = 8
XTAB_WORKSPACE_BYTES = 256


class GemvConfig(ctypes.Structure):
    """b4_gemv_config (include/b4gemv.h)."""

    _fields_ = [
        ("vec_words", ctypes.c_int),
        ("rows_per_warp", ctypes.c_int),
        ("warps_k", ctypes.c_int),
        ("row_groups", ctypes.c_int),
        ("batch_tile", ctypes.c_int),
        ("nf4_lut", ctypes.c_int),
        ("x_tile", ctypes.c_int),
        ("flags", ctypes.c_int),
        ("engine", ctypes.c_int),
        ("stages", ctypes.c_int),
        ("stage_groups", ctypes.c_int),
        ("tile_rows", ctypes.c_int),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}

    @classmethod
    def from_dict(cls, d: dict) -> "GemvConfig":
        c = cls()
        for name, _ in cls._fields_:
            setattr(c, name, int(d.get(name, 0)))
        return c


class GemvSegment(ctypes.Structure):
    """b4_gemv_segment (include/b4gemv.h)."""

    _fields_ = [
        ("qw", ctypes.c_void_p),
        ("scale", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("out_f", ctypes.c_int),
    ]


MAX_SEGMENTS = 4

_P = ctypes.c_void_p
_I = ctypes.c_int

# name -> (restype, argtypes); every symbol of include/b4gemv.h
SIGNATURES = {
    "b4_gemv_int4_g128": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "b4_gemv_nf4_b64": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "b4_gemv_default_config": (_I, [_I, _I, _I, _I, ctypes.POINTER(GemvConfig)]),
    "b4_gemv_ex": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, ctypes.POINTER(GemvConfig), _P]),
    "b4_gemv_workspace_size": (_I, [_I, _I, _I, _I, ctypes.POINTER(GemvConfig), ctypes.POINTER(ctypes.c_size_t)]),
    "b4_gemv_default_config_ws": (_I, [_I, _I, _I, _I, ctypes.POINTER(GemvConfig)]),
    "b4_gemv_ws": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, ctypes.POINTER(GemvConfig), _P, ctypes.c_size_t, _P]),
    "b4_gemv_split_noalloc": (_I, [_I, _P, _P, _P, _P, _I, _I, ctypes.POINTER(GemvConfig), _P]),
    "b4_gemv_nf4_b64_block_per_row": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "b4_gemv_multi": (_I, [_I, ctypes.POINTER(GemvSegment), _I, _P, _I, _I, ctypes.POINTER(GemvConfig), _P]),
    "b4_gemv_multi_default_config": (_I, [_I, ctypes.POINTER(GemvSegment), _I, _I, _I,
                                          ctypes.POINTER(GemvConfig)]),
    "b4_gemv_multi_default_config_ws": (_I, [_I, ctypes.POINTER(GemvSegment), _I, _I, _I,
                                             ctypes.POINTER(GemvConfig)]),
    "b4_gemv_multi_ws": (_I, [_I, ctypes.POINTER(GemvSegment), _I, _P, _I, _I, ctypes.POINTER(GemvConfig), _P,
                              ctypes.c_size_t, _P]),
    "b4_dequant_int4_g128": (_I, [_P, _P, _P, _I, _I, _P]),
    "b4_dequant_nf4_b64": (_I, [_P, _P, _P, _I, _I, _P]),
    "b4_unpack_codes": (_I, [_P, _P, _I, _I, _P]),
    "b4_repack_bnb_nf4": (_I, [_P, _P, _I, _I, _P]),
    "b4_quantise_int4_g128": (_I, [_P, _I, _I, _P, _P, _P, _I]),
    "b4_quantise_nf4_b64": (_I, [_P, _I, _I, _P, _P, _P, _I]),
    "b4_quantise_int4_g128_device": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "b4_quantise_nf4_b64_device": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "b4_empty_launch": (_I, [_P]),
    "b4_nccl_get_unique_id": (_I, [_P]),
    "b4_nccl_comm_init": (_I, [ctypes.POINTER(ctypes.c_void_p), _I, _P, _I]),
    "b4_nccl_comm_destroy": (_I, [_P]),
    "b4_nccl_wait": (_I, [_P, _P, _I]),
    "b4_shard_columns": (_I, [_I, _P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "b4_tp_gemv_allreduce": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "b4_tp_gemv_allreduce_ws": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, _P, ctypes.c_size_t, _P, _P]),
    "b4_p2p_create": (_I, [_I, _I, _I, ctypes.POINTER(ctypes.c_void_p)]),
    "b4_p2p_ipc_handle": (_I, [_P, _P]),
    "b4_p2p_open_peer": (_I, [_P, _I, _P]),
    "b4_p2p_status": (_I, [_P, _I]),
    "b4_p2p_destroy": (_I, [_P]),
    "b4_tp_gemv_p2p": (_I, [_I, _P, _P, _P, _P, _I, _I, _P, _I, _P]),
    "b4_tp_gemv_p2p_ex": (_I, [_I, _P, _P, _P, _P, _P, _I, _I, _P, _I, _P]),
    "b4_swiglu_f16": (_I, [_P, _P, _P, ctypes.c_longlong, _P]),
    "b4_cast_f16": (_I, [_P, _P, ctypes.c_longlong, _P]),
    "b4_nccl_error_string": (ctypes.c_char_p, [_I]),
    "b4_device_error": (_I, [_I]),
    "b4_status_string": (ctypes.c_char_p, [_I]),
    "b4_abi_version": (_I, []),
}

_lib = None


def load() -> ctypes.CDLL:
    """Loads (once) and returns libb4gemv.so with every signature declared."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library first "
            "(make -C int4-gemv_b200, or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class B4Error(RuntimeError):
    """A non-zero status (a cudaError_t value) from the C ABI."""

    def __init__(self, fn: str, status: int):
        msg = load().b4_status_string(status)
        super().__init__(f"{fn} failed: status {status} ({msg.decode() if msg else '?'})")
        self.status = status


def check(fn: str, status: int) -> None:
    if status != 0:
        raise B4Error(fn, status)
