"""ctypes binding of libb200q8_host.so: seeded synthetic inputs and the CPU thread rule."""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
HOST_LIB = os.path.join(PKG, "libb200q8_host.so")
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(HOST_LIB):
            raise RuntimeError(f"{HOST_LIB} is not built: run __graft_entry__.build()")
        L = ctypes.CDLL(HOST_LIB)
        L.b200q8h_normal_fill.argtypes = [ctypes.c_uint64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t]
        L.b200q8h_normal_fill_many.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_int]
        L.b200q8h_default_threads.argtypes = [ctypes.c_int]
        L.b200q8h_default_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def normal(seed: int, count: int, scale: float = 1.0) -> np.ndarray:
    """`count` draws of the seeded N(0,1) stream (synth::NormalRandomStream semantics), times scale."""
    out = np.empty(count, dtype=np.float32)
    lib().b200q8h_normal_fill(seed, scale, out.ctypes.data, count)
    return out


def normal_many(seeds, scales, outs, threads: int = 0) -> None:
    """Fills each float32 array outs[j] from its own stream seeds[j], in parallel on host threads."""
    n = len(outs)
    s = (ctypes.c_uint64 * n)(*seeds)
    f = (ctypes.c_float * n)(*scales)
    p = (ctypes.c_void_p * n)(*[o.ctypes.data for o in outs])
    c = (ctypes.c_size_t * n)(*[o.size for o in outs])
    lib().b200q8h_normal_fill_many(n, s, f, p, c, threads)


def default_threads(available: int) -> int:
    """The reference's default synthesis thread count, min(n/2, n-1)."""
    return int(lib().b200q8h_default_threads(available))
