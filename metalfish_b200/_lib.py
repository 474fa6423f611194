"""Loader for the in-tree CUDA library ``libmfb200.so``.

There is no fallback: if the library is missing or fails to load, every
entry point raises. Build it with ``python -c "import __graft_entry__ as g;
g.build()"`` (or ``make -C metalfish_b200/csrc``).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmfb200.so")

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libmfb200.so not built ({LIB_PATH}); the B200 path has no CPU fallback")
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    c_int, c_float, vp = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
    L.mfb200_debug_gemm.restype = c_int
    L.mfb200_debug_gemm.argtypes = [c_int, c_int, c_int, c_int, c_int, vp, vp, vp, c_int, c_int,
                                    vp, c_float, vp, vp, c_float, vp, c_float, c_int, c_int, vp, vp]
    L.mfb200_debug_set_pdl.restype = None
    L.mfb200_debug_set_pdl.argtypes = [c_int]
    L.mfb200_debug_set_gemm_pairs.restype = None
    L.mfb200_debug_set_gemm_pairs.argtypes = [c_int]
    L.mfb200_debug_set_fold_ln.restype = None
    L.mfb200_debug_set_fold_ln.argtypes = [c_int]
    L.mfb200_debug_set_auto_split.restype = None
    L.mfb200_debug_set_auto_split.argtypes = [c_int]
    L.mfb200_debug_gemm_bench.restype = c_int
    L.mfb200_debug_gemm_bench.argtypes = [c_int] * 9 + [ctypes.POINTER(c_float)]
    L.mfb200_debug_gemm_ln.restype = c_int
    L.mfb200_debug_gemm_ln.argtypes = [c_int, c_int, c_int, c_int, vp, vp, vp, vp, c_float, vp, vp,
                                       c_float, vp, vp, vp]
    L.mfb200_debug_gemm_withheld.restype = c_int
    L.mfb200_debug_gemm_withheld.argtypes = [c_int, c_int, c_int, c_int, ctypes.c_ulonglong,
                                             ctypes.POINTER(ctypes.c_uint)]
    L.mfb200_debug_forward_withheld.restype = c_int
    L.mfb200_debug_forward_withheld.argtypes = [vp, c_int, ctypes.c_ulonglong]
    L.mfb200_debug_gemm_trace.restype = c_int
    L.mfb200_debug_gemm_trace.argtypes = [c_int] * 9 + [ctypes.POINTER(c_float),
                                                        ctypes.POINTER(ctypes.c_ulonglong)]
