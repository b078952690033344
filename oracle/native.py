"""ctypes access to the reference's own C++ CPU routines (``_ref/libkqref.so``).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). The library is built
by ``oracle/Makefile`` from kernelevalplus-main/include/{quantize.h,
gemm_reference.h} and wraps, unchanged:

    quantize_row_q8_1_ref   include/quantize.h:165-193
    gemm_w4a8_reference     include/gemm_reference.h:175-222
    gemm_w8a8_reference     include/gemm_reference.h:233-267

The reference C++ path accumulates in fp32 per output and quantises with
x * (1/d) and roundf, so its bytes and outputs differ in the last bits from
the Python reference (quantize.py uses x / d and round-half-even); parity is
pinned to the Python reference, and this library is the timed CPU baseline.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(_HERE, "_ref", "libkqref.so")
_lib = None


def available() -> bool:
    return os.path.exists(REF_LIB)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{REF_LIB} not built (make -C oracle ref)")
        L = ctypes.CDLL(REF_LIB)
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.kqref_quantize_q8_1.argtypes = [vp, vp, i, i, i]
        L.kqref_gemm_w4a8.argtypes = [vp, vp, vp, i, i, i, i]
        L.kqref_gemm_w8a8.argtypes = [vp, vp, vp, i, i, i, i]
        for f in (L.kqref_quantize_q8_1, L.kqref_gemm_w4a8, L.kqref_gemm_w8a8):
            f.restype = i
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def quantize_q8_1(x: np.ndarray, threads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    out = np.empty((M, K // 32, 36), dtype=np.uint8)
    assert lib().kqref_quantize_q8_1(_ptr(x), _ptr(out), M, K, threads) == 0
    return out


def gemm(wtype: str, w: np.ndarray, a_q8_1: np.ndarray, M: int, N: int, K: int, threads: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    a = np.ascontiguousarray(a_q8_1, dtype=np.uint8)
    c = np.empty((M, N), dtype=np.float32)
    f = {"q4_0": lib().kqref_gemm_w4a8, "q8_0": lib().kqref_gemm_w8a8}[wtype]
    assert f(_ptr(a), _ptr(w), _ptr(c), M, N, K, threads) == 0
    return c
