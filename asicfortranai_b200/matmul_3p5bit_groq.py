"""Host mirror of the reference module ``matmul_3p5bit_groq``
(matmul_3p5bit_dynamic.f90): same procedure names, argument order and meaning, over
numpy arrays in the reference's Fortran layout.  The work runs on the GPU through
libq35.so.

    C   = matmul_3p5bit_awq(A, W_Q, W_scales, W_offsets, M, N, K)   # int32 (M,N)
    Out = dequantize_output_3p5bit(C, W_scales, W_offsets, M, N)    # float32 (M,N)
"""
from __future__ import annotations

import numpy as np

from . import _lib


def _f(a, dt, shape):
    a = np.asfortranarray(a, dtype=dt)
    if a.shape != shape:
        raise ValueError(f"expected shape {shape}, got {a.shape}")
    return a


def matmul_3p5bit_awq(A, W_Q, W_scales, W_offsets, M, N, K):
    """matmul_3p5bit_dynamic.f90:28-65: int8 A(M,K) x 3.5-bit W_Q(K/2,N) -> int32 C(M,N)."""
    L = _lib.load()
    A = _f(A, np.int8, (M, K))
    W_Q = _f(W_Q, np.int8, (K // 2, N))
    s = _f(W_scales, np.float32, (N,))
    o = _f(W_offsets, np.float32, (N,))
    C = np.zeros((M, N), np.int32, order="F")
    _lib.check(L.q35_matmul_3p5bit_awq(A.ctypes.data, W_Q.ctypes.data, s.ctypes.data,
                                       o.ctypes.data, C.ctypes.data, M, N, K), "matmul_3p5bit_awq")
    return C


def dequantize_output_3p5bit(C, W_scales, W_offsets, M, N):
    """matmul_3p5bit_dynamic.f90:69-82: Out = (real(C) + W_offsets) * W_scales."""
    L = _lib.load()
    C = _f(C, np.int32, (M, N))
    s = _f(W_scales, np.float32, (N,))
    o = _f(W_offsets, np.float32, (N,))
    Out = np.zeros((M, N), np.float32, order="F")
    _lib.check(L.q35_dequantize_output_3p5bit(C.ctypes.data, s.ctypes.data, o.ctypes.data,
                                              Out.ctypes.data, M, N), "dequantize_output_3p5bit")
    return Out
