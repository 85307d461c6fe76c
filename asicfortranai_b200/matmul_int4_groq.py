"""Host mirror of the reference module ``matmul_int4_groq`` (matmul_int4_groq.f90) and
of the GPU backends with the same contract (matmul_cuda_fortran.cuf,
matmul_openacc.f90, matmul_cublas.f90): numpy arrays in Fortran layout, GPU work
through libq35.so."""
from __future__ import annotations

import numpy as np

from . import _lib
from .matmul_3p5bit_groq import _f


def matmul_int4_awq(A, W_Q, W_scales, M, N, K_dim):
    """matmul_int4_groq.f90:19-54: int8 A(M,K) x INT4 W_Q(K/2,N) -> int32 C(M,N)."""
    L = _lib.load()
    A = _f(A, np.int8, (M, K_dim))
    W_Q = _f(W_Q, np.int8, (K_dim // 2, N))
    s = _f(W_scales, np.float32, (N,))
    C = np.zeros((M, N), np.int32, order="F")
    _lib.check(L.q35_matmul_int4_awq(A.ctypes.data, W_Q.ctypes.data, s.ctypes.data, C.ctypes.data,
                                     M, N, K_dim), "matmul_int4_awq")
    return C


def dequantize_output(C, W_scales, M, N):
    """matmul_int4_groq.f90:58-69: Out = real(C) * W_scales."""
    L = _lib.load()
    C = _f(C, np.int32, (M, N))
    s = _f(W_scales, np.float32, (N,))
    Out = np.zeros((M, N), np.float32, order="F")
    _lib.check(L.q35_dequantize_output(C.ctypes.data, s.ctypes.data, Out.ctypes.data, M, N),
               "dequantize_output")
    return Out


def matmul_int4_cuda_fused(A, W_Q, W_scales, M, N, K):
    """matmul_cuda_fortran.cuf:233-276 / matmul_int4_cublas (matmul_cublas.f90:222-274):
    dequantized fp32 Out(M,N) in one call.  (The reference CUDA-Fortran kernel folds the
    scale into an fp32 accumulation; this one accumulates exactly in int32 first.)"""
    L = _lib.load()
    A = _f(A, np.int8, (M, K))
    W_Q = _f(W_Q, np.int8, (K // 2, N))
    s = _f(W_scales, np.float32, (N,))
    Out = np.zeros((M, N), np.float32, order="F")
    _lib.check(L.q35_matmul_int4_fused(A.ctypes.data, W_Q.ctypes.data, s.ctypes.data,
                                       Out.ctypes.data, M, N, K), "matmul_int4_cuda_fused")
    return Out
