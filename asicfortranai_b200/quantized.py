"""Device-resident quantized matrices (the cached path of the reference's cuBLAS
backend, matmul_cublas.f90:175-217 / :279-325) over libq35.so."""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import _lib


PATH_AUTO, PATH_CUDA_CORES, PATH_TENSOR_CORES = 0, 1, 2


class Context:
    """A device and a CUDA stream (q35_ctx).  ``stream`` is a cudaStream_t handle (int)
    or None for a stream owned by the context."""

    def __init__(self, device: int = 0, stream: int | None = None):
        L = _lib.load()
        h = C.c_void_p()
        _lib.check(L.q35_ctx_create(device, stream, C.byref(h)), "q35_ctx_create")
        self.h = h
        self.device = device
        self._children = weakref.WeakSet()   # objects living on this context

    def adopt(self, obj):
        """Register an object (matrix, graph, model) that must be closed before the context."""
        self._children.add(obj)

    @property
    def stream(self) -> int:
        return _lib.load().q35_ctx_stream(self.h) or 0

    def synchronize(self):
        _lib.check(_lib.load().q35_ctx_synchronize(self.h), "q35_ctx_synchronize")

    def set_gemm_path(self, path: int):
        """PATH_AUTO (CUDA cores up to 4 rows, tensor cores from 5), PATH_CUDA_CORES or
        PATH_TENSOR_CORES for the matmuls issued on this context."""
        _lib.check(_lib.load().q35_ctx_set_gemm_path(self.h, path), "q35_ctx_set_gemm_path")

    def device_error(self):
        """Raise if a kernel on this context recorded a bounded wait that gave up."""
        _lib.check(_lib.load().q35_ctx_device_error(self.h), "device error")

    def capture(self, fn):
        """Capture the library calls made by fn() on this context's stream into a
        CUDA graph; returns a Graph.  fn must have run once before (no allocation
        may happen while capturing)."""
        L = _lib.load()
        _lib.check(L.q35_ctx_capture_begin(self.h), "capture_begin")
        try:
            fn()
        finally:
            g = C.c_void_p()
            st = L.q35_ctx_capture_end(self.h, C.byref(g))
        _lib.check(st, "capture_end")
        return Graph(self, g)

    def close(self):
        if self.h:
            # communicators last: the models' decode graphs hold their collectives
            for ch in sorted(self._children, key=lambda c: getattr(c, "_close_last", False)):
                try:
                    ch.close()
                except Exception:
                    pass
            _lib.load().q35_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Graph:
    """An instantiated CUDA graph replayed on its context's stream."""

    def __init__(self, ctx: Context, h):
        self.ctx, self.h = ctx, h
        ctx.adopt(self)

    def launch(self):
        _lib.check(_lib.load().q35_graph_launch(self.h, self.ctx.h), "graph_launch")

    def close(self):
        if self.h:
            _lib.load().q35_graph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QuantizedMatrix:
    """One W_Q(K/2,N) matrix (3.5-bit with offsets, or INT4) resident on the device."""

    def __init__(self, ctx: Context, W_Q, scales, offsets=None, fmt: int | None = None):
        L = _lib.load()
        if fmt is None:
            fmt = _lib.Q35_FMT_3P5BIT if offsets is not None else _lib.Q35_FMT_INT4
        W_Q = np.asfortranarray(W_Q, np.int8)
        KH, N = W_Q.shape
        self.K, self.N, self.fmt, self.ctx = 2 * KH, N, fmt, ctx
        s = np.ascontiguousarray(scales, np.float32)
        o = np.ascontiguousarray(offsets, np.float32) if offsets is not None else None
        h = C.c_void_p()
        _lib.check(L.q35_weights_upload(ctx.h, fmt, W_Q.ctypes.data, s.ctypes.data,
                                        o.ctypes.data if o is not None else None, N, self.K, 0,
                                        C.byref(h)), "q35_weights_upload")
        self.h = h
        ctx.adopt(self)

    @classmethod
    def from_handle(cls, ctx: Context, h, K: int, N: int, fmt: int):
        qm = cls.__new__(cls)
        qm.h, qm.K, qm.N, qm.fmt, qm.ctx = h, K, N, fmt, ctx
        ctx.adopt(qm)
        return qm

    @property
    def device_bytes(self) -> int:
        return int(_lib.load().q35_weights_device_bytes(self.h))

    def download_ref(self):
        out = np.zeros((self.K // 2, self.N), np.int8, order="F")
        _lib.check(_lib.load().q35_weights_download_ref(self.ctx.h, self.h, out.ctypes.data),
                   "q35_weights_download_ref")
        return out

    def gemm_dev(self, x_ptr: int, M: int, C_ptr: int | None, y_ptr: int | None,
                 x_layout: int = _lib.Q35_LAYOUT_ROWMAJOR, out_layout: int = _lib.Q35_LAYOUT_ROWMAJOR):
        """Asynchronous device matmul on the context's stream (raw device pointers)."""
        _lib.check(_lib.load().q35_gemm_dev(self.ctx.h, self.h, x_ptr, M, x_layout, C_ptr, y_ptr,
                                            out_layout), "q35_gemm_dev")

    def matmul(self, A, want_C=True, want_out=True):
        """Host arrays in, host arrays out (Fortran layout), synchronous."""
        A = np.asfortranarray(A, np.int8)
        M = A.shape[0]
        Cm = np.zeros((M, self.N), np.int32, order="F") if want_C else None
        Out = np.zeros((M, self.N), np.float32, order="F") if want_out else None
        _lib.check(_lib.load().q35_matmul_cached(self.ctx.h, self.h, A.ctypes.data, M,
                                                 Cm.ctypes.data if want_C else None,
                                                 Out.ctypes.data if want_out else None),
                   "q35_matmul_cached")
        return Cm, Out

    def close(self):
        if self.h:
            _lib.load().q35_weights_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
