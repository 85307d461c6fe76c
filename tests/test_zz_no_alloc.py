"""q35_gemm_dev_noalloc -- the decode matmul for callers that cannot allocate device
memory (real-time loops that must not enter the driver's allocator, processes whose free
HBM is owned by another pool) -- must give the oracle's results and the same results as
q35_gemm_dev, call after call.  Its split-K scratch is a fixed array inside the library
rather than memory allocated per context, and its failure record is read with
q35_gemm_noalloc_device_error.

Kept in its own file, collected last, so a failure here comes after every other test."""

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _case(K, N, M, fmt):
    W = orc.gen_normal((K, N), 41, K + N)
    A = orc.gen_int8((M, K), 43, M)
    if fmt == 0:
        wq, s, o = orc.quantize_3p5bit(W)
        Cref = orc.matmul_3p5bit_awq(A, wq, s, o)
        Yref = orc.dequantize_output_3p5bit(Cref, s, o)
    else:
        (wq, s), o = orc.quantize_int4(W), None
        Cref = orc.matmul_int4_awq(A, wq, s)
        Yref = orc.dequantize_output(Cref, s)
    return A, wq, s, o, Cref, Yref


def _dev(arr, layout):
    """numpy (M, X) -> a device tensor holding it in the given layout."""
    import torch
    from asicfortranai_b200 import _lib
    a = np.asfortranarray(arr) if layout == _lib.Q35_LAYOUT_COLMAJOR else np.ascontiguousarray(arr)
    flat = a.ravel(order="F" if layout == _lib.Q35_LAYOUT_COLMAJOR else "C")
    return torch.from_numpy(flat.copy()).cuda()


def _host(t, M, N, layout):
    from asicfortranai_b200 import _lib
    v = t.cpu().numpy()
    return v.reshape((M, N), order="F" if layout == _lib.Q35_LAYOUT_COLMAJOR else "C")


@pytest.mark.parametrize("fmt,K,N,M,lay", [(0, 8192, 28672, 1, 1), (0, 28672, 8192, 4, 1), (0, 8192, 1024, 16, 1),
                                           (1, 8192, 8192, 2, 1), (0, 258, 33, 3, 1), (0, 8192, 1024, 3, 0),
                                           (1, 1030, 96, 5, 0)])
def test_noalloc_matches_oracle_and_allocating_entry_point(fmt, K, N, M, lay):
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    L = _lib.load()
    ctx = Context(0)
    A, wq, s, o, Cref, Yref = _case(K, N, M, fmt)
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=fmt)
    x = _dev(A, lay)
    C_ref = torch.zeros(M * N, dtype=torch.int32, device="cuda")
    y_ref = torch.zeros(M * N, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    _lib.check(L.q35_gemm_dev(ctx.h, qm.h, x.data_ptr(), M, lay, C_ref.data_ptr(), y_ref.data_ptr(), lay),
               "q35_gemm_dev")
    ctx.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):                         # two calls in a row share the scratch
        C_na = torch.full((M * N,), -7, dtype=torch.int32, device="cuda")
        y_na = torch.full((M * N,), -7.0, dtype=torch.float32, device="cuda")
        st = L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), M, lay, C_na.data_ptr(), y_na.data_ptr(), lay, stream)
        _lib.check(st, "q35_gemm_dev_noalloc")
        assert L.q35_gemm_noalloc_device_error(stream) == 0, _lib.last_error()
        # int32 accumulators: bit-exact against the oracle and the allocating entry point
        np.testing.assert_array_equal(_host(C_na, M, N, lay), Cref, err_msg=f"oracle, call {call}")
        assert torch.equal(C_na, C_ref), f"int32 accumulators differ from q35_gemm_dev on call {call}"
        # dequantized fp32: the path's bar is 1e-5 relative
        np.testing.assert_allclose(_host(y_na, M, N, lay), Yref, rtol=1e-5, atol=0)
        torch.testing.assert_close(y_na, y_ref, rtol=1e-5, atol=0)
    qm.close()
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    L = _lib.load()
    ctx = Context(0)
    _, wq, s, o, _, _ = _case(256, 65536, 1, 0)   # 64 x 65536 partial sums > 1,048,576
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=0)
    x = torch.zeros(64 * 256, dtype=torch.int8, device="cuda")
    y = torch.zeros(64 * 65536, dtype=torch.float32, device="cuda")
    st = L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), 64, _lib.Q35_LAYOUT_ROWMAJOR, None, y.data_ptr(),
                                _lib.Q35_LAYOUT_ROWMAJOR, None)
    assert st == 1 and "exceed the fixed scratch" in _lib.last_error()
    st = L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), 65, _lib.Q35_LAYOUT_ROWMAJOR, None, y.data_ptr(),
                                _lib.Q35_LAYOUT_ROWMAJOR, None)
    assert st == 1 and "M must be in [1,64]" in _lib.last_error()
    qm.close()
    _, wq, s, o, _, _ = _case(2, 65537, 1, 0)     # N above the counter scratch's 65536
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=0)
    st = L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), 1, _lib.Q35_LAYOUT_ROWMAJOR, None, y.data_ptr(),
                                _lib.Q35_LAYOUT_ROWMAJOR, None)
    assert st == 1 and "N above 65536" in _lib.last_error()
    assert L.q35_gemm_noalloc_device_error(None) == 0
    qm.close()
    ctx.close()


def test_noalloc_under_graph_capture():
    """The entry point's main use: one call outside capture (it looks up the scratch
    array's device address), then a call captured into a CUDA graph on a side stream and
    the graph replayed; every replay must write the allocating entry point's results bit
    for bit, with nothing left over from the replay before."""
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    L = _lib.load()
    ctx = Context(0)
    K, N, M, lay = 8192, 1024, 3, _lib.Q35_LAYOUT_ROWMAJOR
    A, wq, s, o, Cref, Yref = _case(K, N, M, 0)
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=0)
    x = _dev(A, lay)
    C_ref = torch.zeros(M * N, dtype=torch.int32, device="cuda")
    y_ref = torch.zeros(M * N, dtype=torch.float32, device="cuda")
    C_na = torch.full((M * N,), -7, dtype=torch.int32, device="cuda")
    y_na = torch.full((M * N,), -7.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    _lib.check(L.q35_gemm_dev(ctx.h, qm.h, x.data_ptr(), M, lay, C_ref.data_ptr(), y_ref.data_ptr(), lay),
               "q35_gemm_dev")
    ctx.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    _lib.check(L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), M, lay, C_na.data_ptr(), y_na.data_ptr(), lay,
                                      side.cuda_stream), "q35_gemm_dev_noalloc, first call")
    side.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side, capture_error_mode="relaxed"):
        st = L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), M, lay, C_na.data_ptr(), y_na.data_ptr(), lay,
                                    side.cuda_stream)
    _lib.check(st, "q35_gemm_dev_noalloc under capture")
    for replay in range(2):
        C_na.fill_(-7)
        y_na.fill_(-7.0)
        g.replay()
        torch.cuda.synchronize()
        assert L.q35_gemm_noalloc_device_error(None) == 0, _lib.last_error()
        np.testing.assert_array_equal(_host(C_na, M, N, lay), Cref, err_msg=f"oracle, replay {replay}")
        assert torch.equal(C_na, C_ref), f"int32 accumulators differ from q35_gemm_dev on replay {replay}"
        np.testing.assert_allclose(_host(y_na, M, N, lay), Yref, rtol=1e-5, atol=0)
        torch.testing.assert_close(y_na, y_ref, rtol=1e-5, atol=0)
    del g
    qm.close()
    ctx.close()
