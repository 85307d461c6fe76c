"""q35_gemm_dev_noalloc -- the decode matmul for callers that cannot allocate device
memory (graph capture, allocator-free real-time loops, HBM owned by another pool) --
must give the same results as q35_gemm_dev, call after call.  Its split-K scratch is a
fixed array inside the library rather than memory allocated per context.

Kept in its own file, collected last, so a failure here comes after every other test."""

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _weights(ctx, K, N, fmt):
    from asicfortranai_b200.quantized import QuantizedMatrix
    W = orc.gen_normal((K, N), 41, K + N)
    if fmt == 0:
        wq, s, o = orc.quantize_3p5bit(W)
    else:
        (wq, s), o = orc.quantize_int4(W), None
    return QuantizedMatrix(ctx, wq, s, o, fmt=fmt)


@pytest.mark.parametrize("fmt,K,N,M", [(0, 8192, 28672, 1), (0, 28672, 8192, 4), (0, 8192, 1024, 16),
                                       (1, 8192, 8192, 2), (0, 258, 33, 3)])
def test_noalloc_matches_allocating_entry_point(fmt, K, N, M):
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context
    L = _lib.load()
    ctx = Context(0)
    qm = _weights(ctx, K, N, fmt)
    x = torch.from_numpy(np.ascontiguousarray(orc.gen_int8((M, K), 43, M))).cuda()
    C_ref = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    y_ref = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    qm.gemm_dev(x.data_ptr(), M, C_ref.data_ptr(), y_ref.data_ptr())
    ctx.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):                         # two calls in a row share the scratch
        C_na = torch.full((M, N), -7, dtype=torch.int32, device="cuda")
        y_na = torch.full((M, N), -7.0, dtype=torch.float32, device="cuda")
        st = L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), M, _lib.Q35_LAYOUT_ROWMAJOR, C_na.data_ptr(),
                                    y_na.data_ptr(), _lib.Q35_LAYOUT_ROWMAJOR, stream)
        _lib.check(st, "q35_gemm_dev_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(C_na, C_ref), f"int32 accumulators differ on call {call}"
        # the path's fp32 bar is 1e-5 relative; the two entry points run the same kernel
        torch.testing.assert_close(y_na, y_ref, rtol=1e-5, atol=0)
    qm.close()
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context
    L = _lib.load()
    ctx = Context(0)
    qm = _weights(ctx, 256, 65536, 0)             # 64 x 65536 partial sums > 1,048,576
    x = torch.zeros(64 * 256, dtype=torch.int8, device="cuda")
    y = torch.zeros(64 * 65536, dtype=torch.float32, device="cuda")
    st = L.q35_gemm_dev_noalloc(qm.h, x.data_ptr(), 64, _lib.Q35_LAYOUT_ROWMAJOR, None, y.data_ptr(),
                                _lib.Q35_LAYOUT_ROWMAJOR, None)
    assert st == 1 and "exceed the fixed scratch" in _lib.last_error()
    qm.close()
    ctx.close()
