"""Device generator and device quantizers against the oracle (which the golden
fixtures pin to the reference's Python quantizer)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _dev(n, dtype):
    import torch
    return torch.zeros(n, dtype=dtype, device="cuda")


def test_gen_int8_and_tokens_bit_exact():
    import torch
    from asicfortranai_b200 import _lib
    L = _lib.load()
    n = 1 << 20
    d = _dev(n, torch.int8)
    _lib.check(L.q35_gen_int8_dev(d.data_ptr(), n, 0, 2, None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(d.cpu().numpy(), orc.gen_int8((n,), 0, 2))
    t = _dev(4096, torch.int32)
    _lib.check(L.q35_gen_tokens_dev(t.data_ptr(), 4096, 0, 9, 32000, None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(t.cpu().numpy(), orc.gen_tokens(4096, 0, 9, 32000))


def test_gen_normal_matches_host_libm():
    import torch
    from asicfortranai_b200 import _lib
    L = _lib.load()
    n = 1 << 20
    d = _dev(n, torch.float32)
    _lib.check(L.q35_gen_normal_dev(d.data_ptr(), n, 0, 1, 0.02, None))
    torch.cuda.synchronize()
    g, h = d.cpu().numpy(), orc.gen_normal((n,), 0, 1, 0.02)
    # device and host double-precision log/cos may differ in the last bit; after the
    # rounding to fp32 at most a handful of values differ, each by one fp32 ulp
    diff = g != h
    assert diff.sum() <= n // 10000
    np.testing.assert_allclose(g, h, rtol=2e-7, atol=1e-12)


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("K,N", [(2, 3), (256, 64), (1000, 77), (8192, 128)])
def test_device_quantizer_bit_exact(fmt, K, N):
    import torch
    from asicfortranai_b200 import _lib
    L = _lib.load()
    W = orc.gen_normal((K, N), 5, 1)
    W[:, 0] = 0.5                                   # constant column
    dW = torch.from_numpy(np.ascontiguousarray(W.T)).cuda()   # (N,K) C-order == (K,N) F-order
    wq = _dev(K // 2 * N, torch.int8)
    s = _dev(N, torch.float32)
    o = _dev(N, torch.float32)
    _lib.check(L.q35_quantize_dev(fmt, dW.data_ptr(), wq.data_ptr(), s.data_ptr(), o.data_ptr(), K, N, None))
    torch.cuda.synchronize()
    gq = wq.cpu().numpy().reshape(N, K // 2).T
    if fmt == 0:
        rq, rs, ro = orc.quantize_3p5bit(W)
        np.testing.assert_array_equal(o.cpu().numpy().view(np.uint32), ro.view(np.uint32))
    else:
        rq, rs = orc.quantize_int4(W)
    np.testing.assert_array_equal(gq, rq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_golden_quantizer_on_device(golden):
    import torch
    from asicfortranai_b200 import _lib
    L = _lib.load()
    W = golden["quant_W"]
    K, N = W.shape
    dW = torch.from_numpy(np.ascontiguousarray(W.T)).cuda()
    wq = _dev(K // 2 * N, torch.int8)
    s = _dev(N, torch.float32)
    o = _dev(N, torch.float32)
    _lib.check(L.q35_quantize_dev(0, dW.data_ptr(), wq.data_ptr(), s.data_ptr(), o.data_ptr(), K, N, None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(wq.cpu().numpy().reshape(N, K // 2).T, golden["quant_wq"])
    np.testing.assert_array_equal(s.cpu().numpy(), golden["quant_scales"])
    np.testing.assert_array_equal(o.cpu().numpy(), golden["quant_offsets"])


def test_weights_generate_matches_host_pipeline():
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    import ctypes as C
    L = _lib.load()
    ctx = Context(0)
    K, N = 4096, 96
    h = C.c_void_p()
    _lib.check(L.q35_weights_generate(ctx.h, 0, N, K, 3, 17, 0.02, C.byref(h)))
    qm = QuantizedMatrix.from_handle(ctx, h, K, N, 0)
    W = orc.gen_normal((K, N), 3, 17)
    rq, rs, ro = orc.quantize_3p5bit(W)
    back = qm.download_ref()
    # generator last-bit differences can move a code by one at a rounding boundary
    assert (back != rq).mean() < 1e-4
    A = orc.gen_int8((2, K), 3, 18)
    C_, _ = qm.matmul(A)
    np.testing.assert_array_equal(C_, orc.matmul_3p5bit_awq(A, back, rs, ro))
    qm.close()
    ctx.close()
