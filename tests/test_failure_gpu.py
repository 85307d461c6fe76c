"""Failure detection on the GPU without a fault: a bounded wait that nothing satisfies
gives up, the kernel reports Q35_ERR_TIMEOUT, and the context keeps working."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_exchange_wait_gives_up_and_context_survives():
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.matmul_3p5bit_groq import matmul_3p5bit_awq
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    L = _lib.load()
    ctx = Context(0)
    obs = C.c_int32(-1)
    _lib.check(L.q35_tp_wait_selftest(ctx.h, C.byref(obs)), "selftest")
    assert obs.value == 5                           # Q35_ERR_TIMEOUT
    ctx.device_error()                              # the error word was cleared
    # the same context still computes correctly
    K, N = 512, 96
    W = orc.gen_normal((K, N), 1, 2, 0.02)
    wq, s, o = orc.quantize_3p5bit(W)
    A = orc.gen_int8((3, K), 1, 3)
    m = QuantizedMatrix(ctx, wq, s, o)
    Cg, _ = m.matmul(A)
    np.testing.assert_array_equal(Cg, orc.matmul_3p5bit_awq(A, wq, s, o))
    m.close()
    ctx.close()
    # the drop-in path (default context) too
    np.testing.assert_array_equal(matmul_3p5bit_awq(A, wq, s, o, 3, N, K), orc.matmul_3p5bit_awq(A, wq, s, o))
