"""The tensor-parallel exchange fused with the next RMSNorm, on one GPU: with a one-rank view
the fused kernel must reproduce the separate dequant + residual and RMSNorm kernels bit for
bit (x, the fp32 norm and its int8), over three calls in a row -- one row (batch-1 decode)
and several rows (decode batches up to 64)."""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N", [256, 1024, 4096, 5120, 8192, 28672, 32768])
def test_fused_exchange_norm_matches_separate_kernels(N):
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context
    ctx = Context(0)
    mism = C.c_int32(-1)
    _lib.check(_lib.load().q35_tp_norm_selftest(ctx.h, N, 7 + N, C.byref(mism)), "norm self-test")
    assert mism.value == 0
    ctx.close()


@pytest.mark.parametrize("R,N", [(2, 8192), (3, 5120), (16, 8192), (16, 5120), (64, 4096), (5, 28672), (8, 32768)])
def test_fused_exchange_norm_several_rows(R, N):
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import Context
    ctx = Context(0)
    mism = C.c_int32(-1)
    _lib.check(_lib.load().q35_tp_norm_selftest_rows(ctx.h, R, N, 11 + R + N, C.byref(mism)), "norm self-test")
    assert mism.value == 0
    ctx.close()


def test_norm_selftest_rejects_bad_widths():
    from asicfortranai_b200 import Q35Error, _lib
    from asicfortranai_b200.quantized import Context
    ctx = Context(0)
    mism = C.c_int32(-1)
    for bad in (6, 32772):
        with pytest.raises(Q35Error):
            _lib.check(_lib.load().q35_tp_norm_selftest(ctx.h, bad, 1, C.byref(mism)), "norm self-test")
    for R, N in ((65, 1024), (0, 1024), (40, 8192)):    # beyond 64 rows or 262,144 elements
        with pytest.raises(Q35Error):
            _lib.check(_lib.load().q35_tp_norm_selftest_rows(ctx.h, R, N, 1, C.byref(mism)), "norm self-test")
    ctx.close()
