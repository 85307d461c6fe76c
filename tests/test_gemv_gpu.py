"""Parity of the CUDA-core matmul engine (dp4a GEMV, through the C ABI) with the CPU
oracle; the module's context pins that engine for every row count (the tensor-core
engine has its own file, test_mma_gpu.py).

int32 accumulators must be bit-exact; the dequantized fp32 output must equal the
oracle's binary32 (C + offset) * scale exactly as well (same three roundings), which is
tighter than the 1e-5 relative bound the path requires."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

RTOL = 1e-5   # dequantized fp32 bar; the kernels in fact match bit for bit


@pytest.fixture(scope="module")
def ctx():
    from asicfortranai_b200.quantized import PATH_CUDA_CORES, Context
    c = Context(0)
    c.set_gemm_path(PATH_CUDA_CORES)
    yield c
    c.close()


def make_case(K, N, M, seed, fmt):
    W = orc.gen_normal((K, N), seed, 1)
    A = orc.gen_int8((M, K), seed, 2)
    if fmt == 0:
        wq, s, o = orc.quantize_3p5bit(W)
        C_ = orc.matmul_3p5bit_awq(A, wq, s, o)
        Y = orc.dequantize_output_3p5bit(C_, s, o)
    else:
        wq, s = orc.quantize_int4(W)
        o = None
        C_ = orc.matmul_int4_awq(A, wq, s)
        Y = orc.dequantize_output(C_, s)
    return A, wq, s, o, C_, Y


SHAPES = [(2, 1), (16, 8), (30, 5), (256, 32), (258, 33), (512, 100), (1000, 257),
          (2048, 300), (8192, 64), (5120, 96)]


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 8, 13, 64])
def test_cached_matmul_matches_oracle(ctx, fmt, K, N, M):
    from asicfortranai_b200.quantized import QuantizedMatrix
    A, wq, s, o, Cref, Yref = make_case(K, N, M, 1000 + K + N + M, fmt)
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=fmt)
    C_, Y = qm.matmul(A)
    np.testing.assert_array_equal(C_, Cref)
    np.testing.assert_array_equal(Y.view(np.uint32), Yref.view(np.uint32))
    # second call: split-K workspace and tickets must have been left clean
    C2, Y2 = qm.matmul(A)
    np.testing.assert_array_equal(C2, Cref)
    qm.close()


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("K,N", [(16, 8), (258, 33), (1000, 257), (8192, 1024)])
def test_repack_round_trip(ctx, fmt, K, N):
    from asicfortranai_b200.quantized import QuantizedMatrix
    _, wq, s, o, _, _ = make_case(K, N, 1, 7, fmt)
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=fmt)
    back = qm.download_ref()
    ref = wq if fmt == 1 else (wq.view(np.uint8) & 0x7F).view(np.int8)
    np.testing.assert_array_equal(back, ref)


def test_msb_ignored_on_device(ctx):
    from asicfortranai_b200.quantized import QuantizedMatrix
    A, wq, s, o, Cref, _ = make_case(512, 40, 3, 11, 0)
    wq_msb = (wq.view(np.uint8) | 0x80).view(np.int8)
    C_, _ = QuantizedMatrix(ctx, np.asfortranarray(wq_msb), s, o).matmul(A)
    np.testing.assert_array_equal(C_, Cref)


def test_extreme_activations_and_codes(ctx):
    """Largest |C|: all activations -127 and every code at its extreme."""
    from asicfortranai_b200.quantized import QuantizedMatrix
    K, N = 28672, 64
    for byte, act in ((0x40, -127), (0x3B, 127), (0x44, 127), (0x00, -127)):
        wq = np.full((K // 2, N), byte, np.int8, order="F")
        A = np.full((2, K), act, np.int8, order="F")
        s = np.ones(N, np.float32)
        o = np.zeros(N, np.float32)
        C_, _ = QuantizedMatrix(ctx, wq, s, o).matmul(A)
        np.testing.assert_array_equal(C_, orc.matmul_3p5bit_awq(A, wq, s, o))


@pytest.mark.parametrize("K,N", [(8192, 8192), (8192, 1024), (8192, 28672), (28672, 8192)])
def test_full_size_projection_shapes(ctx, K, N):
    """LLaMA-70B projection shapes at full size: rows 0 and M-1 against the oracle for
    M in {1,4,16,64}, the other rows through linearity C(a+b) = C(a) + C(b)."""
    from asicfortranai_b200.quantized import QuantizedMatrix
    W = orc.gen_normal((K, N), 0, 3)
    wq, s, o = orc.quantize_3p5bit(W)
    del W
    qm = QuantizedMatrix(ctx, wq, s, o)
    for M in (1, 4, 16, 64):
        A = orc.gen_int8((M, K), M, 4)
        C_, Y = qm.matmul(A)
        np.testing.assert_array_equal(C_[:1], orc.matmul_3p5bit_awq(A[:1], wq, s, o))
        if M > 1:
            a = (A // 2).astype(np.int8)
            b = (A - a).astype(np.int8)
            Ca, _ = qm.matmul(np.asfortranarray(a))
            Cb, _ = qm.matmul(np.asfortranarray(b))
            np.testing.assert_array_equal(C_, Ca + Cb)
            np.testing.assert_array_equal(C_[-1:], orc.matmul_3p5bit_awq(A[-1:], wq, s, o))
        Yref = orc.dequantize_output_3p5bit(C_, s, o)
        np.testing.assert_array_equal(Y.view(np.uint32), Yref.view(np.uint32))
    qm.close()


def test_golden_fixtures_on_gpu(ctx, golden):
    from asicfortranai_b200.quantized import QuantizedMatrix
    for ci in range(len(golden["mm_cases"])):
        A, wq = golden[f"mm{ci}_A"], golden[f"mm{ci}_wq"]
        sc, of = golden[f"mm{ci}_scales"], golden[f"mm{ci}_offsets"]
        C_, Y = QuantizedMatrix(ctx, np.asfortranarray(wq), sc, of).matmul(np.asfortranarray(A))
        np.testing.assert_array_equal(C_, golden[f"mm{ci}_C"])
        np.testing.assert_allclose(Y, golden[f"mm{ci}_Y"], rtol=RTOL, atol=1e-6)


def test_dropin_reference_signatures():
    from asicfortranai_b200 import matmul_3p5bit_groq as m35, matmul_int4_groq as m4
    A, wq, s, o, Cref, Yref = make_case(1024, 77, 5, 21, 0)
    C_ = m35.matmul_3p5bit_awq(A, wq, s, o, 5, 77, 1024)
    np.testing.assert_array_equal(C_, Cref)
    Y = m35.dequantize_output_3p5bit(C_, s, o, 5, 77)
    np.testing.assert_array_equal(Y.view(np.uint32), Yref.view(np.uint32))
    A, wq, s, _, Cref, Yref = make_case(1024, 77, 5, 22, 1)
    C_ = m4.matmul_int4_awq(A, wq, s, 5, 77, 1024)
    np.testing.assert_array_equal(C_, Cref)
    Y = m4.dequantize_output(C_, s, 5, 77)
    np.testing.assert_array_equal(Y.view(np.uint32), Yref.view(np.uint32))
    Yf = m4.matmul_int4_cuda_fused(A, wq, s, 5, 77, 1024)
    np.testing.assert_array_equal(Yf.view(np.uint32), Yref.view(np.uint32))


def test_dropin_rejects_bad_sizes():
    from asicfortranai_b200 import _lib
    L = _lib.load()
    A = np.zeros(6, np.int8)
    assert L.q35_matmul_3p5bit_awq(A.ctypes.data, A.ctypes.data, A.ctypes.data, A.ctypes.data,
                                   A.ctypes.data, 1, 1, 3) == 1
    for M in (-1, 65537):       # rows outside [0, 65536] (0 rows: an empty call, no work)
        assert L.q35_matmul_3p5bit_awq(A.ctypes.data, A.ctypes.data, A.ctypes.data, A.ctypes.data,
                                       A.ctypes.data, M, 1, 2) == 1
    assert L.q35_matmul_3p5bit_awq(A.ctypes.data, A.ctypes.data, A.ctypes.data, A.ctypes.data,
                                   A.ctypes.data, 1, 1, 131074) == 1     # K above 131072


def test_device_pointer_layouts(ctx):
    import torch
    from asicfortranai_b200.quantized import QuantizedMatrix
    K, N, M = 2048, 300, 6
    A, wq, s, o, Cref, Yref = make_case(K, N, M, 31, 0)
    qm = QuantizedMatrix(ctx, wq, s, o)
    xr = torch.from_numpy(np.ascontiguousarray(A)).cuda()          # row-major (M,K)
    Cd = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    Yd = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    qm.gemm_dev(xr.data_ptr(), M, Cd.data_ptr(), Yd.data_ptr())
    ctx.synchronize()
    np.testing.assert_array_equal(Cd.cpu().numpy(), Cref)
    np.testing.assert_array_equal(Yd.cpu().numpy().view(np.uint32), np.ascontiguousarray(Yref).view(np.uint32))
    # column-major input, output only y
    from asicfortranai_b200 import _lib
    xc = torch.from_numpy(np.ascontiguousarray(A.T)).cuda()        # (K,M) == col-major (M,K)
    Yc = torch.zeros((N, M), dtype=torch.float32, device="cuda")   # col-major (M,N)
    torch.cuda.synchronize()
    qm.gemm_dev(xc.data_ptr(), M, None, Yc.data_ptr(), _lib.Q35_LAYOUT_COLMAJOR, _lib.Q35_LAYOUT_COLMAJOR)
    ctx.synchronize()
    np.testing.assert_array_equal(Yc.cpu().numpy().T.view(np.uint32), np.ascontiguousarray(Yref).view(np.uint32))


# the LLaMA-70B layer's shards under tensor parallelism at 2, 4 and 8 GPUs (q/k/v/gate/up
# split by columns, o/down by rows): few column groups, so the per-group launch splits
# each column group's k-blocks over the CTAs of a cluster
SHARDS = sorted({(8192, 8192 // t) for t in (2, 4, 8)} | {(8192, 1024 // t) for t in (2, 4, 8)} |
                {(8192, 28672 // t) for t in (2, 4, 8)} | {(8192 // t, 8192) for t in (2, 4, 8)} |
                {(28672 // t, 8192) for t in (2, 4, 8)} | {(8192, 1024)})


@pytest.mark.parametrize("K,N", SHARDS)
def test_tensor_parallel_shard_shapes(ctx, K, N):
    from asicfortranai_b200.quantized import QuantizedMatrix
    for fmt in (0, 1):
        A, wq, s, o, Cref, Yref = make_case(K, N, 4, 300 + K + N, fmt)
        qm = QuantizedMatrix(ctx, wq, s, o, fmt=fmt)
        for M in (1, 2, 4):
            for _ in range(2):      # twice: the cluster's shared-memory slots are reused
                C_, Y = qm.matmul(np.asfortranarray(A[:M]))
                np.testing.assert_array_equal(C_, Cref[:M])
                np.testing.assert_array_equal(Y.view(np.uint32), np.ascontiguousarray(Yref[:M]).view(np.uint32))
        qm.close()
