"""The tensor-core engine (tcgen05 kind::i8, q35_mma.cu) against the CPU oracle and
against the CUDA-core engine: int32 accumulators and dequantized outputs bit-exact, on
ragged shapes, every row count class (one tile row, several row tiles, split tiles),
both activation layouts, the LLaMA-70B projection shapes at the sweep's batches and the
prefill GEMMs (M=2048)."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.test_gemv_gpu import make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from asicfortranai_b200.quantized import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture
def tensor_path(ctx):
    from asicfortranai_b200.quantized import PATH_AUTO, PATH_TENSOR_CORES
    ctx.set_gemm_path(PATH_TENSOR_CORES)
    yield ctx
    ctx.set_gemm_path(PATH_AUTO)


SHAPES = [(256, 32), (258, 33), (512, 100), (1000, 257), (2048, 300), (8192, 64), (5120, 96), (1024, 1000)]


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 5, 16, 17, 64, 100, 257])
def test_tensor_engine_matches_oracle(tensor_path, fmt, K, N, M):
    from asicfortranai_b200.quantized import QuantizedMatrix
    ctx = tensor_path
    A, wq, s, o, Cref, Yref = make_case(K, N, M, 3000 + K + N + M, fmt)
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=fmt)
    C_, Y = qm.matmul(A)
    np.testing.assert_array_equal(C_, Cref)
    np.testing.assert_array_equal(Y.view(np.uint32), Yref.view(np.uint32))
    C2, _ = qm.matmul(A)          # split slots and tickets were left clean
    np.testing.assert_array_equal(C2, Cref)
    ctx.device_error()
    qm.close()


def _device_case(ctx, fmt, K, N, M, seed):
    import ctypes as C
    import torch
    from asicfortranai_b200 import _lib
    from asicfortranai_b200.quantized import QuantizedMatrix
    L = _lib.load()
    h = C.c_void_p()
    _lib.check(L.q35_weights_generate(ctx.h, fmt, N, K, seed, 77, 0.02, C.byref(h)), "weights_generate")
    qm = QuantizedMatrix.from_handle(ctx, h, K, N, fmt)
    x = torch.empty(M * K, dtype=torch.int8, device="cuda")
    torch.cuda.synchronize()      # the library's streams are not ordered after torch's
    _lib.check(L.q35_gen_int8_dev(x.data_ptr(), x.numel(), seed, 78, None))
    torch.cuda.synchronize()
    return qm, x


def _run(ctx, qm, x, M, N, path):
    import torch
    from asicfortranai_b200.quantized import PATH_AUTO
    ctx.set_gemm_path(path)
    Cd = torch.full((M * N,), 7, dtype=torch.int32, device="cuda")
    Yd = torch.full((M * N,), 7.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()      # the fills complete before the library's stream writes
    qm.gemm_dev(x.data_ptr(), M, Cd.data_ptr(), Yd.data_ptr())
    ctx.synchronize()
    ctx.set_gemm_path(PATH_AUTO)
    ctx.device_error()
    return Cd.cpu().numpy(), Yd.cpu().numpy()


LLAMA70B = [("q", 8192, 8192), ("k", 8192, 1024), ("o", 8192, 8192), ("gate", 8192, 28672),
            ("down", 28672, 8192)]


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("name,K,N", LLAMA70B)
@pytest.mark.parametrize("M", [16, 64])
def test_engines_agree_on_llama70b_shapes(ctx, fmt, name, K, N, M):
    from asicfortranai_b200.quantized import PATH_CUDA_CORES, PATH_TENSOR_CORES
    qm, x = _device_case(ctx, fmt, K, N, M, 5)
    Cc, Yc = _run(ctx, qm, x, M, N, PATH_CUDA_CORES)
    Ct, Yt = _run(ctx, qm, x, M, N, PATH_TENSOR_CORES)
    np.testing.assert_array_equal(Ct, Cc)
    np.testing.assert_array_equal(Yt.view(np.uint32), Yc.view(np.uint32))
    qm.close()


@pytest.mark.parametrize("name,K,N", [("gate", 8192, 28672), ("down", 28672, 8192)])
def test_prefill_2048_rows(ctx, name, K, N):
    """The prefill GEMMs (M=2048): tensor engine == CUDA-core engine bit for bit, and a
    column sample against the oracle."""
    from asicfortranai_b200.quantized import PATH_CUDA_CORES, PATH_TENSOR_CORES
    M = 2048
    qm, x = _device_case(ctx, 0, K, N, M, 9)
    Ct, Yt = _run(ctx, qm, x, M, N, PATH_TENSOR_CORES)
    Cc, _ = _run(ctx, qm, x, M, N, PATH_CUDA_CORES)
    np.testing.assert_array_equal(Ct, Cc)
    # oracle on 40 columns x 64 rows
    wq = qm.download_ref()                       # (K/2, N) column-major
    cols = np.arange(0, N, N // 40)[:40]
    rows = np.arange(0, M, M // 64)[:64]
    A = np.asfortranarray(x.cpu().numpy().reshape(M, K)[rows])
    s = np.ones(len(cols), np.float32)
    o = np.zeros(len(cols), np.float32)
    ref = orc.matmul_3p5bit_awq(A, np.asfortranarray(wq[:, cols]), s, o)
    np.testing.assert_array_equal(Ct.reshape(M, N)[np.ix_(rows, cols)], ref)
    qm.close()


def test_row_and_column_major_layouts(tensor_path):
    """Row-major x read in place through TMA, column-major x through the workspace copy;
    both output layouts."""
    import torch
    from asicfortranai_b200.quantized import QuantizedMatrix
    ctx = tensor_path
    K, N, M = 1024, 200, 37
    A, wq, s, o, Cref, Yref = make_case(K, N, M, 41, 0)
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=0)
    for x_layout, xa in ((0, np.asfortranarray(A)), (1, np.ascontiguousarray(A))):
        for out_layout in (0, 1):
            xd = torch.from_numpy(xa.ravel(order="K").copy()).cuda()
            Cd = torch.zeros(M * N, dtype=torch.int32, device="cuda")
            Yd = torch.zeros(M * N, dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            qm.gemm_dev(xd.data_ptr(), M, Cd.data_ptr(), Yd.data_ptr(), x_layout=x_layout,
                        out_layout=out_layout)
            ctx.synchronize()
            order = "F" if out_layout == 0 else "C"
            np.testing.assert_array_equal(Cd.cpu().numpy().reshape((M, N), order=order), Cref)
            np.testing.assert_array_equal(Yd.cpu().numpy().reshape((M, N), order=order).view(np.uint32),
                                          Yref.view(np.uint32))
    ctx.device_error()
    qm.close()


def test_capture_in_graph(tensor_path):
    """The tensor engine replays inside a CUDA graph (tensor map baked at capture)."""
    import torch
    from asicfortranai_b200.quantized import QuantizedMatrix
    ctx = tensor_path
    K, N, M = 2048, 512, 24
    A, wq, s, o, Cref, _ = make_case(K, N, M, 43, 1)
    qm = QuantizedMatrix(ctx, wq, s, o, fmt=1)
    xd = torch.from_numpy(np.ascontiguousarray(A).ravel()).cuda()
    Cd = torch.zeros(M * N, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    run = lambda: qm.gemm_dev(xd.data_ptr(), M, Cd.data_ptr(), None, x_layout=1, out_layout=1)
    run()
    ctx.synchronize()
    g = ctx.capture(run)
    Cd.zero_()
    torch.cuda.synchronize()
    for _ in range(3):
        g.launch()
    ctx.synchronize()
    np.testing.assert_array_equal(Cd.cpu().numpy().reshape(M, N), Cref)
    g.close()
    ctx.device_error()
    qm.close()
