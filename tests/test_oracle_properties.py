"""Size-independent properties of the oracle's kernels (matmul_3p5bit_dynamic.f90:28-82,
matmul_int4_groq.f90:19-69, transformer_layer.f90:68-90), checked on the CPU.  They are the
properties the device path is later held to at full size: integer accumulation is linear in
the activations, separable over output columns and additive over K slices (the row-split
tensor-parallel sum), exact at the largest accumulator magnitudes, and the dequantization is
the three binary32 roundings (C -> real, + offset, * scale)."""
import numpy as np
import pytest

from oracle import oracle as orc

F = np.float32


def _weights(K, N, seed, fmt):
    W = orc.gen_normal((K, N), seed, 1)
    if fmt == "3p5":
        return orc.quantize_3p5bit(W)
    wq, s = orc.quantize_int4(W)
    return wq, s, None


def _mm(fmt, A, wq, s, o):
    return orc.matmul_3p5bit_awq(A, wq, s, o) if fmt == "3p5" else orc.matmul_int4_awq(A, wq, s)


@pytest.mark.parametrize("fmt", ["3p5", "int4"])
def test_linear_in_the_activations(fmt):
    M, K, N = 3, 512, 40
    wq, s, o = _weights(K, N, 1, fmt)
    rng = np.random.default_rng(2)
    A1 = rng.integers(-63, 64, (M, K)).astype(np.int8)
    A2 = rng.integers(-63, 64, (M, K)).astype(np.int8)
    A12 = (A1.astype(np.int16) + A2).astype(np.int8)
    np.testing.assert_array_equal(_mm(fmt, A12, wq, s, o), _mm(fmt, A1, wq, s, o) + _mm(fmt, A2, wq, s, o))


@pytest.mark.parametrize("fmt", ["3p5", "int4"])
def test_separable_over_columns(fmt):
    M, K, N = 2, 256, 48
    wq, s, o = _weights(K, N, 3, fmt)
    A = orc.gen_int8((M, K), 4, 0)
    full = _mm(fmt, A, wq, s, o)
    for lo, hi in ((0, 1), (5, 17), (17, 48)):
        part = _mm(fmt, A, np.asfortranarray(wq[:, lo:hi]), s[lo:hi], None if o is None else o[lo:hi])
        np.testing.assert_array_equal(part, full[:, lo:hi])


@pytest.mark.parametrize("fmt", ["3p5", "int4"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_additive_over_k_slices(fmt, world):
    """The row split of o and down: every rank's int32 partial over its K slice, summed,
    equals the one-GPU accumulator bit for bit."""
    M, K, N = 2, 1024, 24
    wq, s, o = _weights(K, N, 5 + world, fmt)
    A = orc.gen_int8((M, K), 6, 0)
    full = _mm(fmt, A, wq, s, o)
    ks = K // world
    acc = np.zeros_like(full)
    for r in range(world):
        Ar = np.asfortranarray(A[:, r * ks:(r + 1) * ks])
        Wr = np.asfortranarray(wq[r * ks // 2:(r + 1) * ks // 2, :])
        acc += _mm(fmt, Ar, Wr, s, o)
    np.testing.assert_array_equal(acc, full)


def test_largest_accumulators_are_exact():
    """K = 28672 (the down projection) with every activation -127 and every code at its
    most negative value (-8 in the 4-bit slot, -4 in the 3-bit slot): |C| = 14336 * 127 * 12,
    far inside int32."""
    K, N = 28672, 3
    A = np.full((1, K), -127, np.int8)
    b35 = np.int8((((-8) & 0xF) << 3) | ((-4) & 0x7))          # 0x44
    wq = np.full((K // 2, N), b35, np.int8, order="F")
    C = orc.matmul_3p5bit_awq(A, wq, np.ones(N, F), np.zeros(N, F))
    assert (C == (K // 2) * 127 * 12).all()
    b4 = np.int8(np.uint8(0x88).view(np.int8))                  # -8 in both nibbles
    wq4 = np.full((K // 2, N), b4, np.int8, order="F")
    C4 = orc.matmul_int4_awq(A, wq4, np.ones(N, F))
    assert (C4 == K * 127 * 8).all()


def test_smallest_shape():
    A = np.array([[3, -5]], np.int8)
    wq = np.array([[np.int8((5 << 3) | 2)]], np.int8)        # n1 = 5, n2 = 2
    assert orc.matmul_3p5bit_awq(A, wq, np.ones(1, F), np.zeros(1, F))[0, 0] == 3 * 5 - 5 * 2
    wq4 = np.array([[np.int8(np.uint8(0x2D).view(np.int8))]], np.int8)   # low 0xD = -3, high 2
    assert orc.matmul_int4_awq(A, wq4, np.ones(1, F))[0, 0] == 3 * -3 - 5 * 2


def test_dequant_is_three_binary32_roundings():
    rng = np.random.default_rng(9)
    M, N = 4, 257
    C = rng.integers(-(1 << 26), 1 << 26, (M, N)).astype(np.int32)
    s = rng.normal(0, 1e-3, N).astype(F)
    o = rng.normal(0, 50.0, N).astype(F)
    want = (C.astype(F) + o[None, :]) * s[None, :]                 # float32 throughout
    got = orc.dequantize_output_3p5bit(np.asfortranarray(C), s, o)
    np.testing.assert_array_equal(got.view(np.uint32), want.astype(F).view(np.uint32))
    want4 = C.astype(F) * s[None, :]
    np.testing.assert_array_equal(orc.dequantize_output(np.asfortranarray(C), s).view(np.uint32),
                                  want4.astype(F).view(np.uint32))


def test_activation_quantization_truncates():
    """int(max(-127., min(127., x*127.))): truncation toward zero, clamp, no rescale."""
    x = np.array([[0.0, 0.5, -0.5, 0.0039, -0.0039, 1.0, -1.0, 3.7, -3.7, 0.99999, 0.7316,
                   -0.7316, 1e-30, np.float32(np.nextafter(F(1), F(0)))]], F)
    want = np.trunc(np.clip(x * F(127), F(-127), F(127))).astype(np.int8)
    np.testing.assert_array_equal(orc.quantize_activations(x), want)
    rng = np.random.default_rng(3)
    y = rng.normal(0, 0.7, (5, 333)).astype(F)
    np.testing.assert_array_equal(orc.quantize_activations(y),
                                  np.trunc(np.clip(y * F(127), F(-127), F(127))).astype(np.int8))


def test_quantizer_codes_stay_in_range_and_scale_matches():
    """scale = (max - min) / 15 per column (1 for a constant column); every 4-bit code (even
    k) decodes to within half a scale step of its weight (the 3-bit slot may wrap,
    convert_weights_3p5bit.py:19-85)."""
    K, N = 128, 20
    W = orc.gen_normal((K, N), 11, 2, sigma=0.05)
    W[:, 7] = 0.25                                                  # constant column
    wq, s, o = orc.quantize_3p5bit(W)
    mx, mn = W.max(0), W.min(0)
    want_s = np.where(mx == mn, F(1), (mx - mn) / F(15)).astype(F)
    np.testing.assert_array_equal(s.view(np.uint32), want_s.view(np.uint32))
    raw = wq.astype(np.int32) & 0x7F
    n1 = raw >> 3
    n1 = np.where(n1 >= 8, n1 - 16, n1)
    assert n1.min() >= -8 and n1.max() <= 7
    deq = n1.astype(F) * s[None, :] + o[None, :]
    assert (np.abs(deq - W[0::2]) <= F(0.5) * s[None, :] * F(1.001) + F(1e-6)).all()


def test_thread_count_does_not_change_results():
    """The oracle's OpenMP loops split independent outputs only (columns, heads, rows), so
    one thread and many give the same bits: the CPU baseline may use every host core."""
    from tests.model_util import TINY, make_weights
    cfg = dict(TINY)
    w = make_weights(cfg, seed=12)
    ids = orc.gen_tokens(7, 4, 5, cfg["vocab"])
    A = orc.gen_int8((3, 1024), 7, 0)
    wq, s, o = _weights(1024, 96, 8, "3p5")
    res = []
    try:
        for n in (1, 4):
            orc.set_threads(n)
            om = orc.OracleModel(cfg, w)
            res.append((om.forward(ids), om.generate(ids, 8), orc.matmul_3p5bit_awq(A, wq, s, o)))
    finally:
        import os
        orc.set_threads(os.cpu_count() or 1)
    (l1, g1, c1), (l4, g4, c4) = res
    np.testing.assert_array_equal(l1.view(np.uint32), l4.view(np.uint32))
    np.testing.assert_array_equal(g1, g4)
    np.testing.assert_array_equal(c1, c4)


def _decode35(wq):
    raw = wq.astype(np.int64) & 0x7F
    n1 = raw >> 3
    n2 = raw & 7
    q = np.empty((2 * wq.shape[0], wq.shape[1]), np.int64)
    q[0::2] = np.where(n1 >= 8, n1 - 16, n1)
    q[1::2] = np.where(n2 >= 4, n2 - 8, n2)
    return q


def _decode4(wq):
    b = wq.astype(np.int64) & 0xFF
    lo, hi = b & 15, b >> 4
    q = np.empty((2 * wq.shape[0], wq.shape[1]), np.int64)
    q[0::2] = np.where(lo >= 8, lo - 16, lo)
    q[1::2] = np.where(hi >= 8, hi - 16, hi)
    return q


from hypothesis import given, settings, strategies as st  # noqa: E402


@settings(max_examples=150, derandomize=True, deadline=None)
@given(M=st.integers(1, 5), P=st.integers(1, 40), N=st.integers(1, 9), seed=st.integers(0, 2**32 - 1))
def test_generated_shapes_against_a_dense_decode(M, P, N, seed):
    """Ragged shapes (K = 2..80, N = 1..9, M = 1..5) and arbitrary bytes (bit 7 set or not):
    both kernels equal A @ decoded codes in int64, and the dequantizations follow."""
    rng = np.random.default_rng(seed)
    K = 2 * P
    A = rng.integers(-128, 128, (M, K)).astype(np.int8)
    wq = rng.integers(-128, 128, (P, N)).astype(np.int8)
    s = rng.normal(0, 0.01, N).astype(F)
    o = rng.normal(0, 5.0, N).astype(F)
    C35 = orc.matmul_3p5bit_awq(A, wq, s, o)
    np.testing.assert_array_equal(C35, A.astype(np.int64) @ _decode35(wq))
    C4 = orc.matmul_int4_awq(A, wq, s)
    np.testing.assert_array_equal(C4, A.astype(np.int64) @ _decode4(wq))
    np.testing.assert_array_equal(orc.dequantize_output_3p5bit(C35, s, o).view(np.uint32),
                                  ((C35.astype(F) + o) * s).astype(F).view(np.uint32))
