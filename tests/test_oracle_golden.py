"""Pins the CPU oracle to the reference's own code (golden fixtures made by
tests/golden/make_golden.py from the reference's Python tooling)."""
import numpy as np
import pytest

from oracle import oracle as orc


def test_quantizer_3p5bit_matches_reference_bytes(golden):
    for pre in ("quant", "quant2"):
        W = golden[f"{pre}_W"]
        wq, s, o = orc.quantize_3p5bit(W)
        np.testing.assert_array_equal(wq, golden[f"{pre}_wq"])
        np.testing.assert_array_equal(s.view(np.uint32), golden[f"{pre}_scales"].view(np.uint32))
        np.testing.assert_array_equal(o.view(np.uint32), golden[f"{pre}_offsets"].view(np.uint32))


def test_quantizer_constant_column_and_wraparound(golden):
    s = golden["quant_scales"]
    assert s[5] == np.float32(1.0)                      # w_max == w_min branch
    # the 3-bit slot keeps only the low 3 bits of the odd-row code: some codes wrap
    W = golden["quant_W"]
    K = W.shape[0]
    wmin, wmax = W.min(0), W.max(0)
    sc = np.where(wmax != wmin, (wmax - wmin) / np.float32(15), np.float32(1.0)).astype(np.float32)
    zp = (wmin - np.float32(-8) * sc).astype(np.float32)
    q = np.clip(np.round((W - zp) / sc), -8, 7).astype(np.int32)
    odd = q[1::2]
    assert np.any((odd > 3) | (odd < -4)), "fixture must exercise wrap-around"
    raw7 = golden["quant_wq"].astype(np.int32) & 0x7F
    n2 = raw7 & 7
    n2 = np.where(n2 >= 4, n2 - 8, n2)
    np.testing.assert_array_equal(n2, ((odd + 8) & 7) - 8 * (((odd + 8) & 7) >= 4))
    assert K == 256


@pytest.mark.parametrize("ci", range(4))
def test_matmul_3p5bit_matches_reference_spec(golden, ci):
    A, wq = golden[f"mm{ci}_A"], golden[f"mm{ci}_wq"]
    sc, of = golden[f"mm{ci}_scales"], golden[f"mm{ci}_offsets"]
    Cref, Yref = golden[f"mm{ci}_C"], golden[f"mm{ci}_Y"]
    C_ = orc.matmul_3p5bit_awq(A, wq, sc, of)
    np.testing.assert_array_equal(C_, Cref)              # int32 bit-exact
    Y = orc.dequantize_output_3p5bit(C_, sc, of)
    # the reference's Python spec widens (int32 + float32) to float64 before rounding;
    # the Fortran rounds after each binary32 operation: 1e-5 relative covers both
    np.testing.assert_allclose(Y, Yref, rtol=1e-5, atol=1e-6)


def test_decode_known_answers(golden):
    for n1, n2, raw7, d1, d2 in golden["fixed_cases"]:
        assert (d1, d2) == (n1, n2)
        A = np.zeros((1, 2), np.int8, order="F")
        A[0, 0], A[0, 1] = 1, 0
        wq = np.array([[raw7]], np.int8, order="F")
        z = np.zeros(1, np.float32)
        assert orc.matmul_3p5bit_awq(A, wq, z, z)[0, 0] == n1
        A[0, 0], A[0, 1] = 0, 1
        assert orc.matmul_3p5bit_awq(A, wq, z, z)[0, 0] == n2
    tab = golden["decode_table"]
    A = np.zeros((2, 256), np.int8, order="F")
    A[0, 0::2] = 0
    wq = np.arange(128, dtype=np.int8).reshape(128, 1, order="F")
    for r in range(128):
        A1 = np.zeros((1, 256), np.int8, order="F")
        A1[0, 2 * r] = 1
        A2 = np.zeros((1, 256), np.int8, order="F")
        A2[0, 2 * r + 1] = 1
        z = np.zeros(1, np.float32)
        assert orc.matmul_3p5bit_awq(A1, wq, z, z)[0, 0] == tab[r, 0]
        assert orc.matmul_3p5bit_awq(A2, wq, z, z)[0, 0] == tab[r, 1]
    assert tab[:, 0].min() == -8 and tab[:, 0].max() == 7
    assert tab[:, 1].min() == -4 and tab[:, 1].max() == 3


def test_msb_of_packed_byte_is_ignored():
    """matmul_3p5bit_dynamic.f90:48 masks with 0x7F: bytes b and b|0x80 decode alike."""
    rng = np.random.default_rng(1)
    A = rng.integers(-127, 128, (3, 64)).astype(np.int8)
    wq = rng.integers(0, 128, (32, 7)).astype(np.int8)
    z = np.zeros(7, np.float32)
    c1 = orc.matmul_3p5bit_awq(A, wq, z, z)
    c2 = orc.matmul_3p5bit_awq(A, (wq.view(np.uint8) | 0x80).view(np.int8), z, z)
    np.testing.assert_array_equal(c1, c2)


def test_int4_quantizer_matches_reference_quality(golden):
    W = golden["qq_W"]
    wq, s = orc.quantize_int4(W)
    q = np.zeros(W.shape, np.int32)
    b = wq.astype(np.int32) & 0xFF
    lo, hi = b & 15, (b >> 4) & 15
    q[0::2] = np.where(lo >= 8, lo - 16, lo)
    q[1::2] = np.where(hi >= 8, hi - 16, hi)
    dq = q.astype(np.int8) * s
    err = np.sqrt(np.mean((W - dq) ** 2)) / (np.std(W) + 1e-8) * 100
    assert err == golden["qq_int4_err"]


def test_int4_matmul_against_dense():
    rng = np.random.default_rng(2)
    M, K, N = 3, 40, 9
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    wq, s = orc.quantize_int4(W)
    A = rng.integers(-127, 128, (M, K)).astype(np.int8)
    b = wq.astype(np.int32) & 0xFF
    q = np.zeros((K, N), np.int64)
    lo, hi = b & 15, (b >> 4) & 15
    q[0::2] = np.where(lo >= 8, lo - 16, lo)
    q[1::2] = np.where(hi >= 8, hi - 16, hi)
    C_ = orc.matmul_int4_awq(A, wq, s)
    np.testing.assert_array_equal(C_, A.astype(np.int64) @ q)


def test_greedy_known_answer():
    """test_sampling.f90:22-39 crafts logits(i) = (V-i)/1000 and then sets
    logits(1:3) = 5,4,3 and logits(100) = 2.5.  Its printed expectation is token 1, but
    logits(4) = 31.996 is the maximum, so sample_greedy (sampling.f90:64-83) returns 4;
    the reference test prints and never asserts.  The oracle follows the code."""
    V = 32000
    logits = (V - np.arange(1, V + 1)).astype(np.float32) / np.float32(1000.0)
    logits[0], logits[1], logits[2], logits[99] = 5.0, 4.0, 3.0, 2.5
    assert orc.sample_greedy(logits) == 4
    logits[3:] = np.minimum(logits[3:], 2.0)           # the distribution the test meant
    assert orc.sample_greedy(logits) == 1
    # ties resolve to the first index (strict '>')
    t = np.zeros(10, np.float32)
    t[3] = t[7] = 1.0
    assert orc.sample_greedy(t) == 4


def test_offby1_mode_differs_only_by_shift():
    """matmul_3p5bit_dynamic.f90:47 reads pair (k+0)/2: the compat mode equals the
    correct kernel applied to the byte stream shifted by one."""
    rng = np.random.default_rng(3)
    M, K, N = 2, 16, 4
    A = rng.integers(-127, 128, (M, K)).astype(np.int8)
    wq = rng.integers(0, 128, (K // 2, N)).astype(np.int8)
    z = np.zeros(N, np.float32)
    c_bug = orc.matmul_3p5bit_awq(A, wq, z, z, mode=1)
    flat = np.concatenate([[0], wq.reshape(-1, order="F")[:-1]]).astype(np.int8)
    shifted = flat.reshape(K // 2, N, order="F")
    np.testing.assert_array_equal(c_bug, orc.matmul_3p5bit_awq(A, shifted, z, z))


def test_symmetric_quantizer_bytes_decode_alike(golden):
    """quantize_weights.py's symmetric quantizer (scale = absmax/3, offset 0, codes clipped
    to [-8,7] / [-4,3]) writes bytes that the kernels' decode reads the same way: the
    oracle's int32 sums equal the reference matmul spec on them, the dequantized outputs
    agree within 1e-5, and the per-element expansion equals dequantize_from_3p5bit."""
    from asicfortranai_b200 import weight_files as wf
    wq, s, o = golden["sym_wq"], golden["sym_scales"], golden["sym_offsets"]
    assert not o.any()
    A = np.asfortranarray(golden["sym_A"])
    C_ = orc.matmul_3p5bit_awq(A, np.asfortranarray(wq), s, o)
    np.testing.assert_array_equal(C_, golden["sym_C"])
    np.testing.assert_allclose(orc.dequantize_output_3p5bit(C_, s, o), golden["sym_Y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(wf.expand_3p5bit(wq, s, o), golden["sym_deq"])
    # its reconstruction stays within half a step of the clipped code range
    W = golden["sym_W"]
    assert np.all(np.abs(golden["sym_deq"] - W)[0::2] <= 0.5 * s * 1.001 + 1e-6)
