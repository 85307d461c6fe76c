"""Generate the golden fixtures that pin the CPU oracle to the reference's own code.

Run once in a checkout that has the reference project next to it:

    python tests/golden/make_golden.py /path/to/asicForTranAI

It imports the reference's Python tooling from ``2025-3.5bit-groq-mvp/`` and writes
``tests/golden/q35_golden.npz``.  The fixtures hold only inputs generated here (seeded)
and the outputs of the reference functions on them:

* ``convert_weights_3p5bit.quantize_3p5bit_asymmetric`` (packed bytes, scales, offsets),
  including a constant column (scale 1.0 branch) and 3-bit-slot wrap-around codes;
* ``test_matmul_small.matmul_3p5bit_reference`` (the reference's executable spec of
  matmul_3p5bit_dynamic.f90 + dequant).  Called once with scales=1, offsets=0, which
  returns float32(C) and so the exact int32 accumulators (|C| < 2**24), and once with
  the real scales/offsets for the dequantized output;
* ``test_fixed.py``'s encode/decode round-trip cases and the 0..127 decode table;
* ``benchmark_3p5bit.test_quantization_quality``'s INT4 and 3.5-bit reconstruction
  errors for a seeded matrix (pins the INT4 quantizer expressions);
* ``quantize_weights.quantize_to_3p5bit`` (the symmetric variant) and its
  ``dequantize_from_3p5bit`` on that tool's own test matrix, with the matmul spec on its
  bytes.

It runs only where the reference sources are present; the tests read only the
.npz it writes.
"""
from __future__ import annotations

import contextlib
import io
import os
import sys

import numpy as np


def main(ref_root: str) -> None:
    mvp = os.path.join(ref_root, "2025-3.5bit-groq-mvp")
    sys.path.insert(0, mvp)
    with contextlib.redirect_stdout(io.StringIO()):
        import convert_weights_3p5bit as cw
        import test_matmul_small as tms
        import test_fixed as tf
        import benchmark_3p5bit as bm
        import quantize_weights as qw

    out = {}
    rng = np.random.default_rng(20251128)

    # 1) asymmetric 3.5-bit quantizer
    W = (rng.standard_normal((256, 64)) * 0.02).astype(np.float32)
    W[:, 5] = 0.25                       # constant column -> scale 1.0 branch
    W[:, 6] = np.linspace(-1, 1, 256, dtype=np.float32)
    wq, s, o = cw.quantize_3p5bit_asymmetric(W.copy())
    out.update(quant_W=W, quant_wq=wq, quant_scales=s, quant_offsets=o)

    W2 = (rng.standard_normal((8192, 8)) * 0.02).astype(np.float32)
    wq2, s2, o2 = cw.quantize_3p5bit_asymmetric(W2.copy())
    out.update(quant2_W=W2, quant2_wq=wq2, quant2_scales=s2, quant2_offsets=o2)

    # 2) matmul + dequant reference on quantizer output
    cases = [(1, 16, 8), (4, 64, 16), (3, 30, 5), (2, 256, 33)]
    for ci, (M, K, N) in enumerate(cases):
        Wm = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        wpk, sc, of = cw.quantize_3p5bit_asymmetric(Wm.copy())
        A = rng.integers(-127, 128, size=(M, K)).astype(np.int8)
        Cf = tms.matmul_3p5bit_reference(A, wpk, np.ones(N, np.float32), np.zeros(N, np.float32))
        Cint = Cf.astype(np.int64)
        assert np.all(np.abs(Cint) < 2 ** 24)
        Y = tms.matmul_3p5bit_reference(A, wpk, sc, of)
        out.update({f"mm{ci}_A": A, f"mm{ci}_wq": wpk, f"mm{ci}_scales": sc,
                    f"mm{ci}_offsets": of, f"mm{ci}_C": Cint.astype(np.int32), f"mm{ci}_Y": Y})
    out["mm_cases"] = np.array(cases, np.int32)

    # 3) encode/decode known answers of test_fixed.py
    enc = []
    for n1, n2 in tf.test_cases:
        raw7 = tf.encode_3p5bit(n1, n2)
        d1, d2 = tf.decode_3p5bit_fixed(raw7)
        enc.append((n1, n2, raw7, d1, d2))
    out["fixed_cases"] = np.array(enc, np.int32)
    out["decode_table"] = np.array([tf.decode_3p5bit_fixed(r) for r in range(128)], np.int32)

    # 4) reconstruction errors of benchmark_3p5bit.test_quantization_quality
    np.random.seed(7)
    with contextlib.redirect_stdout(io.StringIO()):
        res = bm.test_quantization_quality([(512, 96)])
    np.random.seed(7)
    Wq = np.random.randn(512, 96).astype(np.float32)
    out.update(qq_W=Wq, qq_int4_err=np.float64(res["int4_mean_error"]),
               qq_3p5_err=np.float64(res["3p5bit_mean_error"]))

    # 5) the symmetric 3.5-bit quantizer of quantize_weights.py on its own test's matrix
    #    (seed 42, 128 x 64, N(0, 0.1^2)), its per-element dequantization, and the reference
    #    matmul spec on its bytes: checkpoints from that tool decode the same way
    np.random.seed(42)
    Ws = (np.random.randn(128, 64).astype(np.float32) * 0.1).astype(np.float32)
    with contextlib.redirect_stdout(io.StringIO()):
        wps, ss, os_ = qw.quantize_to_3p5bit(Ws.copy())
        deq = qw.dequantize_from_3p5bit(wps, ss, os_)
    As = rng.integers(-127, 128, size=(3, 128)).astype(np.int8)
    Cs = tms.matmul_3p5bit_reference(As, wps, np.ones(64, np.float32), np.zeros(64, np.float32))
    assert np.all(np.abs(Cs) < 2 ** 24)
    Ys = tms.matmul_3p5bit_reference(As, wps, ss, os_)
    out.update(sym_W=Ws, sym_wq=wps, sym_scales=ss, sym_offsets=os_, sym_deq=deq, sym_A=As,
               sym_C=Cs.astype(np.int64).astype(np.int32), sym_Y=Ys)

    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "q35_golden.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
