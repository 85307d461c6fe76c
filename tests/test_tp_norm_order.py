"""Host-side pin of the fused exchange + RMSNorm's reduction order (ar_dequant_norm_kernel):
its element ownership (CTA c of 32 owns the float4 groups j with (j mod 1024) / 32 == c, in
slots (k, lane) = ((slot/4)/32, (slot/4)%32)) partitions the row, and its sums -- per owned
norm thread the squares in group order, a 32-lane xor butterfly per CTA, the same butterfly
over the 32 CTA sums -- give the oracle's tree-order RMSNorm bit for bit."""
import numpy as np
import pytest

from oracle import oracle as orc

F = np.float32


def butterfly(v):
    v = [F(x) for x in v]
    for o in (16, 8, 4, 2, 1):
        v = [F(v[l] + v[l ^ o]) for l in range(32)]
    assert all(x.view(np.uint32) == v[0].view(np.uint32) for x in v)
    return v[0]


def owned(c, N):
    n4, kmax = N // 4, (N // 4 + 1023) // 1024
    out = []
    for sl in range(128 * kmax):
        g, comp = sl >> 2, sl & 3
        l, k = g & 31, g >> 5
        j = 32 * c + l + 1024 * k
        if j < n4:
            out.append(4 * j + comp)
    return out


def fused_sumsq(x):
    N = len(x)
    n4, kmax = N // 4, (N // 4 + 1023) // 1024
    cta = []
    for c in range(32):
        lanes = []
        for t in range(32):
            s = F(0)
            for k in range(kmax):
                j = 32 * c + t + 1024 * k
                if j >= n4:
                    break
                for e in range(4):
                    s = F(s + F(x[4 * j + e] * x[4 * j + e]))
            lanes.append(s)
        cta.append(butterfly(lanes))
    return butterfly(cta)


@pytest.mark.parametrize("N", [256, 1024, 5120, 8192, 28672])
def test_ownership_partitions_the_row(N):
    seen = np.zeros(N, np.int32)
    for c in range(32):
        for i in owned(c, N):
            seen[i] += 1
    assert np.all(seen == 1)


@pytest.mark.parametrize("N", [256, 1024, 5120, 8192])
def test_fused_order_equals_tree_order(N):
    rng = np.random.default_rng(N)
    x = rng.normal(0, 1.0, N).astype(F)
    w = rng.normal(1.0, 0.1, N).astype(F)
    eps = F(1e-5)
    s = fused_sumsq(x)
    rms = np.sqrt(F(F(s / F(N)) + eps), dtype=F)
    ours = (x / rms).astype(F) * w
    ref = np.zeros((1, N), F, order="F")
    orc.lib().orc_rms_norm_tree(np.asfortranarray(x.reshape(1, N)), np.asfortranarray(w), ref, 1, N, eps)
    np.testing.assert_array_equal(ours.astype(F).view(np.uint32), ref[0].view(np.uint32))
