/* q35_expf.h -- the exponential used by every softmax and SwiGLU of the decode path,
 * written once for both the CUDA kernels and their CPU restatement so that both produce
 * the same bits.  Method (Cody and Waite's argument reduction with a Taylor polynomial):
 *   k = rint(x / ln 2),  r = x - k*ln2_hi - k*ln2_lo  (|r| <= ln2/2, two fused steps),
 *   e^r = sum_{n=0..8} r^n / n!  (Horner, fused multiply-adds; truncation < 2e-9 rel.),
 *   e^x = e^r * 2^k  (two exact power-of-two multiplies).
 * Accuracy: about 1 ulp, against ~1 ulp for C's expf and CUDA's expf, which differ from
 * each other in the last bit on a small fraction of inputs.  Every operation is a
 * correctly rounded IEEE binary32 operation, so host and device agree exactly (the host
 * build uses -ffp-contract=off; the fused steps are explicit fmaf). */
#ifndef Q35_EXPF_H
#define Q35_EXPF_H

#ifdef __CUDACC__
#define Q35_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#define Q35_HD static inline
#endif

Q35_HD float q35_pow2i(int k) {        /* 2^k for -126 <= k <= 127 as a float */
    union { unsigned int u; float f; } v;
    v.u = (unsigned int)(k + 127) << 23;
    return v.f;
}

Q35_HD float q35_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float k = rintf(x * 1.44269502162933349609375f);     /* 1/ln2 rounded to binary32 */
    float r = fmaf(-k, 0.693145751953125f, x);                 /* ln2_hi: 16 significant bits */
    r = fmaf(-k, 1.428606765330187045e-06f, r);                /* ln2_lo = ln2 - ln2_hi */
    float p = 2.48015873015873e-05f;                           /* 1/8! */
    p = fmaf(p, r, 1.98412698412698e-04f);                     /* 1/7! */
    p = fmaf(p, r, 1.38888888888889e-03f);                     /* 1/6! */
    p = fmaf(p, r, 8.33333333333333e-03f);                     /* 1/5! */
    p = fmaf(p, r, 4.16666666666667e-02f);                     /* 1/4! */
    p = fmaf(p, r, 1.66666666666667e-01f);                     /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ki = (int)k;                                     /* -150 <= ki <= 128 */
    const int k1 = ki / 2, k2 = ki - k1;
    return (p * q35_pow2i(k1)) * q35_pow2i(k2);
}

#endif
