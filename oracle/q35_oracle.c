/*
 * q35_oracle.c -- CPU restatement (C11 + OpenMP) of asicForTranAI's quantized matmul
 * hot path and LLaMA decode loop.  TEST INFRASTRUCTURE ONLY: used by tests/, the smoke
 * check and bench.py's CPU-baseline leg to produce expected results; never by the
 * product library.
 *
 * Reference files are named relative to the reference project root, directory
 * 2025-3.5bit-groq-mvp/.  Build flags: -O3 -fopenmp -ffp-contract=off (no fast-math),
 * so every float operation rounds exactly once.
 * The reference's own Makefile builds with -ffast-math, which leaves the order of its fp32
 * reductions (RMSNorm, attention, LM head) to the vectoriser.  The model functions take
 * one of three orders (orc_config.order): 0, the sequential loops of the source with the C
 * library's expf; 1, the blocked/tree order of the GPU kernels with their exponential;
 * 2, the source loops as an 8-lane vectorising build would run them (each reduction in 8
 * partial sums with fused multiply-adds, lane i%8, combined by halving: lanes 0-3 + 4-7,
 * then 0-1 + 2-3, then 0 + 1), libm expf -- another compilation the reference's
 * -ffast-math build permits, used only to measure how far the source order itself moves.
 * The integer matmuls, quantizers and elementwise steps are order free.
 */
#include "q35_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------ */
/* Generator: SplitMix64 finaliser applied to a (seed, tensor, index) counter.      */
/* ------------------------------------------------------------------------------ */
static inline uint64_t smix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

uint64_t orc_rng_u64(uint64_t seed, uint64_t tensor_id, uint64_t index) {
    uint64_t key = smix(seed ^ smix(tensor_id + 0x632BE59BD9B4E019ull));
    return smix(key + index * 0x9E3779B97F4A7C15ull);
}

void orc_gen_int8(int8_t *out, int64_t n, uint64_t seed, uint64_t tensor_id) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint64_t r = orc_rng_u64(seed, tensor_id, (uint64_t)i);
        int8_t v = 0;
        for (int b = 0; b < 8; ++b) { /* rejection of -128 on 8-bit draws */
            int8_t c = (int8_t)(uint8_t)(r >> (8 * b));
            if (c != -128) { v = c; break; }
        }
        out[i] = v;
    }
}

void orc_gen_normal(float *out, int64_t n, uint64_t seed, uint64_t tensor_id, double sigma) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint64_t a = orc_rng_u64(seed, tensor_id, 2 * (uint64_t)i);
        uint64_t b = orc_rng_u64(seed, tensor_id, 2 * (uint64_t)i + 1);
        double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0); /* (0,1] */
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);         /* [0,1) */
        double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        out[i] = (float)(sigma * z);
    }
}

void orc_gen_tokens(int32_t *out, int64_t n, uint64_t seed, uint64_t tensor_id, int32_t vocab) {
    for (int64_t i = 0; i < n; ++i)
        out[i] = (int32_t)(orc_rng_u64(seed, tensor_id, (uint64_t)i) % (uint64_t)vocab) + 1;
}

/* ------------------------------------------------------------------------------ */
/* Quantizers                                                                       */
/* ------------------------------------------------------------------------------ */
/* convert_weights_3p5bit.py:19-85 quantize_3p5bit_asymmetric, float32 arithmetic as
 * numpy performs it (NEP 50 keeps the Python-int constants weakly typed). */
void orc_quantize_3p5bit_asym(const float *W, int8_t *W_Q, float *scales, float *offsets,
                              int32_t K, int32_t N) {
    const int32_t KH = K / 2;
#pragma omp parallel for schedule(static)
    for (int32_t j = 0; j < N; ++j) {
        const float *col = W + (int64_t)K * j;
        float wmin = col[0], wmax = col[0];
        for (int32_t k = 1; k < K; ++k) {               /* :47-48 np.min / np.max */
            if (col[k] < wmin) wmin = col[k];
            if (col[k] > wmax) wmax = col[k];
        }
        float scale = (wmax != wmin) ? (wmax - wmin) / 15.0f : 1.0f;  /* :58 */
        float zp = wmin - (-8.0f * scale);                             /* :59 */
        scales[j] = scale;
        offsets[j] = zp;                                                /* :62 */
        for (int32_t p = 0; p < KH; ++p) {
            int32_t q[2];
            for (int t = 0; t < 2; ++t) {                               /* :65-66 */
                float v = (col[2 * p + t] - zp) / scale;
                int32_t r = (int32_t)rintf(v);                          /* round half even */
                q[t] = r < -8 ? -8 : (r > 7 ? 7 : r);
            }
            int32_t v1 = q[0] < 0 ? q[0] + 16 : q[0];                   /* :72-74 */
            int32_t v2 = q[1] < 0 ? q[1] + 8 : q[1];                    /* :77-79 */
            int32_t packed = ((v1 & 0xF) << 3) | (v2 & 0x7);            /* :82 */
            W_Q[(int64_t)KH * j + p] = (int8_t)(packed & 0x7F);         /* :83 */
        }
    }
}

/* benchmark_3p5bit.py:155-159 (symmetric absmax/7 INT4), packed low nibble first as
 * matmul_int4_groq.f90:42-50 decodes it. */
void orc_quantize_int4_sym(const float *W, int8_t *W_Q, float *scales, int32_t K, int32_t N) {
    const int32_t KH = K / 2;
#pragma omp parallel for schedule(static)
    for (int32_t j = 0; j < N; ++j) {
        const float *col = W + (int64_t)K * j;
        float amax = 0.0f;
        for (int32_t k = 0; k < K; ++k) {
            float a = fabsf(col[k]);
            if (a > amax) amax = a;
        }
        float scale = amax / 7.0f;
        if (!(scale > 1e-6f)) scale = 1.0f;
        scales[j] = scale;
        for (int32_t p = 0; p < KH; ++p) {
            int32_t q[2];
            for (int t = 0; t < 2; ++t) {
                int32_t r = (int32_t)(int8_t)(int32_t)rintf(col[2 * p + t] / scale);
                q[t] = r < -8 ? -8 : (r > 7 ? 7 : r);
            }
            W_Q[(int64_t)KH * j + p] = (int8_t)((q[0] & 0xF) | ((q[1] & 0xF) << 4));
        }
    }
}

/* ------------------------------------------------------------------------------ */
/* Matmul kernels                                                                   */
/* ------------------------------------------------------------------------------ */
/* matmul_3p5bit_dynamic.f90:42-64.  mode 0 uses idx=(k+1)/2 (1-based k), the index of
 * matmul_int4_optimized.f90:104, matmul_3p5bit_FIXED.f90:18 and test_matmul_small.py:23;
 * mode 1 reproduces line 47's idx=(k+0)/2, which reads the byte before each column
 * (taken as the previous column's last byte, and 0 before column 1). */
void orc_matmul_3p5bit_awq(const int8_t *A, const int8_t *W_Q, const float *scales,
                           const float *offsets, int32_t *C, int32_t M, int32_t N, int32_t K,
                           int32_t mode) {
    (void)scales; (void)offsets;
    const int64_t KH = K / 2;
#pragma omp parallel for schedule(static)
    for (int32_t j = 0; j < N; ++j) {
        for (int32_t i = 0; i < M; ++i) {
            int32_t acc = 0;
            for (int32_t k = 1; k <= K; k += 2) {                       /* 1-based k */
                int64_t idx = mode ? (k + 0) / 2 : (k + 1) / 2;         /* 1-based */
                int64_t flat = (idx - 1) + KH * j;
                int32_t raw7 = flat < 0 ? 0 : ((int32_t)W_Q[flat] & 0x7F);   /* :48 */
                int32_t n1 = raw7 >> 3;                                  /* :51 */
                if (n1 >= 8) n1 -= 16;                                   /* :52 */
                int32_t n2 = raw7 & 7;                                   /* :55 */
                if (n2 >= 4) n2 -= 8;                                    /* :56 */
                acc += (int32_t)A[i + (int64_t)M * (k - 1)] * n1;        /* :59 */
                if (k + 1 <= K) acc += (int32_t)A[i + (int64_t)M * k] * n2;  /* :60-62 */
            }
            C[i + (int64_t)M * j] = acc;
        }
    }
}

/* matmul_3p5bit_dynamic.f90:78-81 */
void orc_dequantize_output_3p5bit(const int32_t *C, const float *scales, const float *offsets,
                                  float *Out, int32_t M, int32_t N) {
    for (int32_t j = 0; j < N; ++j)
        for (int32_t i = 0; i < M; ++i) {
            float c = (float)C[i + (int64_t)M * j];
            float t = c + offsets[j];
            Out[i + (int64_t)M * j] = t * scales[j];
        }
}

/* matmul_int4_groq.f90:117-137 */
void orc_matmul_int4_awq(const int8_t *A, const int8_t *W_Q, const float *scales, int32_t *C,
                         int32_t M, int32_t N, int32_t K) {
    (void)scales;
    const int64_t KH = K / 2;
#pragma omp parallel for schedule(static)
    for (int32_t j = 0; j < N; ++j) {
        for (int32_t i = 0; i < M; ++i) {
            int32_t acc = 0;
            for (int32_t k = 1; k <= K; k += 2) {
                int64_t kp = (k + 1) / 2;                                    /* :122 */
                int32_t b = (int32_t)W_Q[(kp - 1) + KH * j];                 /* :123 */
                int32_t q = b & 15;                                          /* :126 */
                if (q >= 8) q -= 16;
                acc += (int32_t)A[i + (int64_t)M * (k - 1)] * q;             /* :128 */
                if (k + 1 <= K) {
                    q = (b >> 4) & 15;                                       /* :132 */
                    if (q >= 8) q -= 16;
                    acc += (int32_t)A[i + (int64_t)M * k] * q;               /* :134 */
                }
            }
            C[i + (int64_t)M * j] = acc;
        }
    }
}

/* matmul_simd_optimized.f90:24-112 matmul_int4_simd: the same sums as matmul_int4_awq in the
 * reference's CPU-optimised loop form -- OpenMP over columns, eight k per step through the
 * sign-extension table (:13-14, :46-79), one accumulator per output (:82-89), the ragged
 * tail two k at a time (:93-104).  A timed CPU stand-in (all host threads); not a checker. */
static const int32_t SIGN_EXTEND_4BIT[16] = {0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1};

void orc_matmul_int4_simd(const int8_t *A, const int8_t *W_Q, const float *scales, int32_t *C,
                          int32_t M, int32_t N, int32_t K) {
    (void)scales;
    const int64_t KH = K / 2;
#pragma omp parallel for schedule(static)
    for (int32_t j = 0; j < N; ++j) {
        const uint8_t *wc = (const uint8_t *)W_Q + KH * j;
        for (int32_t i = 0; i < M; ++i) {
            int32_t acc = 0;
            int32_t k = 1;
#pragma omp simd reduction(+ : acc)
            for (k = 1; k <= K - 7; k += 8) {
                const uint8_t *b = wc + (k + 1) / 2 - 1;
                const int8_t *a = A + i + (int64_t)M * (k - 1);
                acc += a[0] * SIGN_EXTEND_4BIT[b[0] & 15] + a[M] * SIGN_EXTEND_4BIT[b[0] >> 4] +
                       a[2 * (int64_t)M] * SIGN_EXTEND_4BIT[b[1] & 15] + a[3 * (int64_t)M] * SIGN_EXTEND_4BIT[b[1] >> 4] +
                       a[4 * (int64_t)M] * SIGN_EXTEND_4BIT[b[2] & 15] + a[5 * (int64_t)M] * SIGN_EXTEND_4BIT[b[2] >> 4] +
                       a[6 * (int64_t)M] * SIGN_EXTEND_4BIT[b[3] & 15] + a[7 * (int64_t)M] * SIGN_EXTEND_4BIT[b[3] >> 4];
            }
            for (k = (K / 8) * 8 + 1; k <= K; k += 2) {
                const int32_t b = wc[(k + 1) / 2 - 1];
                acc += (int32_t)A[i + (int64_t)M * (k - 1)] * SIGN_EXTEND_4BIT[b & 15];
                if (k + 1 <= K) acc += (int32_t)A[i + (int64_t)M * k] * SIGN_EXTEND_4BIT[(b >> 4) & 15];
            }
            C[i + (int64_t)M * j] = acc;
        }
    }
}

/* matmul_int4_groq.f90:150-152 */
void orc_dequantize_output(const int32_t *C, const float *scales, float *Out, int32_t M, int32_t N) {
    for (int32_t j = 0; j < N; ++j)
        for (int32_t i = 0; i < M; ++i)
            Out[i + (int64_t)M * j] = (float)C[i + (int64_t)M * j] * scales[j];
}

/* transformer_layer.f90:81-83: int(max(-127.0, min(127.0, x*127.0)), int8) (truncation) */
void orc_quantize_activations(const float *x, int8_t *x_int8, int64_t n) {
    for (int64_t t = 0; t < n; ++t) {
        float v = x[t] * 127.0f;
        v = fminf(127.0f, v);
        v = fmaxf(-127.0f, v);
        x_int8[t] = (int8_t)(int32_t)v;
    }
}

/* transformer_layer.f90:68-90 int4_linear, with the 3.5-bit kernels substituted for
 * the 3.5-bit format (llama70b_3p5bit.f90:298-299). */
void orc_q35_linear(const float *x, const int8_t *W_Q, const float *scales, const float *offsets,
                    float *out, int32_t M, int32_t N, int32_t K, int32_t wformat) {
    int8_t *xi = (int8_t *)malloc((size_t)M * K);
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)M * N);
    orc_quantize_activations(x, xi, (int64_t)M * K);
    if (wformat == 0) {
        orc_matmul_3p5bit_awq(xi, W_Q, scales, offsets, acc, M, N, K, 0);
        orc_dequantize_output_3p5bit(acc, scales, offsets, out, M, N);
    } else {
        orc_matmul_int4_awq(xi, W_Q, scales, acc, M, N, K);
        orc_dequantize_output(acc, scales, out, M, N);
    }
    free(xi);
    free(acc);
}

/* ------------------------------------------------------------------------------ */
/* Transformer pieces                                                               */
/* ------------------------------------------------------------------------------ */
/* transformer_layer.f90:155-178 */
void orc_rms_norm(const float *x, const float *w, float *out, int32_t S, int32_t dim, float eps) {
    for (int32_t i = 0; i < S; ++i) {
        float rms = 0.0f;
        for (int32_t j = 0; j < dim; ++j) {
            float v = x[i + (int64_t)S * j];
            rms = rms + v * v;
        }
        rms = sqrtf(rms / (float)dim + eps);
        for (int32_t j = 0; j < dim; ++j)
            out[i + (int64_t)S * j] = (x[i + (int64_t)S * j] / rms) * w[j];
    }
}

/* ---- the blocked / tree reduction order of the GPU kernels (orc_config.order = 1) ----
 * The reference builds with -ffast-math, which leaves the order of its fp32 reductions to
 * the vectoriser; this order is the one the CUDA kernels use, restated loop for loop. */

/* 32-lane xor butterfly: at each step every lane adds its partner's value (v += v[l^o]);
 * returns lane 0's total */
static float butterfly_sum(float *v) {
    for (int o = 16; o > 0; o >>= 1) {
        float nv[32];
        for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
        memcpy(v, nv, sizeof(nv));
    }
    return v[0];
}

/* sum of squares of a contiguous row: 1024 threads, thread t over float4 groups
 * t, t+1024, ..., then each warp's butterfly, then a butterfly of the 32 warp sums */
static float sumsq_tree(const float *xr, int32_t dim) {
    float warp_tot[32];
    const int32_t n4 = dim / 4;
    for (int w = 0; w < 32; ++w) {
        float v[32];
        for (int l = 0; l < 32; ++l) {
            float s = 0.0f;
            for (int32_t j = 32 * w + l; j < n4; j += 1024)
                for (int e = 0; e < 4; ++e) s = s + xr[4 * j + e] * xr[4 * j + e];
            v[l] = s;
        }
        warp_tot[w] = butterfly_sum(v);
    }
    return butterfly_sum(warp_tot);
}

void orc_rms_norm_tree(const float *x, const float *w, float *out, int32_t S, int32_t dim, float eps) {
    float *row = (float *)malloc(sizeof(float) * (size_t)dim);
    for (int32_t i = 0; i < S; ++i) {
        for (int32_t j = 0; j < dim; ++j) row[j] = x[i + (int64_t)S * j];
        float rms = sqrtf(sumsq_tree(row, dim) / (float)dim + eps);
        for (int32_t j = 0; j < dim; ++j) out[i + (int64_t)S * j] = (row[j] / rms) * w[j];
    }
    free(row);
}

/* The exponential of the GPU kernels (Cody and Waite's reduction by ln 2 with a Taylor
 * polynomial of degree 8, all steps correctly rounded binary32), restated. */
static float pow2i(int k) {
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)(k + 127) << 23;
    return v.f;
}

static float q35_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float k = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-k, 0.693145751953125f, x);
    r = fmaf(-k, 1.428606765330187045e-06f, r);
    float p = 2.48015873015873e-05f;
    p = fmaf(p, r, 1.98412698412698e-04f);
    p = fmaf(p, r, 1.38888888888889e-03f);
    p = fmaf(p, r, 8.33333333333333e-03f);
    p = fmaf(p, r, 4.16666666666667e-02f);
    p = fmaf(p, r, 1.66666666666667e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ki = (int)k, k1 = ki / 2, k2 = ki - k1;
    return (p * pow2i(k1)) * pow2i(k2);
}

float orc_q35_expf(float x) { return q35_expf(x); }

/* transformer_layer.f90:212-216 */
float orc_swish(float x) { return x / (1.0f + expf(-x)); }
static float swish_q35(float x) { return x / (1.0f + q35_expf(-x)); }

/* transformer_layer.f90:96-118: freqs(pos,d) = real(pos-1)*freq_base**(-2(d-1)/HEAD_DIM) */
void orc_rope_freqs(float *freqs, int32_t max_seq, int32_t head_dim, float theta) {
    for (int32_t d = 0; d < head_dim / 2; ++d) {
        float e = (-2.0f * (float)d) / (float)head_dim;
        float th = powf(theta, e);
        for (int32_t pos = 0; pos < max_seq; ++pos)
            freqs[pos + (int64_t)max_seq * d] = (float)pos * th;
    }
}

/* sampling.f90:64-83 (strict '>' keeps the first maximum); returns a 1-based id */
int32_t orc_sample_greedy(const float *logits, int32_t vocab) {
    float mv = logits[0];
    int32_t mi = 1;
    for (int32_t i = 2; i <= vocab; ++i)
        if (logits[i - 1] > mv) { mv = logits[i - 1]; mi = i; }
    return mi;
}

/* ---- sampling.f90:19-259 ---------------------------------------------------------
 * order 0: the reference's loops (sequential fp32 sums, C expf).
 * order 1: the device sampler's order -- 1024 threads x 32 consecutive entries; T_t the
 * sequential sum of thread t's entries, W_w the sequential sum of T_32w..T_32w+31, Q the
 * running sum over the W's; the running sum at entry i of thread t = Q_w + T_32w + ... +
 * T_t-1 + thread t's entries up to i -- with q35_expf -- for the softmax normaliser; the
 * running sums over probabilities (top-p threshold, draw) are exact integer sums of
 * fx(p) = floor(p * 2^40), compared with fx(top_p) and fx(u).  Its top-p threshold is the
 * largest probability v whose fixed-point mass (the probabilities >= v) reaches
 * fx(top_p): the sorted running sum's crossing value. */
#define ORC_SNT 1024
#define ORC_SCH 32
static const uint64_t ORC_SAMPLE_STREAM = 0x53414D0000000000ull;

/* total of v[0,n) in the blocked order (the softmax normaliser of order 1) */
static float blocked_sum(const float *v, int32_t n) {
    float T[ORC_SNT], W[ORC_SNT / 32], Q[ORC_SNT / 32 + 1];
    for (int t = 0; t < ORC_SNT; ++t) {
        float a = 0.0f;
        for (int j = 0; j < ORC_SCH; ++j) {
            const int64_t i = (int64_t)t * ORC_SCH + j;
            if (i < n) a += v[i];
        }
        T[t] = a;
    }
    for (int w = 0; w < ORC_SNT / 32; ++w) {
        float a = 0.0f;
        for (int l = 0; l < 32; ++l) a += T[w * 32 + l];
        W[w] = a;
    }
    Q[0] = 0.0f;
    for (int w = 0; w < ORC_SNT / 32; ++w) Q[w + 1] = Q[w] + W[w];
    return Q[ORC_SNT / 32];
}

/* the reference's running sums (order 0): first i (0-based) whose sequential fp32 running
 * sum reaches bound -- "bound <= sum" over the entries > 0 (only_positive) or all of them,
 * or "sum >= bound" (ge_mode); n when none */
static int32_t first_crossing(const float *v, int32_t n, float bound, int only_positive, int ge_mode) {
    float cum = 0.0f;
    for (int32_t i = 0; i < n; ++i) {
        if (only_positive && !(v[i] > 0.0f)) continue;
        cum += v[i];
        if (ge_mode ? (cum >= bound) : (bound <= cum)) return i;
    }
    return n;
}

static uint64_t fx40(float p) {
    if (!(p > 0.0f)) return 0;
    const float v = p * 1099511627776.0f;                      /* 2^40, exact */
    if (v >= 18446744073709551616.0f) return UINT64_MAX;
    return (uint64_t)v;                                         /* truncation */
}

static int cmp_desc(const void *a, const void *b) {
    const float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

/* softmax (:35-59) of x into pr; e gets the exponentials; returns max */
static float softmax_into(const float *x, float *e, float *pr, int32_t V, int32_t order) {
    float mx = x[0];
    for (int32_t i = 1; i < V; ++i) mx = x[i] > mx ? x[i] : mx;
    float sum = 0.0f;
    for (int32_t i = 0; i < V; ++i) {
        e[i] = order ? q35_expf(x[i] - mx) : expf(x[i] - mx);
        if (!order) sum += e[i];
    }
    if (order) sum = blocked_sum(e, V);
    for (int32_t i = 0; i < V; ++i) pr[i] = sum > 0.0f ? e[i] / sum : 1.0f / (float)V;
    return mx;
}

float orc_sample_uniform(uint64_t seed, int32_t seq, int32_t n) {
    const uint64_t z = orc_rng_u64(seed, ORC_SAMPLE_STREAM + (uint64_t)seq, (uint64_t)n);
    return (float)(uint32_t)(z >> 40) * 0x1p-24f;
}

int32_t orc_sample(const float *logits, int32_t V, int32_t mode, float temperature, int32_t top_k, float top_p,
                   float u, int32_t order) {
    if (mode == 0) return orc_sample_greedy(logits, V);
    float *x = (float *)malloc(sizeof(float) * (size_t)V);
    float *e = (float *)malloc(sizeof(float) * (size_t)V);
    float *pr = (float *)malloc(sizeof(float) * (size_t)V);
    memcpy(x, logits, sizeof(float) * (size_t)V);
    if (mode == 1 && temperature > 0.0f)                       /* apply_temperature :25-29 */
        for (int32_t i = 0; i < V; ++i) x[i] = x[i] / temperature;
    if (mode == 2) {                                           /* :134-156 */
        float kth = -FLT_MAX;
        if (top_k >= 1 && top_k <= V) {   /* k rounds of max + mask = the k-th of a descending sort */
            memcpy(e, x, sizeof(float) * (size_t)V);
            qsort(e, (size_t)V, sizeof(float), cmp_desc);
            kth = e[top_k - 1];
        }
        for (int32_t i = 0; i < V; ++i)
            if (x[i] < kth) x[i] = -FLT_MAX;
    }
    softmax_into(x, e, pr, V, order);
    if (mode == 3) {                                           /* :194-242 */
        float *srt = (float *)malloc(sizeof(float) * (size_t)V);
        memcpy(srt, pr, sizeof(float) * (size_t)V);
        qsort(srt, (size_t)V, sizeof(float), cmp_desc);
        float thr;
        if (order == 0) {   /* :220-230 the running sum over the sorted probabilities */
            const int32_t i0 = first_crossing(srt, V, top_p, 0, 1);
            thr = i0 < V ? srt[i0] : 0.0f;
        } else {            /* fixed point: the first sorted entry whose running mass reaches fx(p) */
            thr = 0.0f;
            if (top_p == top_p) {
                const uint64_t target = fx40(top_p);
                uint64_t cum = 0;
                for (int32_t i = 0; i < V; ++i) {
                    cum += fx40(srt[i]);
                    if (cum >= target) { thr = srt[i]; break; }
                }
            }
        }
        for (int32_t i = 0; i < V; ++i) x[i] = pr[i] >= thr ? logits[i] : -FLT_MAX;
        softmax_into(x, e, pr, V, order);
        free(srt);
    }
    int32_t i = V;                                             /* :106-117, :162-175 */
    if (order == 0) {
        i = first_crossing(pr, V, u, mode != 1, 0);
    } else {
        const uint64_t ufx = fx40(u);
        uint64_t cum = 0;
        for (int32_t j = 0; j < V; ++j) {
            cum += fx40(pr[j]);
            if ((mode == 1 || pr[j] > 0.0f) && ufx <= cum) { i = j; break; }
        }
    }
    free(x); free(e); free(pr);
    return i < V ? i + 1 : V;
}

/* ------------------------------------------------------------------------------ */
/* Model                                                                            */
/* ------------------------------------------------------------------------------ */
struct orc_model {
    orc_config cfg;
    orc_layer_weights *layers;
    const float *embed, *final_norm, *lm_head;
    float *freqs;           /* (max_seq, head_dim/2) */
    float **kc, **vc;       /* per layer (max_seq, kv_heads, head_dim) */
    int32_t *cache_pos;
};

orc_model *orc_model_create(const orc_config *cfg, const orc_layer_weights *layers,
                            const float *embed, const float *final_norm, const float *lm_head) {
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->cfg = *cfg;
    m->layers = (orc_layer_weights *)malloc(sizeof(orc_layer_weights) * cfg->n_layers);
    memcpy(m->layers, layers, sizeof(orc_layer_weights) * cfg->n_layers);
    m->embed = embed;
    m->final_norm = final_norm;
    m->lm_head = lm_head;
    m->freqs = (float *)malloc(sizeof(float) * (size_t)cfg->max_seq * (cfg->head_dim / 2));
    orc_rope_freqs(m->freqs, cfg->max_seq, cfg->head_dim, cfg->rope_theta);
    size_t csz = (size_t)cfg->max_seq * cfg->n_kv_heads * cfg->head_dim;
    m->kc = (float **)malloc(sizeof(float *) * cfg->n_layers);
    m->vc = (float **)malloc(sizeof(float *) * cfg->n_layers);
    m->cache_pos = (int32_t *)calloc(cfg->n_layers, sizeof(int32_t));
    for (int32_t l = 0; l < cfg->n_layers; ++l) {
        m->kc[l] = (float *)calloc(csz, sizeof(float));
        m->vc[l] = (float *)calloc(csz, sizeof(float));
    }
    return m;
}

void orc_model_destroy(orc_model *m) {
    if (!m) return;
    for (int32_t l = 0; l < m->cfg.n_layers; ++l) { free(m->kc[l]); free(m->vc[l]); }
    free(m->kc); free(m->vc); free(m->cache_pos); free(m->freqs); free(m->layers); free(m);
}

/* transformer_layer.f90:145-150 */
void orc_model_reset(orc_model *m) {
    size_t csz = (size_t)m->cfg.max_seq * m->cfg.n_kv_heads * m->cfg.head_dim;
    for (int32_t l = 0; l < m->cfg.n_layers; ++l) {
        m->cache_pos[l] = 0;
        memset(m->kc[l], 0, csz * sizeof(float));
        memset(m->vc[l], 0, csz * sizeof(float));
    }
}

/* order 2: sum of a[i*sa] * b[i*sb] over i < n in 8 fused lanes, combined by halving */
static float dot8(const float *a, int64_t sa, const float *b, int64_t sb, int64_t n) {
    float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = 0; i < n; ++i) l[i & 7] = fmaf(a[i * sa], b[i * sb], l[i & 7]);
    for (int h = 4; h > 0; h >>= 1)
        for (int q = 0; q < h; ++q) l[q] = l[q] + l[q + h];
    return l[0];
}

/* order 2: plain sum of v[i*sv] over i < n in 8 lanes, combined by halving */
static float sum8(const float *v, int64_t sv, int64_t n) {
    float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = 0; i < n; ++i) l[i & 7] = l[i & 7] + v[i * sv];
    for (int h = 4; h > 0; h >>= 1)
        for (int q = 0; q < h; ++q) l[q] = l[q] + l[q + h];
    return l[0];
}

/* transformer_layer.f90:155-178 with the sum of squares in order 2 */
static void rms_norm_vec8(const float *x, const float *w, float *out, int32_t S, int32_t dim, float eps) {
    for (int32_t i = 0; i < S; ++i) {
        float r = dot8(x + i, S, x + i, S, dim);
        r = sqrtf(r / (float)dim + eps);
        for (int32_t j = 0; j < dim; ++j) out[i + (int64_t)S * j] = (x[i + (int64_t)S * j] / r) * w[j];
    }
}

static void norm(const orc_model *m, const float *x, const float *w, float *out, int32_t S) {
    if (m->cfg.order == 1) orc_rms_norm_tree(x, w, out, S, m->cfg.hidden, m->cfg.rms_eps);
    else if (m->cfg.order == 2) rms_norm_vec8(x, w, out, S, m->cfg.hidden, m->cfg.rms_eps);
    else orc_rms_norm(x, w, out, S, m->cfg.hidden, m->cfg.rms_eps);
}

static void linear(const orc_model *m, const float *x, const int8_t *w, const float *s,
                   const float *o, float *out, int32_t S, int32_t N, int32_t K) {
    orc_q35_linear(x, w, s, o, out, S, N, K, m->cfg.wformat);
}

/* transformer_layer.f90:183-205 apply_rope_single on x(S,nh,hd); position index pos0+i */
static void rope(const orc_model *m, float *x, int32_t S, int32_t nh, int32_t pos0) {
    const int32_t hd = m->cfg.head_dim, ms = m->cfg.max_seq;
    for (int32_t i = 0; i < S; ++i)
        for (int32_t h = 0; h < nh; ++h)
            for (int32_t d = 0; d < hd / 2; ++d) {
                float f = m->freqs[(pos0 + i) + (int64_t)ms * d];
                float c = cosf(f), sn = sinf(f);
                float *xr = &x[i + (int64_t)S * (h + (int64_t)nh * (2 * d))];
                float *xi = &x[i + (int64_t)S * (h + (int64_t)nh * (2 * d + 1))];
                float a = *xr, b = *xi;
                *xr = a * c - b * sn;
                *xi = a * sn + b * c;
            }
}

/* transformer_layer.f90:333-402 in the tree order of the GPU kernels: keys in chunks of
 * 64; per key a 32-lane dot (lane l: dims 128t+4l..+3 in one fused chain, t over D/128),
 * butterfly, times the scale; per chunk the max, q35_expf(s - max), a lane-strided sum
 * with butterfly and o = sum_j e_j v_j (fused, in j order); then the chunks merged with
 * q35_expf(m_c - M) and the sum normalised.  Keys j > pos (masked to -1e9 in the
 * reference) carry weight 0 and are skipped. */
enum { ORC_CHUNK = 64 };
static void attention_tree(const orc_model *m, const float *q, const float *kc, const float *vc, float *ao,
                           int32_t S, int32_t cp, float scale) {
    const orc_config *c = &m->cfg;
    const int32_t H = c->n_heads, KVH = c->n_kv_heads, D = c->head_dim, ms = c->max_seq;
    const int32_t grp = H / KVH, nchunk = (ms + ORC_CHUNK - 1) / ORC_CHUNK, D4 = D / 128;
#pragma omp parallel for schedule(static)
    for (int32_t h = 0; h < H; ++h) {
        const int32_t kvh = h / grp;
        float *om = (float *)malloc(sizeof(float) * (size_t)nchunk * (D + 2));
        float qv[256], kv[256], sc[ORC_CHUNK], v[32];
        for (int32_t i = 0; i < S; ++i) {
            const int32_t pos = cp + i;
            for (int32_t d = 0; d < D; ++d) qv[d] = q[i + (int64_t)S * (h + (int64_t)H * d)];
            for (int32_t ch = 0; ch < nchunk; ++ch) {
                float *o = om + (size_t)ch * (D + 2);
                const int32_t j0 = ch * ORC_CHUNK;
                int32_t nj = pos + 1 - j0;
                if (nj > ORC_CHUNK) nj = ORC_CHUNK;
                if (nj <= 0) { o[D] = -INFINITY; o[D + 1] = 0.0f; continue; }
                for (int32_t jj = 0; jj < nj; ++jj) {
                    const int32_t j = j0 + jj;
                    for (int32_t d = 0; d < D; ++d) kv[d] = kc[j + (int64_t)ms * (kvh + (int64_t)KVH * d)];
                    for (int l = 0; l < 32; ++l) {
                        float a = 0.0f;
                        for (int32_t t = 0; t < D4; ++t) {
                            const int32_t b = 128 * t + 4 * l;
                            a = fmaf(qv[b], kv[b], fmaf(qv[b + 1], kv[b + 1], fmaf(qv[b + 2], kv[b + 2], fmaf(qv[b + 3], kv[b + 3], a))));
                        }
                        v[l] = a;
                    }
                    sc[jj] = butterfly_sum(v) * scale;
                }
                float mx = -INFINITY;
                for (int32_t jj = 0; jj < nj; ++jj) mx = fmaxf(mx, sc[jj]);
                for (int32_t jj = 0; jj < nj; ++jj) sc[jj] = q35_expf(sc[jj] - mx);
                for (int l = 0; l < 32; ++l) {
                    float s = 0.0f;
                    for (int32_t jj = l; jj < nj; jj += 32) s = s + sc[jj];
                    v[l] = s;
                }
                o[D] = mx;
                o[D + 1] = butterfly_sum(v);
                for (int32_t d = 0; d < D; ++d) {
                    float a = 0.0f;
                    for (int32_t jj = 0; jj < nj; ++jj)
                        a = fmaf(sc[jj], vc[(j0 + jj) + (int64_t)ms * (kvh + (int64_t)KVH * d)], a);
                    o[d] = a;
                }
            }
            float M = -INFINITY;
            for (int32_t ch = 0; ch < nchunk; ++ch) M = fmaxf(M, om[(size_t)ch * (D + 2) + D]);
            float L = 0.0f;
            for (int32_t ch = 0; ch < nchunk; ++ch) {
                const float mc = om[(size_t)ch * (D + 2) + D];
                if (mc != -INFINITY) L = fmaf(om[(size_t)ch * (D + 2) + D + 1], q35_expf(mc - M), L);
            }
            for (int32_t d = 0; d < D; ++d) {
                float a = 0.0f;
                for (int32_t ch = 0; ch < nchunk; ++ch) {
                    const float mc = om[(size_t)ch * (D + 2) + D];
                    if (mc != -INFINITY) a = fmaf(om[(size_t)ch * (D + 2) + d], q35_expf(mc - M), a);
                }
                ao[i + (int64_t)S * (h + (int64_t)H * d)] = a / L;
            }
        }
        free(om);
    }
}

/* transformer_layer.f90:235-438 grouped_query_attention (weights-allocated branch) */
static void gqa(orc_model *m, int32_t l, const float *xn, float *out, int32_t S) {
    const orc_config *c = &m->cfg;
    const orc_layer_weights *w = &m->layers[l];
    const int32_t H = c->n_heads, KVH = c->n_kv_heads, D = c->head_dim, ms = c->max_seq;
    const int32_t hid = c->hidden, QN = H * D, KN = KVH * D;
    float *q = (float *)malloc(sizeof(float) * (size_t)S * QN);   /* (S,H,D) == q_flat (S,H*D)? */
    float *kf = (float *)malloc(sizeof(float) * (size_t)S * KN);
    float *vf = (float *)malloc(sizeof(float) * (size_t)S * KN);
    float *qf = (float *)malloc(sizeof(float) * (size_t)S * QN);
    float *k = (float *)malloc(sizeof(float) * (size_t)S * KN);
    float *v = (float *)malloc(sizeof(float) * (size_t)S * KN);
    float *ao = (float *)malloc(sizeof(float) * (size_t)S * QN);
    linear(m, xn, w->wq, w->sq, w->oq, qf, S, QN, hid);                 /* :269-274 */
    linear(m, xn, w->wk, w->sk, w->ok, kf, S, KN, hid);
    linear(m, xn, w->wv, w->sv, w->ov, vf, S, KN, hid);
    /* :277-289 reshape q_flat(i,(h-1)*D+d) -> q(i,h,d) ; q(S,H,D) col-major */
    for (int32_t i = 0; i < S; ++i) {
        for (int32_t h = 0; h < H; ++h)
            for (int32_t d = 0; d < D; ++d)
                q[i + (int64_t)S * (h + (int64_t)H * d)] = qf[i + (int64_t)S * (h * D + d)];
        for (int32_t h = 0; h < KVH; ++h)
            for (int32_t d = 0; d < D; ++d) {
                k[i + (int64_t)S * (h + (int64_t)KVH * d)] = kf[i + (int64_t)S * (h * D + d)];
                v[i + (int64_t)S * (h + (int64_t)KVH * d)] = vf[i + (int64_t)S * (h * D + d)];
            }
    }
    int32_t cp = m->cache_pos[l];
    int32_t pos0 = c->rope_mode ? cp : 0;
    rope(m, q, S, H, pos0);                                              /* :313 */
    rope(m, k, S, KVH, pos0);                                            /* :315 */
    float *kc = m->kc[l], *vc = m->vc[l];
    for (int32_t i = 0; i < S; ++i)                                      /* :322-329 */
        for (int32_t h = 0; h < KVH; ++h)
            for (int32_t d = 0; d < D; ++d) {
                int64_t ci = (cp + i) + (int64_t)ms * (h + (int64_t)KVH * d);
                kc[ci] = k[i + (int64_t)S * (h + (int64_t)KVH * d)];
                vc[ci] = v[i + (int64_t)S * (h + (int64_t)KVH * d)];
            }
    const int32_t T = cp + S;                                            /* :333 */
    const float scale = 1.0f / sqrtf((float)D);                          /* :336 */
    const int32_t grp = H / KVH;
    (void)T;
    const int vec = c->order == 2;
    if (c->order == 1) {
        attention_tree(m, q, kc, vc, ao, S, cp, scale);
    } else {
#pragma omp parallel for schedule(static)
    for (int32_t h = 0; h < H; ++h) {                                    /* :340 */
        int32_t kvh = h / grp;                                           /* :342 */
        float *sc = (float *)malloc(sizeof(float) * (size_t)T);
        for (int32_t i = 0; i < S; ++i) {
            for (int32_t j = 0; j < T; ++j) {                            /* :347-366 */
                float s = 0.0f;
                if (vec) {
                    s = dot8(q + i + (int64_t)S * h, (int64_t)S * H, kc + j + (int64_t)ms * kvh,
                             (int64_t)ms * KVH, D);
                } else {
                    for (int32_t d = 0; d < D; ++d) {
                        float kv = kc[j + (int64_t)ms * (kvh + (int64_t)KVH * d)];
                        s = s + q[i + (int64_t)S * (h + (int64_t)H * d)] * kv;
                    }
                }
                s = s * scale;
                if (j + 1 > cp + i + 1) s = -1.0e9f;                     /* :363 */
                sc[j] = s;
            }
            float mx = sc[0];                                            /* :369 maxval */
            for (int32_t j = 1; j < T; ++j) if (sc[j] > mx) mx = sc[j];
            float se = 0.0f;
            for (int32_t j = 0; j < T; ++j) { sc[j] = expf(sc[j] - mx); se = se + sc[j]; }
            if (vec) se = sum8(sc, 1, T);
            if (se > 0.0f)
                for (int32_t j = 0; j < T; ++j) sc[j] = sc[j] / se;      /* :376-378 */
            for (int32_t d = 0; d < D; ++d) {                            /* :388-400 */
                float a = 0.0f;
                if (vec) {
                    a = dot8(sc, 1, vc + (int64_t)ms * (kvh + (int64_t)KVH * d), 1, T);
                } else {
                    for (int32_t j = 0; j < T; ++j)
                        a = a + sc[j] * vc[j + (int64_t)ms * (kvh + (int64_t)KVH * d)];
                }
                ao[i + (int64_t)S * (h + (int64_t)H * d)] = a;
            }
        }
        free(sc);
    }
    }
    for (int32_t i = 0; i < S; ++i)                                      /* :406-412 */
        for (int32_t h = 0; h < H; ++h)
            for (int32_t d = 0; d < D; ++d)
                qf[i + (int64_t)S * (h * D + d)] = ao[i + (int64_t)S * (h + (int64_t)H * d)];
    linear(m, qf, w->wo, w->so, w->oo, out, S, hid, QN);                 /* :415-417 */
    m->cache_pos[l] = cp + S;                                            /* :424-426 */
    free(q); free(kf); free(vf); free(qf); free(k); free(v); free(ao);
}

/* transformer_layer.f90:443-520 swiglu_ffn (weights-allocated branch) */
static void ffn(orc_model *m, int32_t l, const float *xn, float *out, int32_t S) {
    const orc_config *c = &m->cfg;
    const orc_layer_weights *w = &m->layers[l];
    const int32_t F = c->ffn, hid = c->hidden;
    float *g = (float *)malloc(sizeof(float) * (size_t)S * F);
    float *u = (float *)malloc(sizeof(float) * (size_t)S * F);
    linear(m, xn, w->wg, w->sg, w->og, g, S, F, hid);
    linear(m, xn, w->wu, w->su, w->ou, u, S, F, hid);
    for (int64_t t = 0; t < (int64_t)S * F; ++t)                                  /* :226-228 */
        g[t] = (m->cfg.order == 1 ? swish_q35(g[t]) : orc_swish(g[t])) * u[t];
    linear(m, g, w->wd, w->sd, w->od, out, S, hid, F);
    free(g); free(u);
}

/* transformer_layer.f90:527-565 apply_transformer_layer */
void orc_layer_forward(orc_model *m, int32_t l, const float *x, float *out, int32_t S) {
    const int32_t hid = m->cfg.hidden;
    const orc_layer_weights *w = &m->layers[l];
    size_t n = (size_t)S * hid;
    float *xn = (float *)malloc(sizeof(float) * n);
    float *ao = (float *)malloc(sizeof(float) * n);
    float *fo = (float *)malloc(sizeof(float) * n);
    float *res = (float *)malloc(sizeof(float) * n);
    norm(m, x, w->attn_norm, xn, S);                                     /* :546 */
    gqa(m, l, xn, ao, S);                                                /* :547 */
    for (size_t t = 0; t < n; ++t) res[t] = x[t] + ao[t];                /* :550 */
    norm(m, res, w->ffn_norm, xn, S);                                    /* :553 */
    ffn(m, l, xn, fo, S);                                                /* :554 */
    for (size_t t = 0; t < n; ++t) out[t] = res[t] + fo[t];              /* :557 */
    free(xn); free(ao); free(fo); free(res);
}

/* llama_model.f90:105-147 forward_llama */
void orc_forward(orc_model *m, const int32_t *ids, int32_t S, float *logits) {
    const orc_config *c = &m->cfg;
    const int32_t hid = c->hidden, V = c->vocab;
    size_t n = (size_t)S * hid;
    float *x = (float *)malloc(sizeof(float) * n);
    float *y = (float *)malloc(sizeof(float) * n);
    for (int32_t i = 0; i < S; ++i)                                      /* :123-125 */
        for (int32_t j = 0; j < hid; ++j)
            x[i + (int64_t)S * j] = m->embed[(ids[i] - 1) + (int64_t)V * j];
    for (int32_t l = 0; l < c->n_layers; ++l) {                          /* :128-131 */
        orc_layer_forward(m, l, x, y, S);
        memcpy(x, y, sizeof(float) * n);
    }
    norm(m, x, m->final_norm, y, S);                                     /* :134 */
#pragma omp parallel for schedule(static)
    for (int32_t j = 0; j < V; ++j)                                      /* :138-140 */
        for (int32_t i = 0; i < S; ++i) {
            const float *wc = m->lm_head + (int64_t)hid * j;
            if (c->order == 2) {
                logits[i + (int64_t)S * j] = dot8(y + i, S, wc, 1, hid);
            } else if (c->order) {   /* lane l: k = 4l + 128t, one fused chain; then butterfly */
                float v[32];
                for (int l = 0; l < 32; ++l) {
                    float a = 0.0f;
                    for (int32_t k = 4 * l; k < hid; k += 128)
                        a = fmaf(wc[k], y[i + (int64_t)S * k],
                                 fmaf(wc[k + 1], y[i + (int64_t)S * (k + 1)],
                                      fmaf(wc[k + 2], y[i + (int64_t)S * (k + 2)],
                                           fmaf(wc[k + 3], y[i + (int64_t)S * (k + 3)], a))));
                    v[l] = a;
                }
                logits[i + (int64_t)S * j] = butterfly_sum(v);
            } else {
                float a = 0.0f;
                for (int32_t k = 0; k < hid; ++k) a = a + y[i + (int64_t)S * k] * wc[k];
                logits[i + (int64_t)S * j] = a;
            }
        }
    free(x); free(y);
}

/* llama_generate.f90:76-123 with greedy sampling (temperature 0) */
int32_t orc_generate(orc_model *m, const int32_t *prompt, int32_t prompt_len, int32_t n_steps,
                     int32_t stop_at_eos, const orc_sampling *smp, int32_t seq, int32_t *out_tokens,
                     float *all_logits) {
    const int32_t V = m->cfg.vocab;
    float *lg = (float *)malloc(sizeof(float) * (size_t)V * prompt_len);
    float *last = (float *)malloc(sizeof(float) * (size_t)V);
    int32_t total = prompt_len, produced = 0, tok = 0;
    for (int32_t it = 0; it < n_steps; ++it) {
        if (it == 0) {
            orc_forward(m, prompt, prompt_len, lg);
            for (int32_t j = 0; j < V; ++j) last[j] = lg[(prompt_len - 1) + (int64_t)prompt_len * j];
        } else {
            orc_forward(m, &tok, 1, last);
        }
        if (all_logits) memcpy(all_logits + (int64_t)V * it, last, sizeof(float) * V);
        int32_t nt;
        if (!smp || smp->mode == 0)
            nt = orc_sample_greedy(last, V);
        else
            nt = orc_sample(last, V, smp->mode, smp->temperature, smp->top_k, smp->top_p,
                            orc_sample_uniform(smp->seed, seq, it), m->cfg.order == 1);
        if (stop_at_eos && nt == 2) break;                               /* :101 */
        total += 1;
        if (total > m->cfg.max_seq) break;                               /* :109-113 */
        out_tokens[produced++] = nt;
        tok = nt;
    }
    free(lg); free(last);
    return produced;
}

int32_t orc_generate_greedy(orc_model *m, const int32_t *prompt, int32_t prompt_len,
                            int32_t n_steps, int32_t stop_at_eos, int32_t *out_tokens,
                            float *all_logits) {
    return orc_generate(m, prompt, prompt_len, n_steps, stop_at_eos, NULL, 0, out_tokens, all_logits);
}

void orc_set_threads(int32_t n) {
#ifdef _OPENMP
    omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int32_t orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
