/*
 * q35_oracle.h -- CPU restatement of asicForTranAI's quantized-matmul hot path and
 * the LLaMA decode loop that consumes it.
 *
 * TEST INFRASTRUCTURE ONLY.  The test suite, the smoke check and the CPU-baseline leg
 * of bench.py call it to produce expected results.
 * The product (libq35.so) never links, loads or calls anything in this directory.
 *
 * Every array follows the reference's Fortran (column-major) layout:
 *   A(M,K)      element (i,k) at A[i + M*k]          (0-based i,k)
 *   W_Q(K/2,N)  element (p,j) at W_Q[p + (K/2)*j]     (column j holds K/2 bytes)
 *   C(M,N)      element (i,j) at C[i + M*j]
 * Floating point is plain IEEE binary32 with no contraction (-ffp-contract=off); the
 * fp32 reductions of the model run in the source's sequential order or in the GPU
 * kernels' tree order (orc_config.order).
 */
#ifndef Q35_ORACLE_H
#define Q35_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- synthetic input generator (SplitMix64, counter based) ------------------- */
uint64_t orc_rng_u64(uint64_t seed, uint64_t tensor_id, uint64_t index);
void orc_gen_int8(int8_t *out, int64_t n, uint64_t seed, uint64_t tensor_id);      /* uniform [-127,127] */
void orc_gen_normal(float *out, int64_t n, uint64_t seed, uint64_t tensor_id, double sigma);
void orc_gen_tokens(int32_t *out, int64_t n, uint64_t seed, uint64_t tensor_id, int32_t vocab); /* [1,vocab] */

/* ---- quantizers (offline tooling of the reference) ---------------------------- */
/* W fp32 (K,N) column-major -> W_Q int8 (K/2,N), scales[N], offsets[N].  K even. */
void orc_quantize_3p5bit_asym(const float *W, int8_t *W_Q, float *scales, float *offsets,
                              int32_t K, int32_t N);
/* symmetric per-column absmax/7 INT4, nibble-packed low nibble first */
void orc_quantize_int4_sym(const float *W, int8_t *W_Q, float *scales, int32_t K, int32_t N);

/* ---- quantized matmul kernels -------------------------------------------------- */
/* mode 0: pair index (k+1)/2 (the indexing every other reference implementation uses);
 * mode 1: the 1-byte shift of matmul_3p5bit_dynamic.f90:47 ((k+0)/2, byte before
 *         column 1 taken as 0) -- diagnostic only. */
void orc_matmul_3p5bit_awq(const int8_t *A, const int8_t *W_Q, const float *scales,
                           const float *offsets, int32_t *C, int32_t M, int32_t N, int32_t K,
                           int32_t mode);
void orc_dequantize_output_3p5bit(const int32_t *C, const float *scales, const float *offsets,
                                  float *Out, int32_t M, int32_t N);
void orc_matmul_int4_awq(const int8_t *A, const int8_t *W_Q, const float *scales, int32_t *C,
                         int32_t M, int32_t N, int32_t K);
/* matmul_simd_optimized.f90:24-112 (the reference's SIMD/OpenMP INT4 kernel, same sums) */
void orc_matmul_int4_simd(const int8_t *A, const int8_t *W_Q, const float *scales, int32_t *C,
                          int32_t M, int32_t N, int32_t K);
void orc_dequantize_output(const int32_t *C, const float *scales, float *Out, int32_t M, int32_t N);
/* int4_linear: x fp32 (M,K) -> int8 trunc(clamp(x*127)) -> matmul -> dequant */
void orc_quantize_activations(const float *x, int8_t *x_int8, int64_t n);
void orc_q35_linear(const float *x, const int8_t *W_Q, const float *scales, const float *offsets,
                    float *out, int32_t M, int32_t N, int32_t K, int32_t wformat);

/* ---- transformer pieces --------------------------------------------------------- */
void orc_rms_norm(const float *x, const float *w, float *out, int32_t S, int32_t dim, float eps);
/* rms_norm with the sum of squares in the blocked/tree order (1024 partial sums over
 * float4 groups, then 32-lane butterflies) */
void orc_rms_norm_tree(const float *x, const float *w, float *out, int32_t S, int32_t dim, float eps);
float orc_q35_expf(float x);
float orc_swish(float x);
/* rope angle table: freqs[pos + max_seq*d] = (pos)*theta_d, pos 0-based */
void orc_rope_freqs(float *freqs, int32_t max_seq, int32_t head_dim, float theta);
int32_t orc_sample_greedy(const float *logits, int32_t vocab); /* 1-based */
/* sample_temperature / sample_top_k / sample_top_p (sampling.f90:88-259), mode 1/2/3
 * (0: greedy), u the uniform draw that replaces random_number; order 0 = the source's
 * sequential sums with expf, 1 = the device sampler's blocked order with q35_expf */
int32_t orc_sample(const float *logits, int32_t vocab, int32_t mode, float temperature, int32_t top_k,
                   float top_p, float u, int32_t order);
/* the draw of sequence seq's n-th sampled token in a model run (seed, 0x53414D0000000000+seq, n) */
float orc_sample_uniform(uint64_t seed, int32_t seq, int32_t n);
typedef struct {
    int32_t mode;
    float temperature;
    int32_t top_k;
    float top_p;
    uint64_t seed;
} orc_sampling;

typedef struct {
    int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_seq;
    float rms_eps, rope_theta;
    int32_t rope_mode; /* 0: position within the call (reference), 1: absolute position */
    int32_t wformat;   /* 0: 3.5-bit asymmetric, 1: INT4 symmetric */
    int32_t order;     /* fp32 reduction order: 0 = the reference source's sequential loops
                          with the C library's expf; 1 = the blocked/tree order of the GPU
                          kernels with q35_expf (q35_expf.h) */
} orc_config;

/* weights of one layer; packed matrices in W_Q(K/2,N) layout */
typedef struct {
    const int8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *sq, *sk, *sv, *so, *sg, *su, *sd; /* scales */
    const float *oq, *ok, *ov, *oo, *og, *ou, *od; /* offsets (3.5-bit) */
    const float *attn_norm, *ffn_norm;
} orc_layer_weights;

typedef struct orc_model orc_model;
orc_model *orc_model_create(const orc_config *cfg, const orc_layer_weights *layers,
                            const float *embed /* (vocab,hidden) col-major */,
                            const float *final_norm, const float *lm_head /* (hidden,vocab) */);
void orc_model_destroy(orc_model *m);
void orc_model_reset(orc_model *m);
/* forward_llama: token ids (1-based) of S positions -> logits (S,vocab) col-major */
void orc_forward(orc_model *m, const int32_t *ids, int32_t S, float *logits);
/* one transformer layer on x (S,hidden) in place (debug / layer parity) */
void orc_layer_forward(orc_model *m, int32_t layer, const float *x, float *out, int32_t S);
/* generation: prefill prompt, then n_steps greedy tokens; out_tokens[n_steps];
 * last_logits (vocab) of the final step when non-NULL.  Returns tokens produced. */
int32_t orc_generate_greedy(orc_model *m, const int32_t *prompt, int32_t prompt_len,
                            int32_t n_steps, int32_t stop_at_eos, int32_t *out_tokens,
                            float *all_logits /* (vocab, n_steps) or NULL */);
/* the same with the next token drawn by smp (NULL: greedy) from the draws of sequence seq */
int32_t orc_generate(orc_model *m, const int32_t *prompt, int32_t prompt_len, int32_t n_steps,
                     int32_t stop_at_eos, const orc_sampling *smp, int32_t seq, int32_t *out_tokens,
                     float *all_logits);

void orc_set_threads(int32_t n);
int32_t orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
