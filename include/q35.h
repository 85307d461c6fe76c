/*
 * q35.h -- C ABI of libq35, a B200 (sm_100a) implementation of asicForTranAI's
 * quantized-matmul hot path (3.5-bit and INT4 weights, int8 activations, exact int32
 * accumulation, per-column fp32 dequant) and of the LLaMA decode loop built on it.
 *
 * Plain C types only.  Every q35_* function returns a status (Q35_OK == 0); the
 * message of the last failure on the calling thread is q35_last_error().
 *
 * Array layouts follow the reference's Fortran modules (column-major):
 *   A(M,K) int8 at A[i + M*k];  W_Q(K/2,N) int8 at W_Q[p + (K/2)*j];
 *   C(M,N) int32 and Out(M,N) fp32 at [i + M*j].
 * Reference files are named relative to the reference project's directory
 * 2025-3.5bit-groq-mvp/.
 */
#ifndef Q35_H
#define Q35_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    Q35_OK = 0,
    Q35_ERR_INVALID = 1,   /* bad argument (size, layout, null pointer) */
    Q35_ERR_CUDA = 2,      /* CUDA runtime error */
    Q35_ERR_NOMEM = 3,     /* device or host allocation failed */
    Q35_ERR_NCCL = 4,      /* NCCL error */
    Q35_ERR_TIMEOUT = 5,   /* a bounded device wait gave up */
    Q35_ERR_STATE = 6      /* call not valid in the object's current state */
};

enum { Q35_FMT_3P5BIT = 0, Q35_FMT_INT4 = 1 };

/* activation / output layouts for the device-pointer entry points */
enum {
    Q35_LAYOUT_COLMAJOR = 0, /* reference layout: (i,k) at i + M*k ; (i,j) at i + M*j */
    Q35_LAYOUT_ROWMAJOR = 1  /* (i,k) at i*K + k ; (i,j) at i*N + j */
};

/* which engine runs a matmul (q35_ctx_set_gemm_path) */
enum {
    Q35_PATH_AUTO = 0,         /* CUDA cores for M <= 4 rows, tensor cores from 5 rows on */
    Q35_PATH_CUDA_CORES = 1,   /* dp4a GEMV, 64 rows per launch */
    Q35_PATH_TENSOR_CORES = 2  /* tcgen05 kind::i8 GEMM */
};

/* sampling strategies (sampling.f90) */
enum {
    Q35_SAMPLE_GREEDY = 0,       /* sample_greedy, sampling.f90:64-83 */
    Q35_SAMPLE_TEMPERATURE = 1,  /* sample_temperature, :88-118 */
    Q35_SAMPLE_TOP_K = 2,        /* sample_top_k, :123-176 */
    Q35_SAMPLE_TOP_P = 3         /* sample_top_p, :181-259 */
};

typedef struct q35_ctx_s *q35_ctx;         /* device, stream, split-K workspace */
typedef struct q35_weights_s *q35_weights; /* one device-resident quantized matrix */
typedef struct q35_graph_s *q35_graph;     /* an instantiated CUDA graph of captured calls */
typedef struct q35_tp_s *q35_tp;           /* tensor-parallel communicator (NCCL) */

const char *q35_last_error(void);
const char *q35_status_string(int status);
int q35_version(void);

/* Context: device ordinal and a CUDA stream (cudaStream_t, NULL = a new stream owned by
 * the context).  Calls on one context are serialised on its stream. */
int q35_ctx_create(int device, void *stream, q35_ctx *out);
int q35_ctx_destroy(q35_ctx ctx);
int q35_ctx_synchronize(q35_ctx ctx);
void *q35_ctx_stream(q35_ctx ctx);
/* Engine for the matmuls issued on this context (Q35_PATH_*); both compute the same
 * exact int32 sums.  No counterpart in the reference: its backends are chosen at build
 * time. */
int q35_ctx_set_gemm_path(q35_ctx ctx, int path);
/* Synchronise and report a device-side failure recorded by this context's kernels
 * (Q35_ERR_TIMEOUT when a bounded wait gave up); clears the record. */
int q35_ctx_device_error(q35_ctx ctx);
/* CUDA-graph capture of the calls issued on the context's stream between begin and end
 * (every call must have run once before, so that no allocation happens while
 * capturing); the graph replays them with one launch. */
int q35_ctx_capture_begin(q35_ctx ctx);
int q35_ctx_capture_end(q35_ctx ctx, q35_graph *out);
int q35_graph_launch(q35_graph graph, q35_ctx ctx);
int q35_graph_destroy(q35_graph graph);

/* Upload one packed matrix in the reference layout W_Q(K/2,N) with its per-column
 * scales[N] (and offsets[N] for 3.5-bit) and repack it on the device into the
 * streaming format.  Replaces dequantize_weights_gpu (matmul_cublas.f90:175-217), the
 * one-time upload of the cached cuBLAS path.  src_on_device != 0 when the three pointers
 * are device pointers.  K must be even and positive. */
int q35_weights_upload(q35_ctx ctx, int format, const int8_t *W_Q, const float *scales,
                       const float *offsets, int32_t N, int32_t K, int src_on_device,
                       q35_weights *out);
int q35_weights_free(q35_weights w);
size_t q35_weights_device_bytes(q35_weights w);
/* Unpack the device copy back to the reference layout (host pointer, (K/2)*N bytes):
 * a round trip check of the repack. */
int q35_weights_download_ref(q35_ctx ctx, q35_weights w, int8_t *W_Q_host);

/* Device-pointer matmul on the context's stream: x int8 (M,K) in x_layout, C int32 and
 * y fp32 (M,N) in out_layout; C or y may be NULL; 1 <= M <= 65536, K <= 131072.
 * y = (C + offset) * scale (3.5-bit, matmul_3p5bit_dynamic.f90:80) or C * scale (INT4,
 * matmul_int4_groq.f90:151).  Replaces matmul_3p5bit_awq + dequantize_output_3p5bit and
 * matmul_int4_awq + dequantize_output on device-resident data.  The tensor-core path
 * reads x through TMA: row-major x with K a multiple of 16 and a 16-byte aligned base is
 * read in place, other layouts are first copied row-major into the context's workspace.
 * Asynchronous. */
int q35_gemm_dev(q35_ctx ctx, q35_weights w, const int8_t *x, int32_t M, int x_layout,
                 int32_t *C, float *y, int out_layout);

/* q35_gemm_dev for callers that cannot allocate device memory -- real-time loops that
 * must not enter the driver's allocator (which can synchronise the device), processes
 * whose free HBM is owned by another allocator.  No counterpart in the reference.  Same
 * arguments and results as q35_gemm_dev (CUDA-core engine), on the caller's stream
 * (cudaStream_t), with the weights already resident; the split-K scratch is a fixed
 * ~4.1 MiB array inside the library (held on every GPU that loads it), so 1 <= M <= 64,
 * N <= 65536 and M * ceil(N/32)*32 <= 1,048,576, else Q35_ERR_INVALID.  The first call on
 * a device looks up the array's address: make it before any stream capture.  All calls
 * share the array: calls that overlap on the GPU race; each call clears the partial sums
 * and counters it uses first.  Allocates nothing. */
int q35_gemm_dev_noalloc(q35_weights w, const int8_t *x, int32_t M, int x_layout, int32_t *C,
                         float *y, int out_layout, void *stream);
/* Failure record of q35_gemm_dev_noalloc's kernels on the current device: synchronises
 * the stream, returns Q35_ERR_TIMEOUT when a bounded wait in one of them gave up since
 * the last read (their outputs are then incomplete), and clears the record.  No
 * counterpart in the reference.  Allocates nothing. */
int q35_gemm_noalloc_device_error(void *stream);

/* Host-pointer matmul against resident weights (the cached path,
 * matmul_int4_cublas_cached, matmul_cublas.f90:279-325): A(M,K) host int8, C(M,N)
 * host int32 and/or Out(M,N) host fp32 (either may be NULL).  Synchronous. */
int q35_matmul_cached(q35_ctx ctx, q35_weights w, const int8_t *A, int32_t M, int32_t *C,
                      float *Out);

/* ---- synthetic inputs and quantizers on the device (stream = cudaStream_t) ----
 * Counter-based SplitMix64 generator keyed by (seed, tensor_id): int8 uniform in
 * [-127,127], fp32 N(0, sigma^2) by Box-Muller in double, token ids in [1,vocab]. */
int q35_gen_int8_dev(int8_t *out, int64_t n, uint64_t seed, uint64_t tensor_id, void *stream);
int q35_gen_normal_dev(float *out, int64_t n, uint64_t seed, uint64_t tensor_id, double sigma,
                       void *stream);
int q35_gen_tokens_dev(int32_t *out, int64_t n, uint64_t seed, uint64_t tensor_id, int32_t vocab,
                       void *stream);
/* Device twin of quantize_3p5bit_asymmetric (convert_weights_3p5bit.py:19-85,
 * format Q35_FMT_3P5BIT) and of the symmetric absmax/7 INT4 quantizer
 * (benchmark_3p5bit.py:155-159, Q35_FMT_INT4): W fp32 (K,N) column-major ->
 * W_Q(K/2,N), scales[N], offsets[N] (3.5-bit only).  Bit-identical to the reference. */
int q35_quantize_dev(int format, const float *W, int8_t *W_Q, float *scales, float *offsets,
                     int32_t K, int32_t N, void *stream);
/* Random-init resident weights: W ~ N(0, sigma^2) generated, quantized and repacked on
 * the device (no host round trip). */
int q35_weights_generate(q35_ctx ctx, int format, int32_t N, int32_t K, uint64_t seed,
                         uint64_t tensor_id, double sigma, q35_weights *out);

/* ---- tensor parallelism: one process per GPU, NCCL over NVLink (new: the reference
 * has no parallel code) ---- */
/* 128-byte NCCL id made by rank 0 and passed to every rank (any side channel) */
int q35_tp_unique_id(void *out, size_t n);
/* join the communicator; a rank that does not join within timeout_s (<= 0: 120 s) makes
 * every other rank's call fail with Q35_ERR_TIMEOUT instead of hanging */
int q35_tp_create(q35_ctx ctx, int32_t rank, int32_t world, const void *id, size_t n, double timeout_s,
                  q35_tp *out);
/* Q35_ERR_STATE while models built on the group are alive (their decode graphs hold its
 * collectives): destroy them first */
int q35_tp_destroy(q35_tp tp);
/* abandon the communicator after a peer failed (ncclCommAbort): this rank's pending and
 * later collectives return errors instead of waiting; destroy it afterwards */
int q35_tp_abort(q35_tp tp);
int q35_tp_rank(q35_tp tp);
int q35_tp_world(q35_tp tp);
/* in-place int32 sum over the ranks on the context's stream (exact) */
/* The exchange of a row-parallel projection (o, down) in one call: C int32 [rows][N]
 * partial accumulators of this rank (device), summed over the group, then
 * x[rows][N] += (C + offsets) * scales (offsets NULL for INT4), on the context's stream.
 * Over NVLink peer memory when every rank mapped every peer at q35_tp_create (rows * N up
 * to 262,144), else NCCL.  Replaces the epilogue of the reference's
 * int4_linear (transformer_layer.f90:86-89) under tensor parallelism. */
int q35_tp_allreduce_dequant(q35_tp tp, q35_ctx ctx, int32_t *C, int64_t rows, int32_t N, const float *scales,
                             const float *offsets, float *x);
int q35_tp_allreduce_i32(q35_tp tp, q35_ctx ctx, int32_t *buf, size_t count);
/* failure-path self-test of the exchange's bounded waits on one GPU: runs the exchange
 * kernel against a peer that never writes; *observed = the status the kernel recorded
 * (Q35_ERR_TIMEOUT when the waits gave up as designed, after about a second); the context
 * stays usable */
int q35_tp_wait_selftest(q35_ctx ctx, int32_t *observed);
/* self-test of the exchange fused with the next RMSNorm (the tensor-parallel decode step's
 * form) on one GPU, one row, against the separate dequant + residual and RMSNorm kernels
 * on seeded inputs of width N (multiple of 4, up to 32768), three calls in a row;
 * *mismatches = the elements that differ in any bit (0 expected) */
int q35_tp_norm_selftest(q35_ctx ctx, int32_t N, uint64_t seed, int32_t *mismatches);
/* the same for R rows at once (1 <= R <= 64, R * N <= 262144, the decode batches): the
 * several-row form of the fused exchange and norm against the separate kernels */
int q35_tp_norm_selftest_rows(q35_ctx ctx, int32_t R, int32_t N, uint64_t seed, int32_t *mismatches);

/* ---- sampling (sampling.f90) on the device ----
 * One row of logits per CTA; the row's vocabulary is at most 32,768.  Tokens are 1-based.
 * random_number is replaced by the uniform draw u in [0,1), an argument here.  The
 * softmax normaliser is an fp32 sum in a fixed blocked order and the running sums (top-p
 * threshold, draw) are exact sums of the probabilities in 2^-40 fixed point, not the
 * reference's sequential fp32 loops: a draw within rounding distance of a cumulative
 * boundary may pick the neighbour token.
 * The host entry points mirror the reference functions (host logits[vocab]); they run on
 * ctx's stream (ctx NULL: the library's context of the current device, as the drop-in
 * matmuls) and return when *token is set. */
int q35_sample_greedy(q35_ctx ctx, const float *logits, int32_t vocab, int32_t *token);
int q35_sample_temperature(q35_ctx ctx, const float *logits, int32_t vocab, float temperature, float u,
                           int32_t *token);
int q35_sample_top_k(q35_ctx ctx, const float *logits, int32_t vocab, int32_t k, float u, int32_t *token);
int q35_sample_top_p(q35_ctx ctx, const float *logits, int32_t vocab, float p, float u, int32_t *token);
/* device rows: logits[rows][vocab] row-major, u[rows] (unused for greedy), tokens[rows];
 * enqueued on ctx's stream, no synchronisation */
int q35_sample_dev(q35_ctx ctx, int32_t mode, const float *logits, int32_t rows, int32_t vocab, float temperature,
                   int32_t top_k, float top_p, const float *u, int32_t *tokens);

/* ---- LLaMA model (llama_model.f90, transformer_layer.f90, llama_generate.f90) ---- */
typedef struct {
    int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_seq;
    float rms_eps;       /* RMS_NORM_EPS, transformer_layer.f90:26 */
    float rope_theta;    /* freq_base, transformer_layer.f90:109 */
    int32_t rope_mode;   /* 0: angle from the position within the call, as apply_rope_single
                            (transformer_layer.f90:193-196); 1: absolute position */
    int32_t wformat;     /* Q35_FMT_3P5BIT or Q35_FMT_INT4 */
    int32_t max_batch;   /* sequences decoded together (each has its own KV cache) */
} q35_model_config;

/* one layer in the reference layout: W_Q(K/2,N) bytes, scales[N], offsets[N] (3.5-bit;
 * NULL for INT4), norms[hidden] -- the TransformerLayer fields of
 * transformer_layer.f90:30-60 (wq,wk,wv,wo,w_gate,w_up,w_down + scales, attn/ffn norm) */
typedef struct {
    const int8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *sq, *sk, *sv, *so, *sg, *su, *sd;
    const float *oq, *ok, *ov, *oo, *og, *ou, *od;
    const float *attn_norm, *ffn_norm;
} q35_layer_weights;

typedef struct q35_model_s *q35_model;

/* init_llama_model (llama_model.f90:42-100): allocates weights, KV caches (max_batch x
 * n_layers x n_kv_heads x max_seq x head_dim, fp32, zeroed) and activations. */
int q35_model_create(q35_ctx ctx, const q35_model_config *cfg, q35_model *out);
/* the same, sharded over a tensor-parallel group (tp may be NULL: one GPU): rank r holds
 * query heads [r*H/t, (r+1)*H/t), KV heads [r*KVH/t, ...), FFN columns [r*F/t, ...) and
 * vocab rows [r*V/t, ...); o and down are split by rows and their int32 partial sums are
 * all-reduced before the dequant, so every rank's results equal the one-GPU results bit
 * for bit.  H, KVH, F and V must divide by t. */
int q35_model_create_tp(q35_ctx ctx, const q35_model_config *cfg, q35_tp tp, q35_model *out);
/* cleanup_llama_model (llama_model.f90:152-179) */
int q35_model_destroy(q35_model m);
/* load one layer's weights (weight_loader.f90 role), host pointers; attn_norm / ffn_norm
 * may be NULL to keep the current norms (1.0 after q35_model_create, as init_llama_model) */
int q35_model_set_layer(q35_model m, int32_t layer, const q35_layer_weights *w);
/* load_layer_weights (weight_loader.f90:18-182): one layer from the reference's
 * stream-binary file (generate_test_weights.f90:154-183): wq, wk, wv, wo, w_gate, w_up,
 * w_down, each W_Q(K/2,N) INT4 bytes column-major then scales[N] fp32; optionally followed
 * by attn_norm[hidden] and ffn_norm[hidden] fp32 (scripts/convert_weights_to_fortran.py
 * :94-121).  The model's format must be Q35_FMT_INT4; the file size is checked. */
int q35_model_load_layer_file(q35_model m, int32_t layer, const char *path);
/* the 3.5-bit safetensors checkpoint of convert_weights_3p5bit.py:105-139 (one or several
 * shard files): per layer l, model.layers.{l}.self_attn.{q,k,v,o}_proj.weight and
 * model.layers.{l}.mlp.{gate,up,down}_proj.weight as .weight_q (int8 [K/2][N] row-major),
 * .scales and .offsets (fp32 [N]), model.layers.{l}.input_layernorm.weight and
 * .post_attention_layernorm.weight; model.embed_tokens.weight and lm_head.weight
 * ([vocab][hidden], fp16/bf16/fp32, or quantized the same way and expanded as
 * code * scale + zero_point) and model.norm.weight.  The model's format must be
 * Q35_FMT_3P5BIT.  Under tensor parallelism each rank keeps its shard. */
int q35_model_load_safetensors(q35_model m, const char *const *paths, int32_t n_paths);
/* token_embeddings E(vocab,hidden), final_norm[hidden], output_weights(hidden,vocab),
 * column-major host arrays (llama_model.f90:21-30) */
int q35_model_set_embeddings(q35_model m, const float *embed, const float *final_norm,
                             const float *lm_head);
/* random-init weights on the device: every matrix N(0, sigma^2) quantized with the
 * model's format, norms, embeddings and LM head N(0, sigma^2) */
int q35_model_init_random(q35_model m, uint64_t seed, double sigma);
/* reset_kv_cache (transformer_layer.f90:145-150) for every layer and sequence */
int q35_model_reset(q35_model m);
/* forward_llama (llama_model.f90:105-147) of S tokens (1-based ids, host) of sequence
 * seq at its current position; logits (S, vocab) column-major host array or NULL (then
 * only the last position's logits are formed).  The last position's next token (greedy,
 * or drawn by the rule of q35_model_set_sampling) becomes the sequence's current token. */
int q35_model_forward(q35_model m, int32_t seq, const int32_t *ids, int32_t S, float *logits);
/* current token of every sequence (host [max_batch]) */
int q35_model_last_tokens(q35_model m, int32_t *tokens);
/* one decode step of all max_batch sequences (a CUDA graph after the first call): each
 * sequence's current token in (ids overrides them when non-NULL), next tokens (greedy or
 * sampled, q35_model_set_sampling) out to next[max_batch] and logits (max_batch, vocab)
 * column-major when non-NULL */
int q35_model_decode_step(q35_model m, const int32_t *ids, int32_t *next, float *logits);
/* n decode steps enqueued without host synchronisation */
int q35_model_decode_steps_async(q35_model m, int32_t n);
/* the generation loop of llama_generate.f90:76-123 (next tokens by the model's sampling,
 * greedy unless q35_model_set_sampling chose another) for all max_batch sequences:
 * prompts [max_batch][prompt_len], out_tokens [max_batch][n_steps],
 * n_out[max_batch] = tokens produced (stop_at_eos: up to the first token 2) */
int q35_model_generate(q35_model m, const int32_t *prompts, int32_t prompt_len, int32_t n_steps,
                       int32_t stop_at_eos, int32_t *out_tokens, int32_t *n_out);
/* how the model picks each next token (default greedy).  mode Q35_SAMPLE_*; the draw of
 * sequence b's n-th sampled token is u = (top 24 bits of the generator draw (seed,
 * 0x53414D0000000000 + b, n)) * 2^-24 (the q35_gen_* generator), so a run is reproducible
 * and a sequence's draws do not depend on the batch.  q35_model_reset and this call
 * restart every sequence's draw count.  llama_generate.f90:94-98 is mode TOP_P with
 * p = 0.95.  Sampling needs vocab <= 32,768. */
typedef struct {
    int32_t mode;
    float temperature;   /* TEMPERATURE mode */
    int32_t top_k;       /* TOP_K mode */
    float top_p;         /* TOP_P mode */
    uint64_t seed;
} q35_sampling;
int q35_model_set_sampling(q35_model m, const q35_sampling *cfg);
/* apply_transformer_layer (transformer_layer.f90:527-565) of one layer on host x(S,hidden)
 * column-major for sequence seq; advance != 0 moves the sequence's position by S */
int q35_model_layer_forward(q35_model m, int32_t layer, int32_t seq, const float *x, int32_t S,
                            float *out, int32_t advance);
size_t q35_model_weight_bytes(q35_model m);
/* copy the first `bytes` of an internal activation buffer to the host, for layer-level
 * checks: "x", "yqkv", "q", "ygu" (fp32, row-major [rows][width]; gate|up columns
 * interleaved), "xi8", "hq" (int8: matmul inputs; hq the down projection's), "kc",
 * "vc" (KV caches [seq][layer][kv_head][max_seq][head_dim]) */
int q35_model_debug_buffer(q35_model m, const char *name, void *host, size_t bytes);

/* ---- drop-in entry points with the reference's own signatures (host pointers) ----
 * They run on a default context of the current CUDA device, upload their inputs,
 * compute on the GPU and copy the results back before returning.  A failure is
 * reported through q35_last_error() and leaves the outputs untouched.  Empty operands
 * behave like the reference's loops: M = 0 or N = 0 succeeds without touching anything
 * (NULL pointers allowed), K = 0 gives C = 0 (and its dequantization); no device work. */

/* matmul_3p5bit_dynamic.f90:28-34  (bind(C), M/N/K by value); no status return: a failure
 * is also written to stderr (q35_matmul_3p5bit_awq below returns it) */
void matmul_3p5bit_awq(const int8_t *A, const int8_t *W_Q, const float *W_scales,
                       const float *W_offsets, int32_t *C, int32_t M, int32_t N, int32_t K);
/* matmul_3p5bit_dynamic.f90:69-74  (M, N by value) */
int q35_dequantize_output_3p5bit(const int32_t *C, const float *W_scales,
                                 const float *W_offsets, float *Out, int32_t M, int32_t N);
/* matmul_int4_groq.f90:19-25 (M, N, K_dim by reference in Fortran; passed by value here,
 * the Fortran shim dereferences) */
int q35_matmul_int4_awq(const int8_t *A, const int8_t *W_Q, const float *W_scales, int32_t *C,
                        int32_t M, int32_t N, int32_t K);
/* matmul_int4_groq.f90:58-62 */
int q35_dequantize_output(const int32_t *C, const float *W_scales, float *Out, int32_t M,
                          int32_t N);
/* matmul_3p5bit_awq with status return */
int q35_matmul_3p5bit_awq(const int8_t *A, const int8_t *W_Q, const float *W_scales,
                          const float *W_offsets, int32_t *C, int32_t M, int32_t N, int32_t K);
/* matmul_int4_cuda_fused (matmul_cuda_fortran.cuf:233-276) / matmul_int4_cublas
 * (matmul_cublas.f90:222-274): A int8, W_Q INT4, Out = dequantized fp32, all host. */
int q35_matmul_int4_fused(const int8_t *A, const int8_t *W_Q, const float *W_scales, float *Out,
                          int32_t M, int32_t N, int32_t K);
/* The per-call drop-ins keep each matrix they are given resident on the device (the
 * reference re-uploads per call: matmul_cublas.f90:222-274): an entry per (W_Q, scales,
 * offsets addresses, K, N, format), checked against a fingerprint of sampled W_Q bytes and
 * scales, so a caller passing the same layer matrix every token (int4_linear,
 * transformer_layer.f90:86-89) uploads it once.  A matrix edited in place without its
 * sampled bytes or scales changing is not noticed: call q35_dropin_cache_clear after such
 * edits.  Environment Q35_DROPIN_CACHE_MB (default 65536) bounds the cache (least recently
 * used out first); 0 uploads on every call.  No counterpart in the reference. */
int q35_dropin_cache_stats(int64_t *uploads, int64_t *hits, int64_t *entries, size_t *bytes);
int q35_dropin_cache_clear(void);
/* rms_norm (transformer_layer.f90:155-178, eps RMS_NORM_EPS = 1e-5) on the GPU:
 * x(seq_len, dim) and output column-major host arrays, dim a multiple of 4. */
int q35_rms_norm(const float *x, const float *weight, float *output, int32_t seq_len, int32_t dim);

#ifdef __cplusplus
}
#endif
#endif
