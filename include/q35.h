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

typedef struct q35_ctx_s *q35_ctx;         /* device, stream, split-K workspace */
typedef struct q35_weights_s *q35_weights; /* one device-resident quantized matrix */
typedef struct q35_graph_s *q35_graph;     /* an instantiated CUDA graph of captured calls */

const char *q35_last_error(void);
const char *q35_status_string(int status);
int q35_version(void);

/* Context: device ordinal and a CUDA stream (cudaStream_t, NULL = a new stream owned by
 * the context).  Calls on one context are serialised on its stream. */
int q35_ctx_create(int device, void *stream, q35_ctx *out);
int q35_ctx_destroy(q35_ctx ctx);
int q35_ctx_synchronize(q35_ctx ctx);
void *q35_ctx_stream(q35_ctx ctx);
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
 * y fp32 (M,N) in out_layout; C or y may be NULL.  y = (C + offset) * scale (3.5-bit,
 * matmul_3p5bit_dynamic.f90:80) or C * scale (INT4, matmul_int4_groq.f90:151).
 * Replaces matmul_3p5bit_awq + dequantize_output_3p5bit and matmul_int4_awq +
 * dequantize_output on device-resident data.  Asynchronous. */
int q35_gemm_dev(q35_ctx ctx, q35_weights w, const int8_t *x, int32_t M, int x_layout,
                 int32_t *C, float *y, int out_layout);

/* q35_gemm_dev for callers that cannot allocate device memory -- code running during
 * CUDA-graph capture, real-time loops that must not enter the driver's allocator (which
 * can synchronise the device), processes whose free HBM is owned by another allocator.
 * No counterpart in the reference.  Same arguments and results as q35_gemm_dev, on the
 * caller's stream (cudaStream_t), with the weights already resident; the split-K scratch
 * is a fixed ~4.1 MiB array inside the library (held on every GPU that loads it), so
 * M * ceil(N/32)*32 must be <= 1,048,576 and ceil(N/32) * ceil(M/4) <= 32768, else
 * Q35_ERR_INVALID.  The first call on a device looks up the array's address: make it
 * before any stream capture.  All calls share the array: calls that overlap on the GPU
 * race; each call clears what it uses first.  Allocates nothing. */
int q35_gemm_dev_noalloc(q35_weights w, const int8_t *x, int32_t M, int x_layout, int32_t *C,
                         float *y, int out_layout, void *stream);

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

/* ---- drop-in entry points with the reference's own signatures (host pointers) ----
 * They run on a default context of the current CUDA device, upload their inputs,
 * compute on the GPU and copy the results back before returning.  A failure is
 * reported through q35_last_error() and leaves the outputs untouched. */

/* matmul_3p5bit_dynamic.f90:28-34  (bind(C), M/N/K by value) */
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

#ifdef __cplusplus
}
#endif
#endif
