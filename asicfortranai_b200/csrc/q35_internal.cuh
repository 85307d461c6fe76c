// q35_internal.cuh -- shared definitions of libq35 (B200 / sm_100a).
//
// Device weight formats (built once, on the GPU, from the reference's packed bytes):
//
//   The reference stores W_Q(K/2,N) int8, one byte per (even k, odd k) pair: bits 6..3 a
//   4-bit two's-complement code n1 for the even k, bits 2..0 a 3-bit code n2 for the odd
//   k (3.5-bit, matmul_3p5bit_dynamic.f90:48-56), or two 4-bit nibbles (INT4,
//   matmul_int4_groq.f90:126-133).  On the device every code is stored BIASED
//   (b1 = n1 + 8 in [0,15], b2 = n2 + 4 in [0,7], INT4 b = q + 8) so that it can be fed
//   to dp4a / the tensor cores as an unsigned byte; the bias is removed exactly with a
//   per-row integer correction  sum_k a_k*bias_k  (int32 arithmetic, order free).
//
//   The matrix is cut into tiles of 32 columns (a column group) x 256 k (a k-block,
//   128 pairs).  Tiles are stored column-group major, k-block minor, so one column
//   group's whole K range is contiguous.  Inside a tile the data of lane l (column
//   cg*32+l) is split in 16-byte chunks, chunk c of lane l at byte c*512 + l*16, so a
//   warp reading chunk c issues one fully coalesced 512-byte request.
//
//   3.5-bit tile: 7 chunks per lane (112 B = 256 codes at 3.5 bits), four groups of 32
//   pairs, 7 words per group.  Word i (0..6) of group g, byte b, holds pair 32g+4i+b as
//   its 7-bit field  b2 | b1<<3  in bits 0..6, and in bit 7 bit i of the field of pair
//   32g+28+b (the four "stuffed" pairs of the group are spread over the 28 top bits).
//   INT4 tile: 8 chunks per lane (128 B): words 0..15 even-k codes as the nibble plane
//   above, words 16..31 odd-k codes in the same arrangement.
//
//   Activations are staged per k-block as a 256-byte image: 32 words E (even k of pairs
//   0..127, byte b of word q = pair 4q+b) followed by 32 words O (odd k, same order).
//   With that image every extracted weight word meets its activation word directly.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <vector>

#include "q35.h"

namespace q35 {

constexpr int KBLK = 256;              // k per k-block
constexpr int PAIRS = KBLK / 2;        // pairs per k-block
constexpr int CGW = 32;                // columns per column group
constexpr int TILE35 = CGW * 112;      // bytes per 3.5-bit tile
constexpr int TILE4 = CGW * 128;       // bytes per INT4 tile

__host__ __device__ inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }
__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct Weights {
    int format;            // Q35_FMT_3P5BIT or Q35_FMT_INT4
    int32_t K, N;          // logical sizes
    int32_t KB, CG;        // k-blocks, column groups
    int device;
    uint8_t *tiles;        // device, CG*KB tiles
    float *scales;         // device, N
    float *offsets;        // device, N (3.5-bit) or nullptr
    size_t tile_bytes;     // per tile
    size_t bytes;          // total tile bytes
};

struct Workspace {
    int32_t *acc = nullptr;      // split-K accumulators, kept all-zero between calls
    uint32_t *tickets = nullptr; // per column group arrival counters, kept zero
    int *err = nullptr;          // device error word set by bounded waits that gave up
    size_t acc_elems = 0, n_tickets = 0;
    int32_t *corr = nullptr;     // per-row bias corrections of the tensor-core path
    size_t corr_elems = 0;
    int8_t *xt = nullptr;        // row-major copy of column-major activations (tensor-core path)
    size_t xt_bytes = 0;
};

constexpr int GEMM_MAX_K = 131072;   // keeps every int32 accumulator and correction exact
constexpr int GEMM_MAX_M = 65536;    // activation rows per call
constexpr int MMA_MIN_M = 5;         // from this many rows on, the tensor-core path is used

#ifdef __CUDACC__
// int4_linear's activation quantization (transformer_layer.f90:81-83):
// int(max(-127., min(127., x*127.)), int8), truncation toward zero
__device__ __forceinline__ int8_t quant127(float x) {
    float v = __fmul_rn(x, 127.0f);
    v = fminf(127.0f, v);
    v = fmaxf(-127.0f, v);
    return (int8_t)__float2int_rz(v);
}
#endif

// Set the thread-local error message and return the status.
int set_error(int status, const std::string &msg);
#define Q35_CUDA_TRY(expr)                                                              \
    do {                                                                                \
        cudaError_t _e = (expr);                                                        \
        if (_e != cudaSuccess)                                                          \
            return ::q35::set_error(Q35_ERR_CUDA, std::string(#expr ": ") +             \
                                                      cudaGetErrorString(_e));          \
    } while (0)

// ---- kernels' host launchers (q35_pack.cu, q35_gemv.cu) ----
int launch_repack(const Weights &w, const int8_t *d_ref_wq, cudaStream_t s);
int launch_unpack_ref(const Weights &w, int8_t *d_ref_wq, cudaStream_t s);

// q|k|v epilogue of the CUDA-core engine (transformer_layer.f90:183-205 and :322-329):
// the columns are [q heads | k heads | v heads] of width D; q and k are rotated in
// interleaved pairs (2d, 2d+1) at the row's position, q goes to q[row][H*D], k and v to the
// cache at the row's absolute position.  Rows are row0 + the launch's row index.
struct GemvRope {
    float *q = nullptr, *kc = nullptr, *vc = nullptr;
    const int32_t *row_seq = nullptr, *row_i = nullptr, *cache_pos = nullptr;
    const float2 *cs = nullptr;      // [max_seq][D/2] (cos, sin)
    int32_t row0 = 0, layer = 0, n_layers = 0, H = 0, KVH = 0, D = 0, max_seq = 0, rope_mode = 0;
};

struct GemvArgs {
    const int8_t *x;          // activations int8
    int64_t sx_row, sx_k;     // element strides of x (row i, k)
    int32_t M;                // rows
    int32_t *C;               // optional int32 accumulators
    float *y;                 // optional fp32 dequantized output
    int64_t so_row, so_col;   // element strides of C / y (row i, column j)
    const float *res = nullptr;  // optional residual added to y (same strides as y)
    // CUDA-core engine only: SwiGLU of the interleaved (gate, up) column pairs and its int8
    // quantization, row r to swiglu_q[r * N/2 ..] (then C and y are not written)
    int8_t *swiglu_q = nullptr;
    const GemvRope *rope = nullptr;   // CUDA-core engine only: the q|k|v epilogue above
};
int launch_gemv(const Weights &w, const GemvArgs &a, Workspace &ws, cudaStream_t s);
size_t gemv_workspace_acc_elems(const Weights &w, int32_t M);
size_t gemv_workspace_tickets(const Weights &w);
// tensor-core path (q35_mma.cu): any M >= 1, x row-major with 16-byte aligned rows
bool mma_supported(const Weights &w, const GemvArgs &a);
int launch_mma(const Weights &w, const GemvArgs &a, Workspace &ws, cudaStream_t s);
size_t mma_workspace_acc_elems(const Weights &w, int32_t M, int dev);
size_t mma_workspace_tickets(const Weights &w, int32_t M, int dev);
int launch_transpose_i8(const int8_t *src, int8_t *dst, int32_t rows, int32_t cols, int64_t ld, cudaStream_t s);

// sampling (q35_sample.cu): rows row0 .. row0+rows-1 of a logits buffer whose element
// (row r, token g) sits at logits[((g / Vl) * Rtot + r) * Vl + g % Vl] (Vl = V for one
// GPU; the gathered per-rank blocks under tensor parallelism)
struct SampleRows {
    const float *logits = nullptr;
    int32_t Vl = 0, Rtot = 0, V = 0, row0 = 0, rows = 0;
    int32_t mode = 0, top_k = 0;
    float temperature = 0.0f, top_p = 0.0f;
    const float *u = nullptr;          // per sampled row, or nullptr: per-sequence draws
    uint64_t seed = 0;
    const int32_t *row_seq = nullptr;  // sequence of row r at row_seq[row_seq0 + r] (nullptr: r)
    int32_t row_seq0 = 0;
    int32_t *draws = nullptr;          // per-sequence draw counters
    int32_t *tokens = nullptr;         // 1-based tokens of the sampled rows
};
int sample_check(int mode, int V);
int launch_sample(const SampleRows &a, cudaStream_t s);

}  // namespace q35

// the public q35_weights handle wraps one Weights
struct q35_weights_s {
    q35::Weights w;
};

// one matrix of the per-call drop-ins' resident-weight cache: keyed on the caller's
// W_Q / scales / offsets addresses, K, N and the format, and checked against a
// fingerprint of sampled bytes
struct q35_dropin_entry {
    const void *wq = nullptr, *sc = nullptr, *of = nullptr;
    int32_t K = 0, N = 0;
    int format = 0;
    uint64_t fingerprint = 0, last_use = 0;
    q35_weights w = nullptr;
};

// a device, its stream, the split-K workspace and staging for host-pointer calls
struct q35_ctx_s {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    q35::Workspace ws;
    void *d_scratch = nullptr;
    size_t d_scratch_bytes = 0;
    void *h_pinned = nullptr;
    size_t h_pinned_bytes = 0;
    q35_weights transient = nullptr;   // weights of the per-call drop-ins when caching is off
    std::vector<q35_dropin_entry> dropin;   // resident weights of the per-call drop-ins
    uint64_t dropin_tick = 0;
    int64_t dropin_uploads = 0, dropin_hits = 0;
    int gemm_path = 0;                 // Q35_PATH_AUTO / _CUDA_CORES / _TENSOR_CORES
    std::mutex mu;
};

namespace q35 {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// q35_capi.cu helpers shared with the model runtime
int ensure_workspace(q35_ctx ctx, size_t acc_elems, size_t tickets);
// sizes the workspace for an M-row matmul with w on whichever path gemm_dev picks
int ensure_gemm_workspace(q35_ctx ctx, const Weights &w, int32_t M);
int ensure_scratch(q35_ctx ctx, size_t dbytes, size_t hbytes);
// the library's own context of the current device (the drop-in entry points')
int default_ctx(q35_ctx *out);
int weights_alloc(q35_ctx ctx, int format, int32_t N, int32_t K, q35_weights *io);
int weights_fill(q35_ctx ctx, q35_weights h, const int8_t *W_Q, const float *scales, const float *offsets,
                 int src_on_device);
// device matmul of R rows (any R >= 1, chunked by 64): x int8 [R][K] row-major,
// C / y [R][N] row-major (either may be null), y = res + dequant when res is set
int gemm_rows(q35_ctx ctx, q35_weights w, const int8_t *x, int32_t R, int32_t *C, float *y,
              const float *res);
// gate|up (columns interleaved) followed by SwiGLU and int8 quantization into q [R][N/2]
// (swiglu_kernel, transformer_layer.f90:212-229): fused into the CUDA-core matmul's
// epilogue, or y (a [R][N] fp32 scratch) + the SwiGLU kernel after the tensor cores.
// q must not alias x.
int gemm_rows_swiglu(q35_ctx ctx, q35_weights w, const int8_t *x, int32_t R, float *y, int8_t *q);
// q|k|v with the GemvRope epilogue (RoPE, q, the cache writes) on the CUDA-core engine;
// where the tensor-core engine takes R rows nothing is launched and *fused stays false
int gemm_rows_rope(q35_ctx ctx, q35_weights w, const int8_t *x, int32_t R, float *y, const GemvRope &rope,
                   bool *fused);

}  // namespace q35
