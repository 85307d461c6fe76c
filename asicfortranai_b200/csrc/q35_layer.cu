// q35_layer.cu -- the non-matmul kernels of the LLaMA layer and model
// (transformer_layer.f90, llama_model.f90, sampling.f90), fp32 like the reference.
//
// Rows: a forward processes R rows; row r belongs to sequence row_seq[r] at position
// row_i[r] within the call; its absolute position is cache_pos[seq] + row_i[r].
// Activations are row-major [R][width].  KV cache: [seq][layer][kv_head][max_seq][D].
#include <algorithm>
#include <cfloat>

#include "q35_layer.cuh"

namespace q35 {

// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = (threadIdx.x < nw) ? red[threadIdx.x] : 0.0f;
    if (w == 0)
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[32] = v;
    __syncthreads();
    return red[32];
}

__device__ __forceinline__ float block_max(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = (threadIdx.x < nw) ? red[threadIdx.x] : -FLT_MAX;
    if (w == 0)
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[32] = v;
    __syncthreads();
    return red[32];
}

// int4_linear's activation quantization (transformer_layer.f90:81-83):
// int(max(-127., min(127., x*127.)), int8), truncation toward zero
__device__ __forceinline__ int8_t quant127(float x) {
    float v = __fmul_rn(x, 127.0f);
    v = fminf(127.0f, v);
    v = fmaxf(-127.0f, v);
    return (int8_t)__float2int_rz(v);
}

// ---------------------------------------------------------------------------------------
// llama_model.f90:123-125: x(i,:) = E(id,:), ids 1-based.  E row-major [vocab][hidden].
__global__ void embed_kernel(const int32_t *__restrict__ ids, const float *__restrict__ E,
                             float *__restrict__ x, int32_t hidden, int32_t vocab, int *err) {
    const int r = blockIdx.x;
    const int id = ids[r];
    const bool ok = id >= 1 && id <= vocab;
    if (!ok && threadIdx.x == 0) atomicExch(err, Q35_ERR_INVALID);
    const float *src = E + (size_t)(ok ? id - 1 : 0) * hidden;
    for (int j = threadIdx.x; j < hidden; j += blockDim.x) x[(size_t)r * hidden + j] = ok ? src[j] : 0.0f;
}

// transformer_layer.f90:155-178 rms_norm (+ the int8 quantization of int4_linear when
// q is non-null): one CTA per row.
__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                               float *__restrict__ out, int8_t *__restrict__ q, int32_t dim, float eps) {
    __shared__ float red[33];
    const int r = blockIdx.x;
    const float *xr = x + (size_t)r * dim;
    float s = 0.0f;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) s = __fadd_rn(s, __fmul_rn(xr[j], xr[j]));
    s = block_sum(s, red);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)dim), eps));
    for (int j = threadIdx.x; j < dim; j += blockDim.x) {
        const float v = __fmul_rn(__fdiv_rn(xr[j], rms), w[j]);
        if (out) out[(size_t)r * dim + j] = v;
        if (q) q[(size_t)r * dim + j] = quant127(v);
    }
}

// transformer_layer.f90:183-205 (RoPE on q and k, interleaved pairs (2d, 2d+1)) and
// :322-329 (K/V written to the cache at cache_pos + i).  Input: the fused q|k|v output
// [R][QN + 2KN].  The rotation angle's position is the row's index within the call
// (rope_mode 0, the reference's apply_rope_single, :193-196) or its absolute position
// (rope_mode 1).  cs: [max_seq][D/2] pairs (cos, sin) computed on the host.
__global__ void rope_kv_kernel(const float *__restrict__ yqkv, float *__restrict__ q,
                               float *__restrict__ kc, float *__restrict__ vc,
                               const int32_t *__restrict__ row_seq, const int32_t *__restrict__ row_i,
                               const int32_t *__restrict__ cache_pos, const float2 *__restrict__ cs,
                               int32_t layer, int32_t n_layers, int32_t H, int32_t KVH, int32_t D,
                               int32_t max_seq, int32_t rope_mode, int *err) {
    const int r = blockIdx.x;
    const int s = row_seq[r], i = row_i[r];
    const int pos = cache_pos[s] + i;
    if (pos < 0 || pos >= max_seq) {
        if (threadIdx.x == 0) atomicExch(err, Q35_ERR_INVALID);
        return;
    }
    const int rp = rope_mode ? pos : i;
    const int QN = H * D, KN = KVH * D, W = QN + 2 * KN;
    const float *y = yqkv + (size_t)r * W;
    const int half = D / 2;
    // q: H*D/2 pairs, k: KVH*D/2 pairs
    for (int t = threadIdx.x; t < (H + KVH) * half; t += blockDim.x) {
        const int hh = t / half, d = t % half;
        const float2 c = cs[(size_t)rp * half + d];
        const bool isq = hh < H;
        const int col = isq ? hh * D + 2 * d : QN + (hh - H) * D + 2 * d;
        const float a = y[col], b = y[col + 1];
        const float ra = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
        const float rb = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
        if (isq) {
            q[(size_t)r * QN + hh * D + 2 * d] = ra;
            q[(size_t)r * QN + hh * D + 2 * d + 1] = rb;
        } else {
            const int kh = hh - H;
            float *dst = kc + ((((size_t)s * n_layers + layer) * KVH + kh) * max_seq + pos) * D + 2 * d;
            dst[0] = ra;
            dst[1] = rb;
        }
    }
    for (int t = threadIdx.x; t < KN; t += blockDim.x) {
        const int kh = t / D, d = t % D;
        vc[((((size_t)s * n_layers + layer) * KVH + kh) * max_seq + pos) * D + d] = y[QN + KN + t];
    }
}

// transformer_layer.f90:333-402 + the int8 quantization of the o-projection input:
// one CTA per (row, query head).  Scores over the visible keys j <= pos (the masked
// keys of the reference, -1e9, contribute exp(-1e9 - max) = 0), softmax with max
// subtraction and normalisation, then P.V accumulated over j in order.
constexpr int ATT_THREADS = 128;
__global__ void __launch_bounds__(ATT_THREADS)
attention_kernel(const float *__restrict__ q, const float *__restrict__ kc, const float *__restrict__ vc,
                 int8_t *__restrict__ out_q, float *__restrict__ out_f,
                 const int32_t *__restrict__ row_seq, const int32_t *__restrict__ row_i,
                 const int32_t *__restrict__ cache_pos, int32_t layer, int32_t n_layers, int32_t H,
                 int32_t KVH, int32_t D, int32_t max_seq) {
    extern __shared__ float sm[];          // scores[max_seq] | q[D] | red[33]
    float *sc = sm;
    float *qs = sm + max_seq;
    float *red = qs + D;
    const int r = blockIdx.x, h = blockIdx.y;
    const int s = row_seq[r];
    const int pos = cache_pos[s] + row_i[r];
    if (pos < 0 || pos >= max_seq) return;     // rope_kv_kernel has flagged it
    const int kvh = h / (H / KVH);
    const int QN = H * D;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));   // :336
    for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = q[(size_t)r * QN + h * D + d];
    __syncthreads();
    const size_t base = (((size_t)s * n_layers + layer) * KVH + kvh) * max_seq * D;
    const float *K = kc + base, *V = vc + base;
    const int T = pos + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    // scores: one warp per key, lanes over D (D multiple of 32)
    for (int j = warp; j < T; j += nw) {
        float a = 0.0f;
        for (int d = lane; d < D; d += 32) a = fmaf(qs[d], K[(size_t)j * D + d], a);
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) sc[j] = __fmul_rn(a, scale);
    }
    __syncthreads();
    float m = -FLT_MAX;
    for (int j = threadIdx.x; j < T; j += blockDim.x) m = fmaxf(m, sc[j]);
    m = block_max(m, red);
    float se = 0.0f;
    for (int j = threadIdx.x; j < T; j += blockDim.x) {
        const float e = expf(__fsub_rn(sc[j], m));
        sc[j] = e;
        se += e;
    }
    se = block_sum(se, red);
    for (int j = threadIdx.x; j < T; j += blockDim.x) sc[j] = __fdiv_rn(sc[j], se);   // :376-378
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float a = 0.0f;
        for (int j = 0; j < T; ++j) a = __fadd_rn(a, __fmul_rn(sc[j], V[(size_t)j * D + d]));
        const size_t o = (size_t)r * QN + h * D + d;
        if (out_q) out_q[o] = quant127(a);
        if (out_f) out_f[o] = a;
    }
}

// transformer_layer.f90:212-229 swiglu + the int8 quantization of the down-projection
// input.  y = [R][2F] with gate in [0,F) and up in [F,2F).
__global__ void swiglu_kernel(const float *__restrict__ y, int8_t *__restrict__ out_q,
                              float *__restrict__ out_f, int32_t F, int64_t total) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / F, j = t % F;
        const float g = y[r * 2 * F + j], u = y[r * 2 * F + F + j];
        const float sw = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        const float h = __fmul_rn(sw, u);
        if (out_q) out_q[t] = quant127(h);
        if (out_f) out_f[t] = h;
    }
}

// llama_model.f90:138-140 LM head: logits(i,j) = dot_product(x_norm(i,:), W(:,j)),
// W stored row-major [vocab][hidden] (the reference's column j contiguous), fused with
// a per-CTA greedy candidate (largest logit, lowest index on ties, sampling.f90:64-83).
constexpr int LMH_THREADS = 256;
__global__ void __launch_bounds__(LMH_THREADS)
lmhead_kernel(const float *__restrict__ xn, const float *__restrict__ W, float *__restrict__ logits,
              float2 *__restrict__ cand, int32_t R, int32_t hidden, int32_t vocab) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    const int64_t nwt = (int64_t)gridDim.x * (blockDim.x >> 5);
    __shared__ float bv[LMH_THREADS / 32][8];
    __shared__ int bi[LMH_THREADS / 32][8];
    float best[8];
    int bidx[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) { best[r] = -FLT_MAX; bidx[r] = 0x7fffffff; }
    for (int64_t j = gw; j < vocab; j += nwt) {
        const float *wr = W + (size_t)j * hidden;
        for (int r0 = 0; r0 < R; r0 += 8) {
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int k = lane * 4; k < hidden; k += 128) {
                const float4 w4 = __ldcs(reinterpret_cast<const float4 *>(wr + k));   // streamed once
#pragma unroll
                for (int rr = 0; rr < 8; ++rr) {
                    if (r0 + rr < R) {
                        const float4 x4 = *reinterpret_cast<const float4 *>(xn + (size_t)(r0 + rr) * hidden + k);
                        a[rr] = fmaf(w4.x, x4.x, fmaf(w4.y, x4.y, fmaf(w4.z, x4.z, fmaf(w4.w, x4.w, a[rr]))));
                    }
                }
            }
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) {
                float v = a[rr];
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const int row = r0 + rr;
                if (row < R) {
                    if (lane == 0) logits[(size_t)row * vocab + j] = v;
                    if (r0 == 0 && (v > best[rr] || (v == best[rr] && j < bidx[rr]))) {
                        best[rr] = v;
                        bidx[rr] = (int)j;
                    }
                }
            }
        }
    }
    // candidates of rows 0..7 per CTA (rows >= 8 are reduced from the logits buffer)
    if (lane == 0)
        for (int r = 0; r < 8; ++r) { bv[warp][r] = best[r]; bi[warp][r] = bidx[r]; }
    __syncthreads();
    if (threadIdx.x < 8 && threadIdx.x < R) {
        const int r = threadIdx.x;
        float v = -FLT_MAX;
        int ix = 0x7fffffff;
        for (int w = 0; w < LMH_THREADS / 32; ++w)
            if (bv[w][r] > v || (bv[w][r] == v && bi[w][r] < ix)) { v = bv[w][r]; ix = bi[w][r]; }
        cand[(size_t)r * gridDim.x + blockIdx.x] = make_float2(v, __int_as_float(ix));
    }
}

// greedy token per row (1-based), from the per-CTA candidates (rows < 8) or by a scan of
// the row's logits (rows >= 8); lowest index wins ties.
__global__ void argmax_kernel(const float2 *__restrict__ cand, int32_t ncand, const float *__restrict__ logits,
                              int32_t vocab, int32_t *__restrict__ tok_out) {
    __shared__ float sv[256];
    __shared__ int si[256];
    const int r = blockIdx.x;
    float v = -FLT_MAX;
    int ix = 0x7fffffff;
    if (r < 8) {
        for (int c = threadIdx.x; c < ncand; c += blockDim.x) {
            const float2 e = cand[(size_t)r * ncand + c];
            const int ei = __float_as_int(e.y);
            if (e.x > v || (e.x == v && ei < ix)) { v = e.x; ix = ei; }
        }
    } else {
        for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
            const float e = logits[(size_t)r * vocab + j];
            if (e > v) { v = e; ix = j; }
        }
    }
    sv[threadIdx.x] = v;
    si[threadIdx.x] = ix;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = sv[threadIdx.x + s];
            const int oi = si[threadIdx.x + s];
            if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) tok_out[r] = si[0] + 1;
}

// cache_pos[seq] += n for the sequences of a forward (transformer_layer.f90:424-426)
__global__ void advance_kernel(int32_t *cache_pos, const int32_t *seqs, int32_t nseq, int32_t n) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < nseq) cache_pos[seqs[t]] += n;
}

// ---------------------------------------------------------------------------------------
static int grid_1d(int64_t n, int threads) { return (int)std::min<int64_t>(ceil_div(n, threads), 148 * 16); }

int launch_embed(const int32_t *ids, const float *E, float *x, int R, int hidden, int vocab, int *err,
                 cudaStream_t s) {
    embed_kernel<<<R, 256, 0, s>>>(ids, E, x, hidden, vocab, err);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

int launch_rmsnorm(const float *x, const float *w, float *out, int8_t *q, int R, int dim, float eps,
                   cudaStream_t s) {
    rmsnorm_kernel<<<R, 512, 0, s>>>(x, w, out, q, dim, eps);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

int launch_rope_kv(const float *yqkv, float *q, float *kc, float *vc, const int32_t *row_seq,
                   const int32_t *row_i, const int32_t *cache_pos, const float2 *cs, int layer,
                   int n_layers, int R, int H, int KVH, int D, int max_seq, int rope_mode, int *err,
                   cudaStream_t s) {
    rope_kv_kernel<<<R, 256, 0, s>>>(yqkv, q, kc, vc, row_seq, row_i, cache_pos, cs, layer, n_layers, H,
                                     KVH, D, max_seq, rope_mode, err);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

int launch_attention(const float *q, const float *kc, const float *vc, int8_t *out_q, float *out_f,
                     const int32_t *row_seq, const int32_t *row_i, const int32_t *cache_pos, int layer,
                     int n_layers, int R, int H, int KVH, int D, int max_seq, cudaStream_t s) {
    const size_t smem = sizeof(float) * ((size_t)max_seq + D + 33);
    static size_t configured = 0;
    if (smem > 48 * 1024 && configured < smem) {
        Q35_CUDA_TRY(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    attention_kernel<<<dim3(R, H), ATT_THREADS, smem, s>>>(q, kc, vc, out_q, out_f, row_seq, row_i, cache_pos,
                                                          layer, n_layers, H, KVH, D, max_seq);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

int launch_swiglu(const float *y, int8_t *out_q, float *out_f, int R, int F, cudaStream_t s) {
    const int64_t total = (int64_t)R * F;
    swiglu_kernel<<<grid_1d(total, 256), 256, 0, s>>>(y, out_q, out_f, F, total);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

int lmhead_grid(int dev) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms * 4;
}

int launch_lmhead(const float *xn, const float *W, float *logits, float2 *cand, int32_t *tok, int R,
                  int hidden, int vocab, int grid, cudaStream_t s) {
    lmhead_kernel<<<grid, LMH_THREADS, 0, s>>>(xn, W, logits, cand, R, hidden, vocab);
    Q35_CUDA_TRY(cudaGetLastError());
    argmax_kernel<<<R, 256, 0, s>>>(cand, grid, logits, vocab, tok);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

int launch_advance(int32_t *cache_pos, const int32_t *seqs, int nseq, int n, cudaStream_t s) {
    advance_kernel<<<(nseq + 127) / 128, 128, 0, s>>>(cache_pos, seqs, nseq, n);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

}  // namespace q35
