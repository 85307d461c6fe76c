// q35_quant.cu -- on-device synthetic inputs and the reference's weight quantizers.
//
//  * counter-based generator: SplitMix64 finaliser over (seed, tensor, index); int8
//    uniform in [-127,127] by rejection of -128 over the 8 bytes of one draw; normal
//    values by Box-Muller in double rounded to fp32.
//  * quantize_3p5bit_asymmetric (convert_weights_3p5bit.py:19-85): per column
//    scale = (max-min)/15 (1.0 when max == min), zero_point = min + 8*scale,
//    q = clip(round_half_even((w - zero_point)/scale), -8, 7), byte =
//    ((q1 & 0xF) << 3) | (q2 & 7), each float operation singly rounded in binary32.
//  * symmetric INT4 (benchmark_3p5bit.py:155-159): scale = max|w|/7 (1.0 when not
//    above 1e-6), q = clip(round(w/scale), -8, 7), low nibble first.
#include "q35_internal.cuh"

namespace q35 {

__device__ __forceinline__ uint64_t smix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__device__ __forceinline__ uint64_t rng_key(uint64_t seed, uint64_t tensor) {
    return smix(seed ^ smix(tensor + 0x632BE59BD9B4E019ull));
}

__device__ __forceinline__ uint64_t rng_at(uint64_t key, uint64_t index) {
    return smix(key + index * 0x9E3779B97F4A7C15ull);
}

__global__ void gen_int8_kernel(int8_t *out, int64_t n, uint64_t key) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t r = rng_at(key, (uint64_t)i);
        int8_t v = 0;
        for (int b = 0; b < 8; ++b) {
            int8_t c = (int8_t)(uint8_t)(r >> (8 * b));
            if (c != -128) { v = c; break; }
        }
        out[i] = v;
    }
}

__global__ void gen_normal_kernel(float *out, int64_t n, uint64_t key, double sigma) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t a = rng_at(key, 2 * (uint64_t)i), b = rng_at(key, 2 * (uint64_t)i + 1);
        double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
        double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        out[i] = (float)(sigma * z);
    }
}

__global__ void gen_tokens_kernel(int32_t *out, int64_t n, uint64_t key, int32_t vocab) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (int32_t)(rng_at(key, (uint64_t)i) % (uint64_t)vocab) + 1;
}

// one CTA per column: block min/max (or absmax), then the codes of all pairs
template <int FMT>
__global__ void __launch_bounds__(256) quantize_kernel(const float *__restrict__ W, int8_t *__restrict__ W_Q,
                                                       float *__restrict__ scales, float *__restrict__ offsets,
                                                       int32_t K, int32_t N) {
    const int64_t j = blockIdx.x;
    const float *col = W + (int64_t)K * j;
    float mn = INFINITY, mx = -INFINITY;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float v = col[k];
        if (FMT == Q35_FMT_3P5BIT) { mn = fminf(mn, v); mx = fmaxf(mx, v); }
        else mx = fmaxf(mx, fabsf(v));
    }
    __shared__ float s_mn[8], s_mx[8];
    __shared__ float s_scale, s_zp;
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if ((threadIdx.x & 31) == 0) { s_mn[threadIdx.x >> 5] = mn; s_mx[threadIdx.x >> 5] = mx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) { mn = fminf(mn, s_mn[w]); mx = fmaxf(mx, s_mx[w]); }
        if (FMT == Q35_FMT_3P5BIT) {
            float scale = (mx != mn) ? __fdiv_rn(__fsub_rn(mx, mn), 15.0f) : 1.0f;
            float zp = __fsub_rn(mn, __fmul_rn(-8.0f, scale));
            s_scale = scale;
            s_zp = zp;
            scales[j] = scale;
            offsets[j] = zp;
        } else {
            float scale = __fdiv_rn(mx, 7.0f);
            if (!(scale > 1e-6f)) scale = 1.0f;
            s_scale = scale;
            scales[j] = scale;
        }
    }
    __syncthreads();
    const float scale = s_scale, zp = s_zp;
    const int KH = K / 2;
    for (int p = threadIdx.x; p < KH; p += blockDim.x) {
        int q[2];
        for (int t = 0; t < 2; ++t) {
            float w = col[2 * p + t];
            int r;
            if (FMT == Q35_FMT_3P5BIT) r = __float2int_rn(__fdiv_rn(__fsub_rn(w, zp), scale));
            else r = (int)(int8_t)__float2int_rn(__fdiv_rn(w, scale));
            q[t] = r < -8 ? -8 : (r > 7 ? 7 : r);
        }
        uint8_t byte;
        if (FMT == Q35_FMT_3P5BIT) {
            int v1 = q[0] < 0 ? q[0] + 16 : q[0];
            int v2 = q[1] < 0 ? q[1] + 8 : q[1];
            byte = (uint8_t)((((v1 & 0xF) << 3) | (v2 & 7)) & 0x7F);
        } else {
            byte = (uint8_t)((q[0] & 0xF) | ((q[1] & 0xF) << 4));
        }
        W_Q[(int64_t)KH * j + p] = (int8_t)byte;
    }
}

static int grid_for(int64_t n) { return (int)std::min<int64_t>(ceil_div(n, 256), 148 * 16); }

}  // namespace q35

using namespace q35;

// host twin of rng_key (same arithmetic)
static uint64_t host_key(uint64_t seed, uint64_t tensor_id) {
    auto hs = [](uint64_t x) {
        x += 0x9E3779B97F4A7C15ull;
        x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
        x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
        return x ^ (x >> 31);
    };
    return hs(seed ^ hs(tensor_id + 0x632BE59BD9B4E019ull));
}

extern "C" int q35_gen_int8_dev(int8_t *out, int64_t n, uint64_t seed, uint64_t tensor_id,
                                void *stream) {
    if (!out || n < 0) return set_error(Q35_ERR_INVALID, "gen_int8: bad arguments");
    if (n == 0) return Q35_OK;
    gen_int8_kernel<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, n, host_key(seed, tensor_id));
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

extern "C" int q35_gen_normal_dev(float *out, int64_t n, uint64_t seed, uint64_t tensor_id,
                                  double sigma, void *stream) {
    if (!out || n < 0) return set_error(Q35_ERR_INVALID, "gen_normal: bad arguments");
    if (n == 0) return Q35_OK;
    gen_normal_kernel<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, n, host_key(seed, tensor_id), sigma);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

extern "C" int q35_gen_tokens_dev(int32_t *out, int64_t n, uint64_t seed, uint64_t tensor_id,
                                  int32_t vocab, void *stream) {
    if (!out || n < 0 || vocab < 1) return set_error(Q35_ERR_INVALID, "gen_tokens: bad arguments");
    if (n == 0) return Q35_OK;
    gen_tokens_kernel<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, n, host_key(seed, tensor_id), vocab);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

extern "C" int q35_quantize_dev(int format, const float *W, int8_t *W_Q, float *scales,
                                float *offsets, int32_t K, int32_t N, void *stream) {
    if (!W || !W_Q || !scales || (format == Q35_FMT_3P5BIT && !offsets))
        return set_error(Q35_ERR_INVALID, "quantize: NULL pointer");
    if (K < 2 || (K & 1) || N < 1) return set_error(Q35_ERR_INVALID, "quantize: K even >= 2, N >= 1");
    if (format == Q35_FMT_3P5BIT)
        quantize_kernel<Q35_FMT_3P5BIT><<<N, 256, 0, (cudaStream_t)stream>>>(W, W_Q, scales, offsets, K, N);
    else if (format == Q35_FMT_INT4)
        quantize_kernel<Q35_FMT_INT4><<<N, 256, 0, (cudaStream_t)stream>>>(W, W_Q, scales, nullptr, K, N);
    else
        return set_error(Q35_ERR_INVALID, "quantize: unknown format");
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}
