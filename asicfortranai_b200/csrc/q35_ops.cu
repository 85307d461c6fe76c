// q35_ops.cu -- elementwise kernels of the matmul module: the stand-alone dequant of
// int32 accumulators (dequantize_output_3p5bit / dequantize_output) and their host
// entry points.
#include <cstring>

#include "q35_internal.cuh"

namespace q35 {

// matmul_3p5bit_dynamic.f90:78-81 (offsets != nullptr) and matmul_int4_groq.f90:150-152
__global__ void dequant_kernel(const int32_t *__restrict__ C, const float *__restrict__ scales,
                               const float *__restrict__ offsets, float *__restrict__ Out,
                               int32_t M, int64_t total) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = t / M;
        float f = __int2float_rn(C[t]);
        Out[t] = offsets ? __fmul_rn(__fadd_rn(f, offsets[j]), scales[j]) : __fmul_rn(f, scales[j]);
    }
}

static int dequant_host(const int32_t *C, const float *scales, const float *offsets, float *Out,
                        int32_t M, int32_t N) {
    if (M < 0 || N < 0) return set_error(Q35_ERR_INVALID, "M and N must not be negative");
    if (M == 0 || N == 0) return Q35_OK;   // empty: the reference's loops run no iterations
    if (!C || !scales || !Out) return set_error(Q35_ERR_INVALID, "NULL argument");
    const size_t n = (size_t)M * N;
    int32_t *dC = nullptr;
    float *dS = nullptr, *dO = nullptr, *dY = nullptr;
    cudaStream_t s = nullptr;
    int st = Q35_OK;
    auto fail = [&](cudaError_t e) { st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e)); };
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMallocAsync(&dC, n * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&dY, n * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&dS, (size_t)N * 4, s);
    if (e == cudaSuccess && offsets) e = cudaMallocAsync(&dO, (size_t)N * 4, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dC, C, n * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dS, scales, (size_t)N * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && offsets) e = cudaMemcpyAsync(dO, offsets, (size_t)N * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        int blocks = (int)std::min<int64_t>(ceil_div((int64_t)n, 256), 148 * 8);
        dequant_kernel<<<blocks, 256, 0, s>>>(dC, dS, dO, dY, M, (int64_t)n);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(Out, dY, n * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) fail(e);
    if (s) {
        if (dC) cudaFreeAsync(dC, s);
        if (dY) cudaFreeAsync(dY, s);
        if (dS) cudaFreeAsync(dS, s);
        if (dO) cudaFreeAsync(dO, s);
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
    }
    return st;
}

}  // namespace q35

extern "C" int q35_dequantize_output_3p5bit(const int32_t *C, const float *W_scales,
                                            const float *W_offsets, float *Out, int32_t M,
                                            int32_t N) {
    if (!W_offsets && M > 0 && N > 0) return q35::set_error(Q35_ERR_INVALID, "W_offsets is NULL");
    return q35::dequant_host(C, W_scales, W_offsets, Out, M, N);
}

extern "C" int q35_dequantize_output(const int32_t *C, const float *W_scales, float *Out,
                                     int32_t M, int32_t N) {
    return q35::dequant_host(C, W_scales, nullptr, Out, M, N);
}
