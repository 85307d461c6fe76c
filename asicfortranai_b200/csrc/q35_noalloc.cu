// q35_noalloc.cu -- q35_gemm_dev_noalloc: the decode matmul for callers that must not
// allocate device memory.
//
// Who cannot allocate: real-time decode loops that must never enter the driver's
// allocator (cudaMalloc/cudaFree can synchronise the whole device and stall the loop for
// milliseconds), and processes whose free device memory is owned by another allocator
// (a framework's caching pool that has reserved the remaining HBM, so a cudaMalloc of a
// few MiB fails).  q35_gemm_dev grows a per-context split-K workspace with cudaMalloc on
// first use; this entry point keeps that scratch in a fixed array compiled into the
// library instead, and otherwise runs the same gemv_kernel.
//
// Limits and rules:
//  * 1 <= M <= 64 rows; N <= 65536 columns (the counters: 16 row chunks per 32-column
//    group, ceil(N/32) * 16 <= NOALLOC_MAX_CTR = 32768); M * ceil(N/32)*32 <=
//    NOALLOC_MAX_ACC = 1,048,576 int32 partial sums (4 MiB).  Larger calls are rejected
//    with Q35_ERR_INVALID.  Every GPU that loads libq35 holds this ~4.1 MiB until the
//    process exits.
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, which may load the module); make that first call before any
//    stream capture.
//  * all calls share the one array: calls that overlap on the GPU (different streams
//    without ordering between them) race on it.  Each call clears the partial sums and
//    counters it uses on the given stream before the kernel runs, so a call never depends
//    on what an earlier call left there.
//  * a bounded wait inside the kernel that gives up records Q35_ERR_TIMEOUT in the
//    array's error word; the call itself cannot see that (it returns before the kernel
//    runs).  q35_gemm_noalloc_device_error(stream) synchronises the stream, returns that
//    record and clears it; the calls never clear it, so a failure stays visible until it
//    is read.
//  * the weights must already be resident (q35_weights_upload / q35_weights_generate,
//    done once at load time); the call itself allocates nothing.
#include <mutex>
#include <string>

#include "q35_internal.cuh"

namespace q35 {

constexpr size_t NOALLOC_MAX_ACC = 1u << 20;   // int32 partial sums
constexpr size_t NOALLOC_MAX_CTR = 32768;      // column-group counters
constexpr size_t NOALLOC_ERR = NOALLOC_MAX_ACC + NOALLOC_MAX_CTR;   // index of the error word

// the scratch: partial sums, counters and the device error word, one array (zero at
// module load)
static __device__ __align__(256) int32_t g_noalloc_scratch[NOALLOC_MAX_ACC + NOALLOC_MAX_CTR + 64];

static std::mutex g_noalloc_mu;
static int32_t *g_noalloc_ptr[64] = {nullptr};

// once per device, with that device current: the device address of the scratch array
// (host code cannot use the symbol itself, which names a host-side stand-in)
static int noalloc_scratch(int dev, int32_t **out) {
    if (dev < 0 || dev >= 64) return set_error(Q35_ERR_INVALID, "noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(Q35_ERR_CUDA, std::string("noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_noalloc_ptr[dev] = static_cast<int32_t *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return Q35_OK;
}

}  // namespace q35

extern "C" int q35_gemm_dev_noalloc(q35_weights wh, const int8_t *x, int32_t M, int x_layout,
                                    int32_t *C, float *y, int out_layout, void *stream) {
    using namespace q35;
    if (!wh || !x) return set_error(Q35_ERR_INVALID, "noalloc: NULL weights or activations");
    const Weights &w = wh->w;
    if (M < 1 || M > 64) return set_error(Q35_ERR_INVALID, "noalloc: M must be in [1,64]");
    if (w.N > 65536) return set_error(Q35_ERR_INVALID, "noalloc: N above 65536 (fixed counter scratch)");
    const size_t acc = (size_t)M * w.CG * 32;
    const size_t ctr = gemv_workspace_tickets(w);
    if (acc > NOALLOC_MAX_ACC)
        return set_error(Q35_ERR_INVALID, "noalloc: M * ceil(N/32)*32 = " + std::to_string(acc) +
                                              " partial sums exceed the fixed scratch of " +
                                              std::to_string(NOALLOC_MAX_ACC));
    if (ctr > NOALLOC_MAX_CTR)
        return set_error(Q35_ERR_INVALID, "noalloc: N above 65536 (fixed counter scratch)");
    int cur = -1;
    Q35_CUDA_TRY(cudaGetDevice(&cur));
    if (cur != w.device) return set_error(Q35_ERR_INVALID, "noalloc: make the weights' device current first");
    int32_t *base = nullptr;
    int st = noalloc_scratch(cur, &base);
    if (st) return st;
    Workspace ws;
    ws.acc = base;
    ws.acc_elems = NOALLOC_MAX_ACC;
    ws.tickets = reinterpret_cast<uint32_t *>(base + NOALLOC_MAX_ACC);
    ws.n_tickets = NOALLOC_MAX_CTR;
    ws.err = base + NOALLOC_ERR;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // start from zero whatever an earlier (or failed) call left; the error word is left
    // for q35_gemm_noalloc_device_error
    Q35_CUDA_TRY(cudaMemsetAsync(ws.acc, 0, acc * sizeof(int32_t), s));
    Q35_CUDA_TRY(cudaMemsetAsync(ws.tickets, 0, ctr * sizeof(uint32_t), s));
    GemvArgs a;
    a.x = x;
    a.M = M;
    if (x_layout == Q35_LAYOUT_COLMAJOR) { a.sx_row = 1; a.sx_k = M; }
    else if (x_layout == Q35_LAYOUT_ROWMAJOR) { a.sx_row = w.K; a.sx_k = 1; }
    else return set_error(Q35_ERR_INVALID, "noalloc: bad x_layout");
    if (out_layout == Q35_LAYOUT_COLMAJOR) { a.so_row = 1; a.so_col = M; }
    else if (out_layout == Q35_LAYOUT_ROWMAJOR) { a.so_row = w.N; a.so_col = 1; }
    else return set_error(Q35_ERR_INVALID, "noalloc: bad out_layout");
    a.C = C;
    a.y = y;
    return launch_gemv(w, a, ws, s);
}

// the failure record of q35_gemm_dev_noalloc's kernels on the current device: waits for
// the stream, then returns and clears the array's error word (no allocation)
extern "C" int q35_gemm_noalloc_device_error(void *stream) {
    using namespace q35;
    int cur = -1;
    Q35_CUDA_TRY(cudaGetDevice(&cur));
    int32_t *base = nullptr;
    int st = noalloc_scratch(cur, &base);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    int32_t v = 0;
    Q35_CUDA_TRY(cudaMemcpy(&v, base + NOALLOC_ERR, sizeof(int32_t), cudaMemcpyDeviceToHost));
    if (v != 0) {
        Q35_CUDA_TRY(cudaMemset(base + NOALLOC_ERR, 0, sizeof(int32_t)));
        return set_error(v, "q35_gemm_dev_noalloc: a kernel reported a bounded wait that gave up");
    }
    return Q35_OK;
}
