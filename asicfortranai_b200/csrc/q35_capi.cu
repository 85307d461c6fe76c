// q35_capi.cu -- the C ABI of libq35: contexts, resident weights, the device-pointer
// matmul and the drop-in entry points with the reference's signatures.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "q35_layer.cuh"

namespace q35 {

static thread_local std::string g_err;

int set_error(int status, const std::string &msg) {
    if (status != Q35_OK) g_err = msg;
    return status;
}

}  // namespace q35

using namespace q35;

struct q35_graph_s {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int device = 0;
};

namespace q35 {

int ensure_workspace(q35_ctx ctx, size_t acc_elems, size_t tickets) {
    Workspace &ws = ctx->ws;
    if (!ws.err) {
        Q35_CUDA_TRY(cudaMalloc(&ws.err, sizeof(int)));
        Q35_CUDA_TRY(cudaMemsetAsync(ws.err, 0, sizeof(int), ctx->stream));
    }
    if (acc_elems > ws.acc_elems) {
        if (ws.acc) cudaFree(ws.acc);
        ws.acc = nullptr;
        ws.acc_elems = 0;
        size_t n = std::max<size_t>(acc_elems, 64 * 1024);
        Q35_CUDA_TRY(cudaMalloc(&ws.acc, n * sizeof(int32_t)));
        Q35_CUDA_TRY(cudaMemsetAsync(ws.acc, 0, n * sizeof(int32_t), ctx->stream));
        ws.acc_elems = n;
    }
    if (tickets > ws.n_tickets) {
        if (ws.tickets) cudaFree(ws.tickets);
        ws.tickets = nullptr;
        ws.n_tickets = 0;
        size_t n = std::max<size_t>(tickets, 4096);
        Q35_CUDA_TRY(cudaMalloc(&ws.tickets, n * sizeof(uint32_t)));
        Q35_CUDA_TRY(cudaMemsetAsync(ws.tickets, 0, n * sizeof(uint32_t), ctx->stream));
        ws.n_tickets = n;
    }
    return Q35_OK;
}

static bool use_mma(q35_ctx ctx, int32_t M) {
    if (ctx->gemm_path == Q35_PATH_CUDA_CORES) return false;
    if (ctx->gemm_path == Q35_PATH_TENSOR_CORES) return true;
    return M >= MMA_MIN_M;
}

int ensure_gemm_workspace(q35_ctx ctx, const Weights &w, int32_t M) {
    size_t acc = gemv_workspace_acc_elems(w, std::min<int32_t>(M, 64)), tk = gemv_workspace_tickets(w);
    if (use_mma(ctx, M)) {
        acc = std::max(acc, mma_workspace_acc_elems(w, M, ctx->device));
        tk = std::max(tk, mma_workspace_tickets(w, M, ctx->device));
        Workspace &ws = ctx->ws;
        if ((size_t)M > ws.corr_elems) {
            if (ws.corr) cudaFree(ws.corr);
            ws.corr = nullptr;
            ws.corr_elems = 0;
            const size_t n = std::max<size_t>(M, 256);
            Q35_CUDA_TRY(cudaMalloc(&ws.corr, n * sizeof(int32_t)));
            ws.corr_elems = n;
        }
    }
    return ensure_workspace(ctx, acc, tk);
}

int ensure_scratch(q35_ctx ctx, size_t dbytes, size_t hbytes) {
    if (dbytes > ctx->d_scratch_bytes) {
        if (ctx->d_scratch) cudaFree(ctx->d_scratch);
        ctx->d_scratch = nullptr;
        ctx->d_scratch_bytes = 0;
        Q35_CUDA_TRY(cudaMalloc(&ctx->d_scratch, dbytes));
        ctx->d_scratch_bytes = dbytes;
    }
    if (hbytes > ctx->h_pinned_bytes) {
        if (ctx->h_pinned) cudaFreeHost(ctx->h_pinned);
        ctx->h_pinned = nullptr;
        ctx->h_pinned_bytes = 0;
        Q35_CUDA_TRY(cudaMallocHost(&ctx->h_pinned, hbytes));
        ctx->h_pinned_bytes = hbytes;
    }
    return Q35_OK;
}

int check_format(int format) {
    if (format != Q35_FMT_3P5BIT && format != Q35_FMT_INT4)
        return set_error(Q35_ERR_INVALID, "unknown weight format");
    return Q35_OK;
}

// allocate (or reuse) device storage for an N x K matrix of the given format
int weights_alloc(q35_ctx ctx, int format, int32_t N, int32_t K, q35_weights *io) {
    Weights w{};
    w.format = format;
    w.K = K;
    w.N = N;
    w.KB = (int32_t)ceil_div(K, KBLK);
    w.CG = (int32_t)ceil_div(N, CGW);
    w.device = ctx->device;
    w.tile_bytes = format == Q35_FMT_3P5BIT ? TILE35 : TILE4;
    w.bytes = (size_t)w.KB * w.CG * w.tile_bytes;
    q35_weights h = *io;
    if (h && h->w.format == format && h->w.K == K && h->w.N == N) return Q35_OK;
    if (h) q35_weights_free(h);
    *io = nullptr;
    h = new q35_weights_s();
    h->w = w;
    cudaError_t e = cudaMalloc(&h->w.tiles, w.bytes);
    if (e == cudaSuccess) e = cudaMalloc(&h->w.scales, sizeof(float) * (size_t)N);
    if (e == cudaSuccess && format == Q35_FMT_3P5BIT)
        e = cudaMalloc(&h->w.offsets, sizeof(float) * (size_t)N);
    if (e != cudaSuccess) {
        q35_weights_free(h);
        return set_error(Q35_ERR_NOMEM, std::string("weights allocation: ") + cudaGetErrorString(e));
    }
    *io = h;
    return Q35_OK;
}

// copy reference bytes (+ scales/offsets) to the device and repack into *io
int weights_fill(q35_ctx ctx, q35_weights h, const int8_t *W_Q, const float *scales,
                 const float *offsets, int src_on_device) {
    Weights &w = h->w;
    const size_t ref_bytes = (size_t)(w.K / 2) * w.N;
    const int8_t *d_ref = W_Q;
    if (!src_on_device) {
        int st = ensure_scratch(ctx, std::max(ref_bytes, ctx->d_scratch_bytes), 0);
        if (st) return st;
        Q35_CUDA_TRY(cudaMemcpyAsync(ctx->d_scratch, W_Q, ref_bytes, cudaMemcpyHostToDevice, ctx->stream));
        d_ref = reinterpret_cast<const int8_t *>(ctx->d_scratch);
    }
    cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    Q35_CUDA_TRY(cudaMemcpyAsync(w.scales, scales, sizeof(float) * (size_t)w.N, kind, ctx->stream));
    if (w.format == Q35_FMT_3P5BIT)
        Q35_CUDA_TRY(cudaMemcpyAsync(w.offsets, offsets, sizeof(float) * (size_t)w.N, kind, ctx->stream));
    return launch_repack(w, d_ref, ctx->stream);
}

int check_sizes(int32_t M, int32_t N, int32_t K) {
    if (M < 1 || M > GEMM_MAX_M) return set_error(Q35_ERR_INVALID, "M must be in [1,65536]");
    if (K > GEMM_MAX_K) return set_error(Q35_ERR_INVALID, "K above 131072");
    if (N < 1) return set_error(Q35_ERR_INVALID, "N must be positive");
    if (K < 2 || (K & 1)) return set_error(Q35_ERR_INVALID, "K must be even and >= 2");
    return Q35_OK;
}

int gemm_dev(q35_ctx ctx, q35_weights h, const int8_t *x, int32_t M, int x_layout, int32_t *C,
             float *y, int out_layout) {
    const Weights &w = h->w;
    if (M < 1 || M > GEMM_MAX_M) return set_error(Q35_ERR_INVALID, "M must be in [1,65536]");
    if (!x) return set_error(Q35_ERR_INVALID, "x is NULL");
    if (w.device != ctx->device) return set_error(Q35_ERR_INVALID, "weights live on another device");
    if (x_layout != Q35_LAYOUT_COLMAJOR && x_layout != Q35_LAYOUT_ROWMAJOR) return set_error(Q35_ERR_INVALID, "bad x_layout");
    GemvArgs a;
    a.x = x;
    a.M = M;
    if (x_layout == Q35_LAYOUT_COLMAJOR) { a.sx_row = 1; a.sx_k = M; }
    else { a.sx_row = w.K; a.sx_k = 1; }
    if (out_layout == Q35_LAYOUT_COLMAJOR) { a.so_row = 1; a.so_col = M; }
    else if (out_layout == Q35_LAYOUT_ROWMAJOR) { a.so_row = w.N; a.so_col = 1; }
    else return set_error(Q35_ERR_INVALID, "bad out_layout");
    a.C = C;
    a.y = y;
    int st = ensure_gemm_workspace(ctx, w, M);
    if (st) return st;
    if (use_mma(ctx, M)) {
        if (!mma_supported(w, a)) {
            // column-major activations, or rows TMA cannot address (K not a multiple of
            // 16, unaligned base): one row-major copy with 16-byte aligned rows
            const int64_t Kp = round_up(w.K, 16);
            const size_t need = (size_t)M * Kp;
            Workspace &ws = ctx->ws;
            if (ws.xt_bytes < need) {
                if (ws.xt) cudaFree(ws.xt);
                ws.xt = nullptr;
                ws.xt_bytes = 0;
                Q35_CUDA_TRY(cudaMalloc(&ws.xt, need));
                ws.xt_bytes = need;
            }
            if (x_layout == Q35_LAYOUT_COLMAJOR) st = launch_transpose_i8(x, ws.xt, w.K, M, Kp, ctx->stream);
            else Q35_CUDA_TRY(cudaMemcpy2DAsync(ws.xt, Kp, x, w.K, w.K, M, cudaMemcpyDeviceToDevice, ctx->stream));
            if (st) return st;
            a.x = ws.xt;
            a.sx_row = Kp;
            a.sx_k = 1;
            if (!mma_supported(w, a)) return set_error(Q35_ERR_INVALID, "tensor-core path: unsupported activation layout");
        }
        return launch_mma(w, a, ctx->ws, ctx->stream);
    }
    for (int32_t r0 = 0; r0 < M; r0 += 64) {   // CUDA cores: 64 rows per launch
        GemvArgs b = a;
        b.M = std::min<int32_t>(64, M - r0);
        b.x = x + (size_t)r0 * a.sx_row;
        b.C = C ? C + (size_t)r0 * a.so_row : nullptr;
        b.y = y ? y + (size_t)r0 * a.so_row : nullptr;
        st = launch_gemv(w, b, ctx->ws, ctx->stream);
        if (st) return st;
    }
    return Q35_OK;
}

int gemm_rows(q35_ctx ctx, q35_weights h, const int8_t *x, int32_t R, int32_t *C, float *y,
              const float *res) {
    const Weights &w = h->w;
    if (R < 1) return set_error(Q35_ERR_INVALID, "gemm_rows: no rows");
    int st = ensure_gemm_workspace(ctx, w, R);
    if (st) return st;
    GemvArgs a;
    a.M = R;
    a.x = x;
    a.sx_row = w.K;
    a.sx_k = 1;
    a.so_row = w.N;
    a.so_col = 1;
    a.C = C;
    a.y = y;
    a.res = res;
    if (use_mma(ctx, R) && mma_supported(w, a)) return launch_mma(w, a, ctx->ws, ctx->stream);
    for (int32_t r0 = 0; r0 < R; r0 += 64) {
        GemvArgs b = a;
        b.M = std::min<int32_t>(64, R - r0);
        b.x = x + (size_t)r0 * w.K;
        b.C = C ? C + (size_t)r0 * w.N : nullptr;
        b.y = y ? y + (size_t)r0 * w.N : nullptr;
        b.res = res ? res + (size_t)r0 * w.N : nullptr;
        st = launch_gemv(w, b, ctx->ws, ctx->stream);
        if (st) return st;
    }
    return Q35_OK;
}

int gemm_rows_rope(q35_ctx ctx, q35_weights h, const int8_t *x, int32_t R, float *y, const GemvRope &rope,
                   bool *fused) {
    *fused = false;
    const Weights &w = h->w;
    if (R < 1) return set_error(Q35_ERR_INVALID, "gemm_rows_rope: no rows");
    int st = ensure_gemm_workspace(ctx, w, R);
    if (st) return st;
    GemvArgs a;
    a.M = R;
    a.x = x;
    a.sx_row = w.K;
    a.sx_k = 1;
    a.so_row = w.N;
    a.so_col = 1;
    a.C = nullptr;
    a.y = y;
    if (use_mma(ctx, R) && mma_supported(w, a)) return Q35_OK;   // the caller runs the separate kernel
    for (int32_t r0 = 0; r0 < R; r0 += 64) {
        GemvArgs b = a;
        GemvRope g = rope;
        g.row0 = rope.row0 + r0;
        b.M = std::min<int32_t>(64, R - r0);
        b.x = x + (size_t)r0 * w.K;
        b.y = y ? y + (size_t)r0 * w.N : nullptr;
        b.rope = &g;
        st = launch_gemv(w, b, ctx->ws, ctx->stream);
        if (st) return st;
    }
    *fused = true;
    return Q35_OK;
}

int gemm_rows_swiglu(q35_ctx ctx, q35_weights h, const int8_t *x, int32_t R, float *y, int8_t *q) {
    const Weights &w = h->w;
    if (R < 1) return set_error(Q35_ERR_INVALID, "gemm_rows_swiglu: no rows");
    if (w.N % 2) return set_error(Q35_ERR_INVALID, "gemm_rows_swiglu: N must be even (gate, up pairs)");
    int st = ensure_gemm_workspace(ctx, w, R);
    if (st) return st;
    GemvArgs a;
    a.M = R;
    a.x = x;
    a.sx_row = w.K;
    a.sx_k = 1;
    a.so_row = w.N;
    a.so_col = 1;
    if (use_mma(ctx, R) && mma_supported(w, a)) {
        st = gemm_rows(ctx, h, x, R, nullptr, y, nullptr);
        return st ? st : launch_swiglu(y, q, nullptr, R, w.N / 2, ctx->stream);
    }
    for (int32_t r0 = 0; r0 < R; r0 += 64) {
        GemvArgs b = a;
        b.M = std::min<int32_t>(64, R - r0);
        b.x = x + (size_t)r0 * w.K;
        b.swiglu_q = q + (size_t)r0 * (w.N / 2);
        st = launch_gemv(w, b, ctx->ws, ctx->stream);
        if (st) return st;
    }
    return Q35_OK;
}

// a host pointer inside page-locked memory (cudaMallocHost / cudaHostRegister): copies
// can go to and from it directly
static bool host_pinned(const void *p) {
    if (!p) return false;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

// host A (M,K) col-major -> device, run, copy C and/or Out back; synchronous.  Calls on a
// context are ordered on its stream, so nothing waits before the copies are enqueued;
// page-locked caller buffers are copied directly (one cudaMemcpyAsync each), others go
// through the context's page-locked staging buffer.
int matmul_host(q35_ctx ctx, q35_weights h, const int8_t *A, int32_t M, int32_t *C, float *Out) {
    const Weights &w = h->w;
    const size_t a_bytes = (size_t)M * w.K;
    const size_t c_bytes = (size_t)M * w.N * sizeof(int32_t);
    const size_t y_bytes = (size_t)M * w.N * sizeof(float);
    const size_t a_off = 0, c_off = round_up(a_bytes, 256), y_off = c_off + round_up(c_bytes, 256);
    const size_t total = y_off + round_up(y_bytes, 256);
    const bool a_pin = host_pinned(A), c_pin = host_pinned(C), y_pin = host_pinned(Out);
    const size_t hneed = (a_pin && (!C || c_pin) && (!Out || y_pin)) ? 0 : total;
    int st = ensure_scratch(ctx, total, hneed);
    if (st) return st;
    uint8_t *d = reinterpret_cast<uint8_t *>(ctx->d_scratch);
    uint8_t *hp = reinterpret_cast<uint8_t *>(ctx->h_pinned);
    const void *src = A;
    if (!a_pin) {
        std::memcpy(hp + a_off, A, a_bytes);
        src = hp + a_off;
    }
    Q35_CUDA_TRY(cudaMemcpyAsync(d + a_off, src, a_bytes, cudaMemcpyHostToDevice, ctx->stream));
    int32_t *dC = C ? reinterpret_cast<int32_t *>(d + c_off) : nullptr;
    float *dY = Out ? reinterpret_cast<float *>(d + y_off) : nullptr;
    st = gemm_dev(ctx, h, reinterpret_cast<const int8_t *>(d + a_off), M, Q35_LAYOUT_COLMAJOR, dC, dY,
                  Q35_LAYOUT_COLMAJOR);
    if (st) return st;
    if (C) Q35_CUDA_TRY(cudaMemcpyAsync(c_pin ? (void *)C : (void *)(hp + c_off), dC, c_bytes,
                                        cudaMemcpyDeviceToHost, ctx->stream));
    if (Out) Q35_CUDA_TRY(cudaMemcpyAsync(y_pin ? (void *)Out : (void *)(hp + y_off), dY, y_bytes,
                                          cudaMemcpyDeviceToHost, ctx->stream));
    Q35_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    if (C && !c_pin) std::memcpy(C, hp + c_off, c_bytes);
    if (Out && !y_pin) std::memcpy(Out, hp + y_off, y_bytes);
    return Q35_OK;
}

std::mutex g_default_mu;
q35_ctx g_default[64] = {nullptr};

int default_ctx(q35_ctx *out) {
    int dev = 0;
    Q35_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(Q35_ERR_INVALID, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_default_mu);
    if (!g_default[dev]) {
        int st = q35_ctx_create(dev, nullptr, &g_default[dev]);
        if (st) return st;
    }
    *out = g_default[dev];
    return Q35_OK;
}

// The per-call entry points with the reference's signatures keep every matrix they are
// given resident on the device: entries keyed on (W_Q, scales, offsets addresses, K, N,
// format), each checked against a fingerprint of 64 sampled 64-byte windows of W_Q and
// up to 256 sampled scales and offsets, so the reference's caller that passes the same
// layer matrix on every token (int4_linear, transformer_layer.f90:86-89) uploads and
// repacks it once.  A matrix re-quantized at the same address changes its sampled bytes
// and is uploaded again; one edited in place in unsampled bytes only is not noticed --
// q35_dropin_cache_clear drops every entry.  The cache holds at most
// Q35_DROPIN_CACHE_MB megabytes (default 65536; least recently used entries go first);
// 0 turns it off (every call uploads, the reference's behaviour).
static uint64_t fnv1a(uint64_t h, const void *p, size_t n) {
    const uint8_t *b = static_cast<const uint8_t *>(p);
    for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}

static uint64_t dropin_fingerprint(const int8_t *wq, size_t wq_bytes, const float *sc, const float *of, int32_t N) {
    uint64_t h = 1469598103934665603ull;
    if (wq_bytes <= 4096) {
        h = fnv1a(h, wq, wq_bytes);
    } else {
        for (int i = 0; i < 64; ++i) h = fnv1a(h, wq + (wq_bytes - 64) * i / 63, 64);
    }
    const int ns = std::min<int32_t>(N, 256);
    for (int i = 0; i < ns; ++i) {
        const size_t j = ns > 1 ? (size_t)(N - 1) * i / (ns - 1) : 0;
        h = fnv1a(h, sc + j, sizeof(float));
        if (of) h = fnv1a(h, of + j, sizeof(float));
    }
    return h;
}

static size_t dropin_budget() {
    static size_t cached = (size_t)-1;
    if (cached == (size_t)-1) {
        const char *e = std::getenv("Q35_DROPIN_CACHE_MB");
        long long mb = e && *e ? std::atoll(e) : 65536;
        cached = mb > 0 ? (size_t)mb << 20 : 0;
    }
    return cached;
}

// the resident copy of a caller's matrix (uploaded on first sight or when its fingerprint
// changed); ctx->mu held
static int dropin_weights(q35_ctx ctx, int format, const int8_t *W_Q, const float *scales, const float *offsets,
                          int32_t N, int32_t K, q35_weights *out) {
    const size_t budget = dropin_budget();
    if (budget == 0) {
        int st = weights_alloc(ctx, format, N, K, &ctx->transient);
        if (st) return st;
        ++ctx->dropin_uploads;
        *out = ctx->transient;
        return weights_fill(ctx, ctx->transient, W_Q, scales, offsets, 0);
    }
    const uint64_t fp = dropin_fingerprint(W_Q, (size_t)(K / 2) * N, scales, offsets, N);
    const uint64_t tick = ++ctx->dropin_tick;
    for (q35_dropin_entry &e : ctx->dropin) {
        if (e.wq != W_Q || e.sc != scales || e.of != offsets || e.K != K || e.N != N || e.format != format) continue;
        e.last_use = tick;
        *out = e.w;
        if (e.fingerprint == fp) {
            ++ctx->dropin_hits;
            return Q35_OK;
        }
        e.fingerprint = fp;
        ++ctx->dropin_uploads;
        return weights_fill(ctx, e.w, W_Q, scales, offsets, 0);
    }
    q35_dropin_entry e;
    e.wq = W_Q; e.sc = scales; e.of = offsets; e.K = K; e.N = N; e.format = format;
    e.fingerprint = fp;
    e.last_use = tick;
    int st = weights_alloc(ctx, format, N, K, &e.w);
    if (st) return st;
    st = weights_fill(ctx, e.w, W_Q, scales, offsets, 0);
    if (st) {
        q35_weights_free(e.w);
        return st;
    }
    ++ctx->dropin_uploads;
    ctx->dropin.push_back(e);
    // least recently used entries out until the cache fits (the new entry stays)
    size_t bytes = 0;
    for (const q35_dropin_entry &x : ctx->dropin) bytes += q35_weights_device_bytes(x.w);
    while (bytes > budget && ctx->dropin.size() > 1) {
        size_t lru = 0;
        for (size_t i = 1; i < ctx->dropin.size(); ++i)
            if (ctx->dropin[i].last_use < ctx->dropin[lru].last_use) lru = i;
        if (ctx->dropin[lru].w == e.w) break;
        bytes -= q35_weights_device_bytes(ctx->dropin[lru].w);
        cudaStreamSynchronize(ctx->stream);   // an evicted matrix may still be read by queued work
        q35_weights_free(ctx->dropin[lru].w);
        ctx->dropin.erase(ctx->dropin.begin() + lru);
    }
    *out = ctx->dropin.back().w;
    return Q35_OK;
}

void dropin_release(q35_ctx ctx) {
    for (q35_dropin_entry &e : ctx->dropin) q35_weights_free(e.w);
    ctx->dropin.clear();
}

// per-call path of the reference signatures: the resident copy of the matrix, then the
// host matmul
int percall(int format, const int8_t *A, const int8_t *W_Q, const float *scales,
            const float *offsets, int32_t *C, float *Out, int32_t M, int32_t N, int32_t K) {
    // empty operands: the reference's loops run no iterations, and with K = 0 every
    // C(i,j) keeps its initial 0 (matmul_3p5bit_dynamic.f90:42-64, matmul_int4_groq.f90:33-53)
    if (M >= 0 && N >= 0 && K >= 0 && (K & 1) == 0 && (M == 0 || N == 0 || K == 0)) {
        if (M == 0 || N == 0) return Q35_OK;
        if (Out && (!scales || (format == Q35_FMT_3P5BIT && !offsets)))
            return set_error(Q35_ERR_INVALID, "NULL scales/offsets");
        for (int64_t j = 0; j < N; ++j)
            for (int64_t i = 0; i < M; ++i) {
                if (C) C[i + (int64_t)M * j] = 0;
                if (Out)
                    Out[i + (int64_t)M * j] = format == Q35_FMT_3P5BIT ? (0.0f + offsets[j]) * scales[j]
                                                                       : 0.0f * scales[j];
            }
        return Q35_OK;
    }
    int st = check_sizes(M, N, K);
    if (st) return st;
    if (!A || !W_Q || !scales || (format == Q35_FMT_3P5BIT && !offsets))
        return set_error(Q35_ERR_INVALID, "NULL input pointer");
    q35_ctx ctx;
    st = default_ctx(&ctx);
    if (st) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard g(ctx->device);
    q35_weights w = nullptr;
    st = dropin_weights(ctx, format, W_Q, scales, format == Q35_FMT_3P5BIT ? offsets : nullptr, N, K, &w);
    if (st) return st;
    return matmul_host(ctx, w, A, M, C, Out);
}

}  // namespace q35

extern "C" {

const char *q35_last_error(void) { return g_err.c_str(); }

const char *q35_status_string(int status) {
    switch (status) {
        case Q35_OK: return "ok";
        case Q35_ERR_INVALID: return "invalid argument";
        case Q35_ERR_CUDA: return "CUDA error";
        case Q35_ERR_NOMEM: return "out of memory";
        case Q35_ERR_NCCL: return "NCCL error";
        case Q35_ERR_TIMEOUT: return "device wait timed out";
        case Q35_ERR_STATE: return "invalid state";
        default: return "unknown status";
    }
}

int q35_version(void) { return 100; }

int q35_ctx_create(int device, void *stream, q35_ctx *out) {
    if (!out) return set_error(Q35_ERR_INVALID, "out is NULL");
    *out = nullptr;
    int n = 0;
    Q35_CUDA_TRY(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return set_error(Q35_ERR_INVALID, "no such CUDA device");
    DeviceGuard g(device);
    q35_ctx c = new q35_ctx_s();
    c->device = device;
    if (stream) {
        c->stream = reinterpret_cast<cudaStream_t>(stream);
    } else {
        cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete c;
            return set_error(Q35_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(e));
        }
        c->own_stream = true;
    }
    *out = c;
    return Q35_OK;
}

int q35_ctx_destroy(q35_ctx c) {
    if (!c) return Q35_OK;
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->transient) q35_weights_free(c->transient);
    dropin_release(c);
    if (c->ws.acc) cudaFree(c->ws.acc);
    if (c->ws.tickets) cudaFree(c->ws.tickets);
    if (c->ws.err) cudaFree(c->ws.err);
    if (c->ws.corr) cudaFree(c->ws.corr);
    if (c->ws.xt) cudaFree(c->ws.xt);
    if (c->d_scratch) cudaFree(c->d_scratch);
    if (c->h_pinned) cudaFreeHost(c->h_pinned);
    if (c->own_stream) cudaStreamDestroy(c->stream);
    for (auto &d : g_default)
        if (d == c) d = nullptr;
    delete c;
    return Q35_OK;
}

int q35_ctx_set_gemm_path(q35_ctx c, int path) {
    if (!c) return set_error(Q35_ERR_INVALID, "ctx is NULL");
    if (path != Q35_PATH_AUTO && path != Q35_PATH_CUDA_CORES && path != Q35_PATH_TENSOR_CORES)
        return set_error(Q35_ERR_INVALID, "bad gemm path");
    c->gemm_path = path;
    return Q35_OK;
}

int q35_ctx_synchronize(q35_ctx c) {
    if (!c) return set_error(Q35_ERR_INVALID, "ctx is NULL");
    DeviceGuard g(c->device);
    Q35_CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q35_OK;
}

int q35_ctx_device_error(q35_ctx c) {
    if (!c) return set_error(Q35_ERR_INVALID, "ctx is NULL");
    DeviceGuard g(c->device);
    Q35_CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (!c->ws.err) return Q35_OK;
    int v = 0;
    Q35_CUDA_TRY(cudaMemcpy(&v, c->ws.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) {
        Q35_CUDA_TRY(cudaMemset(c->ws.err, 0, sizeof(int)));
        return set_error(v, "a kernel on this context reported a bounded wait that gave up");
    }
    return Q35_OK;
}

int q35_ctx_capture_begin(q35_ctx c) {
    if (!c) return set_error(Q35_ERR_INVALID, "ctx is NULL");
    DeviceGuard g(c->device);
    Q35_CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
    return Q35_OK;
}

int q35_ctx_capture_end(q35_ctx c, q35_graph *out) {
    if (!c || !out) return set_error(Q35_ERR_INVALID, "NULL ctx/out");
    *out = nullptr;
    DeviceGuard g(c->device);
    q35_graph gr = new q35_graph_s();
    gr->device = c->device;
    cudaError_t e = cudaStreamEndCapture(c->stream, &gr->graph);
    if (e == cudaSuccess) e = cudaGraphInstantiate(&gr->exec, gr->graph, 0);
    if (e != cudaSuccess) {
        if (gr->graph) cudaGraphDestroy(gr->graph);
        delete gr;
        return set_error(Q35_ERR_CUDA, std::string("capture: ") + cudaGetErrorString(e));
    }
    *out = gr;
    return Q35_OK;
}

int q35_graph_launch(q35_graph gr, q35_ctx c) {
    if (!gr || !c) return set_error(Q35_ERR_INVALID, "NULL graph/ctx");
    DeviceGuard g(c->device);
    Q35_CUDA_TRY(cudaGraphLaunch(gr->exec, c->stream));
    return Q35_OK;
}

int q35_graph_destroy(q35_graph gr) {
    if (!gr) return Q35_OK;
    DeviceGuard g(gr->device);
    if (gr->exec) cudaGraphExecDestroy(gr->exec);
    if (gr->graph) cudaGraphDestroy(gr->graph);
    delete gr;
    return Q35_OK;
}

void *q35_ctx_stream(q35_ctx c) { return c ? reinterpret_cast<void *>(c->stream) : nullptr; }

int q35_weights_upload(q35_ctx ctx, int format, const int8_t *W_Q, const float *scales,
                       const float *offsets, int32_t N, int32_t K, int src_on_device,
                       q35_weights *out) {
    if (!ctx || !out) return set_error(Q35_ERR_INVALID, "NULL ctx/out");
    *out = nullptr;
    int st = check_format(format);
    if (st) return st;
    st = check_sizes(1, N, K);
    if (st) return st;
    if (!W_Q || !scales || (format == Q35_FMT_3P5BIT && !offsets))
        return set_error(Q35_ERR_INVALID, "NULL input pointer");
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard g(ctx->device);
    q35_weights h = nullptr;
    st = weights_alloc(ctx, format, N, K, &h);
    if (st) return st;
    st = weights_fill(ctx, h, W_Q, scales, offsets, src_on_device);
    if (st == Q35_OK) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, std::string("upload: ") + cudaGetErrorString(e));
    }
    if (st) {
        q35_weights_free(h);
        return st;
    }
    *out = h;
    return Q35_OK;
}

int q35_weights_generate(q35_ctx ctx, int format, int32_t N, int32_t K, uint64_t seed,
                         uint64_t tensor_id, double sigma, q35_weights *out) {
    if (!ctx || !out) return set_error(Q35_ERR_INVALID, "NULL ctx/out");
    *out = nullptr;
    int st = check_format(format);
    if (st) return st;
    st = check_sizes(1, N, K);
    if (st) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard g(ctx->device);
    float *W = nullptr;
    int8_t *wq = nullptr;
    float *sc = nullptr, *of = nullptr;
    const size_t n = (size_t)K * N;
    cudaError_t e = cudaMallocAsync(&W, n * sizeof(float), ctx->stream);
    if (e == cudaSuccess) e = cudaMallocAsync(&wq, n / 2, ctx->stream);
    if (e == cudaSuccess) e = cudaMallocAsync(&sc, (size_t)N * 4, ctx->stream);
    if (e == cudaSuccess) e = cudaMallocAsync(&of, (size_t)N * 4, ctx->stream);
    if (e != cudaSuccess) st = set_error(Q35_ERR_NOMEM, std::string("generate: ") + cudaGetErrorString(e));
    if (!st) st = q35_gen_normal_dev(W, (int64_t)n, seed, tensor_id, sigma, ctx->stream);
    if (!st) st = q35_quantize_dev(format, W, wq, sc, of, K, N, ctx->stream);
    q35_weights h = nullptr;
    if (!st) st = weights_alloc(ctx, format, N, K, &h);
    if (!st) st = weights_fill(ctx, h, wq, sc, of, 1);
    if (W) cudaFreeAsync(W, ctx->stream);
    if (wq) cudaFreeAsync(wq, ctx->stream);
    if (sc) cudaFreeAsync(sc, ctx->stream);
    if (of) cudaFreeAsync(of, ctx->stream);
    e = cudaStreamSynchronize(ctx->stream);
    if (!st && e != cudaSuccess) st = set_error(Q35_ERR_CUDA, std::string("generate: ") + cudaGetErrorString(e));
    if (st) {
        if (h) q35_weights_free(h);
        return st;
    }
    *out = h;
    return Q35_OK;
}

int q35_weights_free(q35_weights h) {
    if (!h) return Q35_OK;
    DeviceGuard g(h->w.device);
    if (h->w.tiles) cudaFree(h->w.tiles);
    if (h->w.scales) cudaFree(h->w.scales);
    if (h->w.offsets) cudaFree(h->w.offsets);
    delete h;
    return Q35_OK;
}

size_t q35_weights_device_bytes(q35_weights h) {
    if (!h) return 0;
    return h->w.bytes + sizeof(float) * (size_t)h->w.N * (h->w.offsets ? 2 : 1);
}

int q35_weights_download_ref(q35_ctx ctx, q35_weights h, int8_t *W_Q_host) {
    if (!ctx || !h || !W_Q_host) return set_error(Q35_ERR_INVALID, "NULL argument");
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard g(ctx->device);
    const size_t ref_bytes = (size_t)(h->w.K / 2) * h->w.N;
    Q35_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    int st = ensure_scratch(ctx, ref_bytes, 0);
    if (st) return st;
    st = launch_unpack_ref(h->w, reinterpret_cast<int8_t *>(ctx->d_scratch), ctx->stream);
    if (st) return st;
    Q35_CUDA_TRY(cudaMemcpyAsync(W_Q_host, ctx->d_scratch, ref_bytes, cudaMemcpyDeviceToHost, ctx->stream));
    Q35_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    return Q35_OK;
}

int q35_gemm_dev(q35_ctx ctx, q35_weights w, const int8_t *x, int32_t M, int x_layout,
                 int32_t *C, float *y, int out_layout) {
    if (!ctx || !w) return set_error(Q35_ERR_INVALID, "NULL ctx/weights");
    DeviceGuard g(ctx->device);
    return gemm_dev(ctx, w, x, M, x_layout, C, y, out_layout);
}

int q35_matmul_cached(q35_ctx ctx, q35_weights w, const int8_t *A, int32_t M, int32_t *C, float *Out) {
    if (!ctx || !w || !A) return set_error(Q35_ERR_INVALID, "NULL argument");
    int st = check_sizes(M, w->w.N, w->w.K);
    if (st) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard g(ctx->device);
    return matmul_host(ctx, w, A, M, C, Out);
}

int q35_matmul_3p5bit_awq(const int8_t *A, const int8_t *W_Q, const float *W_scales,
                          const float *W_offsets, int32_t *C, int32_t M, int32_t N, int32_t K) {
    if (!C && M > 0 && N > 0) return set_error(Q35_ERR_INVALID, "C is NULL");
    return percall(Q35_FMT_3P5BIT, A, W_Q, W_scales, W_offsets, C, nullptr, M, N, K);
}

// the reference's void signature has no status channel: a failure is also reported on
// stderr (the reference prints and stops, matmul_cublas.f90:116-117)
void matmul_3p5bit_awq(const int8_t *A, const int8_t *W_Q, const float *W_scales,
                       const float *W_offsets, int32_t *C, int32_t M, int32_t N, int32_t K) {
    if (q35_matmul_3p5bit_awq(A, W_Q, W_scales, W_offsets, C, M, N, K) != Q35_OK)
        std::fprintf(stderr, "matmul_3p5bit_awq: %s\n", g_err.c_str());
}

int q35_matmul_int4_awq(const int8_t *A, const int8_t *W_Q, const float *W_scales, int32_t *C,
                        int32_t M, int32_t N, int32_t K) {
    if (!C && M > 0 && N > 0) return set_error(Q35_ERR_INVALID, "C is NULL");
    return percall(Q35_FMT_INT4, A, W_Q, W_scales, nullptr, C, nullptr, M, N, K);
}

int q35_matmul_int4_fused(const int8_t *A, const int8_t *W_Q, const float *W_scales, float *Out,
                          int32_t M, int32_t N, int32_t K) {
    if (!Out && M > 0 && N > 0) return set_error(Q35_ERR_INVALID, "Out is NULL");
    return percall(Q35_FMT_INT4, A, W_Q, W_scales, nullptr, nullptr, Out, M, N, K);
}

int q35_dropin_cache_stats(int64_t *uploads, int64_t *hits, int64_t *entries, size_t *bytes) {
    q35_ctx ctx;
    int st = default_ctx(&ctx);
    if (st) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    size_t b = 0;
    for (const q35_dropin_entry &e : ctx->dropin) b += q35_weights_device_bytes(e.w);
    if (uploads) *uploads = ctx->dropin_uploads;
    if (hits) *hits = ctx->dropin_hits;
    if (entries) *entries = (int64_t)ctx->dropin.size();
    if (bytes) *bytes = b;
    return Q35_OK;
}

int q35_dropin_cache_clear(void) {
    q35_ctx ctx;
    int st = default_ctx(&ctx);
    if (st) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard g(ctx->device);
    Q35_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    dropin_release(ctx);
    return Q35_OK;
}

// rms_norm of transformer_layer.f90:155-178 on the GPU (rmsnorm_kernel, eps 1e-5 as
// RMS_NORM_EPS): x(seq_len, dim) and output column-major host arrays
int q35_rms_norm(const float *x, const float *weight, float *output, int32_t seq_len, int32_t dim) {
    if (seq_len == 0) return Q35_OK;
    if (seq_len < 0 || dim < 4 || dim % 4) return set_error(Q35_ERR_INVALID, "rms_norm: seq_len >= 0, dim a positive multiple of 4");
    if (!x || !weight || !output) return set_error(Q35_ERR_INVALID, "rms_norm: NULL argument");
    q35_ctx ctx;
    int st = default_ctx(&ctx);
    if (st) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    DeviceGuard g(ctx->device);
    const size_t n = (size_t)seq_len * dim, xb = round_up(n * 4, 256), wb = round_up((size_t)dim * 4, 256);
    st = ensure_scratch(ctx, 2 * xb + wb, xb);
    if (st) return st;
    float *hx = reinterpret_cast<float *>(ctx->h_pinned);
    uint8_t *d = reinterpret_cast<uint8_t *>(ctx->d_scratch);
    float *dx = reinterpret_cast<float *>(d), *dout = reinterpret_cast<float *>(d + xb);
    float *dw = reinterpret_cast<float *>(d + 2 * xb);
    for (int64_t i = 0; i < seq_len; ++i)            // (seq_len, dim) column-major -> rows
        for (int64_t j = 0; j < dim; ++j) hx[i * dim + j] = x[i + (int64_t)seq_len * j];
    Q35_CUDA_TRY(cudaMemcpyAsync(dx, hx, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    Q35_CUDA_TRY(cudaMemcpyAsync(dw, weight, (size_t)dim * 4, cudaMemcpyHostToDevice, ctx->stream));
    st = launch_rmsnorm(dx, dw, dout, nullptr, seq_len, dim, 1.0e-5f, ctx->stream);
    if (st) return st;
    Q35_CUDA_TRY(cudaMemcpyAsync(hx, dout, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    Q35_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    for (int64_t i = 0; i < seq_len; ++i)
        for (int64_t j = 0; j < dim; ++j) output[i + (int64_t)seq_len * j] = hx[i * dim + j];
    return Q35_OK;
}

}  // extern "C"
