// q35_tp.cu -- tensor-parallel communicator: one process per GPU, NCCL over NVLink.
//
// The reference has no parallel code; the LLaMA-70B shapes are split the Megatron way:
// q/k/v and gate/up by columns, o and down by rows.  A row-split matmul leaves an exact
// int32 partial accumulator on every rank; they are summed with one int32 all-reduce
// (integer addition is order free, so the sum equals the single-GPU accumulator bit for
// bit) before the (C + offset) * scale dequant.  Greedy sampling over a vocab-split LM
// head exchanges one (value, index) pair per row and rank.
//
// Failure handling: the communicator is created non-blocking and its initialisation is
// polled with a deadline; a rank that never joins makes q35_tp_create fail with
// Q35_ERR_TIMEOUT after ncclCommAbort instead of hanging the others.  A rank that learns
// of a failed peer (on the host: a flag, a store, a heartbeat) calls q35_tp_abort, from
// any thread; NCCL kernels still waiting for the peer then return and so does the stream.
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <cstdlib>
#include <thread>
#include <type_traits>
#include <vector>

#include "q35_layer.cuh"

struct q35_tp_s {
    std::atomic<ncclComm_t> comm{nullptr};
    int rank = 0, world = 1, device = 0;
    double timeout_s = 120.0;
    std::atomic<int> users{0};   // models built on this group (their graphs hold its collectives)
    // Buffers that collectives read or write.  NCCL registers the buffers of collectives
    // captured in CUDA graphs and releases the registration after the graph is gone, at a
    // time of its choosing; memory freed and reallocated in between could be reached
    // through a stale registration.  These buffers therefore belong to the communicator:
    // they only grow, and nothing is freed before the communicator is destroyed.
    struct Slot { void *p = nullptr; size_t bytes = 0; };
    std::vector<Slot> slots;
    std::vector<void *> retired;
    std::mutex mu;
    // one-shot all-reduce over NVLink peer memory (q35::ArView): this rank's receive area
    // (mapped by every peer through an IPC handle), the peers' areas mapped here, and the
    // per-CTA epoch counters
    bool ar_ok = false;
    void *ar_base = nullptr;
    uint32_t *ar_epoch = nullptr;
    std::vector<void *> ar_peer;   // [world], ar_peer[rank] = ar_base
};

namespace q35 {

// NCCL is bound at run time, on first use: the library itself carries no NCCL
// dependency, and a process that already holds an NCCL (the one a framework such as
// torch loaded) shares it instead of loading a second, possibly different, copy.
// Q35_NCCL_LIBRARY names a specific file.
struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

static const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = nullptr;
        if (const char *path = std::getenv("Q35_NCCL_LIBRARY")) h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char *e = dlerror();
            api.why = std::string("NCCL library not found: ") + (e ? e : "libnccl.so.2");
            return;
        }
        bool all = true;
        auto sym = [&](auto &fp, const char *name) {
            fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(h, name));
            if (!fp) all = false;
        };
        sym(api.GetUniqueId, "ncclGetUniqueId");
        sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(api.CommFinalize, "ncclCommFinalize");
        sym(api.CommDestroy, "ncclCommDestroy");
        sym(api.CommAbort, "ncclCommAbort");
        sym(api.AllReduce, "ncclAllReduce");
        sym(api.AllGather, "ncclAllGather");
        sym(api.GetErrorString, "ncclGetErrorString");
        api.ok = all;
        if (!all) api.why = "NCCL library lacks a required entry point (NCCL >= 2.18 needed)";
    });
    return api;
}

static int nccl_missing() { return set_error(Q35_ERR_NCCL, nccl().why); }

static int nccl_error(ncclResult_t r, const char *what) {
    return set_error(Q35_ERR_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
}

// wait until a non-blocking communicator has no operation in progress
static int nccl_settle(q35_tp t, const char *what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclComm_t comm = t->comm;
        if (!comm) return set_error(Q35_ERR_NCCL, std::string(what) + ": communicator aborted");
        ncclResult_t r = nccl().CommGetAsyncError(comm, &st);
        if (r != ncclSuccess) return nccl_error(r, what);
        if (st == ncclSuccess) return Q35_OK;
        if (st != ncclInProgress) return nccl_error(st, what);
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > t->timeout_s) return set_error(Q35_ERR_TIMEOUT, std::string(what) + ": timed out");
        // an enqueue settles within microseconds: poll without sleeping for the first
        // milliseconds, then back off (initialisation and teardown take longer)
        if (el < 2e-3) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

int tp_allreduce_i32(q35_tp t, int32_t *buf, size_t count, cudaStream_t s) {
    if (!t || t->world == 1) return Q35_OK;
    ncclComm_t comm = t->comm;
    if (!comm) return set_error(Q35_ERR_NCCL, "all-reduce: communicator aborted");
    ncclResult_t r = nccl().AllReduce(buf, buf, count, ncclInt32, ncclSum, comm, s);
    if (r == ncclInProgress) return nccl_settle(t, "all-reduce");
    if (r != ncclSuccess) return nccl_error(r, "all-reduce");
    return Q35_OK;
}

int tp_allgather(q35_tp t, const void *send, void *recv, size_t bytes, cudaStream_t s) {
    if (!t || t->world == 1) {
        if (send != recv) Q35_CUDA_TRY(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, s));
        return Q35_OK;
    }
    ncclComm_t comm = t->comm;
    if (!comm) return set_error(Q35_ERR_NCCL, "all-gather: communicator aborted");
    ncclResult_t r = nccl().AllGather(send, recv, bytes, ncclUint8, comm, s);
    if (r == ncclInProgress) return nccl_settle(t, "all-gather");
    if (r != ncclSuccess) return nccl_error(r, "all-gather");
    return Q35_OK;
}

// communicator-owned device buffer `slot` of at least `bytes` (grow-only)
int tp_buffer(q35_tp t, int slot, size_t bytes, void **out) {
    std::lock_guard<std::mutex> lk(t->mu);
    if ((int)t->slots.size() <= slot) t->slots.resize(slot + 1);
    q35_tp_s::Slot &b = t->slots[slot];
    if (b.bytes < bytes) {
        if (b.p) t->retired.push_back(b.p);
        b.p = nullptr;
        b.bytes = 0;
        DeviceGuard g(t->device);
        Q35_CUDA_TRY(cudaMalloc(&b.p, bytes));
        Q35_CUDA_TRY(cudaMemset(b.p, 0, bytes));
        b.bytes = bytes;
    }
    *out = b.p;
    return Q35_OK;
}

// ---- one-shot all-reduce of int32 partial accumulators, fused with the dequant and the
// residual add (x += (C + offset) * scale).  Receive area of each rank:
// [2 epoch parities][world source ranks][AR_MAX] 64-bit words, each word = (epoch << 32) |
// value.  CTA b of every rank owns slice b: it writes its slice of C into every rank's
// area (NVLink peer stores of whole words), then reads the slice from every rank, polling
// each word until its epoch is this call's: an aligned 64-bit store is single-copy atomic,
// so a word with the right epoch carries the right value -- no fences, no separate flags.
// The sum is integer (order free, equal to the one-GPU accumulator).  Two parities let a
// fast rank write the next call while a slow one still reads this one; a rank cannot get
// two calls ahead, since finishing a call needs every peer's words of it.  The grid is
// AR_CTAS <= the SM count, so every waiting CTA is resident.  Launched with programmatic
// dependent launch: CTAs that start early wait (griddepcontrol.wait) for the matmul that
// writes C before touching anything, and the kernel after this one waits for it before
// reading x, so calls still run one after another on each GPU.
constexpr int AR_CTAS = 32;
constexpr int AR_THREADS = 256;
constexpr int64_t AR_MAX = 1 << 18;   // int32 elements per call (decode: rows x hidden)
constexpr int AR_MAX_WORLD = 8;

struct ArView {
    uint64_t *buf[AR_MAX_WORLD];   // every rank's receive area (buf[rank] = this rank's own)
    uint32_t *epoch;               // this rank's per-CTA call counters
    uint64_t *wsum;                // [2 parities][rows][AR_CTAS] tagged partial sums of the fused norm
    int world, rank;
};

__global__ void __launch_bounds__(AR_THREADS)
ar_dequant_kernel(ArView v, const int32_t *__restrict__ C, int64_t n, int32_t N, const float *__restrict__ scales,
                  const float *__restrict__ offsets, float *__restrict__ x, int *err) {
    const int b = blockIdx.x, tid = threadIdx.x;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t per = ceil_div(n, (int64_t)gridDim.x);
    const int64_t lo = min(n, (int64_t)b * per), hi = min(n, lo + per);
    const uint32_t e = v.epoch[b] + 1u;
    const int par = (int)(e & 1u);
    const uint64_t tag = (uint64_t)e << 32;
    // 1) this rank's slice, tagged with the call's epoch, to every rank
    for (int p = 0; p < v.world; ++p) {
        uint64_t *dst = v.buf[p] + ((size_t)par * v.world + v.rank) * AR_MAX;
        for (int64_t i = lo + tid; i < hi; i += blockDim.x) {
            const uint64_t w = tag | (uint32_t)C[i];
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + i), "l"(w) : "memory");
        }
    }
    // 2) every rank's words of the slice (bounded polling), summed, dequant, residual
    const uint64_t *mine = v.buf[v.rank] + (size_t)par * v.world * AR_MAX;
    bool ok = true;
    for (int64_t i = lo + tid; i < hi && ok; i += blockDim.x) {
        int32_t acc = 0;
        for (int p = 0; p < v.world && ok; ++p) {
            const uint64_t *src = mine + (size_t)p * AR_MAX + i;
            uint64_t w = 0;
            uint32_t it = 0;
            for (;;) {
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
                if ((uint32_t)(w >> 32) == e) break;
                if (++it == (1u << 22)) { ok = false; break; }
                if (it > 64) __nanosleep(100);
            }
            acc += (int32_t)(uint32_t)w;
        }
        if (!ok) break;
        const int64_t j = i % N;
        const float f = __int2float_rn(acc);
        const float y = offsets ? __fmul_rn(__fadd_rn(f, offsets[j]), scales[j]) : __fmul_rn(f, scales[j]);
        x[i] = __fadd_rn(x[i], y);
    }
    if (!ok) atomicExch(err, Q35_ERR_TIMEOUT);
    __syncthreads();
    if (tid == 0) v.epoch[b] = e;
}

// The exchange of up to ARN_MAX_ROWS rows fused with the RMSNorm (+ int8 quantization) of
// the new rows that the next matmul consumes (rmsnorm_kernel, q35_layer.cu), bit for bit:
// rmsnorm_kernel gives each row one CTA, whose 1024 threads each sum the squares of float4
// groups t, t+1024, ... and whose 32 warps reduce by xor butterflies; here CTA c owns, in
// every row, exactly the groups of that kernel's warp c (j with (j mod 1024) / 32 == c),
// forms the warp's butterfly sum from the new values, and publishes it as a 64-bit word
// tagged with the call's epoch (one word per row and CTA); for each row the 32 words are
// read back (bounded polling; the 32 CTAs are resident together) and the same final
// butterfly is taken, so every CTA holds each row's one-kernel total and normalises its own
// elements.  The CTA's warps share the rows' publish-and-poll work.  The rows' new values
// stay in dynamic shared memory (rows x 128 x groups-per-thread floats).
constexpr int ARN_MAX_K = 8;                 // float4 groups per norm thread: hidden <= 8 * 4096
constexpr int ARN_MAX_ROWS = 64;             // rows of one fused call (decode batches)
constexpr int ARN_SMEM_MAX = 64 * 1024;      // the rows' new values in shared memory

struct NormOut {
    const float *w;   // norm weights [hidden]
    float eps;
    int8_t *q;        // int8 of the normalised rows (the next matmul's input), or null
    float *out;       // fp32 of the normalised rows, or null
};

__global__ void __launch_bounds__(AR_THREADS)
ar_dequant_norm_kernel(ArView v, const int32_t *__restrict__ C, int32_t R, int32_t N, const float *__restrict__ scales,
                       const float *__restrict__ offsets, float *__restrict__ x, NormOut no, int *err) {
    extern __shared__ float xs[];            // [R][ne]: this CTA's elements of every row
    __shared__ float rms_s[ARN_MAX_ROWS];
    const int c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t e = v.epoch[c] + 1u;
    const int par = (int)(e & 1u);
    const uint64_t tag = (uint64_t)e << 32;
    const int n4 = N / 4, kmax = (n4 + 1023) / 1024;
    const int ne = 128 * kmax;   // element slots per row: slot s -> group s/4 = (k, lane) = ((s/4)/32, (s/4)%32)
    const int tot = R * ne;
    auto elem = [&](int sl) -> int {   // element index (within a row) of slot sl, or -1
        const int g = sl >> 2, l = g & 31, k = g >> 5;
        const int j = 32 * c + l + 1024 * k;
        return j < n4 ? 4 * j + (sl & 3) : -1;
    };
    // 1) this rank's elements of every row, tagged, to every rank
    for (int p = 0; p < v.world; ++p) {
        uint64_t *dst = v.buf[p] + ((size_t)par * v.world + v.rank) * AR_MAX;
        for (int t = tid; t < tot; t += blockDim.x) {
            const int r = t / ne, i = elem(t - r * ne);
            if (i < 0) continue;
            const int64_t idx = (int64_t)r * N + i;
            const uint64_t w = tag | (uint32_t)C[idx];
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + idx), "l"(w) : "memory");
        }
    }
    // 2) sum every rank's words, dequant, residual: the new row values
    const uint64_t *mine = v.buf[v.rank] + (size_t)par * v.world * AR_MAX;
    bool ok = true;
    for (int t = tid; t < tot && ok; t += blockDim.x) {
        const int r = t / ne, i = elem(t - r * ne);
        if (i < 0) { xs[t] = 0.0f; continue; }
        const int64_t idx = (int64_t)r * N + i;
        int32_t acc = 0;
        for (int p = 0; p < v.world && ok; ++p) {
            const uint64_t *src = mine + (size_t)p * AR_MAX + idx;
            uint64_t w = 0;
            uint32_t it = 0;
            for (;;) {
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
                if ((uint32_t)(w >> 32) == e) break;
                if (++it == (1u << 22)) { ok = false; break; }
                if (it > 64) __nanosleep(100);
            }
            acc += (int32_t)(uint32_t)w;
        }
        if (!ok) break;
        const float f = __int2float_rn(acc);
        const float y = offsets ? __fmul_rn(__fadd_rn(f, offsets[i]), scales[i]) : __fmul_rn(f, scales[i]);
        const float nx = __fadd_rn(x[idx], y);
        x[idx] = nx;
        xs[t] = nx;
    }
    if (!ok) atomicExch(err, Q35_ERR_TIMEOUT);
    __syncthreads();
    // 3) per row, rmsnorm_kernel's warp c: its 32 threads' sums of squares, the butterfly,
    //    the tagged word; 4) the row's 32 words and the final butterfly
    uint64_t *ws = v.wsum + (size_t)par * ARN_MAX_ROWS * AR_CTAS;
    for (int r = wp; r < R; r += AR_THREADS / 32) {
        const float *xr = xs + (size_t)r * ne;
        float sq = 0.0f;
        for (int k = 0; k < kmax; ++k) {
            const int j = 32 * c + lane + 1024 * k;
            if (j >= n4) break;
            const float *g4 = xr + (k * 32 + lane) * 4;
            sq = __fadd_rn(sq, __fmul_rn(g4[0], g4[0]));
            sq = __fadd_rn(sq, __fmul_rn(g4[1], g4[1]));
            sq = __fadd_rn(sq, __fmul_rn(g4[2], g4[2]));
            sq = __fadd_rn(sq, __fmul_rn(g4[3], g4[3]));
        }
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) {
            const uint64_t w = tag | (uint64_t)__float_as_uint(sq);
            asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(ws + (size_t)r * AR_CTAS + c), "l"(w) : "memory");
        }
        uint64_t w = 0;
        uint32_t it = 0;
        bool got = true;
        for (;;) {
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(ws + (size_t)r * AR_CTAS + lane) : "memory");
            if ((uint32_t)(w >> 32) == e) break;
            if (++it == (1u << 22)) { got = false; break; }
            if (it > 64) __nanosleep(100);
        }
        if (!got) atomicExch(err, Q35_ERR_TIMEOUT);
        float t = got ? __uint_as_float((uint32_t)w) : 0.0f;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0) rms_s[r] = __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)N), no.eps));
    }
    __syncthreads();
    // 5) normalise this CTA's elements of every row (rmsnorm_kernel's arithmetic)
    for (int t = tid; t < tot; t += blockDim.x) {
        const int r = t / ne, i = elem(t - r * ne);
        if (i < 0) continue;
        const int64_t idx = (int64_t)r * N + i;
        const float o = __fmul_rn(__fdiv_rn(xs[t], rms_s[r]), no.w[i]);
        if (no.out) no.out[idx] = o;
        if (no.q) no.q[idx] = quant127(o);
    }
    __syncthreads();
    if (tid == 0) v.epoch[c] = e;
}

// shared-memory bytes of a fused call of R rows of width N, 0 when the fused form cannot
// take it
static size_t arn_smem(int32_t R, int32_t N) {
    if (R < 1 || R > ARN_MAX_ROWS || N < 4 || N % 4 || N > 4 * 1024 * ARN_MAX_K || (int64_t)R * N > AR_MAX) return 0;
    const size_t b = sizeof(float) * (size_t)R * 128 * ((N / 4 + 1023) / 1024);
    return b <= (size_t)ARN_SMEM_MAX ? b : 0;
}

static int arn_attr() {
    static bool set[64] = {false};
    int dev = 0;
    Q35_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !set[dev]) {
        Q35_CUDA_TRY(cudaFuncSetAttribute(ar_dequant_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          ARN_SMEM_MAX));
        set[dev] = true;
    }
    return Q35_OK;
}

// maps every rank's receive area into this process (IPC handles exchanged through the
// communicator); leaves t->ar_ok false (NCCL carries the exchange) unless every rank
// mapped every peer.  Every rank takes part in the same two collectives whatever fails
// locally, so no rank waits for a collective the others skip.
static void ar_setup(q35_tp t, cudaStream_t s) {
    if (t->world > AR_MAX_WORLD) return;
    const size_t bytes = sizeof(uint64_t) * 2 * t->world * AR_MAX;
    cudaIpcMemHandle_t h;
    std::memset(&h, 0, sizeof(h));
    bool ok = cudaMalloc(&t->ar_base, bytes) == cudaSuccess;
    if (!ok) t->ar_base = nullptr;
    // per-CTA epochs, then [2][ARN_MAX_ROWS][AR_CTAS] tagged words of the fused norm
    // (8-byte aligned)
    const size_t eb = sizeof(uint32_t) * AR_CTAS + sizeof(uint64_t) * 2 * ARN_MAX_ROWS * AR_CTAS;
    ok = ok && cudaMalloc(&t->ar_epoch, eb) == cudaSuccess;
    if (!ok && t->ar_epoch == nullptr) cudaGetLastError();
    ok = ok && cudaMemset(t->ar_base, 0, bytes) == cudaSuccess &&
         cudaMemset(t->ar_epoch, 0, eb) == cudaSuccess &&
         cudaIpcGetMemHandle(&h, t->ar_base) == cudaSuccess;
    cudaGetLastError();
    // the handles travel in a communicator-owned buffer (slot 5): a rank whose preparation
    // failed sends zeros and reports failure in the agreement below
    void *dv = nullptr;
    const size_t hb = sizeof(h) * t->world + sizeof(int32_t);
    if (tp_buffer(t, 5, hb, &dv) != Q35_OK) return;   // only if 1 KB cannot be allocated
    uint8_t *dh = static_cast<uint8_t *>(dv);
    int32_t *dflag = reinterpret_cast<int32_t *>(dh + sizeof(h) * t->world);
    cudaMemcpy(dh + sizeof(h) * t->rank, &h, sizeof(h), cudaMemcpyHostToDevice);
    ncclComm_t comm = t->comm;
    std::vector<cudaIpcMemHandle_t> all(t->world);
    ncclResult_t r = nccl().AllGather(dh + sizeof(h) * t->rank, dh, sizeof(h), ncclUint8, comm, s);
    if (r == ncclInProgress) r = nccl_settle(t, "all-reduce setup") == Q35_OK ? ncclSuccess : ncclInternalError;
    ok = ok && r == ncclSuccess && cudaStreamSynchronize(s) == cudaSuccess &&
         cudaMemcpy(all.data(), dh, sizeof(h) * t->world, cudaMemcpyDeviceToHost) == cudaSuccess;
    t->ar_peer.assign(t->world, nullptr);
    t->ar_peer[t->rank] = t->ar_base;
    for (int p = 0; ok && p < t->world; ++p) {
        if (p == t->rank) continue;
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
            break;
        }
        t->ar_peer[p] = ptr;
    }
    // every rank must agree: the peer-memory path runs only if all ranks mapped all peers
    const int32_t mine = ok ? 1 : 0;
    cudaMemcpy(dflag, &mine, sizeof(int32_t), cudaMemcpyHostToDevice);
    ncclResult_t r2 = nccl().AllReduce(dflag, dflag, 1, ncclInt32, ncclMin, comm, s);
    if (r2 == ncclInProgress) r2 = nccl_settle(t, "all-reduce setup") == Q35_OK ? ncclSuccess : ncclInternalError;
    int32_t all_ok = 0;
    if (r2 == ncclSuccess && cudaStreamSynchronize(s) == cudaSuccess)
        cudaMemcpy(&all_ok, dflag, sizeof(int32_t), cudaMemcpyDeviceToHost);
    t->ar_ok = ok && all_ok == 1;
}

// closes this rank's mappings of the peers' areas; with a healthy communicator, waits
// until every rank closed its mappings (a barrier through the communicator, taken by all
// ranks in q35_tp_destroy) before any area is freed
static void ar_close(q35_tp t, bool barrier) {
    for (int p = 0; p < (int)t->ar_peer.size(); ++p)
        if (p != t->rank && t->ar_peer[p]) cudaIpcCloseMemHandle(t->ar_peer[p]);
    t->ar_peer.clear();
    t->ar_ok = false;
    if (!barrier || !t->comm) return;
    void *dv = nullptr;
    cudaStream_t s = nullptr;
    if (tp_buffer(t, 5, sizeof(int32_t), &dv) == Q35_OK &&
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess) {
        ncclResult_t r = nccl().AllReduce(dv, dv, 1, ncclInt32, ncclSum, t->comm, s);
        if (r == ncclInProgress) nccl_settle(t, "teardown barrier");
        cudaStreamSynchronize(s);
    }
    if (s) cudaStreamDestroy(s);
}

static void ar_free(q35_tp t) {
    if (!t->ar_peer.empty()) ar_close(t, false);
    if (t->ar_base) cudaFree(t->ar_base);
    if (t->ar_epoch) cudaFree(t->ar_epoch);
    t->ar_base = nullptr;
    t->ar_epoch = nullptr;
}

int tp_allreduce_dequant(q35_tp t, int32_t *C, int64_t n, int32_t N, const float *scales, const float *offsets,
                         float *x, int *err, cudaStream_t s) {
    if (t && t->world > 1 && t->ar_ok && n <= AR_MAX) {
        ArView v{};
        for (int p = 0; p < t->world; ++p) v.buf[p] = static_cast<uint64_t *>(t->ar_peer[p]);
        v.epoch = t->ar_epoch;
        v.wsum = reinterpret_cast<uint64_t *>(t->ar_epoch + AR_CTAS);
        v.world = t->world;
        v.rank = t->rank;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(AR_CTAS);
        cfg.blockDim = dim3(AR_THREADS);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, ar_dequant_kernel, v, (const int32_t *)C, n, N, scales, offsets, x, err));
        return Q35_OK;
    }
    int st = tp_allreduce_i32(t, C, (size_t)n, s);
    if (st) return st;
    return launch_dequant_residual(C, scales, offsets, x, (int)(n / N), N, s);
}

int tp_allreduce_dequant_norm(q35_tp t, int32_t *C, int32_t R, int32_t N, const float *scales, const float *offsets,
                              float *x, const float *norm_w, float eps, int8_t *q, float *out, int *err, cudaStream_t s,
                              bool *fused) {
    *fused = false;
    const size_t smem = arn_smem(R, N);
    if (!(t && t->world > 1 && t->ar_ok && smem > 0)) return Q35_OK;
    int st = arn_attr();
    if (st) return st;
    ArView v{};
    for (int p = 0; p < t->world; ++p) v.buf[p] = static_cast<uint64_t *>(t->ar_peer[p]);
    v.epoch = t->ar_epoch;
    v.wsum = reinterpret_cast<uint64_t *>(t->ar_epoch + AR_CTAS);
    v.world = t->world;
    v.rank = t->rank;
    NormOut no{norm_w, eps, q, out};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(AR_CTAS);
    cfg.blockDim = dim3(AR_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, ar_dequant_norm_kernel, v, (const int32_t *)C, R, N, scales, offsets, x,
                                    no, err));
    *fused = true;
    return Q35_OK;
}

void tp_attach(q35_tp t, int delta) {
    if (t) t->users += delta;
}

int tp_rank(q35_tp t) { return t ? t->rank : 0; }
int tp_world(q35_tp t) { return t ? t->world : 1; }

}  // namespace q35

using namespace q35;

namespace {
__global__ void selftest_ints_kernel(const float *g, int32_t *C, int32_t n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        C[i] = __float2int_rz(g[i] * 1048576.0f);
}
__global__ void selftest_cmp_kernel(const float *a, const float *b, const float *c, const float *d, const int8_t *e,
                                    const int8_t *f, int32_t n, int32_t *mism) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int bad = (__float_as_uint(a[i]) != __float_as_uint(b[i])) + (__float_as_uint(c[i]) != __float_as_uint(d[i])) +
                        (e[i] != f[i]);
        if (bad) atomicAdd(mism, bad);
    }
}
}  // namespace

// Self-test of the exchange fused with RMSNorm on one GPU: a one-rank view (the kernel's own
// words, no peers) against the separate dequant + residual and RMSNorm kernels on the same
// seeded inputs of R rows, three calls in a row (both parities of the tagged words);
// *mismatches counts the elements of x, the fp32 norm and its int8 that differ in any bit.
extern "C" int q35_tp_norm_selftest_rows(q35_ctx ctx, int32_t R, int32_t N, uint64_t seed, int32_t *mismatches) {
    if (!ctx || !mismatches) return set_error(Q35_ERR_INVALID, "NULL argument");
    if (N < 4 || N % 4 || N > 4 * 1024 * ARN_MAX_K)
        return set_error(Q35_ERR_INVALID, "norm self-test: N must be a multiple of 4 up to 32768");
    if (arn_smem(R, N) == 0)
        return set_error(Q35_ERR_INVALID, "norm self-test: rows outside the fused form (1..64, rows x N <= 262144)");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->mu);
    int st = ensure_workspace(ctx, 1, 1);
    if (st) return st;
    st = arn_attr();
    if (st) return st;
    cudaStream_t s = ctx->stream;
    const int64_t n = (int64_t)R * N;
    const size_t area_bytes = sizeof(uint64_t) * 2 * AR_MAX;
    const size_t eb = sizeof(uint32_t) * AR_CTAS + sizeof(uint64_t) * 2 * ARN_MAX_ROWS * AR_CTAS;
    void *p[14] = {};
    const size_t fb = sizeof(float) * n, nb = sizeof(float) * N;
    const size_t sizes[14] = {area_bytes, eb, sizeof(int32_t) * n, fb, nb, nb, fb, fb, fb, nb, fb, (size_t)n, (size_t)n,
                              sizeof(int32_t)};
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 14 && e == cudaSuccess; ++i) e = cudaMalloc(&p[i], sizes[i]);
    uint64_t *area = (uint64_t *)p[0];
    uint32_t *epoch = (uint32_t *)p[1];
    int32_t *C = (int32_t *)p[2];
    float *gtmp = (float *)p[3], *sc = (float *)p[4], *of = (float *)p[5], *x0 = (float *)p[6], *x1 = (float *)p[7],
          *x2 = (float *)p[8], *w = (float *)p[9], *o1 = (float *)p[10];
    int8_t *q1 = (int8_t *)p[11], *q2 = (int8_t *)p[12];
    int32_t *mism = (int32_t *)p[13];
    float *o2 = gtmp;   // reused after C is made
    if (e == cudaSuccess) e = cudaMemsetAsync(area, 0, area_bytes, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(epoch, 0, eb, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(mism, 0, sizeof(int32_t), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->ws.err, 0, sizeof(int), s);
    if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    if (!st) st = q35_gen_normal_dev(gtmp, n, seed, 1, 1.0, s);
    if (!st) {
        selftest_ints_kernel<<<64, 256, 0, s>>>(gtmp, C, (int32_t)n);
        if (cudaGetLastError() != cudaSuccess) st = set_error(Q35_ERR_CUDA, "self-test kernel launch");
    }
    if (!st) st = q35_gen_normal_dev(sc, N, seed, 2, 1e-3, s);
    if (!st) st = q35_gen_normal_dev(of, N, seed, 3, 5.0, s);
    if (!st) st = q35_gen_normal_dev(x0, n, seed, 4, 1.0, s);
    if (!st) st = q35_gen_normal_dev(w, N, seed, 5, 1.0, s);
    const size_t smem = arn_smem(R, N);
    for (int round = 0; round < 3 && !st; ++round) {
        e = cudaMemcpyAsync(x1, x0, fb, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(x2, x0, fb, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) { st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e)); break; }
        st = launch_dequant_residual(C, sc, round == 1 ? nullptr : of, x1, R, N, s);
        if (!st) st = launch_rmsnorm(x1, w, o1, q1, R, N, 1e-5f, s);
        if (st) break;
        ArView v{};
        v.buf[0] = area;
        v.epoch = epoch;
        v.wsum = reinterpret_cast<uint64_t *>(epoch + AR_CTAS);
        v.world = 1;
        v.rank = 0;
        NormOut no{w, 1e-5f, q2, o2};
        ar_dequant_norm_kernel<<<AR_CTAS, AR_THREADS, smem, s>>>(v, C, R, N, sc, round == 1 ? nullptr : of, x2, no,
                                                                  ctx->ws.err);
        selftest_cmp_kernel<<<64, 256, 0, s>>>(x1, x2, o1, o2, q1, q2, (int32_t)n, mism);
        if (cudaGetLastError() != cudaSuccess) st = set_error(Q35_ERR_CUDA, "self-test kernel launch");
    }
    int h = 0, errv = 0;
    e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = cudaMemcpy(&h, mism, sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&errv, ctx->ws.err, sizeof(int), cudaMemcpyDeviceToHost);
    for (void *q : p)
        if (q) cudaFree(q);
    if (st) return st;
    if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    if (errv) {
        cudaMemset(ctx->ws.err, 0, sizeof(int));
        return set_error(errv, "norm self-test: the fused kernel reported a failed wait");
    }
    *mismatches = h;
    return Q35_OK;
}

extern "C" int q35_tp_norm_selftest(q35_ctx ctx, int32_t N, uint64_t seed, int32_t *mismatches) {
    return q35_tp_norm_selftest_rows(ctx, 1, N, seed, mismatches);
}

// Failure-path self-test of the exchange's bounded waits: a two-rank view whose both
// receive areas are this GPU's one area, so the "peer" words this rank polls for are never
// written.  Every wait gives up after its iteration limit (about a second), the kernel
// records Q35_ERR_TIMEOUT and returns; the context stays usable.
extern "C" int q35_tp_wait_selftest(q35_ctx ctx, int32_t *observed) {
    if (!ctx || !observed) return set_error(Q35_ERR_INVALID, "NULL argument");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->mu);
    int st = ensure_workspace(ctx, 1, 1);
    if (st) return st;
    cudaStream_t s = ctx->stream;
    const int64_t n = 1024;
    const int32_t N = 1024;
    uint64_t *area = nullptr;
    uint32_t *epoch = nullptr;
    int32_t *C = nullptr;
    float *sc = nullptr, *x = nullptr;
    const size_t area_bytes = sizeof(uint64_t) * 2 * 2 * AR_MAX;
    cudaError_t e = cudaMalloc(&area, area_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&epoch, sizeof(uint32_t) * AR_CTAS);
    if (e == cudaSuccess) e = cudaMalloc(&C, sizeof(int32_t) * n);
    if (e == cudaSuccess) e = cudaMalloc(&sc, sizeof(float) * N);
    if (e == cudaSuccess) e = cudaMalloc(&x, sizeof(float) * n);
    if (e == cudaSuccess) e = cudaMemsetAsync(area, 0, area_bytes, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(epoch, 0, sizeof(uint32_t) * AR_CTAS, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(C, 0, sizeof(int32_t) * n, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(sc, 0, sizeof(float) * N, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(x, 0, sizeof(float) * n, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->ws.err, 0, sizeof(int), s);
    if (e == cudaSuccess) {
        ArView v{};
        v.buf[0] = area;
        v.buf[1] = area;      // the peer's area is our own: its words of this call never arrive
        v.epoch = epoch;
        v.world = 2;
        v.rank = 0;
        ar_dequant_kernel<<<AR_CTAS, AR_THREADS, 0, s>>>(v, C, n, N, sc, nullptr, x, ctx->ws.err);
        e = cudaGetLastError();
    }
    int h = 0;
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = cudaMemcpy(&h, ctx->ws.err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(ctx->ws.err, 0, sizeof(int));
    for (void *p : {(void *)area, (void *)epoch, (void *)C, (void *)sc, (void *)x})
        if (p) cudaFree(p);
    if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    *observed = h;
    return Q35_OK;
}

extern "C" {

int q35_tp_unique_id(void *out, size_t n) {
    if (!out || n < sizeof(ncclUniqueId)) return set_error(Q35_ERR_INVALID, "tp_unique_id: buffer below 128 bytes");
    ncclUniqueId id;
    if (!nccl().ok) return nccl_missing();
    ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
    std::memcpy(out, &id, sizeof(id));
    return Q35_OK;
}

int q35_tp_create(q35_ctx ctx, int32_t rank, int32_t world, const void *id, size_t n, double timeout_s,
                  q35_tp *out) {
    if (!ctx || !id || !out || n < sizeof(ncclUniqueId)) return set_error(Q35_ERR_INVALID, "tp_create: bad arguments");
    if (world < 1 || rank < 0 || rank >= world) return set_error(Q35_ERR_INVALID, "tp_create: rank outside [0, world)");
    *out = nullptr;
    q35_tp t = new q35_tp_s();
    t->rank = rank;
    t->world = world;
    t->device = ctx->device;
    if (timeout_s > 0) t->timeout_s = timeout_s;
    if (world == 1) {
        *out = t;
        return Q35_OK;
    }
    if (!nccl().ok) {
        delete t;
        return nccl_missing();
    }
    DeviceGuard g(ctx->device);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = nccl().CommInitRankConfig(&comm, world, uid, rank, &cfg);
    t->comm = comm;
    int st = Q35_OK;
    if (r != ncclSuccess && r != ncclInProgress) st = nccl_error(r, "ncclCommInitRankConfig");
    if (!st) st = nccl_settle(t, "communicator initialisation");
    if (st) {
        if (comm) nccl().CommAbort(comm);
        delete t;
        return st;
    }
    ar_setup(t, ctx->stream);
    *out = t;
    return Q35_OK;
}

int q35_tp_destroy(q35_tp t) {
    if (!t) return Q35_OK;
    if (t->users > 0) return set_error(Q35_ERR_STATE, "tp_destroy: models built on this group are still alive");
    DeviceGuard g(t->device);
    if (ncclComm_t comm = t->comm.exchange(nullptr)) {
        // a communicator that carries an error (a peer failed) is aborted: finalising it
        // would wait for the peer
        ncclResult_t ae = ncclSuccess;
        bool clean = nccl().CommGetAsyncError(comm, &ae) == ncclSuccess && ae == ncclSuccess;
        if (clean) {
            t->comm = comm;
            ar_close(t, true);   // mappings closed on every rank before any area is freed
            const ncclResult_t fr = nccl().CommFinalize(comm);
            clean = (fr == ncclSuccess || fr == ncclInProgress) && nccl_settle(t, "finalize") == Q35_OK;
            t->comm = nullptr;
        }
        if (clean) nccl().CommDestroy(comm);
        else nccl().CommAbort(comm);
    }
    cudaDeviceSynchronize();
    ar_free(t);
    for (auto &b : t->slots)
        if (b.p) cudaFree(b.p);
    for (void *p : t->retired) cudaFree(p);
    delete t;
    return Q35_OK;
}

// abandon the communicator (a peer failed): outstanding and later collectives of this
// rank return instead of waiting for the peer
int q35_tp_abort(q35_tp t) {
    if (!t) return Q35_OK;
    if (ncclComm_t comm = t->comm.exchange(nullptr)) nccl().CommAbort(comm);
    return Q35_OK;
}

int q35_tp_rank(q35_tp t) { return tp_rank(t); }
int q35_tp_world(q35_tp t) { return tp_world(t); }

int q35_tp_allreduce_dequant(q35_tp t, q35_ctx ctx, int32_t *C, int64_t rows, int32_t N, const float *scales,
                             const float *offsets, float *x) {
    if (!t || !ctx || !C || !scales || !x || rows < 1 || N < 1)
        return set_error(Q35_ERR_INVALID, "tp_allreduce_dequant: bad arguments");
    DeviceGuard g(ctx->device);
    int st = ensure_workspace(ctx, 0, 0);
    if (st) return st;
    return tp_allreduce_dequant(t, C, rows * N, N, scales, offsets, x, ctx->ws.err, ctx->stream);
}

int q35_tp_allreduce_i32(q35_tp t, q35_ctx ctx, int32_t *buf, size_t count) {
    if (!t || !ctx || !buf) return set_error(Q35_ERR_INVALID, "tp_allreduce: NULL argument");
    DeviceGuard g(ctx->device);
    return tp_allreduce_i32(t, buf, count, ctx->stream);
}

}  // extern "C"
