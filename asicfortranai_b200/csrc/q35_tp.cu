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

#include "q35_internal.cuh"

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
        std::this_thread::sleep_for(std::chrono::microseconds(200));
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

void tp_attach(q35_tp t, int delta) {
    if (t) t->users += delta;
}

int tp_rank(q35_tp t) { return t ? t->rank : 0; }
int tp_world(q35_tp t) { return t ? t->world : 1; }

}  // namespace q35

using namespace q35;

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
            const ncclResult_t fr = nccl().CommFinalize(comm);
            clean = (fr == ncclSuccess || fr == ncclInProgress) && nccl_settle(t, "finalize") == Q35_OK;
            t->comm = nullptr;
        }
        if (clean) nccl().CommDestroy(comm);
        else nccl().CommAbort(comm);
    }
    cudaDeviceSynchronize();
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

int q35_tp_allreduce_i32(q35_tp t, q35_ctx ctx, int32_t *buf, size_t count) {
    if (!t || !ctx || !buf) return set_error(Q35_ERR_INVALID, "tp_allreduce: NULL argument");
    DeviceGuard g(ctx->device);
    return tp_allreduce_i32(t, buf, count, ctx->stream);
}

}  // extern "C"
