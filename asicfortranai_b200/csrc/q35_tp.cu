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
// Q35_ERR_TIMEOUT after ncclCommAbort instead of hanging the others.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <string>
#include <thread>

#include "q35_internal.cuh"

struct q35_tp_s {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1, device = 0;
    double timeout_s = 120.0;
};

namespace q35 {

static int nccl_error(ncclResult_t r, const char *what) {
    return set_error(Q35_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

// wait until a non-blocking communicator has no operation in progress
static int nccl_settle(q35_tp t, const char *what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(t->comm, &st);
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
    ncclResult_t r = ncclAllReduce(buf, buf, count, ncclInt32, ncclSum, t->comm, s);
    if (r == ncclInProgress) return nccl_settle(t, "all-reduce");
    if (r != ncclSuccess) return nccl_error(r, "all-reduce");
    return Q35_OK;
}

int tp_allgather(q35_tp t, const void *send, void *recv, size_t bytes, cudaStream_t s) {
    if (!t || t->world == 1) {
        if (send != recv) Q35_CUDA_TRY(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, s));
        return Q35_OK;
    }
    ncclResult_t r = ncclAllGather(send, recv, bytes, ncclUint8, t->comm, s);
    if (r == ncclInProgress) return nccl_settle(t, "all-gather");
    if (r != ncclSuccess) return nccl_error(r, "all-gather");
    return Q35_OK;
}

int tp_rank(q35_tp t) { return t ? t->rank : 0; }
int tp_world(q35_tp t) { return t ? t->world : 1; }

}  // namespace q35

using namespace q35;

extern "C" {

int q35_tp_unique_id(void *out, size_t n) {
    if (!out || n < sizeof(ncclUniqueId)) return set_error(Q35_ERR_INVALID, "tp_unique_id: buffer below 128 bytes");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
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
    DeviceGuard g(ctx->device);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&t->comm, world, uid, rank, &cfg);
    int st = Q35_OK;
    if (r != ncclSuccess && r != ncclInProgress) st = nccl_error(r, "ncclCommInitRankConfig");
    if (!st) st = nccl_settle(t, "communicator initialisation");
    if (st) {
        if (t->comm) ncclCommAbort(t->comm);
        delete t;
        return st;
    }
    *out = t;
    return Q35_OK;
}

int q35_tp_destroy(q35_tp t) {
    if (!t) return Q35_OK;
    if (t->comm) {
        DeviceGuard g(t->device);
        ncclCommFinalize(t->comm);
        nccl_settle(t, "finalize");
        ncclCommDestroy(t->comm);
    }
    delete t;
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
