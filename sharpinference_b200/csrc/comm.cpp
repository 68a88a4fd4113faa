// Row-sharded mat-vec across GPUs: each rank owns a contiguous slice of the
// weight rows, runs the GEMV on it, and the output slices are all-gathered
// (NCCL, on the caller's stream) into the full vector on every rank.
//
// NCCL is loaded at first use with dlopen("libnccl.so.2"), so the library has
// no link-time NCCL dependency; when the process already holds an NCCL (for
// example one loaded by PyTorch) that copy is reused. Communicator creation
// is non-blocking with a host-side deadline: a rank that never joins makes
// si_comm_create return SI_ERR_TIMEOUT (after aborting the half-built
// communicator) instead of hanging.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "si_internal.h"

struct si_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0;
    int rank = 0;
    int device = 0;
};

namespace si {
namespace {

struct Nccl {
    void *handle = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

Nccl &nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        n.handle = h;
        n.GetUniqueId = reinterpret_cast<decltype(n.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        n.CommInitRankConfig = reinterpret_cast<decltype(n.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
        n.CommGetAsyncError = reinterpret_cast<decltype(n.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        n.CommDestroy = reinterpret_cast<decltype(n.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        n.CommAbort = reinterpret_cast<decltype(n.CommAbort)>(dlsym(h, "ncclCommAbort"));
        n.AllGather = reinterpret_cast<decltype(n.AllGather)>(dlsym(h, "ncclAllGather"));
        n.GetErrorString = reinterpret_cast<decltype(n.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.GetUniqueId && n.CommInitRankConfig && n.CommGetAsyncError && n.CommDestroy && n.CommAbort &&
               n.AllGather && n.GetErrorString;
    });
    return n;
}

si_status nccl_fail(ncclResult_t r, const char *what) {
    return fail(SI_ERR_NCCL, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "NCCL error");
}

}  // namespace
}  // namespace si

using namespace si;

extern "C" {

si_status si_rowshard_plan(int64_t rows, int nranks, int rank, int64_t *row_begin, int64_t *row_count,
                           int64_t *rows_per_rank) {
    if (rows <= 0 || nranks <= 0 || rank < 0 || rank >= nranks || !row_begin || !row_count || !rows_per_rank)
        return fail(SI_ERR_INVALID_ARGUMENT, "row-shard plan needs rows > 0 and 0 <= rank < nranks");
    const int64_t per = (rows + nranks - 1) / nranks;
    const int64_t b = std::min<int64_t>(rows, per * rank);
    const int64_t e = std::min<int64_t>(rows, per * (rank + 1));
    *row_begin = b;
    *row_count = e - b;
    *rows_per_rank = per;
    return SI_OK;
}

si_status si_comm_unique_id(uint8_t *id, size_t capacity) {
    if (!id || capacity < sizeof(ncclUniqueId)) return fail(SI_ERR_INVALID_ARGUMENT, "id buffer needs 128 bytes");
    Nccl &n = nccl();
    if (!n.ok) return fail(SI_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    ncclUniqueId uid;
    if (ncclResult_t r = n.GetUniqueId(&uid)) return nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id, &uid, sizeof uid);
    return SI_OK;
}

si_status si_comm_create(int device, int nranks, int rank, const uint8_t *id, int timeout_ms, si_comm **out) {
    if (!out || !id || nranks <= 0 || rank < 0 || rank >= nranks || timeout_ms <= 0)
        return fail(SI_ERR_INVALID_ARGUMENT, "communicator needs an id, 0 <= rank < nranks and a timeout");
    *out = nullptr;
    Nccl &n = nccl();
    if (!n.ok) return fail(SI_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return fail(SI_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", device);
    }
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclComm_t comm = nullptr;
    const ncclResult_t r = n.CommInitRankConfig(&comm, nranks, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (comm) n.CommAbort(comm);
        if (prev >= 0) cudaSetDevice(prev);
        return nccl_fail(r, "ncclCommInitRankConfig");
    }
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        ncclResult_t state = ncclInProgress;
        n.CommGetAsyncError(comm, &state);
        if (state == ncclSuccess) break;
        if (state != ncclInProgress || std::chrono::steady_clock::now() > deadline) {
            n.CommAbort(comm);
            if (prev >= 0) cudaSetDevice(prev);
            if (state != ncclInProgress) return nccl_fail(state, "ncclCommInitRankConfig");
            return fail(SI_ERR_TIMEOUT, "NCCL communicator rank %d/%d not complete after %d ms", rank, nranks,
                        timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    auto *c = new si_comm();
    c->comm = comm;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    *out = c;
    if (prev >= 0) cudaSetDevice(prev);
    return SI_OK;
}

si_status si_comm_destroy(si_comm *comm) {
    if (!comm) return SI_OK;
    Nccl &n = nccl();
    if (n.ok && comm->comm) n.CommDestroy(comm->comm);
    delete comm;
    return SI_OK;
}

si_status si_rowshard_matvec_allgather(si_comm *comm, uint32_t weight_type, const void *weight_shard,
                                       const float *input, float *output_full, int64_t rows, int64_t cols,
                                       void *stream) {
    if (!comm) return fail(SI_ERR_INVALID_ARGUMENT, "null communicator");
    int64_t begin, count, per;
    if (si_status st = si_rowshard_plan(rows, comm->nranks, comm->rank, &begin, &count, &per)) return st;
    float *slice = output_full + per * comm->rank;
    if (count > 0)
        if (si_status st = si_matvec(weight_type, weight_shard, SI_TYPE_F32, input, SI_TYPE_F32, slice, count, cols,
                                     SI_MATVEC_DEFAULT, stream))
            return st;
    Nccl &n = nccl();
    ncclResult_t r =
        n.AllGather(slice, output_full, size_t(per), ncclFloat32, comm->comm, static_cast<cudaStream_t>(stream));
    // A non-blocking communicator may still be enqueueing the collective.
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(10);
    while (r == ncclInProgress) {
        if (std::chrono::steady_clock::now() > deadline)
            return fail(SI_ERR_TIMEOUT, "ncclAllGather still being enqueued after 10 s");
        std::this_thread::yield();
        n.CommGetAsyncError(comm->comm, &r);
    }
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return SI_OK;
}

}  // extern "C"
