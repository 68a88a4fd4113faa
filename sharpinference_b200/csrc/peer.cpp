// Row-sharded GEMV with the output exchange fused into the GEMV kernel.
//
// Every rank owns an "arena": a device buffer exported with CUDA IPC and
// mapped by every other rank of the node (NVLink / NVSwitch peer memory, plain
// loads and stores, no multicast objects). Output vectors live at the same
// byte offset in every arena. In si_rowshard_matvec_peer each rank computes
// its row slice (si_rowshard_plan) and its reducer warps store every output
// row into all ranks' arenas; the last CTA of the launch then publishes a
// per-call epoch into every rank's flag slot and waits, bounded, for all
// ranks' epochs, so the gathered vector is complete in every arena when the
// kernel completes in stream order. There is no separate collective launch.
//
// The last 4 KB of every arena hold the group's state: flags[nranks]
// (written by peers) at +0, the CTA ticket at +256 and the call epoch at
// +512. A rank can run at most one call ahead of another, so two consecutive
// calls must not use the same output offset.
#include <cuda_runtime.h>

#include <cstring>

#include "si_internal.h"

namespace {
constexpr uint64_t kStateBytes = 4096;
}

struct si_peer_group {
    int device = 0;
    int nranks = 0;
    int rank = 0;
    uint8_t *arenas[si::kernels::kMaxPeerRanks] = {};
    uint64_t arena_bytes = 0;
    uint64_t data_bytes = 0;  // arena_bytes - kStateBytes
};

using namespace si;

namespace {

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int device) {
        cudaGetDevice(&prev);
        cudaSetDevice(device);
    }
    ~DeviceScope() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

si_status cuda_fail(cudaError_t e, const char *what) {
    cudaGetLastError();
    return fail(SI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

extern "C" {

si_status si_ipc_export(const void *device_ptr, uint8_t *handle, size_t capacity) {
    if (!device_ptr || !handle || capacity < sizeof(cudaIpcMemHandle_t))
        return fail(SI_ERR_INVALID_ARGUMENT, "IPC export needs a device allocation and a 64-byte handle buffer");
    cudaIpcMemHandle_t h;
    if (cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(device_ptr))) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle, &h, sizeof h);
    return SI_OK;
}

si_status si_ipc_open(int device, const uint8_t *handle, void **ptr) {
    if (!handle || !ptr) return fail(SI_ERR_INVALID_ARGUMENT, "IPC open needs a handle and an output pointer");
    *ptr = nullptr;
    DeviceScope scope(device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    if (cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess))
        return cuda_fail(e, "cudaIpcOpenMemHandle");
    return SI_OK;
}

si_status si_ipc_close(int device, void *ptr) {
    if (!ptr) return SI_OK;
    DeviceScope scope(device);
    if (cudaError_t e = cudaIpcCloseMemHandle(ptr)) return cuda_fail(e, "cudaIpcCloseMemHandle");
    return SI_OK;
}

si_status si_peer_group_create(int device, int nranks, int rank, const uint64_t *arena_addrs, uint64_t arena_bytes,
                               si_peer_group **out) {
    if (!out || !arena_addrs || nranks < 1 || nranks > kernels::kMaxPeerRanks || rank < 0 || rank >= nranks)
        return fail(SI_ERR_INVALID_ARGUMENT, "peer group needs 1..%d ranks, a valid rank and the arena addresses",
                    kernels::kMaxPeerRanks);
    if (arena_bytes <= kStateBytes || arena_bytes % 256 != 0)
        return fail(SI_ERR_INVALID_ARGUMENT, "arena size must be a multiple of 256 bytes above 4 KB");
    *out = nullptr;
    auto *g = new si_peer_group();
    g->device = device;
    g->nranks = nranks;
    g->rank = rank;
    g->arena_bytes = arena_bytes;
    g->data_bytes = arena_bytes - kStateBytes;
    for (int q = 0; q < nranks; ++q) {
        if (!arena_addrs[q] || arena_addrs[q] % 256 != 0) {
            delete g;
            return fail(SI_ERR_INVALID_ARGUMENT, "arena %d is null or not 256-byte aligned", q);
        }
        g->arenas[q] = reinterpret_cast<uint8_t *>(arena_addrs[q]);
    }
    DeviceScope scope(device);
    if (cudaError_t e = cudaMemset(g->arenas[rank] + g->data_bytes, 0, kStateBytes)) {
        delete g;
        return cuda_fail(e, "peer group state reset");
    }
    if (cudaError_t e = cudaDeviceSynchronize()) {
        delete g;
        return cuda_fail(e, "peer group state reset");
    }
    *out = g;
    return SI_OK;
}

}  // extern "C"

namespace si {
uint8_t *peer_group_arena(si_peer_group *g, int *nranks, int *rank, uint64_t *data_bytes) {
    *nranks = g->nranks;
    *rank = g->rank;
    *data_bytes = g->data_bytes;
    return g->arenas[g->rank];
}

si_status peer_gather_desc(si_peer_group *g, uint64_t output_offset, int64_t row_base, int64_t rows,
                           kernels::PeerGather *out) {
    if (output_offset % 16 != 0 || row_base < 0 ||
        output_offset + uint64_t(row_base + rows) * 4 > g->data_bytes)
        return fail(SI_ERR_INVALID_ARGUMENT, "peer output rows [%lld, +%lld) at offset %llu leave the arena",
                    (long long)row_base, (long long)rows, (unsigned long long)output_offset);
    kernels::PeerGather pg{};
    for (int q = 0; q < g->nranks; ++q) {
        pg.ys[q] = reinterpret_cast<float *>(g->arenas[q] + output_offset);
        pg.flags[q] = reinterpret_cast<uint32_t *>(g->arenas[q] + g->data_bytes);
    }
    pg.ticket = reinterpret_cast<uint32_t *>(g->arenas[g->rank] + g->data_bytes + 256);
    pg.epoch = reinterpret_cast<uint32_t *>(g->arenas[g->rank] + g->data_bytes + 512);
    pg.nranks = g->nranks;
    pg.rank = g->rank;
    pg.row_base = row_base;
    *out = pg;
    return SI_OK;
}

// State area after the data bytes: flags (+0), ticket (+256), epoch (+512),
// publish-only counts (+1024: four kinds of kMaxPeerRanks u64), kind epochs (+1536).
si_status peer_gather_desc_nowait(si_peer_group *g, uint64_t output_offset, int64_t row_base, int64_t rows, int kind,
                                  kernels::PeerGather *out) {
    if (kind < 0 || kind > 3) return fail(SI_ERR_INVALID_ARGUMENT, "exchange kind %d", kind);
    if (si_status st = peer_gather_desc(g, output_offset, row_base, rows, out)) return st;
    for (int q = 0; q < g->nranks; ++q)
        out->counts[q] = reinterpret_cast<unsigned long long *>(g->arenas[q] + g->data_bytes + 1024 + 64 * kind);
    out->kind_epoch = reinterpret_cast<uint32_t *>(g->arenas[g->rank] + g->data_bytes + 1536 + 4 * kind);
    out->nowait = 1;
    return SI_OK;
}

si_status peer_counts(si_peer_group *g, int kind, const unsigned long long **counts, const uint32_t **epoch) {
    if (kind < 0 || kind > 3) return fail(SI_ERR_INVALID_ARGUMENT, "exchange kind %d", kind);
    *counts = reinterpret_cast<const unsigned long long *>(g->arenas[g->rank] + g->data_bytes + 1024 + 64 * kind);
    *epoch = reinterpret_cast<const uint32_t *>(g->arenas[g->rank] + g->data_bytes + 1536 + 4 * kind);
    return SI_OK;
}
}  // namespace si

extern "C" {

si_status si_peer_group_destroy(si_peer_group *group) {
    delete group;
    return SI_OK;
}

si_status si_rowshard_matvec_peer(si_peer_group *g, uint32_t weight_type, const void *weight_shard,
                                  const float *input, uint64_t output_offset, int64_t rows, int64_t cols,
                                  void *stream) {
    if (!g) return fail(SI_ERR_INVALID_ARGUMENT, "null peer group");
    if (weight_type != SI_TYPE_Q4_K && weight_type != SI_TYPE_Q8_0)
        return fail(SI_ERR_UNSUPPORTED, "row-sharded peer GEMV takes Q4_K or Q8_0 weights");
    if (!weight_shard || !input) return fail(SI_ERR_INVALID_ARGUMENT, "null weight shard or input");
    int64_t begin, count, per;
    if (si_status st = si_rowshard_plan(rows, g->nranks, g->rank, &begin, &count, &per)) return st;
    if (int64_t(per) * (g->nranks - 1) >= rows)
        return fail(SI_ERR_UNSUPPORTED, "%lld rows leave a rank of %d without rows", (long long)rows, g->nranks);
    if (output_offset % 16 != 0 || output_offset + uint64_t(rows) * 4 > g->data_bytes)
        return fail(SI_ERR_INVALID_ARGUMENT, "output [%llu, +%lld floats) is not 16-byte aligned inside the arena",
                    (unsigned long long)output_offset, (long long)rows);
    kernels::PeerGather pg{};
    for (int q = 0; q < g->nranks; ++q) {
        pg.ys[q] = reinterpret_cast<float *>(g->arenas[q] + output_offset);
        pg.flags[q] = reinterpret_cast<uint32_t *>(g->arenas[q] + g->data_bytes);
    }
    pg.ticket = reinterpret_cast<uint32_t *>(g->arenas[g->rank] + g->data_bytes + 256);
    pg.epoch = reinterpret_cast<uint32_t *>(g->arenas[g->rank] + g->data_bytes + 512);
    pg.nranks = g->nranks;
    pg.rank = g->rank;
    pg.row_base = begin;
    DeviceScope scope(g->device);
    const si_status st = kernels::matvec_quant_mma(weight_type, weight_shard, input, nullptr, count, cols, stream, &pg);
    if (st == SI_ERR_UNSUPPORTED)
        return fail(SI_ERR_UNSUPPORTED, "row-sharded peer GEMV: %lldx%lld shard is not on the tensor-core path",
                    (long long)count, (long long)cols);
    return st;
}

}  // extern "C"
