// core.matrix-multiply (transpose_right) without any device allocation: the
// tensor-core path's BF16 split of X (its only scratch) lives in a fixed,
// file-scope device array instead of caller-provided or context-owned
// memory.
//
// Who needs this: a host that owns every byte of device memory through its
// own pool (an executor that sizes all slots up front and must not see the
// library allocate behind it), or code that must not allocate at the call
// site at all — cudaMalloc/cudaFree can synchronise the whole device, which a
// decode loop with a fixed latency budget cannot afford.
//
// Cost and limits: every GPU that loads this library reserves the array
// (kStaticWorkspaceBytes = 64 MiB) until the process exits. A call whose
// workspace requirement (si_matrix_multiply_workspace_bytes: 4 * m * k bytes
// of BF16 split on the tensor-core path, plus the K-split partial sums when
// the GEMM splits K) exceeds it is refused. All calls share the one
// array, so two calls whose executions overlap on the GPU (different
// streams, or different host threads) race on it; serialise them. The
// contents left by the previous call are never read: the split kernel
// rewrites every element the GEMM reads, rows past m come from the TMA's
// zero fill and every partial sum is written before the reduction reads it,
// so nothing has to be cleared first.
#include <cuda_runtime.h>

#include <mutex>

#include "si_internal.h"

namespace {

constexpr uint64_t kStaticWorkspaceBytes = 64ull << 20;

static __device__ __align__(256) uint8_t g_static_workspace[kStaticWorkspaceBytes];

// Device address of g_static_workspace per device. In host code the symbol
// is only a stand-in; the real address comes from cudaGetSymbolAddress with
// the device current, on the device's first successful call. Only a
// successful lookup is kept: a failed one (for example a first call made
// while the stream is being captured) clears the runtime's error state and
// is tried again on the next call.
std::mutex g_slots_mu;
void *g_slots[si::kMaxDevices];

si_status workspace_for_current_device(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return si::fail(SI_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= si::kMaxDevices) return si::fail(SI_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
    std::lock_guard<std::mutex> g(g_slots_mu);
    if (!g_slots[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_workspace);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return si::fail(SI_ERR_CUDA, "cudaGetSymbolAddress(static workspace) failed on device %d: %s", dev,
                            cudaGetErrorString(e));
        }
        g_slots[dev] = p;
    }
    *out = g_slots[dev];
    return SI_OK;
}

}  // namespace

extern "C" {

si_status si_matrix_multiply_static_workspace(uint32_t weight_type, const float *x, const void *weight, float *y,
                                              int64_t m, int64_t n, int64_t k, void *stream) {
    uint64_t need = 0;
    if (si_status st = si_matrix_multiply_workspace_bytes(weight_type, m, n, k, &need)) return st;
    if (need > kStaticWorkspaceBytes)
        return si::fail(SI_ERR_INVALID_ARGUMENT,
                        "core.matrix-multiply (static workspace): m=%lld, k=%lld needs %llu bytes of scratch, "
                        "above the fixed %llu-byte workspace; use si_matrix_multiply with a larger workspace",
                        (long long)m, (long long)k, (unsigned long long)need,
                        (unsigned long long)kStaticWorkspaceBytes);
    void *ws = nullptr;
    if (si_status st = workspace_for_current_device(&ws)) return st;
    return si_matrix_multiply(weight_type, x, weight, y, m, n, k, ws, kStaticWorkspaceBytes, stream);
}

}  // extern "C"
