// Per-device launch state shared by every kernel wrapper of the library.
//
// The dynamic shared-memory opt-in (cudaFuncAttributeMaxDynamicSharedMemorySize)
// and the SM count belong to a device, and one process may drive several
// devices from several host threads (one context per executor, as the
// reference's engine pools executors). So both are looked up per (device,
// kernel) under a lock instead of behind process-wide flags.
#include <cuda_runtime.h>

#include <mutex>
#include <unordered_map>

#include "si_internal.h"

namespace si {
namespace {

std::mutex g_mu;
int g_sms[kMaxDevices];                         // 0 = not yet queried
std::unordered_map<const void *, int> g_opted[kMaxDevices];  // per device: kernel -> limit already set

}  // namespace

int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return dev;
}

int device_sm_count() {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n > 0 ? n : 148;
    }
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_sms[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        g_sms[dev] = n > 0 ? n : 148;
    }
    return g_sms[dev];
}

int opt_in_smem(const void *kernel, int bytes) {
    const int dev = current_device();
    if (dev >= 0 && dev < kMaxDevices) {
        std::lock_guard<std::mutex> g(g_mu);
        const auto it = g_opted[dev].find(kernel);
        if (it != g_opted[dev].end() && it->second >= bytes) return cudaSuccess;
    }
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return e;
    }
    if (dev >= 0 && dev < kMaxDevices) {
        std::lock_guard<std::mutex> g(g_mu);
        int &v = g_opted[dev][kernel];
        if (v < bytes) v = bytes;
    }
    return cudaSuccess;
}

}  // namespace si
