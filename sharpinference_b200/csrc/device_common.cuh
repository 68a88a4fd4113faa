// Device-side helpers shared by the sm_100a kernels of libsharpinfer_cuda:
// mbarrier / bulk-copy wrappers with bounded waits, the device error word,
// binary16 loads and the Neumaier step of the cooperative mat-vec.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace si::dev {

// Device error word, one per translation unit (internal linkage, so no
// relocatable device code is needed). A bounded wait that runs out sets a
// bit here instead of trapping; each unit's host code reads and clears its
// word, and si_device_error_take() ORs them.
enum : uint32_t {
    kErrFullBarrierTimeout = 1u,
    kErrEmptyBarrierTimeout = 2u,
    kErrMmaBarrierTimeout = 4u,
    kErrEpilogueTimeout = 8u,
    kErrPeerTimeout = 16u,  // a row-sharded GEMV's rank never published its rows
    // a Q8_0 block scale above 512 or a Q4_K minimum scale above 1024 reached the
    // few-row GEMM's FP16 operands (gemm_fewrow.cu): those rows are not exact
    kErrRange = 32u,
};
static __device__ uint32_t g_error_word;

// Waits suspend in hardware: each try_wait may park the warp until the
// phase completes or kSuspendHintNs elapse, so a waiting warp takes no issue
// slots and does not hammer the barrier that TMA completions update. Every
// wait is still bounded: by kWaitLimitNs of %globaltimer and by kMaxPolls.
constexpr uint32_t kSuspendHintNs = 10000000u;    // 10 ms per poll at most
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s in total
constexpr uint32_t kMaxPolls = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and records `err`) when
// the time or poll budget runs out, so the caller can carry on without hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    atomicOr(&g_error_word, err);
    return false;
}

// 1-D bulk copy global -> shared (TMA, no tensor map, no multicast); bytes
// and both addresses must be multiples of 16. Completion is signalled as
// transaction bytes on `bar`.
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Programmatic dependent launch. `pdl_trigger` lets the next kernel in the
// stream start launching (its CTAs still wait for free SM resources);
// `pdl_wait` blocks until every prerequisite grid has completed and its
// memory is visible. Kernels read their activations and write their outputs
// only after pdl_wait; read-only weights may be prefetched before it.
// Both are no-ops when the kernel was launched without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float ldf(const float *p) { return *p; }
__device__ __forceinline__ float ldf(const __half *p) { return __half2float(*p); }
__device__ __forceinline__ void stf(float *p, float v) { *p = v; }
__device__ __forceinline__ void stf(__half *p, float v) { *p = __float2half_rn(v); }

// Neumaier step (add32 of the reference's cooperative mat-vec): rounding
// error of each addition is collected in `correction`; a non-finite total
// clears the correction so +/-Inf and NaN survive the final sum.
__device__ __forceinline__ void add32(float &sum, float &correction, float value) {
    const float total = __fadd_rn(sum, value);
    if (isfinite(total)) {
        const float residual = fabsf(sum) >= fabsf(value) ? __fadd_rn(__fsub_rn(sum, total), value)
                                                          : __fadd_rn(__fsub_rn(value, total), sum);
        correction = __fadd_rn(correction, residual);
    } else {
        correction = 0.0f;
    }
    sum = total;
}

}  // namespace si::dev
