// Few-row quantized GEMM with the weights dequantised into tensor memory:
// Y[m, n] = X[m, k] W[n, k]^T for 2..32 input rows and Q4_K / Q8_0 weights
// (transformer.batch-shared-matvec at the reference's 16 rows and config 5's
// 32 streams, GpuBatchTransformerInstructions.cs:224-279; core.matrix-multiply
// with a few rows).
//
// Why a second few-row kernel: the BF16 hi/lo scheme of gemm_skinny.cu splits
// every dequantised weight into two BF16 halves in shared memory, ~14 thread
// instructions per weight, so it runs at a fifth of the weight stream. Here
// the weight operand needs no split:
//   * Q4_K: A = sc * q (6-bit scale times 4-bit code, at most 945) is exact
//     in FP16, built from the nibbles with one LOP3 (0x6400 exponent trick)
//     and one fused HFMA2 per two weights. The super-block scale d is applied
//     in FP32 when the accumulator of that super-block is read back (one FMA
//     per output per 256 weights); the mins term sum_s dmin m_s sum(x_s) is a
//     K = 16 MMA per super-block (A = dmin m_s as FP16 hi + lo, exact; B = the
//     32-element sums of X) into an accumulator of its own.
//   * Q8_0: A = d * q as FP16 hi + lo (q exact, the hi / lo split of the
//     product exact), one accumulator per 256-column stage, read back and
//     added in FP32.
//   * X (the B operand, in shared memory) is split once per stage into FP16
//     hi + lo, rows scaled by a power of two chosen per launch so that the
//     values and the 32-element sums stay inside FP16's range.
// The weight operand lives in tensor memory (tcgen05.mma with A from TMEM,
// written with tcgen05.st by the threads that dequantise it), so the
// dequantised weights never touch shared memory: the shared-memory traffic
// is the raw GGUF bytes (TMA in, one read) and the X tiles.
//
// K order. Inside each group of four consecutive columns the A operand holds
// the weights in the order 0, 2, 1, 3 (the LOP3 unpacking gives bytes 0 / 2
// and 1 / 3 as pairs); the X tiles use the same order, so the products pair
// up exactly and the sum is the same dot product.
//
// Roles (one CTA per SM, persistent over 128-row weight tiles; the K range
// optionally split over the CTAs of a cluster, partial sums added by the
// cluster's first CTA through distributed shared memory in rank order):
//   warp 0      lane 0: weight TMA (128 rows x one 256-column stage per copy)
//               lane 1: X TMA (FP32, 32-column boxes, 128-byte swizzle)
//   warp 1      TMEM allocation and the MMA issue (one thread)
//   warps 2-9   dequantise (two warps per TMEM lane quarter, one half of each
//               stage each), read the accumulators back, write Y
//   warps 10-   split X into FP16 hi / lo (+ 32-element sums), one thread per
//               (row, half sub-block)
// Every mbarrier wait is bounded (device error word, no trap, no hang).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "device_common.cuh"
#include "gemm_core.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

constexpr int kFwRows = 128;       // weight rows per tile (MMA M)
constexpr int kFwStageK = 256;     // columns per stage: one Q4_K super-block, eight Q8_0 blocks
constexpr int kFwDeqWarp0 = 2;     // warps 2..9 dequantise
constexpr int kFwDeqThreads = 256;
constexpr int kFwConvWarp0 = 10;   // then the X converters

template <int FMT, int BN>
struct FwCfg {
    static constexpr bool kQ4K = FMT == SI_TYPE_Q4_K;
    static constexpr uint32_t kSS = kQ4K ? 144u : 272u;       // raw bytes of one row's stage
    static constexpr uint32_t kRawBytes = kFwRows * kSS;
    static constexpr int kConvWarps = BN / 4;                 // 8 * BN threads: (input row, sub-block) of a stage
    static constexpr int kConvThreads = 32 * kConvWarps;
    static constexpr int kThreads = 32 * kFwConvWarp0 + kConvThreads;
    // X operand of half a stage (128 columns), hi and lo concatenated along N:
    // rows 0..BN-1 = FP16 hi, rows BN..2BN-1 = FP16 lo; two 64-column atoms,
    // 128-byte swizzle. One MMA with N = 2 BN covers both.
    static constexpr int kN = 2 * BN;
    static constexpr uint32_t kBHalf = uint32_t(kN) * 256u;
    static constexpr int kBStages = 3;                        // X operand ring depth in stages
    static constexpr int kBSlots = 2 * kBStages;
    // Q4_K: the stage's 32-column sums (rows as above, columns 0..15 of a 128-byte row)
    static constexpr uint32_t kBMin = kQ4K ? uint32_t(kN) * 128u : 0u;
    static constexpr int kBMinSlots = kQ4K ? kBStages : 0;
    static constexpr int kScaleSlots = 8;                     // per-(input row, stage) 1 / scale
    static constexpr int kRedStride = BN + 1;
    static constexpr uint32_t kRed = kFwRows * kRedStride * 4u;
    static constexpr uint32_t kFixed = kBSlots * kBHalf + kBMinSlots * kBMin + kRed + kScaleSlots * BN * 4u + 512u;
    static constexpr int kRawFit = int((227u * 1024u - 1024u - kFixed) / kRawBytes);
    static constexpr int kRaw = kRawFit > 8 ? 8 : kRawFit;
    static constexpr size_t kSmem = 1024 + kFixed + size_t(kRaw) * kRawBytes;
    // tensor memory (512 columns): A slots (half a stage each; Q8_0 hi then lo),
    // Q4_K mins operand slots (one per stage, 8 columns), stage accumulators (2 BN
    // columns: the products with X hi and with X lo, added at read-back)
    static constexpr int kACols = kQ4K ? 64 : 128;
    static constexpr int kASlots = kQ4K ? (BN == 16 ? 5 : 4) : 3;
    static constexpr int kMinCol0 = kASlots * kACols;
    static constexpr int kAMinSlots = kQ4K ? 3 : 0;
    static constexpr int kAccSlots = kQ4K ? 3 : (BN == 16 ? 3 : 2);
    static constexpr int kAccCol0 = 512 - kAccSlots * kN;
    static constexpr int kLag = kAccSlots - 1;                // read-back this many stages behind the dequantisation
    // kind::f16: D F32, A and B F16, both K-major, N = 2 BN, M = 128
    static constexpr uint32_t kIdesc = (1u << 4) | (uint32_t(kN >> 3) << 17) | (uint32_t(kFwRows >> 4) << 24);
    static_assert(kRaw >= 3, "weight ring");
    static_assert(kSmem <= 227u * 1024u, "shared memory");
    static_assert(kMinCol0 + kAMinSlots * 8 <= kAccCol0, "tensor memory");
    static_assert(BN == 16 || BN == 32, "rows per pass");
};

struct FwParams {
    const uint8_t *w;        // raw GGUF rows (also behind the tensor map), for the L2 prefetch
    uint64_t row_bytes;
    const float *x;
    float *y;
    const int32_t *control;  // null: every row; else rows t < control[1]
    int m, n, k;
    int splits;  // CTAs per cluster sharing one tile's K range
    int tiles;   // 128-row weight tiles
};

__device__ __forceinline__ uint32_t fw_cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void fw_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t fw_mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void fw_remote_arrive(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ float fw_ld_cluster(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
// Bounded mbarrier wait. The first wait of the CTA that runs out raises the
// CTA's abort flag; every later wait sees it and gives up at once, so a
// broken pipeline costs one time limit, not one per stage.
// Non-blocking phase test (no suspend): the common case of a phase that has
// already completed costs no sleep / wake-up.
__device__ __forceinline__ bool fw_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool fw_wait(uint64_t *bar, uint32_t parity, uint32_t err, volatile uint32_t *abort) {
    if (fw_test(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (*abort) return false;
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    *abort = 1u;
    atomicOr(&g_error_word, err);
    return false;
}
// Before the CTA exits: the last copy or MMA that this thread issued on
// `bar` has completed (already so unless a wait ran out). Bounded, and not
// cut short by the abort flag.
__device__ __forceinline__ void fw_drain(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return;
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    atomicOr(&g_error_word, kErrEpilogueTimeout);
}
// The same with cluster-scope acquire (the partial sums of another CTA).
__device__ __forceinline__ bool fw_wait_cluster(uint64_t *bar, uint32_t parity, uint32_t err,
                                                volatile uint32_t *abort) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (*abort) return false;
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
            : "memory");
        if (ok) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    *abort = 1u;
    atomicOr(&g_error_word, err);
    return false;
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (FP16 operands, FP32 accumulator).
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t t, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(t), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t t, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            t),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t t, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(t),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
// tcgen05.ld of 8 / 16 columns without the wait (tc_wait_ld after a batch of loads)
__device__ __forceinline__ void tmem_ld8_nw(uint32_t t, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(t));
}
__device__ __forceinline__ void tmem_ld16_nw(uint32_t t, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(t));
}
template <int N>
__device__ __forceinline__ void tmem_ld_nw(uint32_t t, uint32_t (&v)[N]) {
    if constexpr (N == 8) tmem_ld8_nw(t, v);
    else tmem_ld16_nw(t, v);
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed FP16 arithmetic on 32-bit registers (round to nearest, fused FMA).
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// FP32 pair -> FP16 hi + lo (hi = round(v), lo = round(v - hi)).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    hi = h2bits(h);
    // (a, b) - hi in one packed FMA (x * -1 + y is exact)
    const float2 r = __ffma2_rn(hf, make_float2(-1.0f, -1.0f), make_float2(a, b));
    lo = h2bits(__floats2half2_rn(r.x, r.y));
}

// One Q4_K half stage of this thread's weight row (sub-blocks 4h .. 4h+3)
// into tensor memory as sc * q (FP16, exact). The row's stage is read back as
// c * accumulator with c = d (dmin when d is zero); for h = 1 also the mins
// operand of the stage: a_s = -dmin m_s / c (s = 0..7) as FP16 hi (columns
// 0..7 of K) and lo (8..15), so that the mins term lands in the same
// accumulator. Returns c.
__device__ __forceinline__ float dequant_q4k_half(const uint8_t *src, int h, uint32_t ta, uint32_t tmin) {
    const uint4 hd = *reinterpret_cast<const uint4 *>(src);
    const uint32_t d_bits = hd.x & 0xffffu, dmin_bits = hd.x >> 16;
    const bool dz = (d_bits & 0x7fffu) == 0u;
    const float d = h16(d_bits), dmin = h16(dmin_bits);
    const float c = dz ? dmin : d;
    const uint32_t sc_lo = hd.y & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
    const uint32_t scw = h ? sc_hi : sc_lo;  // byte i: scale of sub-block 4h + i
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int j = 2 * h + cc;  // 64-column chunk: low nibbles sub-block 2j, high nibbles 2j + 1
        const uint4 qa = *reinterpret_cast<const uint4 *>(src + 16 + 32 * j);
        const uint4 qb = *reinterpret_cast<const uint4 *>(src + 32 + 32 * j);
        // (1024 + q) * sc - 1024 sc and (1024 + 16 q) * sc / 16 - 64 sc: one rounding of an exact
        // value; all zero when d is zero (the row's stage is then its mins term alone)
        const float sl = dz ? 0.0f : float((scw >> (16 * cc)) & 0xffu);
        const float sh = dz ? 0.0f : float((scw >> (16 * cc + 8)) & 0xffu);
        const uint32_t fl = h2bits(__float2half2_rn(sl)), nl = h2bits(__float2half2_rn(-1024.0f * sl));
        const uint32_t fh = h2bits(__float2half2_rn(sh * 0.0625f)), nh = h2bits(__float2half2_rn(-64.0f * sh));
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint32_t out[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = q[i], w8 = q[i] >> 8;
            out[2 * i] = hfma2u((w & 0x000F000Fu) | 0x64006400u, fl, nl);
            out[2 * i + 1] = hfma2u((w8 & 0x000F000Fu) | 0x64006400u, fl, nl);
            out[16 + 2 * i] = hfma2u((w & 0x00F000F0u) | 0x64006400u, fh, nh);
            out[16 + 2 * i + 1] = hfma2u((w8 & 0x00F000F0u) | 0x64006400u, fh, nh);
        }
        tmem_st32(ta + 32u * uint32_t(cc), out);
    }
    if (h == 1) {
        if (!dz && fabsf(dmin) > 1000.0f * fabsf(d) && (dmin_bits & 0x7fffu) < 0x7c00u)
            atomicOr(&g_error_word, kErrRange);
        const float rc = c != 0.0f ? __frcp_rn(c) : 0.0f;
        const float nd = -dmin * rc;
        const uint32_t mn_lo = hd.z & 0x3F3F3F3Fu;
        const uint32_t mn_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        uint32_t mo[8];
#pragma unroll
        for (int s = 0; s < 8; s += 2) {
            const uint32_t mw = s < 4 ? mn_lo : mn_hi;
            split_pair(nd * float((mw >> (8 * (s & 3))) & 0xffu), nd * float((mw >> (8 * ((s + 1) & 3))) & 0xffu),
                       mo[s / 2], mo[4 + s / 2]);
        }
        tmem_st8(tmin, mo);
    }
    return c;
}

// One Q8_0 half stage (blocks 4h .. 4h+3 of the row's eight) into tensor
// memory as d * q in FP16 hi (columns 0..63) and lo (64..127).
__device__ __forceinline__ void dequant_q80_half(const uint8_t *src, int h, uint32_t ta) {
    const uint2 *p = reinterpret_cast<const uint2 *>(src + 136 * h);  // 136 bytes = 4 blocks of 34, 8-byte aligned
    uint32_t wv[34];
#pragma unroll
    for (int i = 0; i < 17; ++i) {
        const uint2 t = p[i];
        wv[2 * i] = t.x;
        wv[2 * i + 1] = t.y;
    }
#pragma unroll
    for (int bl = 0; bl < 4; ++bl) {
        // block bl starts at byte 34 bl: d in the low half of word 17 bl / 2 for even bl
        // (codes from byte 2, realigned), in the high half of word 8 + 17 (bl - 1) / 2
        // for odd bl (codes word-aligned after it)
        const int w0 = (bl & 1) ? 8 + 17 * (bl >> 1) : 17 * (bl >> 1);
        const uint32_t dbits = (bl & 1) ? wv[w0] >> 16 : wv[w0] & 0xffffu;
        if ((dbits & 0x7fffu) > 0x6000u && (dbits & 0x7fffu) < 0x7c00u) atomicOr(&g_error_word, kErrRange);
        const uint32_t d2 = dbits | (dbits << 16);
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = (bl & 1) ? wv[w0 + 1 + i] : prmt(wv[w0 + i], wv[w0 + i + 1], 0x5432u);
            // bytes 0 / 2 and 1 / 3 as FP16 1152 + q (sign bit flipped into the mantissa), minus 1152: q exact
            const uint32_t v0 = ((w ^ 0x64806480u) & 0x00FF00FFu) | (0x64806480u & 0xFF00FF00u);
            const uint32_t v1 = (((w >> 8) ^ 0x64806480u) & 0x00FF00FFu) | (0x64806480u & 0xFF00FF00u);
            const uint32_t q0 = hsub2u(v0, 0x64806480u), q1 = hsub2u(v1, 0x64806480u);
            const uint32_t h0 = hmul2u(q0, d2), h1 = hmul2u(q1, d2);
            hi[2 * i] = h0;
            hi[2 * i + 1] = h1;
            lo[2 * i] = hfma2u(q0, d2, h0 ^ 0x80008000u);
            lo[2 * i + 1] = hfma2u(q1, d2, h1 ^ 0x80008000u);
        }
        tmem_st16(ta + 16u * uint32_t(bl), hi);
        tmem_st16(ta + 64u + 16u * uint32_t(bl), lo);
    }
}

template <int FMT, int BN>
__global__ void __launch_bounds__(FwCfg<FMT, BN>::kThreads, 1)
    fewrow_ts_kernel(const __grid_constant__ CUtensorMap wmap, const FwParams p) {
    using C = FwCfg<FMT, BN>;
    constexpr int kR = C::kRaw, kA = C::kASlots, kNB = C::kBSlots, kNAcc = C::kAccSlots, kHalfBN = BN / 2;
    constexpr int kNS = C::kScaleSlots, kLag = C::kLag, kSD = 8;
    constexpr bool kEarly = BN == 16;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t *bring = smem;                                  // kNB half-stage slots of the X operand
    uint8_t *bmin = bring + kNB * C::kBHalf;               // Q4_K: kBMinSlots stage slots of X sums
    uint8_t *raw = bmin + C::kBMinSlots * C::kBMin;        // kR stage slots of raw weight rows
    float *red = reinterpret_cast<float *>(raw + size_t(kR) * C::kRawBytes);
    float *scale_inv = red + kFwRows * C::kRedStride;      // [kNS][BN]: 1 / (power-of-two scale) per stage and row
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(scale_inv + kNS * BN);
    uint64_t *raw_empty = raw_full + kR;
    uint64_t *a_full = raw_empty + kR;
    uint64_t *xb_full = a_full + kA;
    uint64_t *acc_empty = xb_full + kNB;
    uint64_t *stage_done = acc_empty + kNAcc;  // [kSD]: every MMA of the stage has completed (one commit)
    uint64_t *scale_full = stage_done + kSD;
    uint64_t *red_full = scale_full + kNS;
    uint64_t *red_free = red_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(red_free + 1);
    volatile uint32_t *abort = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int splits = p.splits;
    const uint32_t rank = splits > 1 ? fw_cluster_rank() : 0u;
    const int cluster_id = int(blockIdx.x) / splits, nclusters = int(gridDim.x) / splits;
    const int stages_total = p.k / kFwStageK;
    const int st0 = int(int64_t(stages_total) * rank / splits);
    const int nst = int(int64_t(stages_total) * (rank + 1) / splits) - st0;
    const int my_tiles = cluster_id < p.tiles ? (p.tiles - 1 - cluster_id) / nclusters + 1 : 0;

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kR; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kFwDeqThreads);
        }
        for (int i = 0; i < kA; ++i) mbar_init(&a_full[i], kFwDeqThreads / 2);
        for (int i = 0; i < kNB; ++i) mbar_init(&xb_full[i], C::kConvThreads / 2);
        for (int i = 0; i < kNAcc; ++i) mbar_init(&acc_empty[i], kFwDeqThreads);
        for (int i = 0; i < kSD; ++i) mbar_init(&stage_done[i], 1);
        for (int i = 0; i < kNS; ++i) mbar_init(&scale_full[i], C::kConvThreads);
        mbar_init(red_full, kFwDeqThreads * (splits > 1 ? splits - 1 : 1));
        mbar_init(red_free, kFwDeqThreads);
        *abort = 0u;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (splits > 1) fw_cluster_sync();  // every CTA's barriers exist before any remote arrive
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // weights: read-only, streamed before the dependency wait; rows past n read as zeros
            uint32_t g = 0;
            for (int ti = 0; ti < my_tiles; ++ti) {
                const int tile = cluster_id + ti * nclusters;
                for (int s = 0; s < nst; ++s, ++g) {
                    const uint32_t slot = g % kR;
                    if (g >= uint32_t(kR))
                        fw_wait(&raw_empty[slot], ((g / kR) - 1) & 1, kErrEmptyBarrierTimeout, abort);
                    mbar_arrive_expect_tx(&raw_full[slot], C::kRawBytes);
                    tma_load_2d(raw + slot * C::kRawBytes, &wmap, (st0 + s) * int(C::kSS / 2), tile * kFwRows,
                                &raw_full[slot]);
                }
            }
            for (uint32_t q = g > uint32_t(kR) ? g - kR : 0; q < g; ++q) fw_drain(&raw_full[q % kR], (q / kR) & 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t g = 0;
            for (int ti = 0; ti < my_tiles; ++ti)
                for (int s = 0; s < nst; ++s, ++g) {
                    const uint32_t acs = g % kNAcc;
                    if (g >= uint32_t(kNAcc))
                        fw_wait(&acc_empty[acs], ((g / kNAcc) - 1) & 1, kErrEmptyBarrierTimeout, abort);
                    const uint32_t dacc = tmem + uint32_t(C::kAccCol0) + acs * C::kN;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t u = 2 * g + h, as = u % kA, bs = u % kNB;
                        fw_wait(&xb_full[bs], (u / kNB) & 1, kErrFullBarrierTimeout, abort);
                        fw_wait(&a_full[as], (u / kA) & 1, kErrFullBarrierTimeout, abort);
                        tc_fence_after();
                        const uint32_t bh = smem_u32(bring + bs * C::kBHalf);
                        const uint32_t acol = tmem + as * C::kACols;
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint64_t db = smem_desc(bh + uint32_t(kk >> 2) * (C::kN * 128) + uint32_t(kk & 3) * 32);
                            mma_ts(dacc, acol + 8 * kk, db, C::kIdesc, (h | kk) != 0);
                            if constexpr (!C::kQ4K) mma_ts(dacc, acol + 64 + 8 * kk, db, C::kIdesc, 1);
                        }
                        if constexpr (C::kQ4K) {
                            if (h == 1) {  // the stage's mins term, into the same accumulator
                                const uint32_t amin = tmem + uint32_t(C::kMinCol0) + (g % C::kAMinSlots) * 8;
                                mma_ts(dacc, amin, smem_desc(smem_u32(bmin + (g % C::kBStages) * C::kBMin)), C::kIdesc, 1);
                            }
                        }
                    }
                    // one commit per stage frees its A and X slots and publishes its accumulator
                    mma_commit(&stage_done[g % kSD]);
                }
            if (g > 0) fw_drain(&stage_done[(g - 1) % kSD], ((g - 1) / kSD) & 1);  // the last MMAs done
        }
        __syncwarp();
    } else if (warp < kFwConvWarp0) {
        // dequantise: TMEM lane quarter = warp % 4 holds weight rows 32 * quarter ..;
        // warps 2..5 take the first half of every stage, 6..9 the second; each also
        // reads back half of every stage accumulator (input rows h * BN / 2 ..)
        const int quarter = warp & 3, h = (warp - kFwDeqWarp0) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t tl = tmem + (uint32_t(quarter * 32) << 16);
        int valid = -1;
        uint32_t g = 0;
        // read-back of stage gg in two parts: start the loads (issued before the next stage's
        // dequantisation so that their latency overlaps it), then y += c / scale * (acc_hi + acc_lo)
        uint32_t vh[kHalfBN], vl[kHalfBN];
        auto readback_start = [&](uint32_t gg) {
            fw_wait(&stage_done[gg % kSD], (gg / kSD) & 1, kErrMmaBarrierTimeout, abort);
            fw_wait(&scale_full[gg % kNS], (gg / kNS) & 1, kErrFullBarrierTimeout, abort);
            tc_fence_after();
            const uint32_t col = tl + uint32_t(C::kAccCol0) + (gg % kNAcc) * C::kN + uint32_t(h * kHalfBN);
            tmem_ld_nw<kHalfBN>(col, vh);
            tmem_ld_nw<kHalfBN>(col + BN, vl);
        };
        auto readback_finish = [&](uint32_t gg, float c, float (&y)[kHalfBN]) {
            tc_wait_ld();
            tc_fence_before();
            mbar_arrive(&acc_empty[gg % kNAcc]);
            const float *inv = scale_inv + (gg % kNS) * BN + h * kHalfBN;
#pragma unroll
            for (int j = 0; j < kHalfBN; ++j)
                y[j] = fmaf(c * inv[j], __uint_as_float(vh[j]) + __uint_as_float(vl[j]), y[j]);
        };
        for (int ti = 0; ti < my_tiles; ++ti) {
            const int tile = cluster_id + ti * nclusters;
            float y[kHalfBN];
#pragma unroll
            for (int j = 0; j < kHalfBN; ++j) y[j] = 0.0f;
            float c1 = 1.0f, c2 = 1.0f;  // multipliers of the stages one and two behind
            for (int s = 0; s < nst; ++s, ++g) {
                // 16 input rows: the read-back loads go out before the dequantisation; 32 rows
                // (18 warps, 96 registers a thread) keep them after it
                if (kEarly && s >= kLag) readback_start(g - kLag);
                const uint32_t rs = g % kR;
                fw_wait(&raw_full[rs], (g / kR) & 1, kErrFullBarrierTimeout, abort);
                const uint8_t *src = raw + rs * C::kRawBytes + row * C::kSS;
                const uint32_t u = 2 * g + h, as = u % kA;
                if (u >= uint32_t(kA)) {  // the slot's last user, unit u - kA, belongs to a completed stage
                    const uint32_t prev = (u - kA) >> 1;
                    fw_wait(&stage_done[prev % kSD], (prev / kSD) & 1, kErrEmptyBarrierTimeout, abort);
                }
                float cur = 1.0f;
                if constexpr (C::kQ4K)
                    cur = dequant_q4k_half(src, h, tl + as * C::kACols,
                                           tl + uint32_t(C::kMinCol0) + (g % C::kAMinSlots) * 8);
                else
                    dequant_q80_half(src, h, tl + as * C::kACols);
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(&a_full[as]);
                fence_proxy_async();  // reads of the raw slot before the TMA refills it
                mbar_arrive(&raw_empty[rs]);
                if (s >= kLag) {
                    if (!kEarly) readback_start(g - kLag);
                    readback_finish(g - kLag, kLag == 2 ? c2 : c1, y);
                }
                c2 = c1;
                c1 = cur;
            }
            if (kLag == 2 && nst >= 2) {
                readback_start(g - 2);
                readback_finish(g - 2, c2, y);
            }
            if (nst >= 1) {
                readback_start(g - 1);
                readback_finish(g - 1, c1, y);
            }
            if (valid < 0) {
                pdl_wait();  // control comes from the stream; the previous kernel may still read Y
                valid = p.m;
                if (p.control) valid = min(valid, p.control[1]);
            }
            const int nrow = tile * kFwRows + row;
            bool store = true;
            if (splits > 1) {
                float *mine = red + row * C::kRedStride + h * kHalfBN;
                if (rank != 0) {
                    if (ti > 0) fw_wait_cluster(red_free, (ti - 1) & 1, kErrEpilogueTimeout, abort);
#pragma unroll
                    for (int j = 0; j < kHalfBN; ++j) mine[j] = y[j];
                    fw_remote_arrive(fw_mapa(smem_u32(red_full), 0));
                    store = false;
                } else {
                    fw_wait_cluster(red_full, ti & 1, kErrEpilogueTimeout, abort);
                    for (int q = 1; q < splits; ++q) {
                        const uint32_t peer = fw_mapa(smem_u32(mine), uint32_t(q));
#pragma unroll
                        for (int j = 0; j < kHalfBN; ++j) y[j] += fw_ld_cluster(peer + 4u * uint32_t(j));
                    }
                    for (int q = 1; q < splits; ++q) fw_remote_arrive(fw_mapa(smem_u32(red_free), uint32_t(q)));
                }
            }
            if (store && nrow < p.n) {
#pragma unroll
                for (int j = 0; j < kHalfBN; ++j) {
                    const int t = h * kHalfBN + j;
                    if (t < valid) p.y[size_t(t) * p.n + nrow] = y[j];
                }
            }
        }
        // a peer keeps its shared memory until the first CTA has read the last partials
        if (splits > 1 && rank != 0 && my_tiles > 0)
            fw_wait_cluster(red_free, (my_tiles - 1) & 1, kErrEpilogueTimeout, abort);
    } else {
        // X converters: thread = (input row r, 32-column sub-block u) of every stage; the
        // eight threads of a row are consecutive lanes. Each thread loads its 128 bytes of
        // the next stage into registers while it converts the current one.
        const int cw = warp - kFwConvWarp0;
        const int r = 4 * cw + (lane >> 3), u = lane & 7;
        const bool live = r < p.m;
        const float *xr = p.x + size_t(live ? r : 0) * p.k + 32 * u;
        const uint32_t total = uint32_t(my_tiles) * uint32_t(nst);  // stages of this CTA
        float4 cur[8], nxt[8];
        auto load = [&](uint32_t xg, float4 (&v)[8]) {
            if (live && xg < total) {
                const float4 *src = reinterpret_cast<const float4 *>(xr + (st0 + int(xg % uint32_t(nst))) * kFwStageK);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = src[i];
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        };
        pdl_wait();  // X may come from the previous kernel
        load(0, cur);
        const uint32_t sw = uint32_t(r & 7);
        // stage xg converts from `cur` while the loads of xg + 1 land in `nxt`; the two
        // buffers swap roles every stage (the body is instantiated for both orders)
        auto stage = [&](uint32_t xg, float4 (&cur)[8], float4 (&nxt)[8]) {
            load(xg + 1, nxt);
            const float *v = reinterpret_cast<const float *>(cur);
            // per (row, stage) power-of-two scale: values below 2^10 (32-column sums stay inside
            // FP16), rows whose largest value is below 2^-6 scaled up; others untouched
            float mx = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            float sc = 1.0f, isc = 1.0f;
            if (mx > 0.0f && (mx < 0x1p-6f || mx >= 0x1p10f) && mx <= 3.0e38f) {
                const int e = max(int((__float_as_uint(mx) >> 23) & 0xffu) - 127, -100);
                sc = __uint_as_float(uint32_t(127 + 9 - e) << 23);
                isc = __uint_as_float(uint32_t(127 - 9 + e) << 23);
            }
            if (__any_sync(0xffffffffu, sc != 1.0f)) {
#pragma unroll
                for (int i = 0; i < 8; ++i) cur[i].x *= sc, cur[i].y *= sc, cur[i].z *= sc, cur[i].w *= sc;
            }
            const uint32_t u0 = 2 * xg;
            if (xg >= uint32_t(C::kBStages)) {  // the last user of both slots and of the sums slot completed
                const uint32_t prev = xg - C::kBStages;
                fw_wait(&stage_done[prev % kSD], (prev / kSD) & 1, kErrEmptyBarrierTimeout, abort);
            }
            const uint32_t hs = uint32_t(u >> 2);
            uint8_t *bt = bring + ((u0 + hs) % kNB) * C::kBHalf;
            // columns 32 (u % 4) .. of the half stage: atom (u % 4) / 2, 16-byte chunks 4 (u % 2) ..
            const uint32_t atom = uint32_t((u & 3) >> 1) * (C::kN * 128), c0 = 4u * uint32_t(u & 1);
            uint8_t *rh = bt + atom + uint32_t(r >> 3) * 1024 + sw * 128;
            uint8_t *rl = bt + atom + uint32_t((BN + r) >> 3) * 1024 + sw * 128;  // BN + r has the same row % 8
            // hi / lo in K order: word w holds columns swap01(2w), swap01(2w + 1) of the sub-block;
            // chunk q = words 4q .. 4q+3 = columns 8q .. 8q+7
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int w2 = 0; w2 < 4; ++w2) {
                    const int w = 4 * q + w2;
                    const int e0 = (2 * w & ~3) | ((2 * w >> 1) & 1);
                    const int e1 = (2 * w & ~3) | 2 | ((2 * w >> 1) & 1);
                    split_pair(v[e0], v[e1], hw[w2], lw[w2]);
                }
                *reinterpret_cast<uint4 *>(rh + (((c0 + q) ^ sw) << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4 *>(rl + (((c0 + q) ^ sw) << 4)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
            if constexpr (C::kQ4K) {
                // sub-block sum: columns u and 8 + u of the mins operand, hi in row r, lo in row BN + r
                float2 s2 = make_float2(0.0f, 0.0f);  // even / odd columns, then added
#pragma unroll
                for (int i = 0; i < 32; i += 2) s2 = __fadd2_rn(s2, make_float2(v[i], v[i + 1]));
                const float sum = s2.x + s2.y;
                const __half shi = __float2half_rn(sum);
                const __half slo = __float2half_rn(sum - __half2float(shi));
                uint8_t *mb = bmin + (xg % C::kBStages) * C::kBMin;
                uint8_t *mh = mb + uint32_t(r >> 3) * 1024 + sw * 128;
                uint8_t *ml = mb + uint32_t((BN + r) >> 3) * 1024 + sw * 128;
                *reinterpret_cast<__half *>(mh + ((0u ^ sw) << 4) + 2 * u) = shi;
                *reinterpret_cast<__half *>(mh + ((1u ^ sw) << 4) + 2 * u) = shi;
                *reinterpret_cast<__half *>(ml + ((0u ^ sw) << 4) + 2 * u) = slo;
                *reinterpret_cast<__half *>(ml + ((1u ^ sw) << 4) + 2 * u) = slo;
            }
            if (u == 0) scale_inv[(xg % kNS) * BN + r] = isc;
            fence_proxy_async();  // the X tiles, written through the generic proxy, for the tensor core
            mbar_arrive(&xb_full[(u0 + hs) % kNB]);
            mbar_arrive(&scale_full[xg % kNS]);
        };
        for (uint32_t xg = 0; xg < total; xg += 2) {
            stage(xg, cur, nxt);
            if (xg + 1 < total) stage(xg + 1, nxt, cur);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (splits > 1) fw_cluster_sync();  // no CTA leaves while a peer may still address its shared memory
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn fw_encoder() {
    static EncodeTiledFn fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            ptr = nullptr;
        return reinterpret_cast<EncodeTiledFn>(ptr);
    }();
    return fn;
}

// Raw GGUF rows as 16-bit units: one stage (144 or 272 bytes) x 128 rows per
// box, rows past n read as zeros.
si_status fw_w_map(CUtensorMap *map, const void *w, uint64_t row_bytes, int n, uint32_t ss_bytes) {
    EncodeTiledFn fn = fw_encoder();
    if (!fn) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {cuuint64_t(row_bytes / 2), cuuint64_t(n)};
    const cuuint64_t strides[1] = {cuuint64_t(row_bytes)};
    const cuuint32_t box[2] = {cuuint32_t(ss_bytes / 2), cuuint32_t(kFwRows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(w), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled (W) failed (%d)", int(r));
    return SI_OK;
}

// Clusters of `cluster` CTAs of `kernel` resident at once; cached per device.
int fw_max_clusters(const void *kernel, int cluster, int threads, size_t smem) {
    struct Entry {
        int device;
        const void *kernel;
        int cluster;
        int value;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    const int dev = current_device();
    {
        std::lock_guard<std::mutex> g(mu);
        for (const Entry &e : cache)
            if (e.device == dev && e.kernel == kernel && e.cluster == cluster) return e.value;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(cluster));
    cfg.blockDim = dim3(unsigned(threads));
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = unsigned(cluster);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    std::lock_guard<std::mutex> g(mu);
    cache.push_back({dev, kernel, cluster, n});
    return n;
}

template <int FMT, int BN>
si_status launch_fewrow(const void *w, uint64_t row_bytes, const FwParams &p0, cudaStream_t st) {
    using C = FwCfg<FMT, BN>;
    auto kernel = fewrow_ts_kernel<FMT, BN>;
    const void *kp = reinterpret_cast<const void *>(kernel);
    if (const int ae = opt_in_smem(kp, int(C::kSmem)))
        return fail(SI_ERR_CUDA, "few-row TMEM GEMM shared-memory opt-in failed: %s",
                    cudaGetErrorString(cudaError_t(ae)));
    FwParams p = p0;
    p.tiles = (p.n + kFwRows - 1) / kFwRows;
    const int stages = p.k / kFwStageK;
    // K split over a cluster: the largest split (up to 8) that keeps every
    // tile resident at once and at least two stages per CTA; otherwise one
    // CTA per SM, persistent over the tiles.
    int splits = 1, clusters = fw_max_clusters(kp, 1, C::kThreads, C::kSmem);
    for (int s = 2; s <= 8; ++s) {
        if (stages < 2 * s) break;
        const int fit = fw_max_clusters(kp, s, C::kThreads, C::kSmem);
        if (fit >= p.tiles) splits = s, clusters = fit;
    }
    if (clusters < 1) return fail(SI_ERR_CUDA, "few-row TMEM GEMM: no cluster of %d CTAs fits", splits);
    p.splits = splits;
    const int nclusters = std::min(p.tiles, clusters);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(nclusters * splits));
    cfg.blockDim = dim3(unsigned(C::kThreads));
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = unsigned(splits);
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    CUtensorMap wmap;
    if (si_status ms = fw_w_map(&wmap, w, row_bytes, p.n, C::kSS)) return ms;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, wmap, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(SI_ERR_CUDA, "few-row TMEM GEMM launch failed: %s", cudaGetErrorString(e));
    }
    return SI_OK;
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {
using namespace si::dev;

bool gemm_fewrow_supported(uint32_t wtype, const void *w, const float *x, int64_t m, int64_t n, int64_t k) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0) return false;
    if (m < 1 || m > 32 || n < 1 || k < kFwStageK || k % kFwStageK != 0 || k > (int64_t(1) << 28) ||
        n > (int64_t(1) << 30))
        return false;
    uint64_t rb = 0;
    if (byte_length(wtype, uint64_t(k), &rb) != SI_OK) return false;
    // TMA: 16-byte aligned bases and row strides
    return reinterpret_cast<uintptr_t>(w) % 16 == 0 && rb % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0;
}

si_status gemm_fewrow(uint32_t wtype, const void *w, const float *x, const int32_t *control, float *y, int64_t m,
                      int64_t n, int64_t k, void *stream) {
    if (!gemm_fewrow_supported(wtype, w, x, m, n, k))
        return fail(SI_ERR_UNSUPPORTED, "few-row TMEM GEMM: unsupported type, shape or alignment");
    uint64_t rb = 0;
    byte_length(wtype, uint64_t(k), &rb);
    FwParams p{static_cast<const uint8_t *>(w), rb, x, y, control, int(m), int(n), int(k), 1, 0};
    auto st = static_cast<cudaStream_t>(stream);
    if (wtype == SI_TYPE_Q4_K)
        return m <= 16 ? launch_fewrow<SI_TYPE_Q4_K, 16>(w, rb, p, st) : launch_fewrow<SI_TYPE_Q4_K, 32>(w, rb, p, st);
    return m <= 16 ? launch_fewrow<SI_TYPE_Q8_0, 16>(w, rb, p, st) : launch_fewrow<SI_TYPE_Q8_0, 32>(w, rb, p, st);
}

si_status take_error_gemm_fewrow(int device, uint32_t *code) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return fail(SI_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    uint32_t v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_error_word, sizeof v);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_error_word, &zero, sizeof zero);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "device error word: %s", cudaGetErrorString(e));
    *code |= v;
    return SI_OK;
}

}  // namespace si::kernels
