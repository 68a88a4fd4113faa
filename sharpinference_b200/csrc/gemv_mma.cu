// Q4_K decode GEMV on the sm_100a tensor pipe (mma.sync m16n8k16, FP16 in,
// FP32 accumulate): y[r] = sum_c W[r,c] x[c] with W the raw GGUF Q4_K blocks.
//
// Why tensor cores for a mat-vec: the SIMT form needs one integer op per
// weight just to isolate each nibble into its own register; here one AND
// turns two nibbles into two exact FP16 codes (the subnormals q * 2^-24) and
// one MMA consumes 16 rows x 16 weights.
//
// Layout of the work:
//  * A = weight codes, 16 rows x 16 k per MMA, read straight from shared
//    memory with ldmatrix (the 16-byte nibble groups are exactly the 8x8 b16
//    tiles ldmatrix distributes: lane (g,t) receives bytes 4t..4t+3 of row g).
//    A k16 slice is one 16-byte group: low nibbles (sub-block 2j) or high
//    nibbles (sub-block 2j+1, codes 16q).
//  * B = x, kept in registers for the whole kernel: each compute warp owns
//    one or two superblock columns (256 x values each). Column pair
//    (2(s%4), 2(s%4)+1) of the n8 tile carries x_hi / x_lo of sub-block s
//    (x scaled by a per-superblock power of two, split into two FP16 parts:
//    ~22 significant bits), so sub-blocks land in separate accumulator
//    columns and their 6-bit scales are applied once per (row, sub-block) in
//    the epilogue, together with the d, dmin and min terms.
//  * Rows stream through shared memory in tiles of 16..48 rows (one 1-D TMA
//    bulk copy per row, padded row stride so ldmatrix is bank-conflict free);
//    a producer warp fills the ring, a reducer warp sums the per-warp
//    partials of each row in a fixed order (deterministic) and stores y.
// All mbarrier waits are bounded and report through the device error word.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "device_common.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

constexpr int kMaxComputeWarps = 16;
constexpr int kMaxThreads = (kMaxComputeWarps + 2) * 32;  // + producer + reducer

struct MmaParams {
    const uint8_t *w;
    const float *x;
    float *y;
    int rows;
    int nsb;             // superblocks per row (K / 256)
    int compute_warps;   // C
    int spw;             // superblocks per compute warp (1 or 2)
    int rows_per_tile;   // multiple of 16
    int stages;
    uint32_t row_bytes;  // 144 * nsb
    uint32_t row_stride; // padded shared-memory row stride
    uint32_t stage_bytes;
    int num_tiles;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two nibbles (bits [3:0] and [19:16], or [7:4] and [23:20]) -> two FP16
// values with exponent field 0: the subnormals q * 2^-24 (or 16 q * 2^-24),
// exact, from one AND. The 2^24 is folded into the epilogue scale.
__device__ __forceinline__ uint32_t codes(uint32_t w, uint32_t mask) { return w & mask; }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ float h2f_bits(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xffffu)));
}

// Per-superblock state of a compute warp (B fragments stay in registers).
struct SbState {
    uint32_t b[16][2];  // [slice = 2*group + half][b0, b1]
    float inv_scale;    // 1 / per-superblock power-of-two scale
    float sx_lo_t;      // sum of x over sub-block t   (t = lane % 4)
    float sx_hi_t;      // sum of x over sub-block t+4
};

__device__ __forceinline__ void load_superblock_x(const float *__restrict__ x, int sb, int lane, SbState &st) {
    const float *xs = x + size_t(sb) * 256;
    // 8 consecutive x per lane: lane l covers elements 8l .. 8l+7 (sub-block l/4).
    float v[8];
    const bool aligned = (reinterpret_cast<uintptr_t>(xs) & 15u) == 0;
    if (aligned) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(xs + 8 * lane));
        const float4 b = __ldg(reinterpret_cast<const float4 *>(xs + 8 * lane + 4));
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __ldg(xs + 8 * lane + i);
    }
    float amax = 0.0f, psum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i])), psum += v[i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);  // lanes 4s..4s+3 hold the sum of sub-block s
    const int t = lane & 3, g = lane >> 2;
    st.sx_lo_t = __shfl_sync(0xffffffffu, psum, 4 * t);
    st.sx_hi_t = __shfl_sync(0xffffffffu, psum, 4 * (t + 4));
    // scale = 2^(14 - e) with amax < 2^e, so |x * scale| < 2^14 (FP16 range).
    float scale = 1.0f;
    const uint32_t ebits = (__float_as_uint(amax) >> 23) & 0xffu;
    if (amax > 0.0f && ebits != 0xffu) {
        const int e = int(ebits) - 127 + 1;
        const int se = 14 - e;
        if (se > -126 && se < 127) scale = __uint_as_float(uint32_t(se + 127) << 23);
    }
    st.inv_scale = 16777216.0f / scale;  // undo the 2^-24 of the subnormal weight codes
    // B fragments. Slice (group gamma = 2j + p, half h) covers sub-block
    // s = 2j + h; its x_hi / x_lo go to columns 2(s%4) / 2(s%4)+1. Lane
    // (g,t) holds column g, k rows 2t, 2t+1, 2t+8, 2t+9 = group bytes
    // 4t, 4t+2, 4t+1, 4t+3.
#pragma unroll
    for (int gamma = 0; gamma < 8; ++gamma) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = gamma >> 1, p = gamma & 1, s = 2 * j + h;
            const int col = 2 * (s & 3);
            uint32_t b0 = 0, b1 = 0;
            if (g == col || g == col + 1) {
                const int e0 = 64 * j + 32 * h + 16 * p + 4 * t;
                float q[4];
                if (aligned) {
                    const float4 a = __ldg(reinterpret_cast<const float4 *>(xs + e0));
                    q[0] = a.x, q[1] = a.y, q[2] = a.z, q[3] = a.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) q[i] = __ldg(xs + e0 + i);
                }
                const float f = h ? scale * 0.0625f : scale;  // high nibbles carry codes 16 q
                float part[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float v2 = q[i] * f;
                    const float hi = __half2float(__float2half_rn(v2));
                    part[i] = (g == col) ? hi : v2 - hi;
                }
                b0 = pack_half2(part[0], part[2]);
                b1 = pack_half2(part[1], part[3]);
            }
            st.b[2 * gamma + h][0] = b0;
            st.b[2 * gamma + h][1] = b1;
        }
    }
}

// One superblock column of one 16-row group. Returns this lane's partial
// (before the cross-lane sum) for rows g (first) and g+8 (second).
__device__ __forceinline__ float2 superblock_rows16(uint32_t qs_addr, const uint8_t *hdr_g, const uint8_t *hdr_g8,
                                                    uint32_t row_stride, int lane, const SbState &st) {
    const int t = lane & 3;
    // ldmatrix addresses: matrix m = lane / 8 -> rows (m & 1) * 8 + lane % 8,
    // group offset (m >> 1) (+ 2 per call).
    const int m = lane >> 3;
    const uint32_t base = qs_addr + uint32_t(((m & 1) * 8 + (lane & 7))) * row_stride + uint32_t(m >> 1) * 16;
    float d1[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t w0, w8, v0, v8;  // rows g / g+8 of groups 2q and 2q+1
        ldsm_x4(base + 32u * q, w0, w8, v0, v8);
        const uint32_t gw[2][2] = {{w0, w8}, {v0, v8}};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int gamma = 2 * q + k;
            const uint32_t a = gw[k][0], b = gw[k][1];
            const uint32_t as = a >> 8, bs = b >> 8;
            float(&acc)[4] = gamma < 4 ? d1 : d2;
            // low nibbles: sub-block 2j
            mma16816(acc, codes(a, 0x000F000Fu), codes(b, 0x000F000Fu), codes(as, 0x000F000Fu),
                     codes(bs, 0x000F000Fu), st.b[2 * gamma][0], st.b[2 * gamma][1]);
            // high nibbles: sub-block 2j+1 (codes 16 q, x pre-scaled by 1/16)
            mma16816(acc, codes(a, 0x00F000F0u), codes(b, 0x00F000F0u), codes(as, 0x00F000F0u),
                     codes(bs, 0x00F000F0u), st.b[2 * gamma + 1][0], st.b[2 * gamma + 1][1]);
        }
    }
    // Epilogue: lane (g,t) holds sub-blocks t (d1) and t+4 (d2), columns
    // (x_hi, x_lo) for rows g (c0,c1) and g+8 (c2,c3).
    const uint4 hg = *reinterpret_cast<const uint4 *>(hdr_g);
    const uint4 hg8 = *reinterpret_cast<const uint4 *>(hdr_g8);
    const uint32_t sh = 8u * uint32_t(t);
    float out[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint4 h = r ? hg8 : hg;
        const uint32_t b0 = (h.y >> sh) & 0xffu, b1 = (h.z >> sh) & 0xffu, b2 = (h.w >> sh) & 0xffu;
        const float sc_lo = float(b0 & 63u), mn_lo = float(b1 & 63u);
        const float sc_hi = float((b2 & 15u) | ((b0 >> 6) << 4)), mn_hi = float((b2 >> 4) | ((b1 >> 6) << 4));
        const float d = h2f_bits(h.x), dmin = h2f_bits(h.x >> 16);
        const float q_lo = d1[2 * r] + d1[2 * r + 1], q_hi = d2[2 * r] + d2[2 * r + 1];
        const float main = (sc_lo * q_lo + sc_hi * q_hi) * st.inv_scale;
        const float mins = mn_lo * st.sx_lo_t + mn_hi * st.sx_hi_t;
        out[r] = d * main - dmin * mins;
    }
    return make_float2(out[0], out[1]);
}

template <int SPW>
__global__ void __launch_bounds__(kMaxThreads, 1) gemv_mma_q4k_kernel(const MmaParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int C = p.compute_warps, RT = p.rows_per_tile;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + size_t(p.stages) * p.stage_bytes);
    uint64_t *empty = full + p.stages;
    uint64_t *pfull = empty + p.stages;  // [2]
    uint64_t *pempty = pfull + 2;        // [2]
    float *part = reinterpret_cast<float *>(pempty + 2);  // [2][C][RT]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&pfull[b], C);
            mbar_init(&pempty[b], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == C) {
        // Producer: one bulk copy per row into the padded stage rows.
        int it = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
            const int s = it % p.stages;
            if (it >= p.stages) mbar_wait(&empty[s], ((it / p.stages) - 1) & 1, kErrEmptyBarrierTimeout);
            const int r0 = tile * RT;
            const int nrows = min(RT, p.rows - r0);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], uint32_t(nrows) * p.row_bytes);
            __syncwarp();
            uint8_t *dst = smem + size_t(s) * p.stage_bytes;
            for (int r = lane; r < nrows; r += 32)
                bulk_copy_g2s(dst + size_t(r) * p.row_stride, p.w + size_t(r0 + r) * p.row_bytes, p.row_bytes,
                              &full[s]);
        }
        return;
    }
    if (warp == C + 1) {
        // Reducer: fixed-order sum of the C per-warp partials of each row.
        pdl_wait();  // y may still be read by the previous kernel
        int it = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
            const int b = it & 1;
            mbar_wait(&pfull[b], (it >> 1) & 1, kErrEpilogueTimeout);
            const int r0 = tile * RT;
            const int nrows = min(RT, p.rows - r0);
            const float *pb = part + size_t(b) * C * RT;
            for (int r = lane; r < nrows; r += 32) {
                float a = 0.0f;
                for (int c = 0; c < C; ++c) a += pb[c * RT + r];
                p.y[r0 + r] = a;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pempty[b]);
        }
        return;
    }

    // Compute warp `warp`: superblocks warp, warp + C (when spw == 2).
    SbState st0;
    SbState st1;
    const int sb0 = warp, sb1 = warp + C;
    const bool has1 = SPW == 2 && sb1 < p.nsb;
    pdl_wait();  // x is produced by the previous kernel
    load_superblock_x(p.x, sb0, lane, st0);
    if constexpr (SPW == 2) {
        if (has1) load_superblock_x(p.x, sb1, lane, st1);
    }

    const int g = lane >> 2, t = lane & 3;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        const int s = it % p.stages;
        const int b = it & 1;
        mbar_wait(&full[s], (it / p.stages) & 1, kErrFullBarrierTimeout);
        const uint8_t *stage = smem + size_t(s) * p.stage_bytes;
        const uint32_t stage_addr = smem_u32(stage);
        if (it >= 2) mbar_wait(&pempty[b], ((it >> 1) - 1) & 1, kErrEpilogueTimeout);
        float *pw = part + (size_t(b) * C + warp) * RT;
        for (int rg = 0; rg < RT; rg += 16) {
            const uint8_t *hdr_g = stage + size_t(rg + g) * p.row_stride;
            const uint8_t *hdr_g8 = hdr_g + size_t(8) * p.row_stride;
            float2 acc = superblock_rows16(stage_addr + uint32_t(rg) * p.row_stride + 144u * sb0 + 16u,
                                           hdr_g + 144 * sb0, hdr_g8 + 144 * sb0, p.row_stride, lane, st0);
            if (SPW == 2 && has1) {
                const float2 a1 = superblock_rows16(stage_addr + uint32_t(rg) * p.row_stride + 144u * sb1 + 16u,
                                                    hdr_g + 144 * sb1, hdr_g8 + 144 * sb1, p.row_stride, lane, st1);
                acc.x += a1.x, acc.y += a1.y;
            }
            acc.x += __shfl_xor_sync(0xffffffffu, acc.x, 1);
            acc.y += __shfl_xor_sync(0xffffffffu, acc.y, 1);
            acc.x += __shfl_xor_sync(0xffffffffu, acc.x, 2);
            acc.y += __shfl_xor_sync(0xffffffffu, acc.y, 2);
            if (t == 0) {
                pw[rg + g] = acc.x;
                pw[rg + g + 8] = acc.y;
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty[s]);
            mbar_arrive(&pfull[b]);
        }
    }
}

int g_sms[64];

int num_sms() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!g_sms[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_sms[dev] = n > 0 ? n : 148;
    }
    return g_sms[dev];
}

bool plan_mma(int64_t rows, int64_t cols, const void *w, MmaParams &p, size_t &smem) {
    if (cols % 256 != 0 || rows <= 0 || rows > (int64_t(1) << 30)) return false;
    if (reinterpret_cast<uintptr_t>(w) & 15u) return false;
    const int nsb = int(cols / 256);
    if (nsb > 2 * kMaxComputeWarps) return false;
    p.nsb = nsb;
    p.spw = nsb > kMaxComputeWarps ? 2 : 1;
    p.compute_warps = (nsb + p.spw - 1) / p.spw;
    p.row_bytes = uint32_t(144 * nsb);
    // Row stride / 16 odd: ldmatrix's 8 row addresses hit 8 distinct bank quads.
    p.row_stride = p.row_bytes + ((nsb % 2 == 0) ? 16u : 32u);
    const size_t budget = 220 * 1024;
    // Tile: 32 rows when the ring still holds three stages (measured best
    // across the Phi-4-mini shapes at K = 3072), else 16.
    const int rt = size_t(32) * p.row_stride * 3 <= budget ? 32 : 16;
    p.rows_per_tile = rt;
    p.stage_bytes = uint32_t((uint64_t(rt) * p.row_stride + 127) / 128 * 128);
    p.num_tiles = int((rows + rt - 1) / rt);
    const size_t part_bytes = size_t(2) * p.compute_warps * rt * sizeof(float);
    int stages = int((budget - part_bytes - 512) / p.stage_bytes);
    stages = std::min(stages, 8);
    if (stages < 2) return false;
    p.stages = stages;
    p.rows = int(rows);
    smem = size_t(stages) * p.stage_bytes + size_t(2 * stages + 4) * sizeof(uint64_t) + part_bytes;
    return true;
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {
using namespace si::dev;

// Returns SI_ERR_UNSUPPORTED (without touching the error string) when the
// shape needs the SIMT kernel instead.
si_status matvec_q4k_mma(const void *w, const float *x, float *y, int64_t rows, int64_t cols, void *stream) {
    MmaParams p{};
    size_t smem = 0;
    if (!plan_mma(rows, cols, w, p, smem)) return SI_ERR_UNSUPPORTED;
    p.w = static_cast<const uint8_t *>(w);
    p.x = x;
    p.y = y;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(gemv_mma_q4k_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        cudaFuncSetAttribute(gemv_mma_q4k_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(std::min(p.num_tiles, num_sms())));
    cfg.blockDim = dim3(unsigned((p.compute_warps + 2) * 32));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    // The weight stream starts before the dependency wait: weights are
    // read-only parameters, never produced by the preceding kernel.
    cudaLaunchAttribute attr_pdl{};
    attr_pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr_pdl.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr_pdl;
    cfg.numAttrs = 1;
    const cudaError_t le = p.spw == 2 ? cudaLaunchKernelEx(&cfg, gemv_mma_q4k_kernel<2>, p)
                                      : cudaLaunchKernelEx(&cfg, gemv_mma_q4k_kernel<1>, p);
    const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "tensor-core Q4_K GEMV launch failed: %s", cudaGetErrorString(e));
    return SI_OK;
}

si_status take_error_gemv_mma(int device, uint32_t *code) {
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
