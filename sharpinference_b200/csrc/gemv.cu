// core.mat-vec on sm_100a.
//
//  * matvec_coop_kernel: F32/F16 weights, the "cooperative-matvec"
//    semantics of GpuTierZeroInstruction.cs:44-90 (per-lane Neumaier sum and
//    correction, tree merge of both) with a 32-lane warp per row.
//  * gemv_staged_kernel<FMT>: Q8_0 / Q4_K decode GEMV. HBM-bound: weights are
//    streamed once. A producer warp moves whole row tiles (contiguous GGUF
//    bytes) into shared memory with 1-D TMA bulk copies through a ring of
//    mbarrier-guarded stages; each consumer thread owns one 64-element unit
//    of the row for the whole kernel and keeps its 64 x values in registers,
//    so x is read from HBM once per CTA. Dequantisation is in registers:
//    nibbles / bytes are turned into floats by byte permutes into a float
//    bit pattern, products use packed FP32x2 FMA, block scales are applied
//    once per 32 elements.
//  * gemv_rowwarp_kernel<FMT>: shapes the staged kernel does not cover
//    (Q8_0 rows not 16-byte aligned, very long rows): one warp per row.
#include <cuda_runtime.h>

#include <algorithm>

#include "device_common.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

// ---------------------------------------------------------------------------
// Cooperative dense mat-vec (Neumaier)
// ---------------------------------------------------------------------------
template <typename TW, typename TX, typename TY>
__global__ void __launch_bounds__(256) matvec_coop_kernel(const TW *__restrict__ w, const TX *__restrict__ x,
                                                          TY *__restrict__ y, int64_t rows, int64_t cols) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = warp; row < rows; row += nwarps) {
        const TW *wr = w + row * cols;
        float sum = 0.0f, correction = 0.0f;
        for (int64_t j = lane; j < cols; j += 32) add32(sum, correction, __fmul_rn(ldf(wr + j), ldf(x + j)));
        for (int step = 16; step > 0; step >>= 1) {
            const float s = __shfl_down_sync(0xffffffffu, sum, step);
            const float c = __shfl_down_sync(0xffffffffu, correction, step);
            if (lane < step) {
                add32(sum, correction, s);
                add32(sum, correction, c);
            }
        }
        if (lane == 0) stf(y + row, __fadd_rn(sum, correction));
    }
}

// ---------------------------------------------------------------------------
// Quantized unit kernels (64 elements, x held in registers)
// ---------------------------------------------------------------------------
// Byte b of `v` placed in the low mantissa byte of 2^23: value 2^23 + byte.
__device__ __forceinline__ float byte_as_f23(uint32_t v, uint32_t sel) {
    return __int_as_float(int(__byte_perm(v, 0x4B000000u, sel)));
}

// Q4_K, one 64-element unit = chunk j of a superblock: 32 bytes of nibbles
// (low nibbles: sub-block 2j, high nibbles: sub-block 2j+1) plus the
// superblock header. Returns sum_e w_e x_e.
// A nibble q placed at mantissa bits [19:16] of 0.5 gives f = 0.5 + q/256
// exactly; with S = sum f x and X = sum x over a sub-block,
//   sum (a q - b) x = (256 a) S - (128 a + b) X.
struct Q4KConsts {
    uint32_t sel_byte0, sel_byte1;  // byte permute selectors of sub-blocks 2j, 2j+1
    bool high_half;                 // j >= 2: sub-blocks 4..7 use the split 6-bit encoding
};

__device__ __forceinline__ float q4k_unit(const uint8_t *sb, int j, const Q4KConsts &c, const float (&xv)[64],
                                          float sx_lo, float sx_hi) {
    const uint4 h = *reinterpret_cast<const uint4 *>(sb);
    const uint4 qa = *reinterpret_cast<const uint4 *>(sb + 16 + 32 * j);
    const uint4 qb = *reinterpret_cast<const uint4 *>(sb + 32 + 32 * j);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};

    // 6-bit scales / mins of the 8 sub-blocks, one per byte.
    const uint32_t sc_lo = h.y & 0x3F3F3F3Fu, mn_lo = h.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    const uint32_t scw = c.high_half ? sc_hi : sc_lo, mnw = c.high_half ? mn_hi : mn_lo;
    const float2 sc = __fadd2_rn(make_float2(byte_as_f23(scw, c.sel_byte0), byte_as_f23(scw, c.sel_byte1)),
                                 make_float2(-8388608.0f, -8388608.0f));
    const float2 mn = __fadd2_rn(make_float2(byte_as_f23(mnw, c.sel_byte0), byte_as_f23(mnw, c.sel_byte1)),
                                 make_float2(-8388608.0f, -8388608.0f));
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));  // (d, dmin)

    float2 acc_lo = make_float2(0.0f, 0.0f), acc_hi = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t lo = q[i] & 0x0F0F0F0Fu;
        const uint32_t hi = (q[i] >> 4) & 0x0F0F0F0Fu;
        const float l0 = __int_as_float(int(__byte_perm(lo, 0x3F000000u, 0x7054u)));
        const float l1 = __int_as_float(int(__byte_perm(lo, 0x3F000000u, 0x7154u)));
        const float l2 = __int_as_float(int(__byte_perm(lo, 0x3F000000u, 0x7254u)));
        const float l3 = __int_as_float(int(__byte_perm(lo, 0x3F000000u, 0x7354u)));
        const float h0 = __int_as_float(int(__byte_perm(hi, 0x3F000000u, 0x7054u)));
        const float h1 = __int_as_float(int(__byte_perm(hi, 0x3F000000u, 0x7154u)));
        const float h2 = __int_as_float(int(__byte_perm(hi, 0x3F000000u, 0x7254u)));
        const float h3 = __int_as_float(int(__byte_perm(hi, 0x3F000000u, 0x7354u)));
        acc_lo = __ffma2_rn(make_float2(l0, l1), make_float2(xv[4 * i], xv[4 * i + 1]), acc_lo);
        acc_lo = __ffma2_rn(make_float2(l2, l3), make_float2(xv[4 * i + 2], xv[4 * i + 3]), acc_lo);
        acc_hi = __ffma2_rn(make_float2(h0, h1), make_float2(xv[32 + 4 * i], xv[32 + 4 * i + 1]), acc_hi);
        acc_hi = __ffma2_rn(make_float2(h2, h3), make_float2(xv[32 + 4 * i + 2], xv[32 + 4 * i + 3]), acc_hi);
    }
    // A = 256 d sc, B = A/2 + dmin m for (low, high) sub-blocks.
    const float2 A = __fmul2_rn(make_float2(256.0f * dd.x, 256.0f * dd.x), sc);
    const float2 B = __ffma2_rn(make_float2(dd.y, dd.y), mn, __fmul2_rn(A, make_float2(0.5f, 0.5f)));
    const float s_lo = acc_lo.x + acc_lo.y, s_hi = acc_hi.x + acc_hi.y;
    return (A.x * s_lo - B.x * sx_lo) + (A.y * s_hi - B.y * sx_hi);
}

// Q8_0, one unit = blocks 2g and 2g+1 (68 bytes, 4-byte aligned).
// Bytes XOR 0x80 give u = q + 128 in [0,255]; u placed in the low mantissa
// byte of 2^23 and 2^23 subtracted gives u exactly; then
//   sum d q x = d (sum u x - 128 X).
__device__ __forceinline__ float q8_0_unit(const uint8_t *u8, const float (&xv)[64], float c0, float c1) {
    const uint32_t *u = reinterpret_cast<const uint32_t *>(u8);
    uint32_t wv[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) wv[i] = u[i];
    const float d0 = __half2float(__ushort_as_half(static_cast<unsigned short>(wv[0] & 0xffffu)));
    const float d1 = __half2float(__ushort_as_half(static_cast<unsigned short>(wv[8] >> 16)));
    const float2 bias = make_float2(-8388608.0f, -8388608.0f);
    float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
    // block 0: element i at byte 2 + i -> word (2+i)/4, byte (2+i)%4
#pragma unroll
    for (int p = 0; p < 16; ++p) {
        const int e = 2 * p;  // elements e, e+1 share a word
        const int word = (2 + e) >> 2, byte = (2 + e) & 3;
        const uint32_t v = wv[word] ^ 0x80808080u;
        const float2 f = __fadd2_rn(make_float2(byte_as_f23(v, 0x7540u | byte), byte_as_f23(v, 0x7540u | (byte + 1))),
                                    bias);
        a0 = __ffma2_rn(f, make_float2(xv[e], xv[e + 1]), a0);
    }
    // block 1: element i at byte 36 + i -> word 9 + i/4, byte i%4
#pragma unroll
    for (int p = 0; p < 16; ++p) {
        const int e = 2 * p;
        const int word = 9 + (e >> 2), byte = e & 3;
        const uint32_t v = wv[word] ^ 0x80808080u;
        const float2 f = __fadd2_rn(make_float2(byte_as_f23(v, 0x7540u | byte), byte_as_f23(v, 0x7540u | (byte + 1))),
                                    bias);
        a1 = __ffma2_rn(f, make_float2(xv[32 + e], xv[32 + e + 1]), a1);
    }
    return d0 * ((a0.x + a0.y) - c0) + d1 * ((a1.x + a1.y) - c1);
}

// ---------------------------------------------------------------------------
// Staged GEMV
// ---------------------------------------------------------------------------
struct StagedParams {
    const uint8_t *w;
    const float *x;
    float *y;
    int rows;            // N
    int units;           // G = K / 64
    int slots;           // S row slots; consumer threads = G * S
    int consumer_threads;  // G * S rounded up to whole warps
    int rows_per_tile;   // RT = S * (rows per slot), rows held by one stage
    int segment;         // lanes per shuffle-reduction segment (power of two dividing G, <= 32)
    int stages;
    uint32_t row_bytes;
    uint32_t stage_bytes;  // RT * row_bytes rounded up to 128
    int num_tiles;
};

constexpr int kMaxStagedThreads = 512;

template <int FMT>
__global__ void __launch_bounds__(kMaxStagedThreads, 1) gemv_staged_kernel(const StagedParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *stage_base = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + size_t(p.stages) * p.stage_bytes);
    uint64_t *empty = full + p.stages;
    float *partials = reinterpret_cast<float *>(empty + p.stages);  // [2][RT][G]

    const int tid = threadIdx.x;
    const int consumer_warps = p.consumer_threads >> 5;
    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], consumer_warps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (tid >= p.consumer_threads) {
        // Producer warp: one thread streams row tiles into the stage ring.
        if (tid == p.consumer_threads) {
            int it = 0;
            for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
                const int s = it % p.stages;
                if (it >= p.stages) mbar_wait(&empty[s], ((it / p.stages) - 1) & 1, kErrEmptyBarrierTimeout);
                const int r0 = tile * p.rows_per_tile;
                const int nrows = min(p.rows_per_tile, p.rows - r0);
                const uint32_t bytes = uint32_t(nrows) * p.row_bytes;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_copy_g2s(stage_base + size_t(s) * p.stage_bytes, p.w + size_t(r0) * p.row_bytes, bytes,
                              &full[s]);
            }
        }
        return;
    }

    // Consumer: unit g of row slot `slot`.
    const int g = tid % p.units;
    const int slot = tid / p.units;
    const bool active = tid < p.units * p.slots;

    float xv[64];
    float sx_lo = 0.0f, sx_hi = 0.0f;
    if (active) {
        const float *xs = p.x + size_t(g) * 64;
        if ((reinterpret_cast<uintptr_t>(xs) & 15u) == 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float4 v = __ldg(reinterpret_cast<const float4 *>(xs) + i);
                xv[4 * i] = v.x, xv[4 * i + 1] = v.y, xv[4 * i + 2] = v.z, xv[4 * i + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 64; ++i) xv[i] = __ldg(xs + i);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) sx_lo += xv[i], sx_hi += xv[32 + i];
    } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) xv[i] = 0.0f;
    }
    const float c0 = 128.0f * sx_lo, c1 = 128.0f * sx_hi;  // Q8_0 bias terms

    Q4KConsts qc;
    const int j = g & 3;
    qc.high_half = j >= 2;
    qc.sel_byte0 = 0x7540u | uint32_t((2 * j) & 3);
    qc.sel_byte1 = 0x7540u | uint32_t(((2 * j) & 3) + 1);

    // Lanes are grouped in segments of `seg` consecutive threads (a power of
    // two dividing G, so a segment never straddles two row slots); each
    // segment first reduces its units' partials with shuffles, then one lane
    // per segment stores the segment sum.
    const int seg = p.segment;
    const int lane = tid & 31;
    const int rt = p.rows_per_tile;
    const int rows_per_slot = rt / p.slots;
    const int nseg = p.units / seg;  // partials per row

    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        const int s = it % p.stages;
        const int r0 = tile * rt;
        const int nrows = min(rt, p.rows - r0);
        mbar_wait(&full[s], (it / p.stages) & 1, kErrFullBarrierTimeout);
        const uint8_t *tile_smem = stage_base + size_t(s) * p.stage_bytes;
        float *part = partials + size_t(it & 1) * rt * nseg;
        // Uniform trip count in every consumer thread (shuffles below need
        // the whole warp); rows past the tile end compute on stale shared
        // memory inside the stage and are not stored.
        for (int i = 0; i < rows_per_slot; ++i) {
            const int r = active ? slot + i * p.slots : 0;
            const uint8_t *row = tile_smem + size_t(r) * p.row_bytes;
            float v;
            if constexpr (FMT == SI_TYPE_Q4_K)
                v = q4k_unit(row + (g >> 2) * 144, j, qc, xv, sx_lo, sx_hi);
            else
                v = q8_0_unit(row + g * 68, xv, c0, c1);
            for (int off = seg >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (active && r < nrows && (lane & (seg - 1)) == 0) part[(g / seg) * rt + r] = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // All segment partials of this tile are written.
        asm volatile("bar.sync 1, %0;" ::"r"(p.consumer_threads) : "memory");
        // Warp w sums rows w, w + W, ...: lanes stride the row's segment
        // partials, then a butterfly finishes the sum (fixed order, so the
        // result is deterministic).
        for (int r = tid >> 5; r < nrows; r += consumer_warps) {
            float a = 0.0f;
            for (int q = lane; q < nseg; q += 32) a += part[q * rt + r];
            for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (lane == 0) p.y[r0 + r] = a;
        }
    }
}

// ---------------------------------------------------------------------------
// Row-per-warp fallback for quantized weights
// ---------------------------------------------------------------------------
template <int FMT>
__global__ void __launch_bounds__(256) gemv_rowwarp_kernel(const uint8_t *__restrict__ w, const float *__restrict__ x,
                                                           float *__restrict__ y, int64_t rows, int64_t cols,
                                                           uint64_t row_bytes) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = warp; row < rows; row += nwarps) {
        const uint8_t *wr = w + row * row_bytes;
        float acc = 0.0f;
        if constexpr (FMT == SI_TYPE_Q6_K) {
            // lane l takes 16-element groups l, l + 32, ... of the row; group g of
            // superblock b is elements e = 16 (g % 16) .. + 15 of the GGUF block:
            // low bits ql[64h + l0 + 32(j & 1) + i] nibble j >> 1, high bits
            // (qh[32h + l0 + i] >> 2j) & 3, w = (d * scale[g % 16]) * (q - 32).
            // Superblocks are 210 bytes, so reads are 16-bit.
            for (int64_t g = lane; g < cols / 16; g += 32) {
                const uint8_t *blk = wr + (g >> 4) * kQ6KBytes;
                const int e0 = int(g & 15) * 16, h = e0 >> 7, j = (e0 >> 5) & 3, l0 = e0 & 31;
                const uint16_t *ql = reinterpret_cast<const uint16_t *>(blk + 64 * h + l0 + 32 * (j & 1));
                const uint16_t *qh = reinterpret_cast<const uint16_t *>(blk + 128 + 32 * h + l0);
                const float *xe = x + g * 16;
                const int lshift = 4 * (j >> 1), hshift = 2 * j;
                float sq = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t lw = ql[i], hw = qh[i];
                    const int q0 = int(((lw >> lshift) & 15u) | (((hw >> hshift) & 3u) << 4)) - 32;
                    const int q1 = int(((lw >> (8 + lshift)) & 15u) | (((hw >> (8 + hshift)) & 3u) << 4)) - 32;
                    sq = fmaf(float(q0), xe[2 * i], sq);
                    sq = fmaf(float(q1), xe[2 * i + 1], sq);
                }
                const float d = __half2float(*reinterpret_cast<const __half *>(blk + 208));
                acc = fmaf(d * float(int8_t(blk[192 + (g & 15)])), sq, acc);
            }
        } else if constexpr (FMT == SI_TYPE_Q8_0) {
            for (int64_t b = lane; b < cols / 32; b += 32) {
                const uint8_t *blk = wr + b * 34;
                const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
                float s = 0.0f;
                for (int i = 0; i < 32; ++i) s = fmaf(float(int8_t(blk[2 + i])), x[b * 32 + i], s);
                acc = fmaf(d, s, acc);
            }
        } else {
            for (int64_t b = lane; b < cols / 256; b += 32) {
                const uint8_t *blk = wr + b * 144;
                const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
                const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[2] | (blk[3] << 8))));
                const uint8_t *sc12 = blk + 4;
                for (int s = 0; s < 8; ++s) {
                    int sc, m;
                    if (s < 4) {
                        sc = sc12[s] & 63;
                        m = sc12[s + 4] & 63;
                    } else {
                        sc = (sc12[s + 4] & 0x0f) | ((sc12[s - 4] >> 6) << 4);
                        m = (sc12[s + 4] >> 4) | ((sc12[s] >> 6) << 4);
                    }
                    const int jj = s >> 1, hi = s & 1;
                    float sq = 0.0f, sx = 0.0f;
                    for (int l = 0; l < 32; ++l) {
                        const uint8_t byte = blk[16 + 32 * jj + l];
                        const int q = hi ? (byte >> 4) : (byte & 15);
                        const float xe = x[b * 256 + 32 * s + l];
                        sq = fmaf(float(q), xe, sq);
                        sx += xe;
                    }
                    acc += (d * float(sc)) * sq - (dmin * float(m)) * sx;
                }
            }
        }
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) y[row] = acc;
    }
}

int sm_count() { return device_sm_count(); }

si_status launch_status(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return SI_OK;
}

template <typename TW, typename TX, typename TY>
si_status launch_coop(const void *w, const void *x, void *y, int64_t rows, int64_t cols, cudaStream_t st) {
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((rows + 7) / 8, int64_t(sm_count()) * 8);
    matvec_coop_kernel<TW, TX, TY><<<unsigned(blocks), threads, 0, st>>>(
        static_cast<const TW *>(w), static_cast<const TX *>(x), static_cast<TY *>(y), rows, cols);
    return launch_status("cooperative mat-vec");
}

// Shape plan of the staged kernel; false when the shape needs the fallback.
bool plan_staged(uint32_t wtype, int64_t rows, int64_t cols, const void *w, StagedParams &p, size_t &smem) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0) return false;
    if (cols % 256 != 0 || rows <= 0 || rows > (int64_t(1) << 30)) return false;
    if (reinterpret_cast<uintptr_t>(w) & 15u) return false;
    const int64_t units = cols / 64;
    if (units > 480) return false;
    uint64_t rb;
    if (byte_length(wtype, uint64_t(cols), &rb) != SI_OK || rb % 16 != 0) return false;
    p.units = int(units);
    p.slots = std::max(1, int(480 / units));
    p.consumer_threads = (p.units * p.slots + 31) / 32 * 32;
    p.row_bytes = uint32_t(rb);
    // A tile is R rows per slot (rows_per_tile = S * R) so every slot gets
    // the same work; a stage holds up to ~36 KB of rows.
    const int sms = sm_count();
    const int r_max = std::max(1, int(36 * 1024 / (uint64_t(rb) * p.slots)));
    const int64_t want = (rows + int64_t(sms) * p.slots - 1) / (int64_t(sms) * p.slots);
    const int r = int(std::max<int64_t>(1, std::min<int64_t>(want, r_max)));
    const int rt = p.slots * r;
    if (rt > 32 * (p.consumer_threads / 32)) return false;
    p.rows_per_tile = rt;
    p.stage_bytes = uint32_t((uint64_t(rt) * rb + 127) / 128 * 128);
    p.num_tiles = int((rows + rt - 1) / rt);
    int seg = 32;
    while (p.units % seg) seg >>= 1;
    p.segment = seg;
    const size_t partial_bytes = size_t(2) * rt * (p.units / seg) * sizeof(float);
    const size_t budget = 220 * 1024;
    int stages = int((budget - partial_bytes - 256) / p.stage_bytes);
    stages = std::min(stages, 8);
    if (stages < 2) return false;
    p.stages = stages;
    p.rows = int(rows);
    smem = size_t(stages) * p.stage_bytes + size_t(2 * stages) * sizeof(uint64_t) + partial_bytes;
    return true;
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {
using namespace si::dev;

si_status matvec_dense(uint32_t wtype, const void *w, uint32_t xtype, const void *x, uint32_t ytype, void *y,
                       int64_t rows, int64_t cols, void *stream) {
    auto st = static_cast<cudaStream_t>(stream);
    const int key = (wtype == SI_TYPE_F16) * 4 + (xtype == SI_TYPE_F16) * 2 + (ytype == SI_TYPE_F16);
    switch (key) {
    case 0: return launch_coop<float, float, float>(w, x, y, rows, cols, st);
    case 1: return launch_coop<float, float, __half>(w, x, y, rows, cols, st);
    case 2: return launch_coop<float, __half, float>(w, x, y, rows, cols, st);
    case 3: return launch_coop<float, __half, __half>(w, x, y, rows, cols, st);
    case 4: return launch_coop<__half, float, float>(w, x, y, rows, cols, st);
    case 5: return launch_coop<__half, float, __half>(w, x, y, rows, cols, st);
    case 6: return launch_coop<__half, __half, float>(w, x, y, rows, cols, st);
    default: return launch_coop<__half, __half, __half>(w, x, y, rows, cols, st);
    }
}

si_status matvec_quant(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                       void *stream) {
    auto st = static_cast<cudaStream_t>(stream);
    {
        const si_status ms = matvec_quant_mma(wtype, w, x, y, rows, cols, stream);
        if (ms != SI_ERR_UNSUPPORTED) return ms;
    }
    StagedParams p{};
    size_t smem = 0;
    if (plan_staged(wtype, rows, cols, w, p, smem)) {
        p.w = static_cast<const uint8_t *>(w);
        p.x = x;
        p.y = y;
        const int grid = std::min(p.num_tiles, sm_count());
        const int threads = p.consumer_threads + 32;
        if (wtype == SI_TYPE_Q4_K) {
            if (const int ae = opt_in_smem(reinterpret_cast<const void *>(gemv_staged_kernel<SI_TYPE_Q4_K>), 227 * 1024))
                return fail(SI_ERR_CUDA, "staged GEMV shared-memory opt-in failed: %s",
                            cudaGetErrorString(cudaError_t(ae)));
            gemv_staged_kernel<SI_TYPE_Q4_K><<<grid, threads, smem, st>>>(p);
        } else {
            if (const int ae = opt_in_smem(reinterpret_cast<const void *>(gemv_staged_kernel<SI_TYPE_Q8_0>), 227 * 1024))
                return fail(SI_ERR_CUDA, "staged GEMV shared-memory opt-in failed: %s",
                            cudaGetErrorString(cudaError_t(ae)));
            gemv_staged_kernel<SI_TYPE_Q8_0><<<grid, threads, smem, st>>>(p);
        }
        return launch_status("staged quantized GEMV");
    }
    uint64_t rb;
    if (si_status s = byte_length(wtype, uint64_t(cols), &rb)) return s;
    const int64_t blocks = std::min<int64_t>((rows + 7) / 8, int64_t(sm_count()) * 8);
    if (wtype == SI_TYPE_Q6_K)
        gemv_rowwarp_kernel<SI_TYPE_Q6_K><<<unsigned(blocks), 256, 0, st>>>(static_cast<const uint8_t *>(w), x, y,
                                                                            rows, cols, rb);
    else if (wtype == SI_TYPE_Q4_K)
        gemv_rowwarp_kernel<SI_TYPE_Q4_K><<<unsigned(blocks), 256, 0, st>>>(static_cast<const uint8_t *>(w), x, y,
                                                                            rows, cols, rb);
    else
        gemv_rowwarp_kernel<SI_TYPE_Q8_0><<<unsigned(blocks), 256, 0, st>>>(static_cast<const uint8_t *>(w), x, y,
                                                                            rows, cols, rb);
    return launch_status("row-warp quantized GEMV");
}

si_status take_error_gemv(int device, uint32_t *code) {
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
