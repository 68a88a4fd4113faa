// Device building blocks of the tensor-core quantised GEMV kernels
// (gemv_mma.cu): the input source with its fused transforms, the MMA and
// ldmatrix wrappers, and per weight format the x load (B fragments in
// registers) and the 16-row partial product of one superblock column.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "device_common.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

// Source of the GEMV input as the load paths see it: element i of the
// (transformed) vector. The transform is a template parameter so the plain
// load (M = 0) compiles to bare vector loads the compiler can batch. Modes
// 1 and 2 need 16-byte aligned vectors. kL2 = 1: load through L2 only (the
// vector was written by another CTA of the same kernel); 0: through the
// read-only path (written by an earlier kernel).
// kL2 = 2: generic loads (the vector was staged in shared memory).
template <int kL2>
__device__ __forceinline__ float ldx(const float *p) {
    if constexpr (kL2 == 2) return *p;
    else if constexpr (kL2 == 1) return __ldcg(p);
    else return __ldg(p);
}
template <int kL2>
__device__ __forceinline__ float4 ldx4(const float *p) {
    if constexpr (kL2 == 2) return *reinterpret_cast<const float4 *>(p);
    else if constexpr (kL2 == 1) return __ldcg(reinterpret_cast<const float4 *>(p));
    else return __ldg(reinterpret_cast<const float4 *>(p));
}

// Modes: 0 x as is; 1 (x (+ res)) * scale * w (rms-norm with the scale given
// or applied later); 2 swiglu of [gate | up] (u at offset `up`); 3 the
// residual stream after a K-split exchange: (x + res[0] + ... + res[nparts-1])
// * scale * w, partial vectors `up` floats apart, summed in rank order.
template <int M, int kL2 = 0>
struct XSrc {
    const float *x;
    const float *res;
    const float *w;
    float scale;
    int64_t up;  // mode 2: offset of u; mode 3: floats between partial vectors
    int nparts = 0;  // mode 3
    __device__ __forceinline__ bool aligned(int64_t i) const {
        return M != 0 || (reinterpret_cast<uintptr_t>(x + i) & 15u) == 0;
    }
    static __device__ __forceinline__ float swish_mul(float g, float u) {
        return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
    __device__ __forceinline__ float get(int64_t i) const {
        const float a = ldx<kL2>(x + i);
        if constexpr (M == 0) {
            return a;
        } else if constexpr (M == 1) {
            const float v = res ? __fadd_rn(a, ldx<kL2>(res + i)) : a;
            return __fmul_rn(__fmul_rn(v, scale), ldx<kL2>(w + i));
        } else if constexpr (M == 3) {
            float v = a;
            for (int r = 0; r < nparts; ++r) v = __fadd_rn(v, ldx<kL2>(res + r * up + i));
            return __fmul_rn(__fmul_rn(v, scale), ldx<kL2>(w + i));
        } else {
            return swish_mul(a, ldx<kL2>(x + up + i));
        }
    }
    __device__ __forceinline__ float4 get4(int64_t i) const {
        float4 a = ldx4<kL2>(x + i);
        if constexpr (M == 0) {
            return a;
        } else if constexpr (M == 3) {
            for (int r = 0; r < nparts; ++r) {
                const float4 p = ldx4<kL2>(res + r * up + i);
                a = make_float4(__fadd_rn(a.x, p.x), __fadd_rn(a.y, p.y), __fadd_rn(a.z, p.z), __fadd_rn(a.w, p.w));
            }
            const float4 m = ldx4<kL2>(w + i);
            return make_float4(__fmul_rn(__fmul_rn(a.x, scale), m.x), __fmul_rn(__fmul_rn(a.y, scale), m.y),
                               __fmul_rn(__fmul_rn(a.z, scale), m.z), __fmul_rn(__fmul_rn(a.w, scale), m.w));
        } else if constexpr (M == 1) {
            if (res) {
                const float4 r = ldx4<kL2>(res + i);
                a = make_float4(__fadd_rn(a.x, r.x), __fadd_rn(a.y, r.y), __fadd_rn(a.z, r.z), __fadd_rn(a.w, r.w));
            }
            const float4 m = ldx4<kL2>(w + i);
            return make_float4(__fmul_rn(__fmul_rn(a.x, scale), m.x), __fmul_rn(__fmul_rn(a.y, scale), m.y),
                               __fmul_rn(__fmul_rn(a.z, scale), m.z), __fmul_rn(__fmul_rn(a.w, scale), m.w));
        } else {
            const float4 u = ldx4<kL2>(x + up + i);
            return make_float4(swish_mul(a.x, u.x), swish_mul(a.y, u.y), swish_mul(a.z, u.z), swish_mul(a.w, u.w));
        }
    }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    // Not volatile: a pure register operation, so the compiler may interleave
    // independent accumulator chains (the ldmatrix loads stay volatile and
    // therefore ordered after the stage's mbarrier wait).
    asm(
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

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t bits) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&bits));
}

// Two 6-bit integers v0, v1 in bits 0-5 / 16-21, OR-ed with kU6Bias (the
// FP16 pattern of 1024 in each half), read as FP16 are 1024 + v exactly;
// subtracting 1024 leaves v0, v1 (exact) and the pair widens to floats. The
// bias is folded into the preceding mask, so no integer conversions are needed.
constexpr uint32_t kU6Bias = 0x64006400u;
__device__ __forceinline__ float2 u6pair(uint32_t biased) {
    const uint32_t k1024 = kU6Bias;
    const __half2 v = __hsub2(*reinterpret_cast<const __half2 *>(&biased), *reinterpret_cast<const __half2 *>(&k1024));
    return __half22float2(v);
}
// Same, divided by 16 in the same FP16 operation: (1024 + v) / 16 - 64 = v / 16 (exact).
__device__ __forceinline__ float2 u6pair_div16(uint32_t biased) {
    const uint32_t k16th = 0x2C002C00u, km64 = 0xD400D400u;  // 1/16, -64
    const __half2 v = __hfma2(*reinterpret_cast<const __half2 *>(&biased), *reinterpret_cast<const __half2 *>(&k16th),
                              *reinterpret_cast<const __half2 *>(&km64));
    return __half22float2(v);
}

// Per-superblock state of a compute warp (B fragments stay in registers).
struct SbState {
    uint32_t b[16][2];  // [slice = 2*group + half][b0, b1]
    float inv_scale;    // 1 / per-superblock power-of-two scale
    float sx_lo_t;      // sum of x over sub-block t   (t = lane % 4)
    float sx_hi_t;      // sum of x over sub-block t+4
};

template <class XS>
__device__ __forceinline__ void load_superblock_x(const XS &X, int sb, int lane, SbState &st) {
    const int64_t xb = int64_t(sb) * 256;
    // 8 consecutive x per lane: lane l covers elements 8l .. 8l+7 (sub-block l/4).
    float v[8];
    const bool aligned = X.aligned(xb);
    if (aligned) {
        const float4 a = X.get4(xb + 8 * lane);
        const float4 b = X.get4(xb + 8 * lane + 4);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = X.get(xb + 8 * lane + i);
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
                    const float4 a = X.get4(xb + e0);
                    q[0] = a.x, q[1] = a.y, q[2] = a.z, q[3] = a.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) q[i] = X.get(xb + e0 + i);
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
// ldsm_addr: this lane's ldmatrix row address for the superblock's first
// 16-byte group pair (row (lane/8 % 2) * 8 + lane % 8 of the 16-row unit,
// group lane / 16).
__device__ __forceinline__ float2 superblock_rows16(uint32_t ldsm_addr, const uint8_t *hdr_g, const uint8_t *hdr_g8,
                                                    int lane, const SbState &st) {
    const int t = lane & 3;
    const uint32_t base = ldsm_addr;
    // Four accumulator chains (one per ldmatrix group q), summed pairwise in
    // the epilogue: shorter dependent MMA chains.
    float dq[4][4] = {};
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
            float(&acc)[4] = dq[q];
            // low nibbles: sub-block 2j
            mma16816(acc, codes(a, 0x000F000Fu), codes(b, 0x000F000Fu), codes(as, 0x000F000Fu),
                     codes(bs, 0x000F000Fu), st.b[2 * gamma][0], st.b[2 * gamma][1]);
            // high nibbles: sub-block 2j+1 (codes 16 q, x pre-scaled by 1/16)
            mma16816(acc, codes(a, 0x00F000F0u), codes(b, 0x00F000F0u), codes(as, 0x00F000F0u),
                     codes(bs, 0x00F000F0u), st.b[2 * gamma + 1][0], st.b[2 * gamma + 1][1]);
        }
    }
    float d1[4], d2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) d1[i] = dq[0][i] + dq[1][i], d2[i] = dq[2][i] + dq[3][i];
    // Epilogue: lane (g,t) holds sub-blocks t (d1) and t+4 (d2), columns
    // (x_hi, x_lo) for rows g (c0,c1) and g+8 (c2,c3). The 6-bit scales and
    // mins of both rows are unpacked together: byte t of the row-g and
    // row-(g+8) words goes to bits 0-7 / 16-23 (one byte permute each).
    const uint4 hg = *reinterpret_cast<const uint4 *>(hdr_g);
    const uint4 hg8 = *reinterpret_cast<const uint4 *>(hdr_g8);
    const uint32_t sel = uint32_t(t) | (uint32_t(t + 4) << 8);
    const uint32_t X = __byte_perm(hg.y, hg8.y, sel);  // scale bytes: low 6 bits sub-block t, top 2 of t+4
    const uint32_t Y = __byte_perm(hg.z, hg8.z, sel);  // min bytes: low 6 bits sub-block t, top 2 of t+4
    const uint32_t Z = __byte_perm(hg.w, hg8.w, sel);  // low nibble: scale t+4, high nibble: min t+4
    const float2 sc_lo = u6pair((X & 0x003F003Fu) | kU6Bias);
    const float2 mn_lo = u6pair((Y & 0x003F003Fu) | kU6Bias);
    const float2 sc_hi = u6pair((Z & 0x000F000Fu) | ((X >> 2) & 0x00300030u) | kU6Bias);
    const float2 mn_hi = u6pair(((Z >> 4) & 0x000F000Fu) | ((Y >> 2) & 0x00300030u) | kU6Bias);
    const float2 dm = half2_bits_to_float2(hg.x);   // (d, dmin) of row g
    const float2 dm8 = half2_bits_to_float2(hg8.x);  // (d, dmin) of row g+8
    float out[2];
    {
        const float main = (sc_lo.x * (d1[0] + d1[1]) + sc_hi.x * (d2[0] + d2[1])) * st.inv_scale;
        const float mins = mn_lo.x * st.sx_lo_t + mn_hi.x * st.sx_hi_t;
        out[0] = dm.x * main - dm.y * mins;
    }
    {
        const float main = (sc_lo.y * (d1[2] + d1[3]) + sc_hi.y * (d2[2] + d2[3])) * st.inv_scale;
        const float mins = mn_lo.y * st.sx_lo_t + mn_hi.y * st.sx_hi_t;
        out[1] = dm8.x * main - dm8.y * mins;
    }
    return make_float2(out[0], out[1]);
}

// Roles (warp index): 0..C-1 compute, C producer, C+1 reducer.
//
// K split: with cluster size CS > 1 the CS CTAs of a cluster share every row
// tile; CTA rank k loads and multiplies superblocks [k*nsb/CS, (k+1)*nsb/CS)
// of each row and keeps its per-row sums in its own shared memory. After the
// last tile one cluster barrier makes them visible, and the cluster's rows
// are finished split over its CTAs: y = rank 0 + rank 1 + ... (DSMEM loads,
// fixed order, deterministic). Smaller per-CTA slices let more CTAs stream a
// small matrix at once and leave room for the next kernel's CTAs on the SM.
// MAXW bounds the compute warps of a launch: the register budget ptxas may
// use follows from the warps per SM sub-partition ((MAXW + 2) / 4 rounded
// up), so the 12-warp instantiation (K = 3072 slices) gets up to 128
// registers a thread where the 16-warp one gets 96.
// FP16 path: nibble codes as FP16 subnormals, x as FP16 hi/lo pairs.
struct F16Path {
    using State = SbState;
    static constexpr int kTokens = 1;
    using Out = float2;
    static __device__ __forceinline__ void accumulate(Out &a, const Out &b) { a.x += b.x, a.y += b.y; }
    static constexpr uint32_t kColBytes = 144;  // one Q4_K superblock
    static constexpr uint32_t kQsOffset = 16;   // nibbles follow the 16-byte header
    static constexpr uint32_t kScratchBytes = 0;
    template <class XS>
    static __device__ __forceinline__ void load(const XS &x, int sb, int lane, State &st, uint8_t *, int64_t, int) {
        load_superblock_x(x, sb, lane, st);
    }
    static __device__ __forceinline__ float2 rows16(uint32_t ldsm_addr, const uint8_t *hdr_g, const uint8_t *hdr_g8,
                                                    int lane, const State &st,
                                                    const uint8_t * = nullptr) {
        return superblock_rows16(ldsm_addr, hdr_g, hdr_g8, lane, st);
    }
};

// ---------------------------------------------------------------------------
// INT8 path (mma.sync m16n8k32, u8 x s8 -> s32, exact integer accumulation).
//
//  * A = weight codes as bytes: the low nibbles of a 32-byte chunk j are the
//    32 weights of sub-block 2j in order (k = 0..31), the high nibbles those
//    of sub-block 2j+1. One AND yields four codes: q (mask 0x0F) or 16 q
//    (mask 0xF0, the 1/16 goes into the sub-block scale). One ldmatrix.x4
//    per chunk feeds two MMAs.
//  * B = x as three base-256 digits: per superblock, v = rint(x * 2^(22-e))
//    (|x| < 2^e, so |v| < 2^22) and v = d0 * 2^16 + d1 * 2^8 + d2 with
//    signed 8-bit digits. Columns: sub-block s sits in half s / 4 of the n8
//    tile (columns 0-2 or 4-6 hold d0, d1, d2; 3 and 7 stay zero), so the
//    accumulator set s % 4 collects sub-blocks s and s + 4 side by side.
//  * Lane (g,t) holds columns 2t, 2t+1 of set q: for even t (d0, d1) ->
//    256 * c0 + c1 in units of 2^8, for odd t d2 (c1 is a zero column), so
//    c0 * M + c1 with M = 256 or 1 is exact in int32 and in FP32 (< 2^24);
//    each lane scales it by its sub-block's 6-bit scale and the per-lane
//    digit weight / x scale, and the four lanes of a row are summed.
// Precision: x is carried as 22-bit fixed point per superblock (relative to
// its largest element), the products are exact, the sum is FP32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct I8State {
    uint32_t b[8][2];   // B fragment of sub-block s (zero unless s / 4 is this lane's column half)
    float wt_inv;       // digit weight of this lane's accumulator columns / x scale
    float sx_lo_t;      // sum of x over sub-block t
    float sx_hi_t;      // sum of x over sub-block t+4
    int digit_mul;      // 256 (even t: columns d0, d1) or 1 (odd t: column d2)
    uint32_t sc_shift;  // scale unpack of this lane's sub-block half (t / 2): 0 / 2
    uint32_t sc_wmask;  // 0 / 0x0F0F0F0F
    uint32_t sc_ymask;  // 0x3F3F3F3F / 0x30303030
};

// v = d0 * 2^16 + d1 * 2^8 + d2 with d1, d2 in [-128, 127] (balanced base
// 256): d2 is the low byte of v, d1 the low byte of (v + 2^7) >> 8 and d0 =
// (v + 2^15 + 2^7) >> 16, because adding 128 to each lower digit makes it a
// plain byte without carry. Only the low byte of each is kept (two's
// complement int8), so one add and one shift give a digit.
__device__ __forceinline__ uint32_t digit_byte(int v, int add, uint32_t shift) {
    return uint32_t((v + add) >> shift);
}
// rint(v) for |v| < 2^22 on the FMA pipe instead of the conversion pipe:
// v + 1.5 * 2^23 lies in [2^23, 2^24), where the float spacing is 1, so the
// addition rounds v to the nearest integer (ties to even, as
// __float2int_rn) and the integer is the sum's low mantissa bits. `m` is a
// power of two with |x * m| < 2^22, so x * m is exact and one FMA suffices.
__device__ __forceinline__ int rint_scaled(float x, float m) {
    return __float_as_int(fmaf(x, m, 12582912.0f)) - 0x4B400000;
}
// Low bytes of four words packed into one.
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
}

struct I8Path {
    using State = I8State;
    static constexpr int kTokens = 1;
    using Out = float2;
    static __device__ __forceinline__ void accumulate(Out &a, const Out &b) { a.x += b.x, a.y += b.y; }
    static constexpr uint32_t kColBytes = 144;
    static constexpr uint32_t kQsOffset = 16;
    static constexpr uint32_t kScratchBytes = 0;
    template <class XS>
    static __device__ __forceinline__ void load(const XS &X, int sb, int lane, State &st, uint8_t *, int64_t, int) {
        const int64_t xb = int64_t(sb) * 256;
        const bool aligned = X.aligned(xb);
        const int t = lane & 3, g = lane >> 2;
        const int half = g >> 2, digit = g & 3;
        // Each lane loads (and transforms) eight consecutive values, lane l
        // elements 8l .. 8l+7 of the superblock: one memory round trip, every
        // input transform computed once. The 32 values of the lane's B
        // fragments (sub-blocks 4 * half .. + 3, k = 4t..4t+3 and
        // 16+4t..16+4t+3) are then gathered from the lanes holding them.
        float v[8], q[4][8];
        if (aligned) {
            const float4 a = X.get4(xb + 8 * lane);
            const float4 b = X.get4(xb + 8 * lane + 4);
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = X.get(xb + 8 * lane + i);
        }
        // element 32 s + 4t + i (i < 4) sits in lane 4s + t/2, slot 4(t%2) + i;
        // element 32 s + 16 + 4t + i in lane 4s + 2 + t/2, same slot
        const bool odd_t = (t & 1) != 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int s0 = 4 * (4 * half + j) + (t >> 1);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float lo_a = __shfl_sync(0xffffffffu, v[i], s0), lo_b = __shfl_sync(0xffffffffu, v[4 + i], s0);
                const float hi_a = __shfl_sync(0xffffffffu, v[i], s0 + 2),
                            hi_b = __shfl_sync(0xffffffffu, v[4 + i], s0 + 2);
                q[j][i] = odd_t ? lo_b : lo_a;
                q[j][4 + i] = odd_t ? hi_b : hi_a;
            }
        }
        float amax = 0.0f, psum = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i])), psum += v[i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);  // lanes 4s..4s+3 hold the sum of sub-block s
        st.sx_lo_t = __shfl_sync(0xffffffffu, psum, 4 * t);
        st.sx_hi_t = __shfl_sync(0xffffffffu, psum, 4 * (t + 4));
        // scale = 2^(22 - e) with amax < 2^e: |x * scale| < 2^22.
        float scale = 1.0f, inv = 1.0f;
        const uint32_t ebits = (__float_as_uint(amax) >> 23) & 0xffu;
        if (ebits == 0xffu) {
            inv = __int_as_float(0x7fc00000);  // non-finite activation: the rows become NaN
        } else if (amax > 0.0f) {
            const int e = int(ebits) - 127 + 1;
            const int se = max(-126, min(127, 22 - e));
            scale = __uint_as_float(uint32_t(se + 127) << 23);
            inv = __uint_as_float(uint32_t(127 - se) << 23);
        }
        st.digit_mul = (t & 1) ? 1 : 256;
        st.wt_inv = ((t & 1) ? 1.0f : 256.0f) * inv;
        const bool hi_half = t >= 2;
        st.sc_shift = hi_half ? 2u : 0u;
        st.sc_wmask = hi_half ? 0x0F0F0F0Fu : 0u;
        st.sc_ymask = hi_half ? 0x30303030u : 0x3F3F3F3Fu;
        // B fragments: lane (g,t) holds column g = 4 * half + digit of
        // sub-blocks 4 * half .. 4 * half + 3, k = 4t..4t+3 (b0) and
        // 16+4t..16+4t+3 (b1); column digit 3 stays zero.
        const int dadd = digit == 0 ? 0x8080 : (digit == 1 ? 0x80 : 0);
        const uint32_t dshift = digit == 0 ? 16u : (digit == 1 ? 8u : 0u);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            uint32_t b0 = 0, b1 = 0;
            if ((s >> 2) == half && digit < 3) {
                const float *qs = q[s & 3];
                uint32_t dg[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) dg[i] = digit_byte(rint_scaled(qs[i], scale), dadd, dshift);
                b0 = pack_low_bytes(dg[0], dg[1], dg[2], dg[3]);
                b1 = pack_low_bytes(dg[4], dg[5], dg[6], dg[7]);
            }
            st.b[s][0] = b0;
            st.b[s][1] = b1;
        }
    }

    static __device__ __forceinline__ float2 rows16(uint32_t ldsm_addr, const uint8_t *hdr_g, const uint8_t *hdr_g8,
                                                    int lane, const State &st,
                                                    const uint8_t * = nullptr) {
        const int t = lane & 3;
        const uint32_t base = ldsm_addr;
        int acc[4][4] = {};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t w0, w8, v0, v8;  // rows g / g+8 of the chunk's two 16-byte groups
            ldsm_x4(base + 32u * j, w0, w8, v0, v8);
            constexpr uint32_t L = 0x0F0F0F0Fu, H = 0xF0F0F0F0u;
            imma16832(acc[(2 * j) & 3], w0 & L, w8 & L, v0 & L, v8 & L, st.b[2 * j][0], st.b[2 * j][1]);
            imma16832(acc[(2 * j + 1) & 3], w0 & H, w8 & H, v0 & H, v8 & H, st.b[2 * j + 1][0], st.b[2 * j + 1][1]);
        }
        const uint4 hg = *reinterpret_cast<const uint4 *>(hdr_g);
        const uint4 hg8 = *reinterpret_cast<const uint4 *>(hdr_g8);
        // Scales of this lane's sub-blocks 4 * (t / 2) + q, q = 0..3, one per byte.
        const uint32_t pg = (hg.w & st.sc_wmask) | ((hg.y >> st.sc_shift) & st.sc_ymask);
        const uint32_t pg8 = (hg8.w & st.sc_wmask) | ((hg8.y >> st.sc_shift) & st.sc_ymask);
        float main0 = 0.0f, main1 = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            // Odd sets hold high-nibble sub-blocks (codes 16 q): scale / 16.
            const uint32_t biased = (__byte_perm(pg, pg8, uint32_t(q) | (uint32_t(q + 4) << 8)) & 0x00FF00FFu) | kU6Bias;
            const float2 sc = (q & 1) ? u6pair_div16(biased) : u6pair(biased);
            main0 = fmaf(float(acc[q][0] * st.digit_mul + acc[q][1]), sc.x, main0);
            main1 = fmaf(float(acc[q][2] * st.digit_mul + acc[q][3]), sc.y, main1);
        }
        // Mins of sub-blocks t and t+4 (rows g, g+8).
        const uint32_t sel = uint32_t(t) | (uint32_t(t + 4) << 8);
        const uint32_t Y = __byte_perm(hg.z, hg8.z, sel);
        const uint32_t Z = __byte_perm(hg.w, hg8.w, sel);
        const float2 mn_lo = u6pair((Y & 0x003F003Fu) | kU6Bias);
        const float2 mn_hi = u6pair(((Z >> 4) & 0x000F000Fu) | ((Y >> 2) & 0x00300030u) | kU6Bias);
        const float2 dm = half2_bits_to_float2(hg.x);
        const float2 dm8 = half2_bits_to_float2(hg8.x);
        const float out0 = dm.x * (main0 * st.wt_inv) - dm.y * (mn_lo.x * st.sx_lo_t + mn_hi.x * st.sx_hi_t);
        const float out1 = dm8.x * (main1 * st.wt_inv) - dm8.y * (mn_lo.y * st.sx_lo_t + mn_hi.y * st.sx_hi_t);
        return make_float2(out0, out1);
    }
};

// ---------------------------------------------------------------------------
// Batched INT8 path (Q4_K, up to 8 input rows "tokens" per launch). The n8
// tile of mma.m16n8k32.u8.s8 holds the 8 tokens (column g = token g), one
// tile per base-256 digit of x, so the weight codes of a 16-row unit are
// unpacked once and meet all 8 tokens in 3 MMAs per 32-weight sub-block.
// Lane (g,t) accumulates rows g, g+8 x tokens 2t, 2t+1 (complete sums, no
// cross-lane reduction). The 6-bit sub-block scales are applied in integer
// arithmetic (16 x scale for low-nibble sub-blocks, whose codes are q where
// high-nibble codes are 16 q), exact up to one float conversion per digit
// and superblock. The mins term sum_s m_s * sum(x over s) is three more
// MMAs: A = the packed 6-bit mins (k = sub-block), B = the per-token
// sub-block sums of x as exact digits.
// ---------------------------------------------------------------------------
struct I8T8State {
    uint32_t b[8][3][2];  // [sub-block][digit][b0, b1]
    uint32_t bm[3];       // mins B fragment per digit (k = sub-block 4t..4t+3; b1 = 0)
    float inv[2];         // 1 / x scale of tokens 2t, 2t+1 (0 when absent)
    float inv_m[2];       // 1 / scale of their sub-block sums
};

struct I8T8Path {
    using State = I8T8State;
    static constexpr int kTokens = 8;
    using Out = float4;  // (row g, token 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1)
    static __device__ __forceinline__ void accumulate(Out &a, const Out &b) {
        a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
    }
    static constexpr uint32_t kColBytes = 144;
    static constexpr uint32_t kQsOffset = 16;
    static constexpr uint32_t kScratchBytes = 0;

    // power-of-two scale with |v * scale| < 2^22 for |v| <= amax; inv = 1 / scale
    static __device__ __forceinline__ void fixed_point(float amax, float &scale, float &inv) {
        scale = 1.0f, inv = 1.0f;
        const uint32_t ebits = (__float_as_uint(amax) >> 23) & 0xffu;
        if (ebits == 0xffu) {
            inv = __int_as_float(0x7fc00000);
        } else if (amax > 0.0f) {
            const int e = int(ebits) - 127 + 1;
            const int se = max(-126, min(127, 22 - e));
            scale = __uint_as_float(uint32_t(se + 127) << 23);
            inv = __uint_as_float(uint32_t(127 - se) << 23);
        }
    }

    template <class XS>
    static __device__ __forceinline__ void load(const XS &X, int sb, int lane, State &st, uint8_t *,
                                                int64_t x_stride, int ntok) {
        const float *__restrict__ x = X.x;  // batched launches take x as is (mode 0)
        const int t = lane & 3, g = lane >> 2;
        const bool present = g < ntok;
        const float *xs = x + size_t(present ? g : 0) * x_stride + size_t(sb) * 256;
        // This lane's 64 elements of token g: sub-block s, k = 4t..4t+3 and 16+4t..16+4t+3.
        float amax = 0.0f, ps[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            ps[s] = 0.0f;
            if (present) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(xs + 32 * s + 4 * t));
                const float4 c = __ldg(reinterpret_cast<const float4 *>(xs + 32 * s + 16 + 4 * t));
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(c.x), fabsf(c.y)), fmaxf(fabsf(c.z), fabsf(c.w))));
                ps[s] = ((a.x + a.y) + (a.z + a.w)) + ((c.x + c.y) + (c.z + c.w));
            }
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        float smax = 0.0f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            ps[s] += __shfl_xor_sync(0xffffffffu, ps[s], 1);
            ps[s] += __shfl_xor_sync(0xffffffffu, ps[s], 2);  // sum of token g over sub-block s
            smax = fmaxf(smax, fabsf(ps[s]));
        }
        float scale, inv, scale_m, inv_m;
        fixed_point(amax, scale, inv);
        fixed_point(smax, scale_m, inv_m);
        if (!present) inv = 0.0f, inv_m = 0.0f;
        // accumulator side: tokens 2t, 2t+1 live in lanes 8t and 8t+4
        st.inv[0] = __shfl_sync(0xffffffffu, inv, 8 * t);
        st.inv[1] = __shfl_sync(0xffffffffu, inv, 8 * t + 4);
        st.inv_m[0] = __shfl_sync(0xffffffffu, inv_m, 8 * t);
        st.inv_m[1] = __shfl_sync(0xffffffffu, inv_m, 8 * t + 4);
        constexpr int kAdd[3] = {0x8080, 0x80, 0};
        constexpr uint32_t kShift[3] = {16u, 8u, 0u};
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            int v[8];
            if (present) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(xs + 32 * s + 4 * t));
                const float4 c = __ldg(reinterpret_cast<const float4 *>(xs + 32 * s + 16 + 4 * t));
                v[0] = rint_scaled(a.x, scale), v[1] = rint_scaled(a.y, scale);
                v[2] = rint_scaled(a.z, scale), v[3] = rint_scaled(a.w, scale);
                v[4] = rint_scaled(c.x, scale), v[5] = rint_scaled(c.y, scale);
                v[6] = rint_scaled(c.z, scale), v[7] = rint_scaled(c.w, scale);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = 0;
            }
#pragma unroll
            for (int d = 0; d < 3; ++d) {
                st.b[s][d][0] = pack_low_bytes(digit_byte(v[0], kAdd[d], kShift[d]), digit_byte(v[1], kAdd[d], kShift[d]),
                                               digit_byte(v[2], kAdd[d], kShift[d]), digit_byte(v[3], kAdd[d], kShift[d]));
                st.b[s][d][1] = pack_low_bytes(digit_byte(v[4], kAdd[d], kShift[d]), digit_byte(v[5], kAdd[d], kShift[d]),
                                               digit_byte(v[6], kAdd[d], kShift[d]), digit_byte(v[7], kAdd[d], kShift[d]));
            }
        }
        // mins B: k = sub-block s (t = 0: s 0..3, t = 1: s 4..7, t >= 2: zero), column g = token g
        int vm[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float sv = t == 0 ? ps[i] : ps[4 + i];
            vm[i] = (present && t < 2) ? rint_scaled(sv, scale_m) : 0;
        }
#pragma unroll
        for (int d = 0; d < 3; ++d)
            st.bm[d] = pack_low_bytes(digit_byte(vm[0], kAdd[d], kShift[d]), digit_byte(vm[1], kAdd[d], kShift[d]),
                                      digit_byte(vm[2], kAdd[d], kShift[d]), digit_byte(vm[3], kAdd[d], kShift[d]));
    }

    static __device__ __forceinline__ Out rows16(uint32_t ldsm_addr, const uint8_t *hdr_g, const uint8_t *hdr_g8,
                                                 int lane, const State &st, const uint8_t * = nullptr) {
        const int t = lane & 3;
        const uint4 hg = *reinterpret_cast<const uint4 *>(hdr_g);
        const uint4 hg8 = *reinterpret_cast<const uint4 *>(hdr_g8);
        // 6-bit scales: sub-blocks 0..3 in sl, 4..7 in sh (one per byte); mins likewise.
        const uint32_t sl0 = hg.y & 0x3F3F3F3Fu, sl8 = hg8.y & 0x3F3F3F3Fu;
        const uint32_t sh0 = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
        const uint32_t sh8 = (hg8.w & 0x0F0F0F0Fu) | ((hg8.y >> 2) & 0x30303030u);
        int tot[3][4];
#pragma unroll
        for (int d = 0; d < 3; ++d) tot[d][0] = tot[d][1] = tot[d][2] = tot[d][3] = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t w0, w8, v0, v8;
            ldsm_x4(ldsm_addr + 32u * j, w0, w8, v0, v8);
            constexpr uint32_t L = 0x0F0F0F0Fu, H = 0xF0F0F0F0u;
            const uint32_t p0 = j < 2 ? sl0 : sh0, p8 = j < 2 ? sl8 : sh8;
            const uint32_t sh_lo = 16u * (j & 1), sh_hi = sh_lo + 8u;  // bytes 2(j%2), 2(j%2)+1
            const int s_lo0 = int(((p0 >> sh_lo) & 0xffu) << 4), s_lo8 = int(((p8 >> sh_lo) & 0xffu) << 4);
            const int s_hi0 = int((p0 >> sh_hi) & 0xffu), s_hi8 = int((p8 >> sh_hi) & 0xffu);
#pragma unroll
            for (int d = 0; d < 3; ++d) {
                int lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
                imma16832(lo, w0 & L, w8 & L, v0 & L, v8 & L, st.b[2 * j][d][0], st.b[2 * j][d][1]);
                imma16832(hi, w0 & H, w8 & H, v0 & H, v8 & H, st.b[2 * j + 1][d][0], st.b[2 * j + 1][d][1]);
                tot[d][0] += lo[0] * s_lo0 + hi[0] * s_hi0;
                tot[d][1] += lo[1] * s_lo0 + hi[1] * s_hi0;
                tot[d][2] += lo[2] * s_lo8 + hi[2] * s_hi8;
                tot[d][3] += lo[3] * s_lo8 + hi[3] * s_hi8;
            }
        }
        // mins: A = 6-bit mins (k = sub-block: lane t = 0 holds 0..3, t = 1 holds 4..7)
        const uint32_t ml0 = hg.z & 0x3F3F3F3Fu, ml8 = hg8.z & 0x3F3F3F3Fu;
        const uint32_t mh0 = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
        const uint32_t mh8 = ((hg8.w >> 4) & 0x0F0F0F0Fu) | ((hg8.z >> 2) & 0x30303030u);
        const uint32_t am0 = t == 0 ? ml0 : (t == 1 ? mh0 : 0u), am8 = t == 0 ? ml8 : (t == 1 ? mh8 : 0u);
        int mt[3][4];
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            mt[d][0] = mt[d][1] = mt[d][2] = mt[d][3] = 0;
            imma16832(mt[d], am0, am8, 0u, 0u, st.bm[d], 0u);
        }
        const float2 dm = half2_bits_to_float2(hg.x), dm8 = half2_bits_to_float2(hg8.x);
        float r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float main = (float(tot[0][i]) * 65536.0f + float(tot[1][i]) * 256.0f + float(tot[2][i])) * 0.0625f;
            const float mins = float(mt[0][i]) * 65536.0f + float(mt[1][i]) * 256.0f + float(mt[2][i]);
            const float2 dd = i < 2 ? dm : dm8;
            const int u = i & 1;
            r[i] = dd.x * main * st.inv[u] - dd.y * mins * st.inv_m[u];
        }
        return make_float4(r[0], r[1], r[2], r[3]);
    }
};

// ---------------------------------------------------------------------------
// Q8_0 path (mma.sync m16n8k32, s8 x s8 -> s32). A Q8_0 block is 34 bytes
// (FP16 d, 32 int8 quants), so quants are not 16-byte aligned; instead of
// unpacking, the MMA reads the raw row bytes: a column of 8 blocks (256
// elements, 272 bytes) is covered by nine 32-byte windows (the last half
// window overlaps the next column or the row padding), ldmatrix hands each
// lane bytes 4t..4t+3 of every 16-byte chunk, and B holds the x digits of
// the element at each byte position, zero at the FP16 scale bytes and
// outside the column. Columns of the n8 tile: 2 * digit + parity, i.e. even
// blocks in even columns (0, 2, 4), odd blocks in odd ones (1, 3, 5), 6 and 7
// zero. Lane (g,t) then holds digit t of both block parities, so which block
// a window's accumulator belongs to is the same for every lane: block 2j is
// windows 2j and 2j+1 (even columns), block 2j+1 windows 2j+1 and 2j+2 (odd
// columns). Window sums are exact integers (< 2^21); each lane scales its
// eight block sums by the blocks' FP16 d, by its digit weight 2^16 / 2^8 / 1
// and by the x scale, and the four lanes of a row are summed.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void imma16832_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct Q8State {
    uint32_t b[9][2];  // B fragments of the column's nine windows
    float wt_inv;      // digit weight of this lane's accumulator columns / x scale (0 for t = 3)
};

struct Q8Path {
    using State = Q8State;
    static constexpr int kTokens = 1;
    using Out = float2;
    static __device__ __forceinline__ void accumulate(Out &a, const Out &b) { a.x += b.x, a.y += b.y; }
    static constexpr uint32_t kColBytes = 272;  // eight 34-byte blocks
    static constexpr uint32_t kQsOffset = 0;    // windows start at the column start
    static constexpr uint32_t kImageBytes = 288;            // nine windows
    static constexpr uint32_t kScratchBytes = 3 * kImageBytes;  // per compute warp: one image per digit

    // scratch: this warp's 864-byte area. Image d holds, at each byte
    // position of the column, digit d of the element stored there (0 at the
    // scale bytes and beyond the column); each lane then reads its B words
    // with aligned 32-bit loads.
    template <class XS>
    static __device__ __forceinline__ void load(const XS &X, int sb, int lane, State &st, uint8_t *scratch,
                                                int64_t, int) {
        const int64_t xb = int64_t(sb) * 256;
        float v[8];
        if (X.aligned(xb)) {
            const float4 a = X.get4(xb + 8 * lane);
            const float4 b = X.get4(xb + 8 * lane + 4);
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = X.get(xb + 8 * lane + i);
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        float scale = 1.0f, inv = 1.0f;
        const uint32_t ebits = (__float_as_uint(amax) >> 23) & 0xffu;
        if (ebits == 0xffu) {
            inv = __int_as_float(0x7fc00000);  // non-finite activation: the rows become NaN
        } else if (amax > 0.0f) {
            const int e = int(ebits) - 127 + 1;
            const int se = max(-126, min(127, 22 - e));
            scale = __uint_as_float(uint32_t(se + 127) << 23);
            inv = __uint_as_float(uint32_t(127 - se) << 23);
        }
        const int t = lane & 3, g = lane >> 2;
        st.wt_inv = (t == 0 ? 65536.0f : (t == 1 ? 256.0f : (t == 2 ? 1.0f : 0.0f))) * inv;
        // Images: lane l owns elements 8l..8l+7 = bytes 34 * (l / 4) + 2 + 8 * (l % 4) .. + 7 of the column.
        int vi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) vi[i] = rint_scaled(v[i], scale);
        const uint32_t pos = 34u * uint32_t(lane >> 2) + 2u + 8u * uint32_t(lane & 3);
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            const int add = d == 0 ? 0x8080 : (d == 1 ? 0x80 : 0);
            const uint32_t shift = d == 0 ? 16u : (d == 1 ? 8u : 0u);
            uint16_t *img = reinterpret_cast<uint16_t *>(scratch + d * kImageBytes + pos);  // 2-byte aligned
#pragma unroll
            for (int i = 0; i < 4; ++i)
                img[i] = uint16_t((digit_byte(vi[2 * i], add, shift) & 0xffu) |
                                  ((digit_byte(vi[2 * i + 1], add, shift) & 0xffu) << 8));
            // scale bytes of block `lane` and the tail past the column read as zero
            if (lane < 8) *reinterpret_cast<uint16_t *>(scratch + d * kImageBytes + 34 * lane) = 0;
            if (lane < 4) *reinterpret_cast<uint32_t *>(scratch + d * kImageBytes + 272 + 4 * lane) = 0u;
        }
        __syncwarp();
        // B column g = 2 * digit + parity; digit 3 (g = 6, 7) stays zero.
        const int parity = g & 1, digit = g >> 1;
#pragma unroll
        for (int w = 0; w < 9; ++w) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t p0 = 32u * w + 16u * h + 4u * t;  // 4 positions, all in block p0 / 34 or scale bytes
                uint32_t b = 0;
                if (digit < 3 && p0 < 272u && int((p0 / 34u) & 1u) == parity)
                    b = *reinterpret_cast<const uint32_t *>(scratch + digit * kImageBytes + p0);
                st.b[w][h] = b;
            }
        }
        __syncwarp();
    }

    // hdr_g / hdr_g8: the column's first byte in rows g and g+8.
    static __device__ __forceinline__ float2 rows16(uint32_t ldsm_addr, const uint8_t *hdr_g, const uint8_t *hdr_g8,
                                                    int lane, const State &st,
                                                    const uint8_t * = nullptr) {
        (void)lane;
        int acc[9][4];
#pragma unroll
        for (int w = 0; w < 9; ++w) {
            uint32_t w0, w8, v0, v8;
            ldsm_x4(ldsm_addr + 32u * w, w0, w8, v0, v8);
            acc[w][0] = acc[w][1] = acc[w][2] = acc[w][3] = 0;
            imma16832_s8(acc[w], w0, w8, v0, v8, st.b[w][0], st.b[w][1]);
        }
        const uint16_t *dg = reinterpret_cast<const uint16_t *>(hdr_g);
        const uint16_t *dg8 = reinterpret_cast<const uint16_t *>(hdr_g8);
        float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            // block 2j: windows 2j, 2j+1, even column (c0 row g, c2 row g+8)
            const int e0 = acc[2 * j][0] + acc[2 * j + 1][0], e1 = acc[2 * j][2] + acc[2 * j + 1][2];
            // block 2j+1: windows 2j+1, 2j+2, odd column (c1, c3)
            const int o0 = acc[2 * j + 1][1] + acc[2 * j + 2][1], o1 = acc[2 * j + 1][3] + acc[2 * j + 2][3];
            m0 = fmaf(__half2float(__ushort_as_half(dg[17 * (2 * j)])), float(e0), m0);
            m0 = fmaf(__half2float(__ushort_as_half(dg[17 * (2 * j + 1)])), float(o0), m0);
            m1 = fmaf(__half2float(__ushort_as_half(dg8[17 * (2 * j)])), float(e1), m1);
            m1 = fmaf(__half2float(__ushort_as_half(dg8[17 * (2 * j + 1)])), float(o1), m1);
        }
        return make_float2(m0 * st.wt_inv, m1 * st.wt_inv);
    }
};

}  // namespace
}  // namespace si::dev
