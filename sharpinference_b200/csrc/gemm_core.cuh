// Device pieces shared by the tcgen05 GEMM kernels (gemm.cu: the prefill
// GEMM; gemm_skinny.cu: the few-row GEMM): shared-memory matrix
// descriptors, the BF16 MMA issue and commit, TMEM loads, and the GGUF
// weight fetch / decode of 64 columns of one row.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <type_traits>
#include <cuda_fp16.h>

#include "device_common.cuh"
#include "si_internal.h"

namespace si::dev {

constexpr int kGemmBM = 128;  // weight rows per CTA (MMA M)
constexpr int kGemmBK = 64;   // K per stage (128 B of BF16)
constexpr int kProducers = 256;  // weight-producer threads: two per weight row

// Instruction descriptor, kind::f16: D F32, A/B BF16, both K-major,
// N (bits 17-22: N>>3), M = 128 (bits 24-28: M>>4).
constexpr uint32_t mma_idesc(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(kGemmBM >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major tile in the canonical
// 128-byte swizzled layout: rows of 128 B, 8-row groups 1024 B apart
// (stride byte offset), leading byte offset 16 B, version 1, swizzle 128B.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// D[tmem] (+)= A * B^T, kind::f16 with BF16 operands and an FP32
// accumulator; idesc from mma_idesc.
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float h16(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xffffu)));
}

// 64 consecutive weights of one row, columns k0 .. k0+63 (k0 % 64 == 0), in
// two steps so that the producer issues the next stage's loads before it
// decodes this one: fetch_weights64 loads the raw bytes into registers,
// decode_weights64 turns them into FP32 values.
template <int FMT>
struct RawWeights {
    uint4 v[FMT == SI_TYPE_Q4_K ? 3 : FMT == SI_TYPE_Q8_0 ? 5 : FMT == SI_TYPE_F16 ? 8 : 16];
    int j;  // Q4_K: 64-column group within the super-block
};

template <int FMT>
__device__ __forceinline__ void fetch_weights64(const uint8_t *row, int k0, RawWeights<FMT> &r) {
    if constexpr (FMT == SI_TYPE_Q4_K) {
        const uint8_t *sb = row + (k0 >> 8) * 144;
        r.j = (k0 >> 6) & 3;
        r.v[0] = __ldg(reinterpret_cast<const uint4 *>(sb));
        r.v[1] = __ldg(reinterpret_cast<const uint4 *>(sb + 16 + 32 * r.j));
        r.v[2] = __ldg(reinterpret_cast<const uint4 *>(sb + 32 + 32 * r.j));
    } else if constexpr (FMT == SI_TYPE_Q8_0) {
        const uint32_t *u = reinterpret_cast<const uint32_t *>(row + (k0 >> 5) * 34);  // 68 bytes, 4-byte aligned
#pragma unroll
        for (int i = 0; i < 5; ++i) {
            r.v[i].x = __ldg(u + 4 * i);
            r.v[i].y = i < 4 ? __ldg(u + 4 * i + 1) : 0u;
            r.v[i].z = i < 4 ? __ldg(u + 4 * i + 2) : 0u;
            r.v[i].w = i < 4 ? __ldg(u + 4 * i + 3) : 0u;
        }
    } else if constexpr (FMT == SI_TYPE_F16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + size_t(k0) * 2);
#pragma unroll
        for (int i = 0; i < 8; ++i) r.v[i] = __ldg(p + i);
    } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + size_t(k0) * 4);
#pragma unroll
        for (int i = 0; i < 16; ++i) r.v[i] = __ldg(p + i);
    }
}

template <int FMT>
__device__ __forceinline__ void decode_weights64(const RawWeights<FMT> &r, float (&w)[64]) {
    if constexpr (FMT == SI_TYPE_Q4_K) {
        const uint4 h = r.v[0];
        const uint32_t q[8] = {r.v[1].x, r.v[1].y, r.v[1].z, r.v[1].w, r.v[2].x, r.v[2].y, r.v[2].z, r.v[2].w};
        const int j = r.j;
        const uint32_t sc_lo = h.y & 0x3F3F3F3Fu, mn_lo = h.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
        const uint32_t mn_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
        const uint32_t scw = j >= 2 ? sc_hi : sc_lo, mnw = j >= 2 ? mn_hi : mn_lo;
        const int b0 = (2 * j) & 3;
        const float d = h16(h.x), dmin = h16(h.x >> 16);
        const float a0 = d * float((scw >> (8 * b0)) & 0xffu), a1 = d * float((scw >> (8 * b0 + 8)) & 0xffu);
        const float c0 = dmin * float((mnw >> (8 * b0)) & 0xffu), c1 = dmin * float((mnw >> (8 * b0 + 8)) & 0xffu);
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint32_t byte = (q[i] >> (8 * b)) & 0xffu;
                w[4 * i + b] = a0 * float(byte & 15u) - c0;
                w[32 + 4 * i + b] = a1 * float(byte >> 4) - c1;
            }
    } else if constexpr (FMT == SI_TYPE_Q8_0) {
        uint32_t wv[17];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wv[4 * i] = r.v[i].x, wv[4 * i + 1] = r.v[i].y, wv[4 * i + 2] = r.v[i].z, wv[4 * i + 3] = r.v[i].w;
        }
        wv[16] = r.v[4].x;
        const float d0 = h16(wv[0]), d1 = h16(wv[8] >> 16);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const int b0 = 2 + e, b1 = 36 + e;
            w[e] = d0 * float(int8_t((wv[b0 >> 2] >> (8 * (b0 & 3))) & 0xffu));
            w[32 + e] = d1 * float(int8_t((wv[b1 >> 2] >> (8 * (b1 & 3))) & 0xffu));
        }
    } else if constexpr (FMT == SI_TYPE_F16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t vv[4] = {r.v[i].x, r.v[i].y, r.v[i].z, r.v[i].w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                w[8 * i + 2 * t] = h16(vv[t]);
                w[8 * i + 2 * t + 1] = h16(vv[t] >> 16);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            w[4 * i] = __uint_as_float(r.v[i].x), w[4 * i + 1] = __uint_as_float(r.v[i].y);
            w[4 * i + 2] = __uint_as_float(r.v[i].z), w[4 * i + 3] = __uint_as_float(r.v[i].w);
        }
    }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Half of a stage's 64 columns of one row (columns 32h .. 32h+31): the
// weight producers run two threads per row, each fetching and decoding its
// half, so twice the warps share the dequantisation work.
template <int FMT>
struct RawHalf {
    uint4 v[FMT == SI_TYPE_Q4_K ? 3 : FMT == SI_TYPE_Q8_0 ? 3 : FMT == SI_TYPE_F16 ? 4 : 8];
    uint32_t extra;  // Q8_0: the ninth 32-bit word of the block window
    int j;           // Q4_K: 64-column group within the super-block
};

template <int FMT>
__device__ __forceinline__ void fetch_weights32(const uint8_t *row, int k0, int h, RawHalf<FMT> &r) {
    if constexpr (FMT == SI_TYPE_Q4_K) {
        // both halves need the group's 32 quant bytes (low / high nibbles)
        const uint8_t *sb = row + (k0 >> 8) * 144;
        r.j = (k0 >> 6) & 3;
        r.v[0] = __ldg(reinterpret_cast<const uint4 *>(sb));
        r.v[1] = __ldg(reinterpret_cast<const uint4 *>(sb + 16 + 32 * r.j));
        r.v[2] = __ldg(reinterpret_cast<const uint4 *>(sb + 32 + 32 * r.j));
    } else if constexpr (FMT == SI_TYPE_Q8_0) {
        // blocks 2m (4-byte aligned) and 2m+1 (2 bytes past a 4-byte
        // boundary): 36 bytes from word 0, or from word 8, of the pair
        const uint32_t *u = reinterpret_cast<const uint32_t *>(row + (k0 >> 5) * 34) + 8 * h;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            r.v[i].x = __ldg(u + 4 * i), r.v[i].y = __ldg(u + 4 * i + 1);
            r.v[i].z = __ldg(u + 4 * i + 2), r.v[i].w = __ldg(u + 4 * i + 3);
        }
        r.extra = __ldg(u + 8);
        r.j = h;
    } else if constexpr (FMT == SI_TYPE_F16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + size_t(k0 + 32 * h) * 2);
#pragma unroll
        for (int i = 0; i < 4; ++i) r.v[i] = __ldg(p + i);
    } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + size_t(k0 + 32 * h) * 4);
#pragma unroll
        for (int i = 0; i < 8; ++i) r.v[i] = __ldg(p + i);
    }
}

// The same half-row bytes from a super-stage in shared memory: row_ss is
// the row's 256 columns (Q4_K: one super-block, 144 bytes; Q8_0: eight
// blocks, 272 bytes), `sub` the 64-column stage within it.
template <int FMT>
__device__ __forceinline__ void fetch_weights32_smem(const uint8_t *row_ss, int sub, int h, RawHalf<FMT> &r) {
    static_assert(FMT == SI_TYPE_Q4_K || FMT == SI_TYPE_Q8_0, "super-stages hold Q4_K or Q8_0 rows");
    if constexpr (FMT == SI_TYPE_Q4_K) {
        r.j = sub;
        r.v[0] = *reinterpret_cast<const uint4 *>(row_ss);
        r.v[1] = *reinterpret_cast<const uint4 *>(row_ss + 16 + 32 * sub);
        r.v[2] = *reinterpret_cast<const uint4 *>(row_ss + 32 + 32 * sub);
    } else {
        const uint32_t *u = reinterpret_cast<const uint32_t *>(row_ss + 68 * sub) + 8 * h;
#pragma unroll
        for (int i = 0; i < 2; ++i) r.v[i] = make_uint4(u[4 * i], u[4 * i + 1], u[4 * i + 2], u[4 * i + 3]);
        r.extra = u[8];
        r.j = h;
    }
}

template <int FMT>
__device__ __forceinline__ void decode_weights32(const RawHalf<FMT> &r, int h, float (&w)[32]) {
    if constexpr (FMT == SI_TYPE_Q4_K) {
        const uint4 hd = r.v[0];
        const uint32_t q[8] = {r.v[1].x, r.v[1].y, r.v[1].z, r.v[1].w, r.v[2].x, r.v[2].y, r.v[2].z, r.v[2].w};
        const int j = r.j;
        const uint32_t sc_lo = hd.y & 0x3F3F3F3Fu, mn_lo = hd.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
        const uint32_t mn_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        const uint32_t scw = j >= 2 ? sc_hi : sc_lo, mnw = j >= 2 ? mn_hi : mn_lo;
        const int b = ((2 * j) & 3) + h;  // sub-block byte of this half
        const float a = h16(hd.x) * float((scw >> (8 * b)) & 0xffu);
        const float c = h16(hd.x >> 16) * float((mnw >> (8 * b)) & 0xffu);
        // nibble -> float without the conversion pipe: the byte placed under
        // the exponent of 2^23 (byte permute) gives 2^23 + q exactly.
        const int shift = 4 * h;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t nib = (q[i] >> shift) & 0x0F0F0F0Fu;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float f = __uint_as_float(__byte_perm(nib, 0x4B000000u, uint32_t(t) | 0x7650u)) - 8388608.0f;
                w[4 * i + t] = a * f - c;
            }
        }
    } else if constexpr (FMT == SI_TYPE_Q8_0) {
        uint32_t wv[9];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            wv[4 * i] = r.v[i].x, wv[4 * i + 1] = r.v[i].y, wv[4 * i + 2] = r.v[i].z, wv[4 * i + 3] = r.v[i].w;
        }
        wv[8] = r.extra;
        // the block starts at byte 0 (h = 0) or 2 (h = 1) of the window;
        // two unrolled copies keep every word index a constant
        // int8 -> float without the conversion pipe: with the sign bit
        // flipped the byte is q + 128, placed under the exponent of 2^23.
        auto decode = [&](auto offset) {
            constexpr int o = decltype(offset)::value;
            const float d = h16(o == 0 ? (wv[0] & 0xffffu) : (wv[0] >> 16));
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                constexpr int base = o + 2;
                const int byte = base + e;
                const uint32_t biased = wv[byte >> 2] ^ 0x80808080u;
                const float f = __uint_as_float(__byte_perm(biased, 0x4B000000u, uint32_t(byte & 3) | 0x7650u)) -
                                8388736.0f;  // 2^23 + 128
                w[e] = d * f;
            }
        };
        if (r.j == 0) decode(std::integral_constant<int, 0>{});
        else decode(std::integral_constant<int, 2>{});
    } else if constexpr (FMT == SI_TYPE_F16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t vv[4] = {r.v[i].x, r.v[i].y, r.v[i].z, r.v[i].w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                w[8 * i + 2 * t] = h16(vv[t]);
                w[8 * i + 2 * t + 1] = h16(vv[t] >> 16);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            w[4 * i] = __uint_as_float(r.v[i].x), w[4 * i + 1] = __uint_as_float(r.v[i].y);
            w[4 * i + 2] = __uint_as_float(r.v[i].z), w[4 * i + 3] = __uint_as_float(r.v[i].w);
        }
    }
}

// Stages of raw weight bytes a producer thread keeps in flight (deeper
// rings measured slower: the producers are bound by instruction issue, and
// the ring costs registers).
template <int FMT>
struct PrefetchDepth {
    static constexpr int value = 2;
};

// A producer thread's loop over its K stages: decodes stage it's 32 weights
// (fetched PrefetchDepth stages earlier into a register ring), refills the
// ring slot with stage it + depth, then hands the weights to emit(it, w),
// which waits for the shared-memory slot, stores and arrives. The loop is
// unrolled by the depth so every ring index is a constant.
template <int FMT, class Emit>
__device__ __forceinline__ void produce_weights(const uint8_t *wrow, bool valid, int it0, int iters, int h,
                                                Emit &&emit) {
    constexpr int D = PrefetchDepth<FMT>::value;
    RawHalf<FMT> ring[D];
#pragma unroll
    for (int u = 0; u < D; ++u)
        if (valid && u < iters) fetch_weights32<FMT>(wrow, (it0 + u) * kGemmBK, h, ring[u]);
    for (int base = 0; base < iters; base += D) {
#pragma unroll
        for (int u = 0; u < D; ++u) {
            const int it = base + u;
            if (it >= iters) break;
            float w[32];
            if (valid) {
                decode_weights32<FMT>(ring[u], h, w);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) w[i] = 0.0f;
            }
            if (valid && it + D < iters) fetch_weights32<FMT>(wrow, (it0 + it + D) * kGemmBK, h, ring[u]);
            emit(it, w);
        }
    }
}

// Splits 32 decoded weights (columns 32h ..) into BF16 hi / lo and stores
// them as 16-byte chunks 4h .. 4h+3 of row r in the canonical K-major
// 128-byte-swizzled layout (hi tile at `hi`, lo tile at `lo`).
__device__ __forceinline__ void store_split_half(const float (&w)[32], int r, int h, uint8_t *hi, uint8_t *lo) {
    uint8_t *hi_row = hi + (r >> 3) * 1024 + (r & 7) * 128;
    uint8_t *lo_row = lo + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t hv[4], lv[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float v0 = w[8 * c + 2 * t], v1 = w[8 * c + 2 * t + 1];
            const uint32_t hb = pack_bf16(v0, v1);
            hv[t] = hb;
            lv[t] = pack_bf16(v0 - __uint_as_float(hb << 16), v1 - __uint_as_float(hb & 0xffff0000u));
        }
        const int pc = (4 * h + c) ^ (r & 7);
        *reinterpret_cast<uint4 *>(hi_row + pc * 16) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<uint4 *>(lo_row + pc * 16) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
}


}  // namespace si::dev
