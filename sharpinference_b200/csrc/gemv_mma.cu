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
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "device_common.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

constexpr int kMaxComputeWarps = 16;
constexpr int kMaxWps2Warps = 24;  // compute warps of the two-warps-per-column instantiation

struct MmaParams {
    const uint8_t *w;
    const float *x;
    float *y;
    kernels::PeerGather peer;  // nranks == 0: plain GEMV into y
    const int32_t *control;    // batch-shared: y is written only when token < control[1]
    int token;                 // index of this launch's first input row (batched: of its 8 rows)
    int ntok;                  // batched paths: input rows in this launch (<= 8)
    int64_t x_stride;          // batched paths: floats between input rows (K)
    int64_t y_stride;          // batched paths: floats between output rows (N)
    int rows;
    int nsb;              // superblocks per row (K / 256)
    int cluster;          // CTAs per cluster = K split (1, 2 or 4)
    int nsb_cta;          // superblocks of every row one CTA covers (nsb / cluster)
    int compute_warps;    // C
    int spw;              // superblocks per compute warp (1 or 2)
    int wps;              // compute warps per superblock column (1 or 2)
    int stages;
    uint32_t row_bytes;   // column bytes (144 Q4_K, 272 Q8_0) * nsb, the global row pitch
    uint32_t cta_bytes;   // column bytes * nsb_cta, bytes of each row one CTA loads
    uint32_t row_stride;  // padded shared-memory row stride (per-row copies)
    // Shared-memory row map (see row_offset): rows come in groups of
    // group_rows consecutive rows at pitch row_pitch, groups group_stride
    // apart; class_period P = rows per group that fall in distinct bank
    // classes. copy_groups: one bulk copy per group instead of per row.
    int group_rows;       // power of two
    int class_period;     // power of two
    int log2_group_rows;
    int log2_class_period;
    uint32_t row_pitch;
    uint32_t group_stride;
    int copy_groups;
    uint32_t stage_bytes;
    int num_tiles;
    int path;             // host side: 0 FP16 MMA, 1 INT8 MMA
    int groups;           // clusters (or CTAs when cluster == 1) in the grid
    int max_local_tiles;  // ceil(num_tiles / groups): row-sum slots per CTA when cluster > 1
    // Input transform applied while x is loaded (the decode step's fused
    // prologue; kernels::XForm): 0 x as is; 1 rms-norm, x_j = (x_j + x_res_j)
    // * s * x_norm_w_j with s = 1 / sqrt(mean over all K of (x + x_res)^2 +
    // x_eps), CTA 0 also storing x + x_res to x_updated; 2 swiglu, x_j =
    // g_j / (1 + exp(-g_j)) * u_j with g = x[0, K) and u = x[K, 2K).
    int x_mode;
    float x_eps;
    const float *x_res;
    const float *x_norm_w;
    float *x_updated;
    // Weights of the next projection to pull into L2 once this CTA's ring
    // is full (decode step; null: none).
    const uint8_t *prefetch;
    uint64_t prefetch_bytes;
};

// Source of the GEMV input as the load paths see it: element i of the
// (transformed) vector. The transform is a template parameter so the plain
// load (M = 0) compiles to bare vector loads the compiler can batch. Modes
// 1 and 2 need 16-byte aligned vectors.
template <int M>
struct XSrc {
    const float *x;
    const float *res;
    const float *w;
    float scale;
    int64_t up;  // mode 2: offset of u
    __device__ __forceinline__ bool aligned(int64_t i) const {
        return M != 0 || (reinterpret_cast<uintptr_t>(x + i) & 15u) == 0;
    }
    static __device__ __forceinline__ float swish_mul(float g, float u) {
        return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
    __device__ __forceinline__ float get(int64_t i) const {
        const float a = __ldg(x + i);
        if constexpr (M == 0) {
            return a;
        } else if constexpr (M == 1) {
            const float v = res ? __fadd_rn(a, __ldg(res + i)) : a;
            return __fmul_rn(__fmul_rn(v, scale), __ldg(w + i));
        } else {
            return swish_mul(a, __ldg(x + up + i));
        }
    }
    __device__ __forceinline__ float4 get4(int64_t i) const {
        float4 a = __ldg(reinterpret_cast<const float4 *>(x + i));
        if constexpr (M == 0) {
            return a;
        } else if constexpr (M == 1) {
            if (res) {
                const float4 r = __ldg(reinterpret_cast<const float4 *>(res + i));
                a = make_float4(__fadd_rn(a.x, r.x), __fadd_rn(a.y, r.y), __fadd_rn(a.z, r.z), __fadd_rn(a.w, r.w));
            }
            const float4 m = __ldg(reinterpret_cast<const float4 *>(w + i));
            return make_float4(__fmul_rn(__fmul_rn(a.x, scale), m.x), __fmul_rn(__fmul_rn(a.y, scale), m.y),
                               __fmul_rn(__fmul_rn(a.z, scale), m.z), __fmul_rn(__fmul_rn(a.w, scale), m.w));
        } else {
            const float4 u = __ldg(reinterpret_cast<const float4 *>(x + up + i));
            return make_float4(swish_mul(a.x, u.x), swish_mul(a.y, u.y), swish_mul(a.z, u.z), swish_mul(a.w, u.w));
        }
    }
};

// --- thread-block cluster helpers (distributed shared memory) ---
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
// Output row store: into y, or (row-sharded GEMV) into every rank's output
// vector at this rank's row offset, over NVLink for the peers.
__device__ __forceinline__ void store_y(const MmaParams &p, int row, float v, int tok = 0) {
    if (p.control && p.token + tok >= p.control[1]) return;  // read after the dependency wait
    if (p.peer.nranks == 0) {
        p.y[tok * p.y_stride + row] = v;
        return;
    }
    const int64_t gr = p.peer.row_base + row;
#pragma unroll
    for (int q = 0; q < kernels::kMaxPeerRanks; ++q)
        if (q < p.peer.nranks) p.peer.ys[q][gr] = v;
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t *addr, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *addr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// End of a row-sharded GEMV: the last CTA of this rank (ticket) publishes
// epoch e to every rank's flag slot of this rank, then waits (bounded) until
// every rank has published e here, so the output vector is complete when
// the kernel completes. The warp that stored output rows fenced them at
// system scope before the CTA barrier that precedes the ticket; one more
// system fence after the ticket orders all CTAs' rows before the flags
// (a system fence with remote stores in flight costs ~3 us on NVLink, so
// only the storing warp and the publishing thread fence).
__device__ __forceinline__ void peer_handshake(const MmaParams &p) {
    const kernels::PeerGather &g = p.peer;
    const uint32_t t = atomicAdd(g.ticket, 1u);
    if (t != gridDim.x - 1) return;
    __threadfence_system();
    *g.ticket = 0u;  // every CTA of this launch has taken its ticket
    const uint32_t e = *reinterpret_cast<volatile uint32_t *>(g.epoch) + 1u;
    for (int q = 0; q < g.nranks; ++q) st_relaxed_sys(g.flags[q] + g.rank, e);
    const uint32_t *mine = g.flags[g.rank];
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < g.nranks; ++q) {
        uint32_t polls = 0;
        while (int32_t(ld_acquire_sys(mine + q) - e) < 0) {
            if (++polls > kMaxPolls || globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&g_error_word, kErrPeerTimeout);
                break;
            }
            __nanosleep(64);
        }
    }
    *reinterpret_cast<volatile uint32_t *>(g.epoch) = e;
}

// Every thread of every CTA of the cluster (hardware barrier).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

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
        float v[8];
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
        const int half = g >> 2, digit = g & 3;
        const int dadd = digit == 0 ? 0x8080 : (digit == 1 ? 0x80 : 0);
        const uint32_t dshift = digit == 0 ? 16u : (digit == 1 ? 8u : 0u);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            uint32_t b0 = 0, b1 = 0;
            if ((s >> 2) == half && digit < 3) {
                float q[8];
                const int64_t e0 = xb + 32 * s + 4 * t;
                if (aligned) {
                    const float4 a = X.get4(e0);
                    const float4 c = X.get4(e0 + 16);
                    q[0] = a.x, q[1] = a.y, q[2] = a.z, q[3] = a.w, q[4] = c.x, q[5] = c.y, q[6] = c.z, q[7] = c.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) q[i] = X.get(e0 + i), q[4 + i] = X.get(e0 + 16 + i);
                }
                uint32_t dg[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) dg[i] = digit_byte(__float2int_rn(q[i] * scale), dadd, dshift);
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
                v[0] = __float2int_rn(a.x * scale), v[1] = __float2int_rn(a.y * scale);
                v[2] = __float2int_rn(a.z * scale), v[3] = __float2int_rn(a.w * scale);
                v[4] = __float2int_rn(c.x * scale), v[5] = __float2int_rn(c.y * scale);
                v[6] = __float2int_rn(c.z * scale), v[7] = __float2int_rn(c.w * scale);
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
            vm[i] = (present && t < 2) ? __float2int_rn(sv * scale_m) : 0;
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
        for (int i = 0; i < 8; ++i) vi[i] = __float2int_rn(v[i] * scale);
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

// Tile row of MMA row r (0..15) of 16-row unit u: the unit's two 8-row
// ldmatrix sets k = 2u, 2u+1 take P rows from each of the 8/P groups, so
// their eight row addresses fall in eight distinct bank classes.
__device__ __forceinline__ int unit_row(const MmaParams &p, int u, int r) {
    const int k = 2 * u + (r >> 3), e = r & 7;
    return ((e >> p.log2_class_period) << p.log2_group_rows) + (k << p.log2_class_period) +
           (e & (p.class_period - 1));
}
__device__ __forceinline__ uint32_t row_offset(const MmaParams &p, int row) {
    return uint32_t(row >> p.log2_group_rows) * p.group_stride + uint32_t(row & (p.group_rows - 1)) * p.row_pitch;
}

// Fused rms-norm prologue (x_mode 1): the C compute warps of every CTA
// reduce the sum of squares of x + x_res over all K in one fixed order, so
// every CTA derives the same scale; CTA 0 also stores x + x_res to
// x_updated. `red` is C floats of shared memory the pipeline has not used
// yet; named barrier 1 spans the C compute warps only.
__device__ __forceinline__ float rms_prologue(const MmaParams &p, int warp, int lane, int C, float *red) {
    const int64_t K = int64_t(p.nsb) * 256;
    const bool store = p.x_updated != nullptr && blockIdx.x == 0;
    float s = 0.0f;
    for (int64_t i = (int64_t(warp) * 32 + lane) * 4; i < K; i += int64_t(C) * 128) {
        float4 a = __ldg(reinterpret_cast<const float4 *>(p.x + i));
        if (p.x_res) {
            const float4 r = __ldg(reinterpret_cast<const float4 *>(p.x_res + i));
            a = make_float4(__fadd_rn(a.x, r.x), __fadd_rn(a.y, r.y), __fadd_rn(a.z, r.z), __fadd_rn(a.w, r.w));
        }
        if (store) *reinterpret_cast<float4 *>(p.x_updated + i) = a;
        s = __fadd_rn(s, __fmul_rn(a.x, a.x));
        s = __fadd_rn(s, __fmul_rn(a.y, a.y));
        s = __fadd_rn(s, __fmul_rn(a.z, a.z));
        s = __fadd_rn(s, __fmul_rn(a.w, a.w));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    if (lane == 0) red[warp] = s;
    asm volatile("bar.sync 1, %0;" ::"r"(C * 32) : "memory");
    float total = 0.0f;
    for (int w = 0; w < C; ++w) total = __fadd_rn(total, red[w]);
    asm volatile("bar.sync 1, %0;" ::"r"(C * 32) : "memory");  // red returns to the pipeline
    return 1.0f / sqrtf(__fadd_rn(__fdiv_rn(total, float(K)), p.x_eps));
}

// WPS compute warps share each superblock column (WPS = 2: each takes one
// 16-row half of a 32-row tile), for more warps in flight per SM.
template <class Path, int SPW, int RT, int WPS, int MAXW>
__global__ void __launch_bounds__((MAXW + 2) * 32, 1) gemv_mma_q4k_kernel(const MmaParams p) {
    static_assert(WPS == 1 || (WPS == 2 && SPW == 1 && RT == 32), "two warps per column need 32-row tiles");
    extern __shared__ __align__(128) uint8_t smem[];
    const int C = p.compute_warps, CS = p.cluster;
    const int C0 = C / WPS;  // superblock columns (partial sums per row)
    constexpr int TK = Path::kTokens;  // input rows per launch (1: GEMV)
    constexpr int RTK = RT * TK;       // outputs per tile
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + size_t(p.stages) * p.stage_bytes);
    uint64_t *empty = full + p.stages;
    uint64_t *pfull = empty + p.stages;  // [2] compute warps -> reducer
    uint64_t *pempty = pfull + 2;        // [2] reducer -> compute warps
    float *part = reinterpret_cast<float *>(pempty + 2);  // [2][C0][RT][TK]
    float *rowsum = part + size_t(2) * C0 * RTK;           // [max_local_tiles][RT][TK] when CS > 1
    // Per compute warp scratch of the path, 16-byte aligned.
    uint8_t *scratch = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(rowsum + size_t(p.max_local_tiles) * RTK * (CS > 1)) + 15) & ~uintptr_t(15));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t crank = CS > 1 ? cluster_ctarank() : 0u;
    const int first_tile = CS > 1 ? int(cluster_id_x()) : int(blockIdx.x);
    const int tile_step = CS > 1 ? int(cluster_count_x()) : int(gridDim.x);
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
        // Producer: one bulk copy per row (this CTA's K slice) into the padded stage rows.
        const uint8_t *wsrc = p.w + size_t(crank) * p.cta_bytes;
        int it = 0, s = 0;
        uint32_t ring_phase = 0;
        for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
            if (it >= p.stages) mbar_wait(&empty[s], ring_phase ^ 1u, kErrEmptyBarrierTimeout);
            const int r0 = tile * RT;
            const int nrows = min(RT, p.rows - r0);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], uint32_t(nrows) * p.cta_bytes);
            __syncwarp();
            uint8_t *dst = smem + size_t(s) * p.stage_bytes;
            if (p.copy_groups) {
                // One copy per group of consecutive rows (contiguous in global memory).
                const int G = p.group_rows;
                const int first = lane * G;
                if (first < nrows) {
                    const int cnt = min(G, nrows - first);
                    bulk_copy_g2s(dst + size_t(lane) * p.group_stride, wsrc + size_t(r0 + first) * p.row_bytes,
                                  uint32_t(cnt) * p.cta_bytes, &full[s]);
                }
            } else {
                for (int r = lane; r < nrows; r += 32)
                    bulk_copy_g2s(dst + size_t(r) * p.row_stride, wsrc + size_t(r0 + r) * p.row_bytes, p.cta_bytes,
                                  &full[s]);
            }
            if (it == p.stages - 1) prefetch_l2_share(p.prefetch, p.prefetch_bytes, lane);
            if (++s == p.stages) s = 0, ring_phase ^= 1u;
        }
        if (it < p.stages) prefetch_l2_share(p.prefetch, p.prefetch_bytes, lane);  // fewer tiles than stages
    } else if (warp == C + 1) {
        // Reducer: fixed-order sum of the C0 per-column partials of each
        // output (row r, input row u) = index r * TK + u of the tile.
        if (CS == 1) pdl_wait();  // y may still be read by the previous kernel
        int it = 0;
        for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
            const int b = it & 1;
            mbar_wait(&pfull[b], (it >> 1) & 1, kErrEpilogueTimeout);
            const int r0 = tile * RT;
            const int nrows = min(RT, p.rows - r0);
            const float *pb = part + size_t(b) * C0 * RTK;
#pragma unroll
            for (int o0 = 0; o0 < RTK; o0 += 32) {
                const int o = o0 + lane, r = o / TK, u = o % TK;
                if (o >= RTK) break;  // RT * TK = 16: lanes 16..31 have no output
                float a = 0.0f;
                if (r < nrows)
                    for (int c = 0; c < C0; ++c) a += pb[c * RTK + o];
                if (CS == 1) {
                    if (r < nrows && (TK == 1 || u < p.ntok)) store_y(p, r0 + r, a, u);
                } else {
                    rowsum[it * RTK + o] = a;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pempty[b]);
        }
    } else {
        // Compute warp `warp`: column col = warp % C0, i.e. superblocks col,
        // col + C0 (SPW == 2) of this CTA's slice; row half warp / C0 (WPS == 2).
        typename Path::State st0;
        typename Path::State st1;
        const int col = warp % C0, unit0 = warp / C0;
        const int sb0 = col, sb1 = col + C0;
        const bool has1 = SPW == 2 && sb1 < p.nsb_cta;
        const int gsb = int(crank) * p.nsb_cta;
        pdl_wait();  // x is produced by the previous kernel
        uint8_t *my_scratch = scratch + size_t(warp) * Path::kScratchBytes;
        auto load_x = [&](const auto &X) {
            Path::load(X, gsb + sb0, lane, st0, my_scratch, p.x_stride, p.ntok);
            if constexpr (SPW == 2) {
                if (has1) Path::load(X, gsb + sb1, lane, st1, my_scratch, p.x_stride, p.ntok);
            }
        };
        const int64_t K = int64_t(p.nsb) * 256;
        if (Path::kTokens > 1 || p.x_mode == 0) {
            load_x(XSrc<0>{p.x, nullptr, nullptr, 1.0f, K});
        } else if (p.x_mode == 1) {
            const float scale = rms_prologue(p, warp, lane, C, part);
            load_x(XSrc<1>{p.x, p.x_res, p.x_norm_w, scale, K});
        } else {
            load_x(XSrc<2>{p.x, nullptr, nullptr, 1.0f, K});
        }

        const int g = lane >> 2, t = lane & 3;
        constexpr int kUnits = RT / 16 / WPS;  // 16-row groups per warp per tile
        // Per unit: this lane's ldmatrix row address and the rows g, g+8 it
        // owns in the epilogue (offsets within a stage, superblock 0).
        uint32_t off_ldsm[kUnits], off_g[kUnits], off_g8[kUnits];
        int row_g[kUnits], row_g8[kUnits];
#pragma unroll
        for (int q = 0; q < kUnits; ++q) {
            const int u = q * WPS + unit0;
            const int m = lane >> 3;
            off_ldsm[q] = row_offset(p, unit_row(p, u, (m & 1) * 8 + (lane & 7))) + uint32_t(m >> 1) * 16u + Path::kQsOffset;
            row_g[q] = unit_row(p, u, g);
            row_g8[q] = unit_row(p, u, g + 8);
            off_g[q] = row_offset(p, row_g[q]);
            off_g8[q] = row_offset(p, row_g8[q]);
        }
        int it = 0, s = 0;
        uint32_t ring_phase = 0;
        for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
            const int b = it & 1;
            mbar_wait(&full[s], ring_phase, kErrFullBarrierTimeout);
            const uint8_t *stage = smem + size_t(s) * p.stage_bytes;
            const uint32_t stage_addr = smem_u32(stage);
            if (it >= 2) mbar_wait(&pempty[b], ((it >> 1) - 1) & 1, kErrEpilogueTimeout);
            float *pw = part + (size_t(b) * C0 + col) * RTK;
            typename Path::Out acc[kUnits];
#pragma unroll
            for (int q = 0; q < kUnits; ++q) {
                constexpr uint32_t CB = Path::kColBytes;
                acc[q] = Path::rows16(stage_addr + off_ldsm[q] + CB * sb0, stage + off_g[q] + CB * sb0,
                                      stage + off_g8[q] + CB * sb0, lane, st0, my_scratch);
                if (SPW == 2 && has1) {
                    const typename Path::Out a1 =
                        Path::rows16(stage_addr + off_ldsm[q] + CB * sb1, stage + off_g[q] + CB * sb1,
                                     stage + off_g8[q] + CB * sb1, lane, st1, my_scratch);
                    Path::accumulate(acc[q], a1);
                }
            }
#pragma unroll
            for (int q = 0; q < kUnits; ++q) {
                if constexpr (TK == 1) {
                    float2 v = acc[q];
                    v.x += __shfl_xor_sync(0xffffffffu, v.x, 1);
                    v.y += __shfl_xor_sync(0xffffffffu, v.y, 1);
                    v.x += __shfl_xor_sync(0xffffffffu, v.x, 2);
                    v.y += __shfl_xor_sync(0xffffffffu, v.y, 2);
                    if (t == 0) {
                        pw[row_g[q]] = v.x;
                        pw[row_g8[q]] = v.y;
                    }
                } else {
                    // lane (g,t) owns rows g, g+8 x input rows 2t, 2t+1 (complete sums)
                    const float4 v = acc[q];
                    *reinterpret_cast<float2 *>(pw + row_g[q] * TK + 2 * t) = make_float2(v.x, v.y);
                    *reinterpret_cast<float2 *>(pw + row_g8[q] * TK + 2 * t) = make_float2(v.z, v.w);
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[s]);
                mbar_arrive(&pfull[b]);
            }
            if (++s == p.stages) s = 0, ring_phase ^= 1u;
        }
    }
    if (CS > 1) {
        pdl_wait();          // y may still be read by the previous kernel
        cluster_sync_all();  // every CTA's row sums are complete and visible to the cluster
        const int local_tiles = first_tile < p.num_tiles ? (p.num_tiles - 1 - first_tile) / tile_step + 1 : 0;
        const uint32_t base = smem_u32(rowsum);
        // The reducer warps of the cluster finish the rows (one warp per CTA
        // stores, so only it has output stores to fence on a sharded call).
        for (int i = warp == C + 1 ? int(crank) * 32 + lane : local_tiles * RTK; i < local_tiles * RTK;
             i += CS * 32) {
            const int li = i / RTK, rem = i - li * RTK, r = rem / TK, u = rem % TK;
            const int row = (first_tile + li * tile_step) * RT + r;
            if (row < p.rows && (TK == 1 || u < p.ntok)) {
                float a = 0.0f;
                for (int k = 0; k < CS; ++k) a += ld_cluster_f32(mapa_shared(base + 4u * uint32_t(i), uint32_t(k)));
                store_y(p, row, a, u);
            }
        }
        cluster_sync_all();  // no CTA leaves while a peer may still read its row sums
    }
    if (p.peer.nranks > 0) {
        if (warp == C + 1) __threadfence_system();  // the output stores of the reducer warp, before the ticket
        __syncthreads();
        if (threadIdx.x == 0) peer_handshake(p);
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

// Launch shape of one GEMV: cluster size (K split), row-tile height and the
// shared-memory budget of one CTA.
struct Shape {
    int cluster;
    int rt;
    int budget_kb;
    int path;  // 0: FP16 MMA, 1: INT8 MMA
    int wps;   // compute warps per superblock column (1, or 2 on the INT8 path with 32-row tiles)
    int max_groups;  // 0: one CTA (cluster) per SM; else at most this many
};

// Optional override for tuning sweeps:
// SI_Q4K_GEMV_PLAN="cluster,rows_per_tile,budget_kb[,path[,warps_per_column[,max_groups]]]"
// (for example "2,16,100" or "1,32,226,1,2"); ignored when it does not fit.
bool shape_override(Shape &s) {
    static Shape o{0, 0, 0, 0, 1, 0};
    static bool parsed = false;
    if (!parsed) {
        parsed = true;
        if (const char *e = std::getenv("SI_Q4K_GEMV_PLAN")) {
            Shape t{0, 0, 0, 0, 1, 0};
            if (std::sscanf(e, "%d,%d,%d,%d,%d,%d", &t.cluster, &t.rt, &t.budget_kb, &t.path, &t.wps, &t.max_groups) >=
                3)
                o = t;
        }
    }
    if (o.cluster <= 0) return false;
    s = o;
    return true;
}

// Largest ring budget: the 227 KB a CTA may hold, less 1 KB of headroom.
// The bytes in flight per SM set the bandwidth (Little's law): with one
// stage held by the compute warps, a 4 x 55.8 KB ring (K = 3072, 32-row
// tiles) keeps ~167 KB in flight where 3 stages kept ~111 KB.
constexpr int kMaxBudgetKb = 226;

// Default launch shape: one CTA per SM with the whole shared memory as
// ring and 32-row tiles. K is split over a cluster only when a CTA would
// otherwise give each compute warp two superblocks (K > 4096): the one-
// superblock warps keep the x fragments in registers without spilling.
// (Measured on the Phi-4-mini shapes: splitting K = 3072 halves the compute
// warps per SM and loses; K = 8192 split in two gains about 10%.)
Shape default_shape(int64_t rows, int nsb, int sms, int path) {
    (void)rows;
    (void)sms;
    int cs = 1;
    if (nsb > kMaxComputeWarps) {
        cs = 0;
        for (int c = 2; c <= 8 && !cs; ++c)
            if (nsb % c == 0 && nsb / c <= kMaxComputeWarps) cs = c;
        if (!cs) cs = 1;  // two superblocks per warp
    }
    return {cs, 32, kMaxBudgetKb, path, 1, 0};
}

// path: 0 FP16 / 1 INT8 (Q4_K), 2 Q8_0. col_bytes: bytes of 256 elements;
// scratch_bytes: per compute warp scratch of the path.
// group_cap > 0 limits the clusters (CTAs) of the grid to what can be
// resident at once.
bool plan_mma(int64_t rows, int64_t cols, const void *w, int sms, int path, uint32_t col_bytes,
              uint32_t scratch_bytes, int group_cap, MmaParams &p, size_t &smem, int &rt, int tokens = 1) {
    if (cols % 256 != 0 || rows <= 0 || rows > (int64_t(1) << 30)) return false;
    if (reinterpret_cast<uintptr_t>(w) & 15u) return false;
    const int nsb = int(cols / 256);
    Shape sh = default_shape(rows, nsb, sms, path);
    Shape o;
    if (shape_override(o) && o.cluster >= 1 && o.cluster <= 8 && (o.rt == 16 || o.rt == 32) &&
        o.budget_kb >= 32 && o.budget_kb <= kMaxBudgetKb && (o.wps == 1 || o.wps == 2)) {
        const int opath = path >= 2 ? path : o.path;
        if (opath == path || (path < 2 && (opath == 0 || opath == 1))) {
            sh = o;
            sh.path = opath;
        }
    }
    if (nsb % sh.cluster != 0) sh.cluster = 1;
    const size_t budget = size_t(sh.budget_kb) * 1024;
    for (;;) {
        const int nsb_cta = nsb / sh.cluster;
        if (nsb_cta > 2 * kMaxComputeWarps) return false;
        p.nsb = nsb;
        p.cluster = sh.cluster;
        p.nsb_cta = nsb_cta;
        p.spw = nsb_cta > kMaxComputeWarps ? 2 : 1;
        const int columns = (nsb_cta + p.spw - 1) / p.spw;
        rt = sh.rt;
        p.row_bytes = col_bytes * uint32_t(nsb);
        p.cta_bytes = col_bytes * uint32_t(nsb_cta);
        // Row stride / 16 odd: ldmatrix's 8 row addresses hit 8 distinct bank quads.
        p.row_stride = p.cta_bytes + ((nsb_cta % 2 == 0) ? 16u : 32u);
        // Fall back to 16-row tiles when 32-row tiles leave fewer than 3 stages.
        if (rt == 32 && size_t(32) * p.row_stride * 3 > budget) rt = 16;
        p.wps = (sh.wps == 2 && sh.path == 1 && p.spw == 1 && rt == 32 && 2 * columns <= kMaxWps2Warps) ? 2 : 1;
        const size_t scratch = size_t(columns) * p.wps * scratch_bytes;
        p.compute_warps = columns * p.wps;
        if (p.cluster == 1) {
            // Whole rows are contiguous: copy groups of rows. A row is
            // 144 * nsb bytes = 16 * (9 nsb) with 9 nsb = nsb (mod 8), so
            // consecutive rows repeat their bank class every P rows; 8 / P
            // groups based 16 bytes apart give the 8 classes one ldmatrix needs.
            const int r8 = nsb_cta % 8;
            p.class_period = (r8 & 1) ? 8 : (r8 == 4 ? 2 : (r8 == 0 ? 1 : 4));
            p.group_rows = rt * p.class_period / 8;
            p.log2_class_period = p.class_period == 8 ? 3 : (p.class_period == 4 ? 2 : (p.class_period == 2 ? 1 : 0));
            p.log2_group_rows = rt == 32 ? p.log2_class_period + 2 : p.log2_class_period + 1;
            p.row_pitch = p.cta_bytes;
            p.group_stride = uint32_t(p.group_rows) * p.cta_bytes + 16u;
            p.copy_groups = 1;
            p.stage_bytes = uint32_t((uint64_t(8 / p.class_period) * p.group_stride + 127) / 128 * 128);
        } else {
            // K slices of a row are not contiguous across rows: one copy per row.
            p.class_period = 8;
            p.group_rows = rt;
            p.log2_class_period = 3;
            p.log2_group_rows = rt == 32 ? 5 : 4;
            p.row_pitch = p.row_stride;
            p.group_stride = uint32_t(rt) * p.row_stride;
            p.copy_groups = 0;
            p.stage_bytes = uint32_t((uint64_t(rt) * p.row_stride + 127) / 128 * 128);
        }
        p.num_tiles = int((rows + rt - 1) / rt);
        // One CTA per SM at most: a cluster of CS CTAs takes CS SMs.
        p.groups = std::max(1, std::min(p.num_tiles, sms / p.cluster));
        if (sh.max_groups > 0) p.groups = std::min(p.groups, sh.max_groups);
        if (group_cap > 0) p.groups = std::min(p.groups, group_cap);
        p.max_local_tiles = (p.num_tiles + p.groups - 1) / p.groups;
        const size_t rowsum = p.cluster > 1 ? size_t(p.max_local_tiles) * rt * tokens * sizeof(float) : 0;
        // The K split is for small matrices: the row sums it keeps must stay small.
        if (rowsum > 48 * 1024) {
            sh.cluster = 1;
            continue;
        }
        const size_t tail =
            size_t(2) * columns * rt * tokens * sizeof(float) + rowsum + (scratch ? scratch + 16 : 0);
        const size_t bars = size_t(2 * 8 + 4) * sizeof(uint64_t);
        if (budget < tail + bars + 2 * size_t(p.stage_bytes)) {
            if (sh.cluster == 1) return false;
            sh.cluster = 1;
            continue;
        }
        p.stages = std::min(int((budget - tail - bars) / p.stage_bytes), 8);
        p.rows = int(rows);
        p.path = sh.path;
        smem = size_t(p.stages) * p.stage_bytes + size_t(2 * p.stages + 4) * sizeof(uint64_t) + tail;
        return true;
    }
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {
using namespace si::dev;

// Returns SI_ERR_UNSUPPORTED (without touching the error string) when the
// shape needs the SIMT kernel instead.
// Clusters of `cluster` CTAs of `kernel` that fit on the device at once
// (GPC boundaries leave SMs unusable for some cluster sizes); cached.
int max_active_clusters(void (*kernel)(MmaParams), int cluster, int threads, size_t smem) {
    struct Entry {
        int device;
        void (*kernel)(MmaParams);
        int cluster, threads;
        size_t smem;
        int value;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> g(mu);
        for (const Entry &e : cache)
            if (e.device == dev && e.kernel == kernel && e.cluster == cluster && e.threads == threads && e.smem == smem)
                return e.value;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(cluster));
    cfg.blockDim = dim3(unsigned(threads));
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr{};
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
    cache.push_back({dev, kernel, cluster, threads, smem, n});
    return n;
}

namespace {

// One launch of the tensor-core GEMV skeleton. path: 1 Q4_K INT8 (or FP16
// by override), 2 Q8_0, 3 Q4_K batched (up to 8 input rows).
si_status launch_mma(int path, const void *w, const float *x, float *y, int64_t rows, int64_t cols, void *stream,
                     const PeerGather *peer, const int32_t *control, int token, int ntok, int64_t x_stride,
                     int64_t y_stride, const XForm *xf = nullptr) {
    if (xf && xf->mode) {
        // The transforms read 16-byte vectors of x, the residual and the norm weight.
        auto misaligned = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) != 0; };
        if (path == 3 || (xf->mode != 1 && xf->mode != 2) || misaligned(x) ||
            (xf->mode == 1 && (!xf->norm_weight || misaligned(xf->norm_weight) ||
                               (xf->residual && misaligned(xf->residual)) || (xf->updated && misaligned(xf->updated)))))
            return SI_ERR_UNSUPPORTED;
    }
    MmaParams p{};
    size_t smem = 0;
    int rt = 0;
    const int sms = num_sms();
    using Kernel = void (*)(MmaParams);
#define SI_GEMV_KERNELS(P)                                                                  \
    {{{gemv_mma_q4k_kernel<P, 1, 16, 1, 12>, gemv_mma_q4k_kernel<P, 1, 32, 1, 12>},        \
      {gemv_mma_q4k_kernel<P, 1, 16, 1, 16>, gemv_mma_q4k_kernel<P, 1, 32, 1, 16>}},       \
     {{gemv_mma_q4k_kernel<P, 2, 16, 1, 16>, gemv_mma_q4k_kernel<P, 2, 32, 1, 16>},        \
      {gemv_mma_q4k_kernel<P, 2, 16, 1, 16>, gemv_mma_q4k_kernel<P, 2, 32, 1, 16>}}}
    static const Kernel kernels[3][2][2][2] = {SI_GEMV_KERNELS(F16Path), SI_GEMV_KERNELS(I8Path),
                                               SI_GEMV_KERNELS(Q8Path)};
#undef SI_GEMV_KERNELS
    // batched: one superblock per warp only ([max warps 12 / 16][rows per tile 16 / 32])
    static const Kernel kernels_t8[2][2] = {
        {gemv_mma_q4k_kernel<I8T8Path, 1, 16, 1, 12>, gemv_mma_q4k_kernel<I8T8Path, 1, 32, 1, 12>},
        {gemv_mma_q4k_kernel<I8T8Path, 1, 16, 1, 16>, gemv_mma_q4k_kernel<I8T8Path, 1, 32, 1, 16>}};
    static const Kernel kernel_wps2 = gemv_mma_q4k_kernel<I8Path, 1, 32, 2, kMaxWps2Warps>;
    static std::once_flag attr_once;
    std::call_once(attr_once, [] {
        for (auto &a : kernels)
            for (auto &b : a)
                for (auto &c : b)
                    for (Kernel k : c) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        for (auto &a : kernels_t8)
            for (Kernel k : a) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        cudaFuncSetAttribute(kernel_wps2, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    });
    const bool q8 = path == 2, batched = path == 3;
    const uint32_t col_bytes = q8 ? Q8Path::kColBytes : I8Path::kColBytes;
    // Plan; with a K split, shrink the grid to the clusters that can be
    // resident together (one wave) and plan again.
    Kernel kernel = nullptr;
    int cap = 0;
    for (int attempt = 0; attempt < 4; ++attempt) {
        if (!plan_mma(rows, cols, w, sms, path, col_bytes, q8 ? Q8Path::kScratchBytes : 0u, cap, p, smem, rt,
                      batched ? I8T8Path::kTokens : 1))
            return SI_ERR_UNSUPPORTED;
        if (batched) {
            if (p.spw != 1 || p.wps != 1) return SI_ERR_UNSUPPORTED;
            kernel = kernels_t8[p.compute_warps > 12 ? 1 : 0][rt == 32 ? 1 : 0];
        } else {
            kernel = p.wps == 2 ? kernel_wps2
                                : kernels[p.path][p.spw - 1][p.compute_warps > 12 ? 1 : 0][rt == 32 ? 1 : 0];
        }
        if (p.cluster == 1) break;
        const int fit = max_active_clusters(kernel, p.cluster, (p.compute_warps + 2) * 32, smem);
        if (fit <= 0) return SI_ERR_UNSUPPORTED;
        if (p.groups <= fit) break;
        cap = fit;
    }
    p.w = static_cast<const uint8_t *>(w);
    p.x = x;
    p.y = y;
    if (peer) p.peer = *peer;
    p.control = control;
    p.token = token;
    p.ntok = ntok;
    p.x_stride = x_stride;
    p.y_stride = y_stride;
    if (xf && xf->mode) {
        p.x_mode = xf->mode;
        p.x_eps = xf->eps;
        p.x_res = xf->residual;
        p.x_norm_w = xf->norm_weight;
        p.x_updated = xf->updated;
    }
    if (xf && xf->prefetch && xf->prefetch_bytes >= 16 && !(reinterpret_cast<uintptr_t>(xf->prefetch) & 15u)) {
        p.prefetch = static_cast<const uint8_t *>(xf->prefetch);
        p.prefetch_bytes = xf->prefetch_bytes & ~uint64_t(15);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(p.groups * p.cluster));
    cfg.blockDim = dim3(unsigned((p.compute_warps + 2) * 32));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    // The weight stream starts before the dependency wait: weights are
    // read-only parameters, never produced by the preceding kernel.
    cudaLaunchAttribute attrs[2]{};
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = unsigned(p.cluster);
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = p.cluster > 1 ? 2 : 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, kernel, p);
    const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
    if (e != cudaSuccess)
        return fail(SI_ERR_CUDA, "tensor-core %s GEMV launch failed: %s", q8 ? "Q8_0" : "Q4_K", cudaGetErrorString(e));
    return SI_OK;
}

}  // namespace

// Tensor-core quantised GEMV (Q4_K or Q8_0). Returns SI_ERR_UNSUPPORTED
// (without touching the error string) when the shape needs the SIMT kernel.
si_status matvec_quant_mma(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                           void *stream, const PeerGather *peer, const int32_t *control, int token,
                           const XForm *xform) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0) return SI_ERR_UNSUPPORTED;
    return launch_mma(wtype == SI_TYPE_Q8_0 ? 2 : 1, w, x, y, rows, cols, stream, peer, control, token, 1, cols,
                      rows, xform);
}

// Q4_K batch: y[b] = W x[b] for the m input rows, eight per launch (each
// weight byte read once per eight rows). x rows 16-byte aligned.
si_status matvec_q4k_batched(const void *w, const float *x, float *y, int64_t m, int64_t rows, int64_t cols,
                             void *stream, const int32_t *control) {
    if ((reinterpret_cast<uintptr_t>(x) & 15u) || cols % 4 != 0 || m < 2) return SI_ERR_UNSUPPORTED;
    for (int64_t b0 = 0; b0 < m; b0 += I8T8Path::kTokens) {
        const int n = int(std::min<int64_t>(I8T8Path::kTokens, m - b0));
        const si_status st = launch_mma(3, w, x + b0 * cols, y + b0 * rows, rows, cols, stream, nullptr, control,
                                        int(b0), n, cols, rows);
        if (st != SI_OK) return st;  // the first launch decides (same shape for every group)
    }
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
