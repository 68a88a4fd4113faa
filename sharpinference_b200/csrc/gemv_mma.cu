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
#include "gemv_core.cuh"
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
    // Fused neighbours of the decode program (kernels::GemvFusion):
    int in_mode;          // 0: x as is; 1: rms-norm of x (x * norm_w, rows * 1/rms); 2: swiglu of [gate | up]
    const float *norm_w;  // in_mode 1: the norm weight (K floats)
    float eps;            // in_mode 1
    const float *resid;   // non-null: y[r] = resid[r] + (W x)[r] (resid may equal y)
    // in_mode 3: x + the partial vectors of a K-split exchange, rms-normed
    const float *parts;   // nparts vectors of K floats, part_stride apart
    int nparts;
    int64_t part_stride;
    float *h_out;         // non-null: CTA 0 stores x + the partials (the residual stream) here
    // consumer of a publish-only exchange (see consumer_wait)
    const unsigned long long *wait_counts;
    const uint32_t *wait_epoch;
    int wait_ranks;
    int64_t wait_rows;
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
// `res`: resid[row] when p.resid is set, loaded ahead by the caller.
__device__ __forceinline__ void store_y(const MmaParams &p, int row, float v, int tok = 0, float res = 0.0f) {
    if (p.control && p.token + tok >= p.control[1]) return;  // read after the dependency wait
    if (p.peer.nranks == 0) {
        if (p.resid) v = __fadd_rn(res, v);  // residual add of the decode program (batch 1)
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

// End of a publish-only exchange GEMV (tensor-parallel partial sums): no
// wait for the peers here. The storing warp fenced its rows at system scope
// before the CTA barrier; this thread fences once more (cumulative over them)
// and adds the CTA's stored rows to its slot of every rank's count of this
// kind; the launch's last CTA (ticket) advances this rank's epoch of the
// kind, which the consumer GEMV on this rank reads after the dependency wait.
__device__ __forceinline__ void peer_publish(const MmaParams &p, uint32_t rows) {
    const kernels::PeerGather &g = p.peer;
    __threadfence_system();
    if (rows)
        for (int q = 0; q < g.nranks; ++q)
            asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(g.counts[q] + g.rank),
                         "l"(static_cast<unsigned long long>(rows))
                         : "memory");
    const uint32_t t = atomicAdd(g.ticket, 1u);
    if (t != gridDim.x - 1) return;
    *g.ticket = 0u;
    *reinterpret_cast<volatile uint32_t *>(g.kind_epoch) = *reinterpret_cast<volatile uint32_t *>(g.kind_epoch) + 1u;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long *addr) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// Consumer of a publish-only exchange: every warp that reads x / the parts
// waits (lane 0, bounded) until each rank's count of the exchange reached
// epoch * rows, i.e. every rank has stored and fenced all its rows.
__device__ __forceinline__ void consumer_wait(const MmaParams &p, int lane) {
    if (!p.wait_counts) return;
    if (lane == 0) {
        const unsigned long long target =
            static_cast<unsigned long long>(*reinterpret_cast<const volatile uint32_t *>(p.wait_epoch)) *
            static_cast<unsigned long long>(p.wait_rows);
        const uint64_t t0 = globaltimer_ns();
        for (int q = 0; q < p.wait_ranks; ++q) {
            uint32_t polls = 0;
            while (ld_acquire_sys_u64(p.wait_counts + q) < target) {
                if (++polls > kMaxPolls || globaltimer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(&g_error_word, kErrPeerTimeout);
                    break;
                }
                __nanosleep(32);
            }
        }
    }
    __syncwarp();
}

// 1 / rms of the input vector (transformer.rms-norm, GpuTransformerInstructionCollection.cs:323-368):
// sum of squares over all K elements by one warp (lane-strided partial sums,
// fixed shuffle tree), then 1 / sqrt(sum / K + eps). Called by the reducer
// warp after the dependency wait; the rows it stores are scaled by it.
// The loads of 8 strides are issued before any of them is used, so the warp
// pays one L2 round trip per 1024 elements instead of one per 128; the sums
// keep their element order.
constexpr int kRmsBatch = 8;
__device__ __forceinline__ float sq4(float s, float4 v) {
    return __fadd_rn(s, __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                                  __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w))));
}
__device__ __forceinline__ float inv_rms_warp(const float *x, int64_t k, float eps, int lane) {
    float s = 0.0f;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && k % 128 == 0) {
        for (int64_t i0 = int64_t(lane) * 4; i0 < k; i0 += 128 * kRmsBatch) {
            float4 v[kRmsBatch];
#pragma unroll
            for (int j = 0; j < kRmsBatch; ++j) {
                const int64_t i = i0 + 128 * j;
                v[j] = i < k ? __ldg(reinterpret_cast<const float4 *>(x + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < kRmsBatch; ++j)
                if (i0 + 128 * j < k) s = sq4(s, v[j]);
        }
    } else {
        for (int64_t i = lane; i < k; i += 32) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    return __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(s, float(k)), eps)));
}

// Mode 3: the residual stream after a K-split exchange, x + parts[0] + ...
// (rank order, as the compute warps form it), stored to h_out when given;
// returns 1 / rms of it with the reference's arithmetic.
__device__ __forceinline__ float inv_rms_parts_warp(const MmaParams &p, int64_t k, int lane, float *h_out) {
    float s = 0.0f;
    for (int64_t i0 = int64_t(lane) * 4; i0 < k; i0 += 128 * kRmsBatch) {
        float4 v[kRmsBatch];
#pragma unroll
        for (int j = 0; j < kRmsBatch; ++j) {
            const int64_t i = i0 + 128 * j;
            v[j] = i < k ? __ldg(reinterpret_cast<const float4 *>(p.x + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int r = 0; r < p.nparts; ++r) {
            float4 q[kRmsBatch];
#pragma unroll
            for (int j = 0; j < kRmsBatch; ++j) {
                const int64_t i = i0 + 128 * j;
                q[j] = i < k ? __ldg(reinterpret_cast<const float4 *>(p.parts + r * p.part_stride + i))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < kRmsBatch; ++j)
                v[j] = make_float4(__fadd_rn(v[j].x, q[j].x), __fadd_rn(v[j].y, q[j].y), __fadd_rn(v[j].z, q[j].z),
                                   __fadd_rn(v[j].w, q[j].w));
        }
#pragma unroll
        for (int j = 0; j < kRmsBatch; ++j) {
            const int64_t i = i0 + 128 * j;
            if (i < k) {
                if (h_out) *reinterpret_cast<float4 *>(h_out + i) = v[j];
                s = sq4(s, v[j]);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    return __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(s, float(k)), p.eps)));
}

// The same 1 / rms (mode 1: of x; mode 3: of x + parts[0] + ... in rank
// order, stored to h_out when given) formed by every thread of the CTA: the
// epilogue of a K-split launch, where all warps are free, so the loads go out
// in one batch instead of one warp's serial batches. Per thread the float4
// groups tid, tid + T, .. (T threads); warp trees, then the warp sums added
// in warp order by every thread (`red`: one float per warp of shared memory;
// the caller has synchronised the CTA before its first use).
__device__ float inv_rms_block(const MmaParams &p, int64_t k, float *red, float *h_out) {
    constexpr int kJ = 4;  // float4 groups per thread per pass
    const int nthr = int(blockDim.x), tid = int(threadIdx.x), lane = tid & 31, nw = nthr >> 5;
    float s = 0.0f;
    const bool vec = (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0 && k % 4 == 0 &&
                     (p.in_mode != 3 || p.nparts == 0 || ((reinterpret_cast<uintptr_t>(p.parts) & 15u) == 0 &&
                                                          p.part_stride % 4 == 0));
    if (vec) {
        for (int64_t i0 = int64_t(tid) * 4; i0 < k; i0 += int64_t(nthr) * 4 * kJ) {
            float4 v[kJ];
#pragma unroll
            for (int j = 0; j < kJ; ++j) {
                const int64_t i = i0 + int64_t(j) * nthr * 4;
                v[j] = i < k ? __ldg(reinterpret_cast<const float4 *>(p.x + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (p.in_mode == 3)
                for (int r = 0; r < p.nparts; ++r) {
                    float4 q[kJ];
#pragma unroll
                    for (int j = 0; j < kJ; ++j) {
                        const int64_t i = i0 + int64_t(j) * nthr * 4;
                        q[j] = i < k ? __ldg(reinterpret_cast<const float4 *>(p.parts + r * p.part_stride + i))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int j = 0; j < kJ; ++j)
                        v[j] = make_float4(__fadd_rn(v[j].x, q[j].x), __fadd_rn(v[j].y, q[j].y),
                                           __fadd_rn(v[j].z, q[j].z), __fadd_rn(v[j].w, q[j].w));
                }
#pragma unroll
            for (int j = 0; j < kJ; ++j) {
                const int64_t i = i0 + int64_t(j) * nthr * 4;
                if (i < k) {
                    if (h_out) *reinterpret_cast<float4 *>(h_out + i) = v[j];
                    s = sq4(s, v[j]);
                }
            }
        }
    } else {
        for (int64_t i = tid; i < k; i += nthr) {
            float v = p.x[i];
            if (p.in_mode == 3)
                for (int r = 0; r < p.nparts; ++r) v = __fadd_rn(v, p.parts[r * p.part_stride + i]);
            if (h_out) h_out[i] = v;
            s = __fadd_rn(s, __fmul_rn(v, v));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    if (lane == 0) red[tid >> 5] = s;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < nw; ++w) t = __fadd_rn(t, red[w]);
    return __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, float(k)), p.eps)));
}

// Every thread of every CTA of the cluster (hardware barrier).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

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
    uint32_t peer_rows = 0;  // output rows this thread stored (publish-only exchange count)
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
            if (++s == p.stages) s = 0, ring_phase ^= 1u;
        }
    } else if (warp == C + 1) {
        // Reducer: fixed-order sum of the C0 per-column partials of each
        // output (row r, input row u) = index r * TK + u of the tile.
        if (CS == 1) {
            pdl_wait();  // y may still be read by the previous kernel
            consumer_wait(p, lane);
        }
        const float row_scale =
            CS != 1 ? 1.0f
            : p.in_mode == 1 ? inv_rms_warp(p.x, int64_t(p.nsb) * 256, p.eps, lane)
            : p.in_mode == 3 ? inv_rms_parts_warp(p, int64_t(p.nsb) * 256, lane, blockIdx.x == 0 ? p.h_out : nullptr)
                             : 1.0f;
        int it = 0;
        for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
            const int b = it & 1;
            const int r0 = tile * RT;
            const int nrows = min(RT, p.rows - r0);
            // the residual of this lane's row, loaded while the tile is computed
            const float res = (CS == 1 && TK == 1 && p.resid && lane < nrows) ? p.resid[r0 + lane] : 0.0f;
            mbar_wait(&pfull[b], (it >> 1) & 1, kErrEpilogueTimeout);
            const float *pb = part + size_t(b) * C0 * RTK;
#pragma unroll
            for (int o0 = 0; o0 < RTK; o0 += 32) {
                const int o = o0 + lane, r = o / TK, u = o % TK;
                if (o >= RTK) break;  // RT * TK = 16: lanes 16..31 have no output
                float a = 0.0f;
                if (r < nrows)
                    for (int c = 0; c < C0; ++c) a += pb[c * RTK + o];
                if (CS == 1) {
                    if (r < nrows && (TK == 1 || u < p.ntok)) {
                        store_y(p, r0 + r, __fmul_rn(a, row_scale), u, res);
                        ++peer_rows;
                    }
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
        consumer_wait(p, lane);
        uint8_t *my_scratch = scratch + size_t(warp) * Path::kScratchBytes;
        auto load_x = [&](const auto &X) {
            Path::load(X, gsb + sb0, lane, st0, my_scratch, p.x_stride, p.ntok);
            if constexpr (SPW == 2) {
                if (has1) Path::load(X, gsb + sb1, lane, st1, my_scratch, p.x_stride, p.ntok);
            }
        };
        if (p.in_mode == 1)
            load_x(XSrc<1>{p.x, nullptr, p.norm_w, 1.0f, 0});
        else if (p.in_mode == 3)
            load_x(XSrc<3>{p.x, p.parts, p.norm_w, 1.0f, p.part_stride, p.nparts});
        else if (p.in_mode == 2)
            load_x(XSrc<2>{p.x, nullptr, nullptr, 1.0f, int64_t(p.nsb) * 256});
        else
            load_x(XSrc<0>{p.x, nullptr, nullptr, 1.0f, int64_t(p.nsb) * 256});

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
        if (warp == C + 1) consumer_wait(p, lane);
        float row_scale = 1.0f;
        if (p.in_mode == 1 || p.in_mode == 3) {
            __syncthreads();  // every warp is past its tile loop (the partial buffers are free) and the wait
            row_scale = inv_rms_block(p, int64_t(p.nsb) * 256, part,
                                      p.in_mode == 3 && blockIdx.x == 0 ? p.h_out : nullptr);
        }
        const int local_tiles = first_tile < p.num_tiles ? (p.num_tiles - 1 - first_tile) / tile_step + 1 : 0;
        // residuals of this lane's first rows, loaded before the cluster barrier
        constexpr int kResAhead = 4;
        float res_ahead[kResAhead];
#pragma unroll
        for (int j = 0; j < kResAhead; ++j) {
            res_ahead[j] = 0.0f;
            const int i = int(crank) * 32 + lane + j * CS * 32;
            if (warp == C + 1 && TK == 1 && p.resid && i < local_tiles * RTK) {
                const int li = i / RTK, r = i - li * RTK;
                const int row = (first_tile + li * tile_step) * RT + r;
                if (row < p.rows) res_ahead[j] = p.resid[row];
            }
        }
        cluster_sync_all();  // every CTA's row sums are complete and visible to the cluster
        const uint32_t base = smem_u32(rowsum);
        // The reducer warps of the cluster finish the rows (one warp per CTA
        // stores, so only it has output stores to fence on a sharded call).
        int j = 0;
        for (int i = warp == C + 1 ? int(crank) * 32 + lane : local_tiles * RTK; i < local_tiles * RTK;
             i += CS * 32, ++j) {
            const int li = i / RTK, rem = i - li * RTK, r = rem / TK, u = rem % TK;
            const int row = (first_tile + li * tile_step) * RT + r;
            if (row < p.rows && (TK == 1 || u < p.ntok)) {
                float a = 0.0f;
                for (int k = 0; k < CS; ++k) a += ld_cluster_f32(mapa_shared(base + 4u * uint32_t(i), uint32_t(k)));
                float res = 0.0f;
                if (p.resid) {
                    if (j < kResAhead) {
#pragma unroll
                        for (int q = 0; q < kResAhead; ++q)
                            if (q == j) res = res_ahead[q];
                    } else {
                        res = p.resid[row];
                    }
                }
                store_y(p, row, __fmul_rn(a, row_scale), u, res);
                ++peer_rows;
            }
        }
        cluster_sync_all();  // no CTA leaves while a peer may still read its row sums
    }
    if (p.peer.nranks > 0 && p.peer.nowait) {
        // only the reducer warp stores output rows: it fences them, counts them and publishes
        if (warp == C + 1) {
            __threadfence_system();
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) peer_rows += __shfl_xor_sync(0xffffffffu, peer_rows, off);
            if (lane == 0) peer_publish(p, peer_rows);
        }
    } else if (p.peer.nranks > 0) {
        if (warp == C + 1) __threadfence_system();  // the output stores of the reducer warp, before the ticket
        __syncthreads();
        if (threadIdx.x == 0) peer_handshake(p);
    }
}

int num_sms() { return device_sm_count(); }

// Launch shape of one GEMV: cluster size (K split), row-tile height, the
// shared-memory budget of one CTA, superblocks per compute warp and CTAs
// per SM (si_gemv_plan carries the same fields across the C ABI).
struct Shape {
    int cluster;
    int rt;
    int budget_kb;
    int path;        // 0: FP16 MMA, 1: INT8 MMA
    int wps;         // compute warps per superblock column (1, or 2 on the INT8 path with 32-row tiles)
    int max_groups;  // 0: ctas_per_sm CTAs (clusters of CTAs) per SM; else at most this many
    int spw;         // 0: one superblock per warp while that fits, else 2; or forced 1 / 2
    int per_sm;      // CTAs resident per SM the grid is sized for (1 or 2)
};

// Largest ring budget: the 227 KB a CTA may hold, less 1 KB of headroom.
// The bytes in flight per SM set the bandwidth (Little's law): with one
// stage held by the compute warps, a 4 x 55.8 KB ring (K = 3072, 32-row
// tiles) keeps ~167 KB in flight where 3 stages kept ~111 KB.
constexpr int kMaxBudgetKb = 226;
// Two CTAs per SM: each holds at most half of the SM's 228 KB (less the
// 1 KB the hardware reserves per CTA).
constexpr int kHalfBudgetKb = 112;

// Default launch shape: one CTA per SM with the whole shared memory as
// ring and 32-row tiles. K is split over a cluster only when a CTA would
// otherwise give each compute warp two superblocks (K > 4096): the one-
// superblock warps keep the x fragments in registers without spilling.
// (Measured on the Phi-4-mini shapes: splitting K = 3072 halves the compute
// warps per SM and loses; K = 8192 split in two gains about 10%.)
// Tiles are 32 rows unless the busiest CTA would stream at least 8% fewer
// rows with 16-row tiles, which happens when there are several tiles per CTA
// and 32-row tiles leave a ragged last round (gate_up: 512 tiles of 32 on 148
// CTAs = 4 rounds, 1024 tiles of 16 = 7 rounds, 112 rows instead of 128;
// measured 7.4 us instead of 8.5 us). With one or two tiles per CTA the fixed
// cost of a tile outweighs the balance, and 32-row tiles stay.
Shape default_shape(int64_t rows, int nsb, int sms, int path) {
    int cs = 1;
    if (nsb > kMaxComputeWarps) {
        cs = 0;
        for (int c = 2; c <= 8 && !cs; ++c)
            if (nsb % c == 0 && nsb / c <= kMaxComputeWarps) cs = c;
        if (!cs) cs = 1;  // two superblocks per warp
    }
    int rt = 32;
    const int64_t groups = std::max(1, sms / cs);
    const int64_t tiles32 = (rows + 31) / 32, tiles16 = (rows + 15) / 16;
    if (tiles32 > 2 * groups) {
        const int64_t busiest32 = (tiles32 + groups - 1) / groups * 32;
        const int64_t busiest16 = (tiles16 + groups - 1) / groups * 16;
        if (busiest16 * 100 <= busiest32 * 92) rt = 16;
    }
    return {cs, rt, kMaxBudgetKb, path, 1, 0, 0, 1};
}

Shape shape_from_plan(const si_gemv_plan &g) {
    return {g.cluster, g.rows_per_tile, g.smem_kb, g.mma_path, g.warps_per_column, g.max_groups,
            g.superblocks_per_warp, g.ctas_per_sm};
}

// path: 0 FP16 / 1 INT8 (Q4_K), 2 Q8_0. col_bytes: bytes of 256 elements;
// scratch_bytes: per compute warp scratch of the path.
// group_cap > 0 limits the clusters (CTAs) of the grid to what can be
// resident at once.
// `forced`: an explicit launch shape (si_matvec_quant_planned), else the default.
bool plan_mma(int64_t rows, int64_t cols, const void *w, int sms, int path, uint32_t col_bytes,
              uint32_t scratch_bytes, int group_cap, MmaParams &p, size_t &smem, int &rt, int tokens,
              const Shape *forced) {
    if (cols % 256 != 0 || rows <= 0 || rows > (int64_t(1) << 30)) return false;
    if (reinterpret_cast<uintptr_t>(w) & 15u) return false;
    const int nsb = int(cols / 256);
    Shape sh = forced ? *forced : default_shape(rows, nsb, sms, path);
    if (path >= 2) sh.path = path;  // Q8_0 and the batched path have one MMA path each
    if (nsb % sh.cluster != 0) sh.cluster = 1;
    const size_t budget = size_t(sh.budget_kb) * 1024;
    for (;;) {
        const int nsb_cta = nsb / sh.cluster;
        if (nsb_cta > 2 * kMaxComputeWarps) return false;
        p.nsb = nsb;
        p.cluster = sh.cluster;
        p.nsb_cta = nsb_cta;
        p.spw = (nsb_cta > kMaxComputeWarps || (sh.spw == 2 && nsb_cta >= 2)) ? 2 : 1;
        if (sh.spw == 1 && p.spw == 2) return false;  // one superblock per warp cannot cover this K slice
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
        p.groups = std::max(1, std::min(p.num_tiles, sh.per_sm * sms / p.cluster));
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
// by an explicit shape), 2 Q8_0, 3 Q4_K batched (up to 8 input rows).
si_status launch_mma(int path, const void *w, const float *x, float *y, int64_t rows, int64_t cols, void *stream,
                     const PeerGather *peer, const int32_t *control, int token, int ntok, int64_t x_stride,
                     int64_t y_stride, const Shape *forced = nullptr, const GemvFusion *fusion = nullptr) {
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
    const bool q8 = path == 2, batched = path == 3;
    const uint32_t col_bytes = q8 ? Q8Path::kColBytes : I8Path::kColBytes;
    // Plan; with a K split, shrink the grid to the clusters that can be
    // resident together (one wave) and plan again.
    Kernel kernel = nullptr;
    int cap = 0;
    for (int attempt = 0; attempt < 4; ++attempt) {
        if (!plan_mma(rows, cols, w, sms, path, col_bytes, q8 ? Q8Path::kScratchBytes : 0u, cap, p, smem, rt,
                      batched ? I8T8Path::kTokens : 1, forced))
            return SI_ERR_UNSUPPORTED;
        if (batched) {
            if (p.spw != 1 || p.wps != 1) return SI_ERR_UNSUPPORTED;
            kernel = kernels_t8[p.compute_warps > 12 ? 1 : 0][rt == 32 ? 1 : 0];
        } else {
            kernel = p.wps == 2 ? kernel_wps2
                                : kernels[p.path][p.spw - 1][p.compute_warps > 12 ? 1 : 0][rt == 32 ? 1 : 0];
        }
        // The occupancy query below and the launch both need the kernel's
        // shared-memory opt-in on this device.
        if (const int ae = opt_in_smem(reinterpret_cast<const void *>(kernel), 227 * 1024))
            return fail(SI_ERR_CUDA, "tensor-core GEMV shared-memory opt-in failed: %s",
                        cudaGetErrorString(cudaError_t(ae)));
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
    if (fusion) {
        p.in_mode = fusion->in_mode;
        p.norm_w = fusion->norm_w;
        p.eps = fusion->eps;
        p.resid = fusion->resid;
        p.parts = fusion->parts;
        p.nparts = fusion->nparts;
        p.part_stride = fusion->part_stride;
        p.h_out = fusion->h_out;
        p.wait_counts = fusion->wait_counts;
        p.wait_epoch = fusion->wait_epoch;
        p.wait_ranks = fusion->wait_ranks;
        p.wait_rows = fusion->wait_rows;
    }
    p.token = token;
    p.ntok = ntok;
    p.x_stride = x_stride;
    p.y_stride = y_stride;
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
                           void *stream, const PeerGather *peer, const int32_t *control, int token) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0) return SI_ERR_UNSUPPORTED;
    return launch_mma(wtype == SI_TYPE_Q8_0 ? 2 : 1, w, x, y, rows, cols, stream, peer, control, token, 1, cols,
                      rows);
}

// The decode program's GEMV with its neighbours fused (see GemvFusion).
// SI_ERR_UNSUPPORTED (nothing launched, no error string) when the tensor-core
// GEMV does not take the shape; the caller then runs the instructions apart.
si_status matvec_quant_fused(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                             const GemvFusion &f, void *stream, const PeerGather *peer) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0) return SI_ERR_UNSUPPORTED;
    const auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if ((f.in_mode != 0 && !a16(x)) || ((f.in_mode == 1 || f.in_mode == 3) && (!f.norm_w || !a16(f.norm_w))) ||
        (f.in_mode == 3 && ((f.nparts > 0 && (!f.parts || !a16(f.parts) || f.part_stride % 4)) ||
                            (f.h_out && !a16(f.h_out)))) ||
        (peer && f.resid))
        return SI_ERR_UNSUPPORTED;
    return launch_mma(wtype == SI_TYPE_Q8_0 ? 2 : 1, w, x, y, rows, cols, stream, peer, nullptr, 0, 1, cols, rows,
                      nullptr, &f);
}

// The launch shape si_matvec picks for a Q4_K / Q8_0 GEMV on the current device.
si_status gemv_default_plan(uint32_t wtype, int64_t rows, int64_t cols, si_gemv_plan *plan) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0) return SI_ERR_UNSUPPORTED;
    if (cols % 256 != 0 || rows <= 0) return SI_ERR_UNSUPPORTED;
    const Shape sh = default_shape(rows, int(cols / 256), num_sms(), wtype == SI_TYPE_Q8_0 ? 2 : 1);
    *plan = si_gemv_plan{sh.cluster, sh.rt, sh.budget_kb, sh.path == 0 ? 0 : 1, sh.wps, sh.spw, sh.per_sm,
                         sh.max_groups};
    return SI_OK;
}

// One GEMV with an explicit launch shape. SI_ERR_INVALID_ARGUMENT for a
// shape outside the documented ranges; SI_ERR_UNSUPPORTED when the shape
// cannot cover this matrix (nothing launched).
si_status matvec_quant_planned(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                               const si_gemv_plan &g, void *stream) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0) return fail(SI_ERR_UNSUPPORTED, "planned GEMV: Q8_0 or Q4_K");
    if (g.cluster < 1 || g.cluster > 8 || (g.rows_per_tile != 16 && g.rows_per_tile != 32) || g.smem_kb < 32 ||
        g.smem_kb > kMaxBudgetKb || (g.mma_path != 0 && g.mma_path != 1) ||
        (g.warps_per_column != 1 && g.warps_per_column != 2) || g.superblocks_per_warp < 0 ||
        g.superblocks_per_warp > 2 || (g.ctas_per_sm != 1 && g.ctas_per_sm != 2) || g.max_groups < 0 ||
        (g.ctas_per_sm == 2 && g.smem_kb > kHalfBudgetKb))
        return fail(SI_ERR_INVALID_ARGUMENT,
                    "GEMV plan out of range (cluster 1..8, rows_per_tile 16/32, smem_kb 32..%d and <= %d at two "
                    "CTAs per SM, mma_path 0/1, warps_per_column 1/2, superblocks_per_warp 0..2, ctas_per_sm 1/2)",
                    kMaxBudgetKb, kHalfBudgetKb);
    const Shape sh = shape_from_plan(g);
    const si_status st = launch_mma(wtype == SI_TYPE_Q8_0 ? 2 : 1, w, x, y, rows, cols, stream, nullptr, nullptr, 0,
                                    1, cols, rows, &sh);
    if (st == SI_ERR_UNSUPPORTED) return fail(SI_ERR_UNSUPPORTED, "GEMV plan does not fit this matrix");
    return st;
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
