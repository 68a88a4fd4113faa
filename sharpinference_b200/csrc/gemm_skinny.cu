// Few-row GEMM on the tensor cores: Y[m, n] = X[m, k] W[n, k]^T for a
// handful of input rows (transformer.batch-shared-matvec at the reference's
// 16 rows and config 5's 32 streams, GpuBatchTransformerInstructions.cs:
// 224-279; a prefill chunk's tail). Same arithmetic as the prefill GEMM
// (gemm.cu): X and the dequantised weights are split into BF16 hi/lo pairs
// and Xhi Whi + Xlo Whi + Xhi Wlo accumulate in FP32 in tensor memory.
//
// What differs from the prefill GEMM, for m of 2..64 rows per tile:
//   * The MMA is M = 128 weight rows x N = BN input rows (16, 32 or 64), so
//     the tensor work follows the rows that exist, and the kernel is bound
//     by the weight stream rather than by the MMA.
//   * No workspace: the TMA lands each stage's FP32 X tile in shared
//     memory a few stages ahead (a 2-D tensor map over X, no multicast) and
//     the weight producers split it into hi/lo in the swizzled layout the
//     MMA reads, a few 8-column units each.
//   * K is split over the CTAs of a thread-block cluster (z), so a narrow
//     weight matrix still spreads over the SMs; the partial accumulators
//     are summed through distributed shared memory by the cluster's first
//     CTA in rank order (deterministic), no partial sums in global memory.
//   * Rows t >= control[1] are not written (the batch-shared instruction's
//     validCount, read on the device).
//   * Programmatic dependent launch: the weight producers start streaming
//     before the dependency wait; only the X loads and the stores wait.
// Every mbarrier wait is bounded (device error word, no trap, no hang).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "device_common.cuh"
#include "gemm_core.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

constexpr int kSkThreads = 64 + kProducers;  // 10 warps

// Stage = weight hi / lo tiles (128 x 64 BF16 each), X hi / lo tiles
// (BN x 64 BF16 each) and the FP32 X tile the TMA lands (BN x 64, row-major,
// converted by warp 0 into the X hi / lo tiles).
// TMAW: Q4_K / Q8_0 weights arrive by TMA, 128 rows x 256 columns of raw
// GGUF bytes per transfer ("super-stage": four K stages), into a ring of
// their own; the producers decode them from shared memory.
template <int BN, int FMT, bool TMAW>
struct SkinnyCfg {
    static constexpr uint32_t kSS = FMT == SI_TYPE_Q4_K ? 144 : 272;  // bytes of 256 columns of one row
    static constexpr int kRawStages = TMAW ? (FMT == SI_TYPE_Q4_K ? 3 : 2) : 0;
    static constexpr uint32_t kRawBytes = kGemmBM * kSS;
    static constexpr int kStages = TMAW ? (BN >= 64 ? 2 : 3) : (BN >= 64 ? 3 : 4);
    static constexpr uint32_t kATile = kGemmBM * kGemmBK * 2;  // 16 KB (one of hi / lo)
    static constexpr uint32_t kBTile = BN * kGemmBK * 2;       // BN rows of 128 B
    static constexpr uint32_t kXTile = BN * kGemmBK * 4;       // FP32 X as loaded
    static constexpr uint32_t kStageBytes = 2 * kATile + 2 * kBTile + kXTile;
    static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
    static constexpr uint32_t kIdesc = mma_idesc(BN);
    static constexpr int kRedStride = BN + 1;  // padded row of the split-K exchange buffer
    static constexpr size_t kSmem = size_t(kStages) * kStageBytes + size_t(kRawStages) * kRawBytes + 1024 + 256;
    static_assert(size_t(kGemmBM) * kRedStride * 4 <= size_t(kStages) * kStageBytes, "exchange buffer");
    static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct SkinnyParams {
    const uint8_t *w;
    const float *x;
    float *y;
    const int32_t *control;  // null: every row; else rows t < control[1]
    uint64_t row_bytes;
    int m, n, k;
    int splits;  // K split over the cluster (gridDim.z == cluster size)
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

template <int FMT, int BN, bool TMAW>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                       const SkinnyParams p) {
    using Cfg = SkinnyCfg<BN, FMT, TMAW>;
    constexpr int kSkStages = Cfg::kStages;
    constexpr int kRaw = Cfg::kRawStages > 0 ? Cfg::kRawStages : 1;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);  // 1024-byte aligned tiles
    uint8_t *wraw = smem + kSkStages * Cfg::kStageBytes;                 // raw weight super-stages
    uint64_t *full = reinterpret_cast<uint64_t *>(wraw + Cfg::kRawStages * Cfg::kRawBytes);
    uint64_t *empty = full + kSkStages;
    uint64_t *xfull = empty + kSkStages;   // the FP32 X tile of the stage has landed
    uint64_t *xempty = xfull + kSkStages;  // the producers have converted it: the staging can refill
    uint64_t *wfull = xempty + kSkStages;  // a raw weight super-stage has landed
    uint64_t *wempty = wfull + kRaw;       // every producer has decoded its rows of it
    uint64_t *accum = wempty + kRaw;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kGemmBM, t0 = blockIdx.y * BN;
    int it0, iters;
    if constexpr (TMAW) {  // splits on super-stage boundaries
        const int total_ss = p.k / 256;
        const int ss0 = int(int64_t(total_ss) * blockIdx.z / p.splits);
        it0 = 4 * ss0;
        iters = 4 * (int(int64_t(total_ss) * (blockIdx.z + 1) / p.splits) - ss0);
    } else {
        const int total_iters = p.k / kGemmBK;
        it0 = int(int64_t(total_iters) * blockIdx.z / p.splits);
        iters = int(int64_t(total_iters) * (blockIdx.z + 1) / p.splits) - it0;
    }

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSkStages; ++s) {
            mbar_init(&full[s], kProducers);  // weight producers (they also convert X)
            mbar_init(&empty[s], 1);
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], kProducers);
        }
        for (int s = 0; s < kRaw; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], kProducers);
        }
        mbar_init(accum, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(Cfg::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    float acc[BN < 32 ? 32 : BN];  // epilogue warps: this thread's weight row, BN input rows
    if (warp == 0) {
        // X: the TMA brings each stage's FP32 tile (rows past m read as
        // zeros) into the stage's staging area as soon as the producers have
        // converted the tile it held, so it runs up to kSkStages stages
        // ahead of them, independently of the MMA.
        if (lane == 0) {
            pdl_wait();  // X may come from the previous kernel; the weights never do
            for (int q = 0; q < iters; ++q) {
                const int sq = q % kSkStages;
                if (q >= kSkStages) mbar_wait(&xempty[sq], ((q / kSkStages) - 1) & 1, kErrEmptyBarrierTimeout);
                uint8_t *xs = smem + sq * Cfg::kStageBytes + 2 * Cfg::kATile + 2 * Cfg::kBTile;
                mbar_arrive_expect_tx(&xfull[sq], Cfg::kXTile);
                tma_load_2d(xs, &xmap, (it0 + q) * kGemmBK, t0, &xfull[sq]);
            }
        }
        if constexpr (TMAW) {
            // Weights: read-only, so no dependency wait is needed for them;
            // one super-stage (128 rows x 256 columns) per transfer, rows
            // past n read as zeros. Coordinates in 16-bit units.
            if (lane == 1) {
                for (int q = 0; q < iters / 4; ++q) {
                    const int sq = q % kRaw;
                    if (q >= kRaw) mbar_wait(&wempty[sq], ((q / kRaw) - 1) & 1, kErrEmptyBarrierTimeout);
                    mbar_arrive_expect_tx(&wfull[sq], Cfg::kRawBytes);
                    tma_load_2d(wraw + sq * Cfg::kRawBytes, &wmap, (it0 / 4 + q) * int(Cfg::kSS / 2), n0, &wfull[sq]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            for (int it = 0; it < iters; ++it) {
                const int s = it % kSkStages;
                mbar_wait(&full[s], (it / kSkStages) & 1, kErrFullBarrierTimeout);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t base = smem_u32(smem + s * Cfg::kStageBytes);
                const uint32_t a_hi = base, a_lo = base + Cfg::kATile, b_hi = base + 2 * Cfg::kATile,
                               b_lo = b_hi + Cfg::kBTile;
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk) {
                    const uint32_t off = kk * 32;  // 16 BF16 along K within the 128-byte row
                    mma_bf16(tmem, smem_desc(a_hi + off), smem_desc(b_hi + off), Cfg::kIdesc, (it | kk) != 0);
                    mma_bf16(tmem, smem_desc(a_hi + off), smem_desc(b_lo + off), Cfg::kIdesc, 1);
                    mma_bf16(tmem, smem_desc(a_lo + off), smem_desc(b_hi + off), Cfg::kIdesc, 1);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(accum);
        }
        __syncwarp();
    } else {
        // warps 2..9: weight producers (no dependency wait: weights are
        // read-only), then the accumulator drain.
        // Two threads per weight row, each fetching and decoding 32 of the
        // stage's 64 columns (the dequantisation is the per-stage bound).
        const int pt = threadIdx.x - 64, r = pt >> 1, h = pt & 1;  // row 0..127, half 0..1
        const bool valid_row = n0 + r < p.n;
        const uint8_t *wrow = p.w + size_t(n0 + r) * p.row_bytes;
        auto emit = [&](int it, const float(&w)[32]) {
            const int s = it % kSkStages;
            if (it >= kSkStages) mbar_wait(&empty[s], ((it / kSkStages) - 1) & 1, kErrEmptyBarrierTimeout);
            uint8_t *st = smem + s * Cfg::kStageBytes;
            store_split_half(w, r, h, st, st + Cfg::kATile);
            // this thread's share of the stage's X tile: units of 8 columns
            // of one row, FP32 staging -> BF16 hi / lo, swizzled
            mbar_wait(&xfull[s], (it / kSkStages) & 1, kErrFullBarrierTimeout);
            uint8_t *hi_tile = st + 2 * Cfg::kATile;
            uint8_t *lo_tile = hi_tile + Cfg::kBTile;
            const float *xs = reinterpret_cast<const float *>(hi_tile + 2 * Cfg::kBTile);
#pragma unroll
            for (int u = pt; u < BN * 8; u += kProducers) {
                const int xr = u >> 3, c = u & 7;
                const float4 a = *reinterpret_cast<const float4 *>(xs + xr * kGemmBK + 8 * c);
                const float4 b = *reinterpret_cast<const float4 *>(xs + xr * kGemmBK + 8 * c + 4);
                const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                uint32_t hv[4], lv[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t hb = pack_bf16(v[2 * q], v[2 * q + 1]);
                    hv[q] = hb;
                    lv[q] = pack_bf16(v[2 * q] - __uint_as_float(hb << 16),
                                      v[2 * q + 1] - __uint_as_float(hb & 0xffff0000u));
                }
                const int pc = c ^ (xr & 7);
                *reinterpret_cast<uint4 *>(hi_tile + (xr >> 3) * 1024 + (xr & 7) * 128 + pc * 16) =
                    make_uint4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<uint4 *>(lo_tile + (xr >> 3) * 1024 + (xr & 7) * 128 + pc * 16) =
                    make_uint4(lv[0], lv[1], lv[2], lv[3]);
            }
            fence_proxy_async();  // generic reads of the staging before the next TMA write to it
            mbar_arrive(&xempty[s]);
            mbar_arrive(&full[s]);
        };
        if constexpr (TMAW) {
            for (int it = 0; it < iters; ++it) {
                const int sub = it & 3, q = it >> 2, rs = q % kRaw;
                if (sub == 0) mbar_wait(&wfull[rs], (q / kRaw) & 1, kErrFullBarrierTimeout);
                RawHalf<FMT> rh;
                fetch_weights32_smem<FMT>(wraw + rs * Cfg::kRawBytes + r * Cfg::kSS, sub, h, rh);
                float w[32];
                decode_weights32<FMT>(rh, h, w);
                if (sub == 3) {
                    fence_proxy_async();  // reads of the super-stage before the TMA refills it
                    mbar_arrive(&wempty[rs]);
                }
                emit(it, w);
            }
        } else {
            produce_weights<FMT>(wrow, valid_row, it0, iters, h, emit);
        }
        // TMEM lane quarter (warp % 4) holds weight rows 32 * (warp % 4) ..;
        // warps 2..5 drain it.
        if (warp < 6) {
            mbar_wait(accum, 0, kErrMmaBarrierTimeout);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int quarter = warp & 3;
#pragma unroll
            for (int c0 = 0; c0 < (BN < 32 ? 32 : BN); c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(c0), v);
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[c0 + j] = __uint_as_float(v[j]);
            }
        }
    }

    // Split-K: every CTA but the cluster's first leaves its partial sums in
    // its shared memory (the stage ring is idle: the accumulator barrier
    // completed after the last MMA read it); the first adds them in rank order.
    const bool drain = warp >= 2 && warp < 6;
    const int row_local = (warp & 3) * 32 + lane;
    float *red = reinterpret_cast<float *>(smem);
    const uint32_t crank = p.splits > 1 ? cluster_rank() : 0;
    if (p.splits > 1) {
        if (drain && crank != 0) {
#pragma unroll
            for (int j = 0; j < BN; ++j) red[row_local * Cfg::kRedStride + j] = acc[j];
        }
        cluster_barrier();
        if (drain && crank == 0) {
            for (int q = 1; q < p.splits; ++q) {
                const uint32_t peer = map_to_rank(smem_u32(red + row_local * Cfg::kRedStride), uint32_t(q));
#pragma unroll
                for (int j = 0; j < BN; ++j) acc[j] += ld_cluster_f32(peer + 4u * uint32_t(j));
            }
        }
    }
    if (drain && crank == 0) {
        pdl_wait();  // the previous kernel may still read Y
        const int row = n0 + row_local;
        int valid = p.m;
        if (p.control) valid = min(valid, p.control[1]);
        if (row < p.n) {
#pragma unroll
            for (int j = 0; j < BN; ++j) {
                const int t = t0 + j;
                if (t < valid) p.y[size_t(t) * p.n + row] = acc[j];
            }
        }
    }
    if (p.splits > 1) cluster_barrier();  // peers keep their shared memory until the first CTA has read it
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols)
                     : "memory");
    }
}

int sm_count() { return device_sm_count(); }

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
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

// FP32 X [m, k] as a 2-D tensor map with a 64-column x BN-row box, no
// swizzle; rows past m read as zeros.
si_status make_x_map_f32(CUtensorMap *map, const float *x, int m, int k, int bn) {
    EncodeTiledFn fn = encoder();
    if (!fn) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(m)};
    const cuuint64_t strides[1] = {cuuint64_t(k) * 4};
    const cuuint32_t box[2] = {cuuint32_t(kGemmBK), cuuint32_t(bn)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(x), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled (X) failed (%d)", int(r));
    return SI_OK;
}

// Raw GGUF weight rows as a 2-D tensor map of 16-bit units: 256 columns
// (144 or 272 bytes) x 128 rows per box, rows past n read as zeros.
si_status make_w_map(CUtensorMap *map, const void *w, uint64_t row_bytes, int n, uint32_t ss_bytes) {
    EncodeTiledFn fn = encoder();
    if (!fn) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {cuuint64_t(row_bytes / 2), cuuint64_t(n)};
    const cuuint64_t strides[1] = {cuuint64_t(row_bytes)};
    const cuuint32_t box[2] = {cuuint32_t(ss_bytes / 2), cuuint32_t(kGemmBM)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(w), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled (W) failed (%d)", int(r));
    return SI_OK;
}

template <int FMT, int BN, bool TMAW>
si_status launch_skinny(const SkinnyParams &p0, cudaStream_t st) {
    using Cfg = SkinnyCfg<BN, FMT, TMAW>;
    auto kernel = gemm_skinny_kernel<FMT, BN, TMAW>;
    if (const int ae = opt_in_smem(reinterpret_cast<const void *>(kernel), int(Cfg::kSmem)))
        return fail(SI_ERR_CUDA, "few-row GEMM shared-memory opt-in failed: %s", cudaGetErrorString(cudaError_t(ae)));
    SkinnyParams p = p0;
    const int64_t tiles = ((p.n + kGemmBM - 1) / kGemmBM) * ((p.m + BN - 1) / BN);
    const int iters = p.k / kGemmBK;
    // K split over a cluster of 1, 2 or 4 CTAs: the fewest that come close
    // to one CTA per SM, keeping at least four stages per CTA.
    int splits = 1;
    while (splits < 4 && tiles * splits * 2 <= sm_count() && iters / (splits * 2) >= 4) splits *= 2;
    p.splits = splits;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned((p.n + kGemmBM - 1) / kGemmBM), unsigned((p.m + BN - 1) / BN), unsigned(splits));
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 1;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = unsigned(splits);
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    CUtensorMap xmap, wmap;
    if (si_status ms = make_x_map_f32(&xmap, p.x, p.m, p.k, BN)) return ms;
    if constexpr (TMAW) {
        if (si_status ms = make_w_map(&wmap, p.w, p.row_bytes, p.n, Cfg::kSS)) return ms;
    } else {
        wmap = xmap;  // unused
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, xmap, wmap, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(SI_ERR_CUDA, "tcgen05 few-row GEMM launch failed: %s", cudaGetErrorString(e));
    }
    return SI_OK;
}

template <int BN>
si_status dispatch_type(uint32_t wtype, const SkinnyParams &p, cudaStream_t st) {
    // TMA weight rows: 256-column super-stages, 16-byte aligned rows and base
    const bool tmaw = p.k % 256 == 0 && p.row_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(p.w) % 16 == 0;
    switch (wtype) {
    case SI_TYPE_Q4_K:
        return tmaw ? launch_skinny<SI_TYPE_Q4_K, BN, true>(p, st) : launch_skinny<SI_TYPE_Q4_K, BN, false>(p, st);
    case SI_TYPE_Q8_0:
        return tmaw ? launch_skinny<SI_TYPE_Q8_0, BN, true>(p, st) : launch_skinny<SI_TYPE_Q8_0, BN, false>(p, st);
    case SI_TYPE_F16: return launch_skinny<SI_TYPE_F16, BN, false>(p, st);
    default: return launch_skinny<SI_TYPE_F32, BN, false>(p, st);
    }
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {
using namespace si::dev;

bool gemm_skinny_supported(uint32_t wtype, const void *w, const float *x, int64_t m, int64_t n, int64_t k) {
    if (wtype != SI_TYPE_Q4_K && wtype != SI_TYPE_Q8_0 && wtype != SI_TYPE_F16 && wtype != SI_TYPE_F32) return false;
    if (m < 1 || n < 1 || k % kGemmBK != 0 || k > (int64_t(1) << 30) || n > (int64_t(1) << 30) ||
        m > (int64_t(1) << 24))
        return false;
    if (wtype == SI_TYPE_Q4_K && k % 256 != 0) return false;
    // 16-byte weight and input loads
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) return false;
    uint64_t rb = 0;
    if (byte_length(wtype, uint64_t(k), &rb) != SI_OK) return false;
    const uintptr_t wa = reinterpret_cast<uintptr_t>(w);
    if (wtype == SI_TYPE_Q8_0) return wa % 4 == 0 && rb % 4 == 0;
    return wa % 16 == 0 && rb % 16 == 0;
}

si_status gemm_skinny(uint32_t wtype, const void *w, const float *x, const int32_t *control, float *y, int64_t m,
                      int64_t n, int64_t k, void *stream) {
    if (!gemm_skinny_supported(wtype, w, x, m, n, k))
        return fail(SI_ERR_UNSUPPORTED, "few-row GEMM: unsupported type, shape or alignment");
    uint64_t rb = 0;
    byte_length(wtype, uint64_t(k), &rb);
    SkinnyParams p{static_cast<const uint8_t *>(w), x, y, control, rb, int(m), int(n), int(k), 1};
    auto st = static_cast<cudaStream_t>(stream);
    if (m <= 16) return dispatch_type<16>(wtype, p, st);
    if (m <= 32) return dispatch_type<32>(wtype, p, st);
    return dispatch_type<64>(wtype, p, st);
}

si_status take_error_gemm_skinny(int device, uint32_t *code) {
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
