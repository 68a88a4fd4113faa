// core.matrix-multiply with transpose_right (Y[m,n] = sum_k X[m,k] W[n,k],
// CpuInstructionNumerics.cs:61-82) on the sm_100a tensor cores.
//
// Precision: the parity gate is relative L2 <= 1e-4 against FP32, which a
// single BF16 pass cannot meet (2^-9 operand rounding). Both operands are
// split into BF16 pairs, v = hi + lo with hi = bf16(v), lo = bf16(v - hi),
// and three products are accumulated in FP32 in tensor memory:
//   X W ~= Xhi Whi + Xlo Whi + Xhi Wlo       (dropped term ~2^-18 relative)
//
// Kernel structure (one CTA = 128 weight rows x 256 input rows, K in 64-wide
// stages, two-stage ring in shared memory):
//   warp 0      TMA: X_hi / X_lo tiles (2-D tensor maps, 128-byte swizzle,
//               no multicast) into the stage, completion as tx bytes
//   warp 1      allocates 256 TMEM columns; one thread issues
//               tcgen05.mma (M=128, N=256, K=16, BF16 -> FP32) x 3 products,
//               then tcgen05.commit frees the stage
//   warps 2..9  dequantise this stage's 128x64 weight block (GGUF Q8_0 /
//               Q4_K / F16 / F32) in registers, split hi/lo and store both in
//               the canonical K-major 128B-swizzled layout; after the last
//               stage they drain the accumulator (tcgen05.ld) to Y
// Every mbarrier wait is bounded; a wait that runs out sets the device error
// word and the kernel still runs to completion (no trap, no hang).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "device_common.cuh"
#include "gemm_core.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

constexpr int kBM = kGemmBM;                     // weight rows per CTA (MMA M)
constexpr int kBN = 256;                         // input rows per CTA (MMA N)
constexpr int kBK = kGemmBK;                     // K per stage (128 B of BF16)
constexpr int kStages = 2;
constexpr int kThreads = 64 + kProducers;       // 10 warps
constexpr uint32_t kATile = kBM * kBK * 2;       // 16 KB (one of hi / lo)
constexpr uint32_t kBTile = kBN * kBK * 2;       // 32 KB
constexpr uint32_t kStageBytes = 2 * kATile + 2 * kBTile;  // 96 KB
constexpr uint32_t kTmemCols = 256;

constexpr uint32_t kIdesc = mma_idesc(kBN);

struct GemmParams {
    const uint8_t *w;
    float *y;            // splits == 1: Y; otherwise the partial sums [splits][m][n]
    uint64_t row_bytes;
    int m, n, k;
    int splits;          // K split over gridDim.z CTAs
};

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                        const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);  // 1024-byte aligned tiles
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *accum = empty + kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kBM, t0 = blockIdx.y * kBN;
    // K stages [it0, it0 + iters) of this CTA's split
    const int total_iters = p.k / kBK;
    const int it0 = int(int64_t(total_iters) * blockIdx.z / p.splits);
    const int iters = int(int64_t(total_iters) * (blockIdx.z + 1) / p.splits) - it0;
    float *const y = p.y + size_t(blockIdx.z) * size_t(p.m) * size_t(p.n);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kProducers + 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            for (int it = 0; it < iters; ++it) {
                const int s = it % kStages;
                if (it >= kStages) mbar_wait(&empty[s], ((it / kStages) - 1) & 1, kErrEmptyBarrierTimeout);
                uint8_t *st = smem + s * kStageBytes;
                mbar_arrive_expect_tx(&full[s], 2 * kBTile);
                tma_load_2d(st + 2 * kATile, &map_hi, (it0 + it) * kBK, t0, &full[s]);
                tma_load_2d(st + 2 * kATile + kBTile, &map_lo, (it0 + it) * kBK, t0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int it = 0; it < iters; ++it) {
                const int s = it % kStages;
                mbar_wait(&full[s], (it / kStages) & 1, kErrFullBarrierTimeout);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t base = smem_u32(smem + s * kStageBytes);
                const uint32_t a_hi = base, a_lo = base + kATile, b_hi = base + 2 * kATile,
                               b_lo = base + 2 * kATile + kBTile;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint32_t off = kk * 32;  // 16 BF16 along K within the 128-byte row
                    mma_bf16(tmem, smem_desc(a_hi + off), smem_desc(b_hi + off), kIdesc, (it | kk) != 0);
                    mma_bf16(tmem, smem_desc(a_hi + off), smem_desc(b_lo + off), kIdesc, 1);
                    mma_bf16(tmem, smem_desc(a_lo + off), smem_desc(b_hi + off), kIdesc, 1);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(accum);
        }
        __syncwarp();
    } else {
        // warps 2..9: weight producers, then epilogue.
        // Two threads per weight row, each fetching and decoding 32 of the
        // stage's 64 columns (the dequantisation is the per-stage bound).
        const int pt = threadIdx.x - 64, r = pt >> 1, h = pt & 1;  // row 0..127, half 0..1
        const bool valid_row = n0 + r < p.n;
        const uint8_t *wrow = p.w + size_t(n0 + r) * p.row_bytes;
        produce_weights<FMT>(wrow, valid_row, it0, iters, h, [&](int it, const float(&w)[32]) {
            const int s = it % kStages;
            if (it >= kStages) mbar_wait(&empty[s], ((it / kStages) - 1) & 1, kErrEmptyBarrierTimeout);
            uint8_t *st = smem + s * kStageBytes;
            store_split_half(w, r, h, st, st + kATile);
            fence_proxy_async();
            mbar_arrive(&full[s]);
        });
        // Epilogue: TMEM lane quarter (warp % 4) holds weight rows 32*(warp%4) ..;
        // warps 2..5 drain the first half of the columns, warps 6..9 the second.
        mbar_wait(accum, 0, kErrMmaBarrierTimeout);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int quarter = warp & 3;
        const int row = n0 + quarter * 32 + lane;
        const int c_begin = warp >= 6 ? kBN / 2 : 0;
#pragma unroll 1
        for (int c0 = c_begin; c0 < c_begin + kBN / 2; c0 += 32) {
            uint32_t v[32];
            tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(c0), v);
            if (row < p.n) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int t = t0 + c0 + j;
                    if (t < p.m) y[size_t(t) * p.n + row] = __uint_as_float(v[j]);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// X (fp32, [m,k]) -> X_hi, X_lo (bf16, [m,k]) with hi = bf16(x), lo = bf16(x - hi).
__global__ void split_bf16_kernel(const float4 *__restrict__ x, uint2 *__restrict__ hi, uint2 *__restrict__ lo,
                                  int64_t n4) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
        const float4 v = x[i];
        const uint32_t h01 = pack_bf16(v.x, v.y), h23 = pack_bf16(v.z, v.w);
        const uint32_t l01 = pack_bf16(v.x - __uint_as_float(h01 << 16), v.y - __uint_as_float(h01 & 0xffff0000u));
        const uint32_t l23 = pack_bf16(v.z - __uint_as_float(h23 << 16), v.w - __uint_as_float(h23 & 0xffff0000u));
        hi[i] = make_uint2(h01, h23);
        lo[i] = make_uint2(l01, l23);
    }
}

// Y = sum of the K-split partial sums, in split order (deterministic).
// vec: count % 4 == 0 and y 16-byte aligned (float4 accesses), else scalar.
__global__ void reduce_splits_kernel(const float *__restrict__ part, float *__restrict__ y, int64_t count, int splits,
                                     bool vec) {
    const int64_t n4 = vec ? count / 4 : 0;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
        float4 acc = reinterpret_cast<const float4 *>(part)[i];
        for (int s = 1; s < splits; ++s) {
            const float4 v = reinterpret_cast<const float4 *>(part + size_t(s) * count)[i];
            acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
        }
        reinterpret_cast<float4 *>(y)[i] = acc;
    }
    for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += int64_t(gridDim.x) * blockDim.x) {
        float acc = part[i];
        for (int s = 1; s < splits; ++s) acc += part[size_t(s) * count + i];
        y[i] = acc;
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

si_status make_x_map(CUtensorMap *map, void *base, int m, int k) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(m)};
    const cuuint64_t strides[1] = {cuuint64_t(k) * 2};
    const cuuint32_t box[2] = {kBK, kBN};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SI_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return SI_OK;
}

constexpr size_t kGemmSmem = size_t(kStages) * kStageBytes + 1024 + 256;

bool tensor_core_shape(uint32_t wtype, int64_t m, int64_t n, int64_t k) {
    if (m < 64 || k % kBK != 0 || k > (int64_t(1) << 30) || m > (int64_t(1) << 30) || n > (int64_t(1) << 30))
        return false;
    return wtype == SI_TYPE_Q4_K || wtype == SI_TYPE_Q8_0 || wtype == SI_TYPE_F16 || wtype == SI_TYPE_F32;
}

uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

// K splits for an m x n output: one CTA per SM at most per wave (the
// two-stage ring takes 193 KB of shared memory), so pick the split that
// minimises waves x (stages per CTA + a fixed cost of about four stages
// for the TMEM drain and pipeline fill), keeping at least two stages per CTA.
int gemm_splits(int64_t m, int64_t n, int64_t k) {
    const int sms = device_sm_count();
    const int64_t tiles = ((n + kBM - 1) / kBM) * ((m + kBN - 1) / kBN);
    const int64_t iters = k / kBK;
    int best = 1;
    double best_cost = 1e30;
    for (int s = 1; s <= 16 && iters / s >= 2; ++s) {
        const int64_t waves = (tiles * s + sms - 1) / sms;
        const double cost = double(waves) * (double(iters) / s + 4.0);
        if (cost < best_cost - 1e-9) best_cost = cost, best = s;
    }
    return best;
}

template <int FMT>
si_status launch_gemm(const void *w, float *y, uint64_t rb, int m, int n, int k, int splits, const CUtensorMap &hi,
                      const CUtensorMap &lo, cudaStream_t st) {
    if (const int ae = opt_in_smem(reinterpret_cast<const void *>(gemm_tcgen05_kernel<FMT>), int(kGemmSmem)))
        return fail(SI_ERR_CUDA, "tcgen05 GEMM shared-memory opt-in failed: %s",
                    cudaGetErrorString(cudaError_t(ae)));
    GemmParams p{static_cast<const uint8_t *>(w), y, rb, m, n, k, splits};
    const dim3 grid(unsigned((n + kBM - 1) / kBM), unsigned((m + kBN - 1) / kBN), unsigned(splits));
    gemm_tcgen05_kernel<FMT><<<grid, kThreads, kGemmSmem, st>>>(hi, lo, p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "tcgen05 GEMM launch failed: %s", cudaGetErrorString(e));
    return SI_OK;
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {
using namespace si::dev;

si_status gemm_workspace_bytes(uint32_t wtype, int64_t m, int64_t n, int64_t k, uint64_t *bytes) {
    *bytes = 0;
    if (!tensor_core_shape(wtype, m, n, k)) return SI_OK;
    const int splits = gemm_splits(m, n, k);
    *bytes = 2 * align256(uint64_t(m) * uint64_t(k) * 2) +
             (splits > 1 ? align256(uint64_t(splits) * uint64_t(m) * uint64_t(n) * 4) : 0);
    return SI_OK;
}

si_status gemm_tn(uint32_t wtype, const float *x, const void *w, float *y, int64_t m, int64_t n, int64_t k,
                  void *workspace, uint64_t workspace_bytes, void *stream) {
    auto st = static_cast<cudaStream_t>(stream);
    uint64_t need = 0;
    gemm_workspace_bytes(wtype, m, n, k, &need);
    if (!need || reinterpret_cast<uintptr_t>(w) % 16 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0)
        return shared_weight_matvec(wtype, w, x, nullptr, y, m, n, k, stream);
    uint64_t rb;
    if (si_status s = byte_length(wtype, uint64_t(k), &rb)) return s;
    if (rb % 16 != 0 && wtype != SI_TYPE_Q8_0) return shared_weight_matvec(wtype, w, x, nullptr, y, m, n, k, stream);
    if (wtype == SI_TYPE_Q8_0 && rb % 4 != 0) return shared_weight_matvec(wtype, w, x, nullptr, y, m, n, k, stream);
    if (workspace_bytes < need) return fail(SI_ERR_INVALID_ARGUMENT, "workspace too small");
    auto *hi = static_cast<uint8_t *>(workspace);
    auto *lo = hi + align256(uint64_t(m) * uint64_t(k) * 2);
    const int64_t n4 = m * k / 4;
    const int blocks = int(std::min<int64_t>((n4 + 255) / 256, 148 * 16));
    split_bf16_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4 *>(x), reinterpret_cast<uint2 *>(hi),
                                              reinterpret_cast<uint2 *>(lo), n4);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "split launch failed: %s", cudaGetErrorString(e));
    CUtensorMap map_hi, map_lo;
    if (si_status s = make_x_map(&map_hi, hi, int(m), int(k))) return s;
    if (si_status s = make_x_map(&map_lo, lo, int(m), int(k))) return s;
    const int splits = gemm_splits(m, n, k);
    float *out = splits > 1 ? reinterpret_cast<float *>(lo + align256(uint64_t(m) * uint64_t(k) * 2)) : y;
    si_status ls;
    switch (wtype) {
    case SI_TYPE_Q4_K: ls = launch_gemm<SI_TYPE_Q4_K>(w, out, rb, int(m), int(n), int(k), splits, map_hi, map_lo, st); break;
    case SI_TYPE_Q8_0: ls = launch_gemm<SI_TYPE_Q8_0>(w, out, rb, int(m), int(n), int(k), splits, map_hi, map_lo, st); break;
    case SI_TYPE_F16: ls = launch_gemm<SI_TYPE_F16>(w, out, rb, int(m), int(n), int(k), splits, map_hi, map_lo, st); break;
    default: ls = launch_gemm<SI_TYPE_F32>(w, out, rb, int(m), int(n), int(k), splits, map_hi, map_lo, st); break;
    }
    if (ls != SI_OK || splits == 1) return ls;
    const int64_t count = m * n;
    const int rblocks = int(std::min<int64_t>((count / 4 + 255) / 256 + 1, 148 * 8));
    const bool vec = count % 4 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
    reduce_splits_kernel<<<rblocks, 256, 0, st>>>(out, y, count, splits, vec);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "split reduction launch failed: %s", cudaGetErrorString(e));
    return SI_OK;
}

si_status take_error_gemm(int device, uint32_t *code) {
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
