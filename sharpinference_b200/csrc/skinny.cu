// Weight-shared multi-row mat-vec on sm_100a (SIMT FP32 path):
//  * transformer.batch-shared-matvec (GpuBatchTransformerInstructions.cs:224-275)
//    out[b,o] = sum_i W[o,i] in[b,i] for b < control[1], other rows untouched;
//  * core.matrix-multiply with transpose_right (CpuInstructionNumerics.cs:61-82)
//    when the tensor-core path does not apply.
// Each CTA owns 32 weight rows x 32 input rows. Per 256-column chunk the CTA
// stages the 32 input rows in shared memory (padded rows: conflict-free
// column reads) and each warp dequantises its 4 weight rows into a
// [k][4] layout, so one 128-bit broadcast load feeds four FMAs. Every weight
// block is read once per 32 input rows instead of once per (row, output).
#include <cuda_runtime.h>

#include <algorithm>

#include "device_common.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

constexpr int kChunk = 256;
constexpr int kRowsPerWarp = 4;
constexpr int kWarps = 8;
constexpr int kRowsPerCta = kRowsPerWarp * kWarps;  // 32 weight rows
constexpr int kTokens = 32;                         // input rows per CTA
constexpr int kXStride = kChunk + 1;

__device__ __forceinline__ float h2f(const uint8_t *p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

// Eight consecutive dequantised weights of one row, columns c .. c+7
// (c a multiple of 8); columns >= cols read as 0.
template <int FMT>
__device__ __forceinline__ void dequant8(const uint8_t *row, int64_t c, int64_t cols, float (&v)[8]) {
    if constexpr (FMT == SI_TYPE_F32) {
        const float *r = reinterpret_cast<const float *>(row);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = c + i < cols ? r[c + i] : 0.0f;
    } else if constexpr (FMT == SI_TYPE_F16) {
        const __half *r = reinterpret_cast<const __half *>(row);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = c + i < cols ? __half2float(r[c + i]) : 0.0f;
    } else if constexpr (FMT == SI_TYPE_Q6_K) {
        // eight elements of one 16-element group: same nibble / 2-bit fields
        const uint8_t *blk = row + (c >> 8) * 210;
        const int e0 = int(c & 255), h = e0 >> 7, j = (e0 >> 5) & 3, l0 = e0 & 31;
        const float a = h2f(blk + 208) * float(int8_t(blk[192 + (e0 >> 4)]));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int low = (blk[64 * h + l0 + i + 32 * (j & 1)] >> (4 * (j >> 1))) & 15;
            const int high = (blk[128 + 32 * h + l0 + i] >> (2 * j)) & 3;
            v[i] = a * float((low | (high << 4)) - 32);
        }
    } else if constexpr (FMT == SI_TYPE_Q8_0) {
        const uint8_t *blk = row + (c >> 5) * 34;
        const float d = h2f(blk);
        const int i0 = int(c & 31);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = d * float(int8_t(blk[2 + i0 + i]));
    } else {
        const uint8_t *blk = row + (c >> 8) * 144;
        const int e0 = int(c & 255), s = e0 >> 5, j = s >> 1, hi = s & 1, l0 = e0 & 31;
        const uint8_t *sc12 = blk + 4;
        int sc, m;
        if (s < 4) {
            sc = sc12[s] & 63;
            m = sc12[s + 4] & 63;
        } else {
            sc = (sc12[s + 4] & 0x0f) | ((sc12[s - 4] >> 6) << 4);
            m = (sc12[s + 4] >> 4) | ((sc12[s] >> 6) << 4);
        }
        const float a = h2f(blk) * float(sc), b = h2f(blk + 2) * float(m);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint8_t byte = blk[16 + 32 * j + l0 + i];
            v[i] = a * float(hi ? (byte >> 4) : (byte & 15)) - b;
        }
    }
}

template <int FMT>
__global__ void __launch_bounds__(256) shared_weight_kernel(const uint8_t *__restrict__ w, uint64_t row_bytes,
                                                            const float *__restrict__ x, float *__restrict__ y,
                                                            const int32_t *__restrict__ control, int64_t m,
                                                            int64_t n, int64_t k) {
    extern __shared__ __align__(16) float smem_f[];
    float *xs = smem_f;                                       // [kTokens][kXStride]
    float4 *ws = reinterpret_cast<float4 *>(xs + kTokens * kXStride + 3);  // [kWarps][kChunk]
    ws = reinterpret_cast<float4 *>((reinterpret_cast<uintptr_t>(ws) + 15) & ~uintptr_t(15));

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t n0 = int64_t(blockIdx.x) * kRowsPerCta + warp * kRowsPerWarp;
    const int64_t t0 = int64_t(blockIdx.y) * kTokens;
    int64_t valid = m;
    if (control) {
        const int64_t c = control[1] < 0 ? 0 : int64_t(control[1]);
        valid = c < m ? c : m;
    }
    if (t0 >= valid) return;
    const int64_t token = t0 + lane;

    float acc[kRowsPerWarp] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int64_t c0 = 0; c0 < k; c0 += kChunk) {
        // Stage input rows t0..t0+31, columns c0..c0+255.
        for (int idx = threadIdx.x; idx < kTokens * kChunk; idx += blockDim.x) {
            const int t = idx / kChunk, cc = idx % kChunk;
            const int64_t gt = t0 + t, gc = c0 + cc;
            xs[t * kXStride + cc] = (gt < valid && gc < k) ? x[gt * k + gc] : 0.0f;
        }
        // Dequantise this warp's 4 rows: lane takes columns 8*lane .. +7.
        float4 *wsw = ws + warp * kChunk;
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
            float v[8];
            const int64_t row = n0 + r;
            if (row < n && c0 + 8 * lane < k) {
                dequant8<FMT>(w + row * row_bytes, c0 + 8 * lane, k, v);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) reinterpret_cast<float *>(&wsw[8 * lane + i])[r] = v[i];
        }
        __syncthreads();
        const float *xr = xs + lane * kXStride;
        const int len = int(k - c0 < kChunk ? k - c0 : kChunk);
#pragma unroll 8
        for (int cc = 0; cc < len; ++cc) {
            const float4 wv = wsw[cc];
            const float xv = xr[cc];
            acc[0] = fmaf(wv.x, xv, acc[0]);
            acc[1] = fmaf(wv.y, xv, acc[1]);
            acc[2] = fmaf(wv.z, xv, acc[2]);
            acc[3] = fmaf(wv.w, xv, acc[3]);
        }
        __syncthreads();
    }
    if (token < valid) {
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r)
            if (n0 + r < n) y[token * n + n0 + r] = acc[r];
    }
}

size_t shared_weight_smem() { return (kTokens * kXStride + 3) * sizeof(float) + 16 + kWarps * kChunk * sizeof(float4); }

template <int FMT>
si_status launch_shared(const void *w, const float *x, float *y, const int32_t *control, int64_t m, int64_t n,
                        int64_t k, cudaStream_t st) {
    uint64_t rb;
    if (si_status s = byte_length(FMT, uint64_t(k), &rb)) return s;
    if (const int ae = opt_in_smem(reinterpret_cast<const void *>(shared_weight_kernel<FMT>), int(shared_weight_smem())))
        return fail(SI_ERR_CUDA, "shared-weight mat-vec shared-memory opt-in failed: %s",
                    cudaGetErrorString(cudaError_t(ae)));
    const dim3 grid(unsigned((n + kRowsPerCta - 1) / kRowsPerCta), unsigned((m + kTokens - 1) / kTokens));
    if (grid.y > 65535u) return fail(SI_ERR_INVALID_ARGUMENT, "too many input rows (%lld)", (long long)m);
    shared_weight_kernel<FMT><<<grid, 256, shared_weight_smem(), st>>>(static_cast<const uint8_t *>(w), rb, x, y,
                                                                        control, m, n, k);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "shared-weight mat-vec launch failed: %s", cudaGetErrorString(e));
    return SI_OK;
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {
using namespace si::dev;

si_status shared_weight_matvec(uint32_t wtype, const void *w, const float *x, const int32_t *control, float *y,
                               int64_t m, int64_t n, int64_t k, void *stream) {
    auto st = static_cast<cudaStream_t>(stream);
    // 2..32 rows of Q4_K / Q8_0: the few-row GEMM with the dequantised
    // weights in tensor memory (no split of W; weights read once per call).
    if (m >= 2 && gemm_fewrow_supported(wtype, w, x, m, n, k))
        return gemm_fewrow(wtype, w, x, control, y, m, n, k, stream);
    // Otherwise two or more rows: the few-row tcgen05 GEMM (weights read once
    // per 16, 32 or 64 rows, no workspace) -- except Q4_K up to 16 rows, where
    // the batched integer GEMV below measured faster (lm_head 3072 -> 200064
    // at 16 rows: 255 vs 434 us; at 32 rows the GEMM wins, 468 vs 506 us).
    const bool q4k_small = wtype == SI_TYPE_Q4_K && m <= 16;
    if (m >= 2 && !q4k_small && gemm_skinny_supported(wtype, w, x, m, n, k))
        return gemm_skinny(wtype, w, x, control, y, m, n, k, stream);
    // Q4_K: the batched tensor-core GEMV (eight input rows per weight pass).
    // Otherwise quantised weights: one tensor-core GEMV per input row (the weights are
    // re-read per row, from L2 when they fit, which still beats the SIMT
    // kernel by an order of magnitude). Rows at or past control[1] are not
    // written (the check runs on the device, after the dependency wait).
    if (wtype == SI_TYPE_Q4_K && m >= 2 && m <= 1024) {
        const si_status bs = matvec_q4k_batched(w, x, y, m, n, k, stream, control);
        if (bs != SI_ERR_UNSUPPORTED) return bs;
    }
    if ((wtype == SI_TYPE_Q4_K || wtype == SI_TYPE_Q8_0) && m <= 1024) {
        si_status ms = SI_OK;
        for (int64_t b = 0; b < m && ms == SI_OK; ++b)
            ms = matvec_quant_mma(wtype, w, x + b * k, y + b * n, n, k, stream, nullptr, control, int(b));
        if (ms != SI_ERR_UNSUPPORTED) return ms;  // the first call decides: the shape is the same for every row
    }
    switch (wtype) {
    case SI_TYPE_F32: return launch_shared<SI_TYPE_F32>(w, x, y, control, m, n, k, st);
    case SI_TYPE_F16: return launch_shared<SI_TYPE_F16>(w, x, y, control, m, n, k, st);
    case SI_TYPE_Q8_0: return launch_shared<SI_TYPE_Q8_0>(w, x, y, control, m, n, k, st);
    case SI_TYPE_Q4_K: return launch_shared<SI_TYPE_Q4_K>(w, x, y, control, m, n, k, st);
    case SI_TYPE_Q6_K: return launch_shared<SI_TYPE_Q6_K>(w, x, y, control, m, n, k, st);
    default: return fail(SI_ERR_UNSUPPORTED, "unsupported weight type %u", wtype);
    }
}

si_status batch_shared_matvec(uint32_t wtype, const void *w, const float *in, const int32_t *control, float *out,
                              int64_t batch, int64_t out_features, int64_t in_features, void *stream) {
    return shared_weight_matvec(wtype, w, in, control, out, batch, out_features, in_features, stream);
}

}  // namespace si::kernels
