// Seeded synthetic weights generated in device memory: the same definition
// as the host generator (si_synth_weight_rows in host_codecs.cpp) -- element
// e of the row-major matrix is N(0, sigma) from a Box-Muller pair of
// splitmix64 draws (cos for even e, sin for odd e, double precision), then
// quantised per block -- so a multi-gigabyte model (Phi-4-14B's 15 GB of
// Q8_0) is made in HBM in well under a second instead of minutes of host
// work. The double-precision log / sin / cos are the device library's, so a
// value can differ from the host generator's in its last bit; the bytes
// match the host's except where that moves a rounding boundary.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "si_internal.h"

namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t seed, uint64_t index) {
    uint64_t z = seed + (index + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// The pair (2p, 2p + 1) of normals.
__device__ __forceinline__ void normal_pair(uint64_t seed, uint64_t p, float sigma, float &even, float &odd) {
    constexpr double kTwoPi = 6.283185307179586476925286766559;
    const double u1 = double((splitmix64(seed, 2 * p) >> 11) + 1) * 0x1.0p-53;
    const double u2 = double(splitmix64(seed, 2 * p + 1) >> 11) * 0x1.0p-53;
    const double r = sqrt(-2.0 * log(u1));
    double s, c;
    sincos(kTwoPi * u2, &s, &c);
    even = float(r * c * double(sigma));
    odd = float(r * s * double(sigma));
}

// binary32 -> binary16, round to nearest even: the host conversion
// (float_to_half in host_codecs.cpp) bit for bit.
__device__ __forceinline__ uint16_t half_bits_rne(float f) {
    const uint32_t b = __float_as_uint(f);
    const uint16_t sign = uint16_t((b >> 16) & 0x8000u);
    const uint32_t a = b & 0x7fffffffu;
    if (a >= 0x7f800000u)
        return uint16_t(sign | 0x7c00u | (a > 0x7f800000u ? (0x200u | ((a >> 13) & 0x3ffu)) : 0u));
    if (a >= 0x477ff000u) return uint16_t(sign | 0x7c00u);
    if (a < 0x38800000u) {
        if (a <= 0x33000000u) return sign;
        const uint32_t m = (a & 0x7fffffu) | 0x800000u, shift = 126u - (a >> 23);
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return uint16_t(sign | h);
    }
    uint32_t h = (a >> 13) - (112u << 10);
    const uint32_t rem = a & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return uint16_t(sign | h);
}

// One thread per 32-element block of the block [row_begin, + rows) x
// [col_begin, + out_cols) of the [*, cols] matrix: F32, F16 or Q8_0; dst
// rows are row_bytes apart and hold the out_cols columns.
__global__ void synth_rows_kernel(uint32_t type, uint64_t seed, int64_t row_begin, int64_t rows, int64_t cols,
                                  int64_t col_begin, int64_t out_cols, float sigma, uint8_t *dst, uint64_t row_bytes) {
    const int64_t blocks_per_row = out_cols / 32, total = rows * blocks_per_row;
    for (int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; b < total; b += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = b / blocks_per_row, c0 = (b - r * blocks_per_row) * 32;
        // even: cols, col_begin and c0 are multiples of 32
        const uint64_t e0 = uint64_t(row_begin + r) * uint64_t(cols) + uint64_t(col_begin + c0);
        float v[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) normal_pair(seed, (e0 >> 1) + i, sigma, v[2 * i], v[2 * i + 1]);
        uint8_t *row = dst + uint64_t(r) * row_bytes;
        if (type == SI_TYPE_F32) {
            float *o = reinterpret_cast<float *>(row) + c0;
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = v[i];
        } else if (type == SI_TYPE_F16) {
            __half *o = reinterpret_cast<__half *>(row) + c0;
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float2half_rn(v[i]);
        } else {
            // Q8_0: d = absmax / 127 as binary16, q = round(v * 127 / absmax)
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            uint8_t *o = row + (c0 / 32) * 34;
            const uint16_t bits = half_bits_rne(d);
            o[0] = uint8_t(bits & 0xffu);
            o[1] = uint8_t(bits >> 8);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float q = fminf(fmaxf(roundf(__fmul_rn(v[i], id)), -127.0f), 127.0f);
                o[2 + i] = uint8_t(int8_t(q));
            }
        }
    }
}

}  // namespace

extern "C" si_status si_synth_weight_block_device(uint32_t type, uint64_t seed, int64_t row_begin, int64_t rows,
                                                  int64_t col_begin, int64_t col_count, int64_t cols, float sigma,
                                                  void *dst, void *stream) {
    if (!dst || rows <= 0 || cols <= 0 || row_begin < 0 || col_begin < 0 || col_count <= 0 ||
        col_begin + col_count > cols)
        return si::fail(SI_ERR_INVALID_ARGUMENT, "invalid shape or null destination");
    if (type != SI_TYPE_F32 && type != SI_TYPE_F16 && type != SI_TYPE_Q8_0)
        return si::fail(SI_ERR_UNSUPPORTED, "device synthesis makes F32, F16 or Q8_0 weights");
    if (cols % 32 != 0 || col_begin % 32 != 0 || col_count % 32 != 0)
        return si::fail(SI_ERR_INVALID_ARGUMENT, "cols, col_begin and col_count must be multiples of 32");
    uint64_t rb = 0;
    if (si_status st = si::byte_length(type, uint64_t(col_count), &rb)) return st;
    if (si_status st = si::device_range("destination", dst, rb * uint64_t(rows))) return st;
    const int64_t total = rows * (col_count / 32);
    const int grid = int(std::min<int64_t>((total + 127) / 128, 148 * 32));
    synth_rows_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        type, seed, row_begin, rows, cols, col_begin, col_count, sigma, static_cast<uint8_t *>(dst), rb);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return si::fail(SI_ERR_CUDA, "synthesis launch failed: %s", cudaGetErrorString(e));
    return SI_OK;
}

extern "C" si_status si_synth_weight_rows_device(uint32_t type, uint64_t seed, int64_t row_begin, int64_t rows,
                                                 int64_t cols, float sigma, void *dst, void *stream) {
    return si_synth_weight_block_device(type, seed, row_begin, rows, 0, cols, cols, sigma, dst, stream);
}
