// Host-side GGUF helpers of libsharpinfer_cuda: error state, byte-length
// table, binary16 conversion, Q8_0/Q4_K block codecs and the seeded
// synthetic-weight generator. Compiled with -ffp-contract=off so every
// product is rounded once and results are identical on every host.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "si_internal.h"

namespace si {

static thread_local std::string g_last_error;

si_status fail(si_status status, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

void clear_error() { g_last_error.clear(); }

const std::string &last_error() { return g_last_error; }

// GgufModelFile.GetByteLength (GgufModelFile.cs:301-331), extended with the
// K-quant superblocks of the GGUF format (256 elements: Q2_K 84 B, Q3_K 110,
// Q4_K 144, Q5_K 176, Q6_K 210, Q8_K 292), which the reference rejects.
si_status byte_length(uint32_t type, uint64_t elements, uint64_t *bytes) {
    uint64_t block = 1, per = 0;
    switch (type) {
    case 0: per = 4; break;                      // F32
    case 1: case 30: per = 2; break;             // F16, BF16
    case 24: per = 1; break;                     // I8
    case 25: per = 2; break;                     // I16
    case 26: per = 4; break;                     // I32
    case 27: case 28: per = 8; break;            // I64, F64
    case 2: block = 32, per = 18; break;         // Q4_0
    case 3: block = 32, per = 20; break;         // Q4_1
    case 6: block = 32, per = 22; break;         // Q5_0
    case 7: block = 32, per = 24; break;         // Q5_1
    case 8: block = 32, per = 34; break;         // Q8_0
    case 9: block = 32, per = 36; break;         // Q8_1
    case 10: block = 256, per = 84; break;       // Q2_K
    case 11: block = 256, per = 110; break;      // Q3_K
    case 12: block = 256, per = 144; break;      // Q4_K
    case 13: block = 256, per = 176; break;      // Q5_K
    case 14: block = 256, per = 210; break;      // Q6_K
    case 15: block = 256, per = 292; break;      // Q8_K
    default: return fail(SI_ERR_UNSUPPORTED, "GGUF tensor type '%u' is not supported.", type);
    }
    if (elements % block)
        return fail(SI_ERR_INVALID_DATA, "Quantized tensor element count %llu is not divisible by block size %llu.",
                    (unsigned long long)elements, (unsigned long long)block);
    const uint64_t blocks = elements / block;
    if (blocks > UINT64_MAX / per) return fail(SI_ERR_INVALID_DATA, "tensor byte length overflows");
    *bytes = blocks * per;
    return SI_OK;
}

static inline uint32_t bits_of(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float float_of(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

float half_to_float(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    const uint32_t exponent = (h >> 10) & 0x1fu, mantissa = h & 0x3ffu;
    if (exponent == 0) {
        const float v = float(mantissa) * 0x1.0p-24f;
        return sign ? -v : v;
    }
    if (exponent == 31) return float_of(sign | 0x7f800000u | (mantissa << 13));
    return float_of(sign | ((exponent + 112u) << 23) | (mantissa << 13));
}

uint16_t float_to_half(float f) {
    const uint32_t b = bits_of(f);
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

namespace {

inline uint64_t splitmix64(uint64_t seed, uint64_t index) {
    uint64_t z = seed + (index + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

inline float normal_at(uint64_t seed, uint64_t e, float sigma) {
    constexpr double kTwoPi = 6.283185307179586476925286766559;
    const uint64_t p = e >> 1;
    const double u1 = double((splitmix64(seed, 2 * p) >> 11) + 1) * 0x1.0p-53;
    const double u2 = double(splitmix64(seed, 2 * p + 1) >> 11) * 0x1.0p-53;
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double z = (e & 1) ? r * std::sin(kTwoPi * u2) : r * std::cos(kTwoPi * u2);
    return float(z * double(sigma));
}

inline void put16(uint8_t *p, uint16_t v) { p[0] = uint8_t(v); p[1] = uint8_t(v >> 8); }
inline uint16_t get16(const uint8_t *p) { return uint16_t(p[0] | (p[1] << 8)); }
inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Q8_0: d = absmax/127 (stored binary16), q = round(x * 127/absmax) in [-127,127].
void quantize_q8_0_block(const float *v, uint8_t *o) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(v[i]));
    const float d = amax / 127.0f;
    const float id = amax > 0.0f ? 127.0f / amax : 0.0f;
    put16(o, float_to_half(d));
    for (int i = 0; i < 32; ++i) {
        const float q = clampf(std::round(v[i] * id), -127.0f, 127.0f);
        o[2 + i] = uint8_t(int8_t(q));
    }
}

// Q4_K superblock: per 32-element sub-block an asymmetric range
// [min(0,lo), hi] split into 15 steps; sub-block scales and mins are
// quantized to 6 bits against binary16 d = max scale/63 and
// dmin = max min/63. Byte layout is the GGUF Q4_K block.
void quantize_q4_k_block(const float *v, uint8_t *o) {
    float scale[8], minv[8], smax = 0.0f, mmax = 0.0f;
    for (int s = 0; s < 8; ++s) {
        float lo = 0.0f, hi = 0.0f;
        for (int i = 0; i < 32; ++i) {
            lo = std::min(lo, v[32 * s + i]);
            hi = std::max(hi, v[32 * s + i]);
        }
        scale[s] = (hi - lo) / 15.0f;
        minv[s] = -lo;
        smax = std::max(smax, scale[s]);
        mmax = std::max(mmax, minv[s]);
    }
    const uint16_t dh = float_to_half(smax / 63.0f), mh = float_to_half(mmax / 63.0f);
    const float d = half_to_float(dh), dmin = half_to_float(mh);
    int sc[8], mn[8];
    for (int s = 0; s < 8; ++s) {
        sc[s] = d > 0.0f ? int(clampf(std::round(scale[s] / d), 0.0f, 63.0f)) : 0;
        if (sc[s] == 0 && scale[s] > 0.0f && d > 0.0f) sc[s] = 1;
        mn[s] = dmin > 0.0f ? int(clampf(std::round(minv[s] / dmin), 0.0f, 63.0f)) : 0;
    }
    put16(o, dh);
    put16(o + 2, mh);
    uint8_t *packed = o + 4;
    for (int s = 0; s < 4; ++s) {
        packed[s] = uint8_t((sc[s] & 63) | ((sc[s + 4] >> 4) << 6));
        packed[s + 4] = uint8_t((mn[s] & 63) | ((mn[s + 4] >> 4) << 6));
        packed[s + 8] = uint8_t((sc[s + 4] & 15) | ((mn[s + 4] & 15) << 4));
    }
    uint8_t q[256];
    for (int s = 0; s < 8; ++s) {
        const float a = d * float(sc[s]), m = dmin * float(mn[s]);
        for (int i = 0; i < 32; ++i)
            q[32 * s + i] = a > 0.0f ? uint8_t(clampf(std::round((v[32 * s + i] + m) / a), 0.0f, 15.0f)) : 0;
    }
    uint8_t *qs = o + 16;
    for (int j = 0; j < 4; ++j)
        for (int l = 0; l < 32; ++l) qs[32 * j + l] = uint8_t(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
}

void scale_min_q4_k(const uint8_t *packed, int s, int *sc, int *m) {
    if (s < 4) {
        *sc = packed[s] & 63;
        *m = packed[s + 4] & 63;
    } else {
        *sc = (packed[s + 4] & 0x0f) | ((packed[s - 4] >> 6) << 4);
        *m = (packed[s + 4] >> 4) | ((packed[s] >> 6) << 4);
    }
}

// Q6_K superblock (GGUF layout, 210 bytes): ql[128] low four bits, qh[64]
// high two bits, 16 int8 sub-block scales, binary16 d. Element e = 128h +
// 32j + l: low bits in ql[64h + l + 32(j & 1)] (nibble j >> 1), high bits
// (qh[32h + l] >> 2j) & 3; w = (d * scale[e / 16]) * (q - 32).
// Quantiser: per 16 elements s = absmax / 31, d = max s / 127 (binary16),
// scale = round(s / d) in [0, 127] (1 when a non-zero s rounds to 0),
// q = round(x / (d * scale)) + 32 in [0, 63].
void quantize_q6_k_block(const float *v, uint8_t *o) {
    float gs[16], smax = 0.0f;
    for (int g = 0; g < 16; ++g) {
        float amax = 0.0f;
        for (int i = 0; i < 16; ++i) amax = std::max(amax, std::fabs(v[16 * g + i]));
        gs[g] = amax / 31.0f;
        smax = std::max(smax, gs[g]);
    }
    const uint16_t dh = float_to_half(smax / 127.0f);
    const float d = half_to_float(dh);
    int sc[16];
    for (int g = 0; g < 16; ++g) {
        sc[g] = d > 0.0f ? int(clampf(std::round(gs[g] / d), 0.0f, 127.0f)) : 0;
        if (sc[g] == 0 && gs[g] > 0.0f && d > 0.0f) sc[g] = 1;
    }
    std::memset(o, 0, kQ6KBytes);
    for (int e = 0; e < 256; ++e) {
        const float a = d * float(sc[e / 16]);
        const int q = a > 0.0f ? int(clampf(std::round(v[e] / a), -32.0f, 31.0f) + 32.0f) : 32;
        const int h = e >> 7, j = (e >> 5) & 3, l = e & 31;
        o[64 * h + l + 32 * (j & 1)] |= uint8_t((q & 15) << (4 * (j >> 1)));
        o[128 + 32 * h + l] |= uint8_t((q >> 4) << (2 * j));
    }
    for (int g = 0; g < 16; ++g) o[192 + g] = uint8_t(int8_t(sc[g]));
    put16(o + 208, dh);
}

void dequantize_q6_k_block(const uint8_t *o, float *w) {
    const float d = half_to_float(get16(o + 208));
    for (int e = 0; e < 256; ++e) {
        const int h = e >> 7, j = (e >> 5) & 3, l = e & 31;
        const int low = (o[64 * h + l + 32 * (j & 1)] >> (4 * (j >> 1))) & 15;
        const int high = (o[128 + 32 * h + l] >> (2 * j)) & 3;
        w[e] = (d * float(int8_t(o[192 + e / 16]))) * float((low | (high << 4)) - 32);
    }
}

template <class F>
void parallel_for(int64_t n, int threads, F &&body, int64_t grain = 1024) {
    if (threads <= 0) threads = int(std::max(1u, std::thread::hardware_concurrency()));
    if (n < 4 * grain || threads == 1) {
        body(int64_t(0), n);
        return;
    }
    threads = int(std::min<int64_t>(threads, n / grain + 1));
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t)
        pool.emplace_back([&, t] { body(n * t / threads, n * (t + 1) / threads); });
    for (auto &th : pool) th.join();
}

}  // namespace
}  // namespace si

using namespace si;

extern "C" {

int si_abi_version(void) { return SI_ABI_VERSION; }

si_status si_last_error(char *buffer, size_t capacity) {
    if (!buffer || capacity == 0) return SI_ERR_INVALID_ARGUMENT;
    const std::string &e = si::last_error();
    const size_t n = std::min(capacity - 1, e.size());
    std::memcpy(buffer, e.data(), n);
    buffer[n] = '\0';
    return SI_OK;
}

si_status si_tensor_byte_length(uint32_t type, const uint64_t *dims, int rank, uint64_t *bytes) {
    if (!bytes || rank < 0 || (rank > 0 && !dims)) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    uint64_t elements = 1;
    for (int i = 0; i < rank; ++i) {
        if (dims[i] && elements > UINT64_MAX / dims[i])
            return fail(SI_ERR_INVALID_ARGUMENT, "element count overflows 64 bits");
        elements *= dims[i];
    }
    return byte_length(type, elements, bytes);
}

si_status si_row_bytes(uint32_t type, int64_t cols, uint64_t *bytes) {
    if (!bytes || cols <= 0) return fail(SI_ERR_INVALID_ARGUMENT, "row requires a positive column count");
    return byte_length(type, uint64_t(cols), bytes);
}

si_status si_quantize(uint32_t type, const float *src, int64_t count, void *dst) {
    if (!src || !dst || count < 0) return fail(SI_ERR_INVALID_ARGUMENT, "null argument or negative count");
    uint64_t bytes;
    if (si_status st = byte_length(type, uint64_t(count), &bytes)) return st;
    auto *o = static_cast<uint8_t *>(dst);
    switch (type) {
    case SI_TYPE_F32: std::memcpy(o, src, bytes); return SI_OK;
    case SI_TYPE_F16:
        for (int64_t i = 0; i < count; ++i) put16(o + 2 * i, float_to_half(src[i]));
        return SI_OK;
    case SI_TYPE_Q8_0:
        parallel_for(count / 32, 0, [&](int64_t b0, int64_t b1) {
            for (int64_t b = b0; b < b1; ++b) quantize_q8_0_block(src + 32 * b, o + 34 * b);
        });
        return SI_OK;
    case SI_TYPE_Q4_K:
        parallel_for(count / 256, 0, [&](int64_t b0, int64_t b1) {
            for (int64_t b = b0; b < b1; ++b) quantize_q4_k_block(src + 256 * b, o + 144 * b);
        });
        return SI_OK;
    case SI_TYPE_Q6_K:
        parallel_for(count / 256, 0, [&](int64_t b0, int64_t b1) {
            for (int64_t b = b0; b < b1; ++b) quantize_q6_k_block(src + 256 * b, o + kQ6KBytes * b);
        });
        return SI_OK;
    }
    return fail(SI_ERR_UNSUPPORTED, "unsupported type");
}

si_status si_dequantize(uint32_t type, const void *src, int64_t count, float *dst) {
    if (!src || !dst || count < 0) return fail(SI_ERR_INVALID_ARGUMENT, "null argument or negative count");
    uint64_t bytes;
    if (si_status st = byte_length(type, uint64_t(count), &bytes)) return st;
    const auto *p = static_cast<const uint8_t *>(src);
    switch (type) {
    case SI_TYPE_F32: std::memcpy(dst, p, bytes); return SI_OK;
    case SI_TYPE_F16:
        for (int64_t i = 0; i < count; ++i) dst[i] = half_to_float(get16(p + 2 * i));
        return SI_OK;
    case SI_TYPE_Q8_0:
        for (int64_t b = 0; b < count / 32; ++b) {
            const float d = half_to_float(get16(p + 34 * b));
            for (int i = 0; i < 32; ++i) dst[32 * b + i] = d * float(int8_t(p[34 * b + 2 + i]));
        }
        return SI_OK;
    case SI_TYPE_Q4_K:
        for (int64_t b = 0; b < count / 256; ++b) {
            const uint8_t *o = p + 144 * b;
            const float d = half_to_float(get16(o)), dmin = half_to_float(get16(o + 2));
            for (int s = 0; s < 8; ++s) {
                int sc, m;
                scale_min_q4_k(o + 4, s, &sc, &m);
                const float a = d * float(sc), c = dmin * float(m);
                const int j = s >> 1, hi = s & 1;
                for (int l = 0; l < 32; ++l) {
                    const int q = hi ? (o[16 + 32 * j + l] >> 4) : (o[16 + 32 * j + l] & 15);
                    dst[256 * b + 32 * s + l] = a * float(q) - c;
                }
            }
        }
        return SI_OK;
    case SI_TYPE_Q6_K:
        for (int64_t b = 0; b < count / 256; ++b) dequantize_q6_k_block(p + kQ6KBytes * b, dst + 256 * b);
        return SI_OK;
    }
    return fail(SI_ERR_UNSUPPORTED, "unsupported type");
}

si_status si_synth_normal(uint64_t seed, uint64_t offset, int64_t count, float sigma, float *dst,
                          int threads) {
    if (!dst || count < 0) return fail(SI_ERR_INVALID_ARGUMENT, "null argument or negative count");
    parallel_for(count, threads, [&](int64_t i0, int64_t i1) {
        for (int64_t i = i0; i < i1; ++i) dst[i] = normal_at(seed, offset + uint64_t(i), sigma);
    });
    return SI_OK;
}

si_status si_synth_weights(uint32_t type, uint64_t seed, int64_t rows, int64_t cols, float sigma,
                           void *dst, int threads) {
    return si_synth_weight_rows(type, seed, 0, rows, cols, sigma, dst, threads);
}

si_status si_synth_weight_rows(uint32_t type, uint64_t seed, int64_t row_begin, int64_t rows, int64_t cols,
                               float sigma, void *dst, int threads) {
    if (!dst || rows <= 0 || cols <= 0 || row_begin < 0) return fail(SI_ERR_INVALID_ARGUMENT, "invalid shape");
    if (!known_type(type)) return fail(SI_ERR_UNSUPPORTED, "GGUF tensor type '%u' is not supported.", type);
    uint64_t rb;
    if (si_status st = byte_length(type, uint64_t(cols), &rb)) return st;
    auto *o = static_cast<uint8_t *>(dst);
    parallel_for(rows, threads, [&](int64_t r0, int64_t r1) {
        std::vector<float> row(static_cast<size_t>(cols));
        for (int64_t r = r0; r < r1; ++r) {
            for (int64_t c = 0; c < cols; ++c)
                row[size_t(c)] = normal_at(seed, uint64_t((row_begin + r) * cols + c), sigma);
            uint8_t *dr = o + uint64_t(r) * rb;
            if (type == SI_TYPE_F32) std::memcpy(dr, row.data(), rb);
            else if (type == SI_TYPE_F16) for (int64_t c = 0; c < cols; ++c) put16(dr + 2 * c, float_to_half(row[size_t(c)]));
            else if (type == SI_TYPE_Q8_0) for (int64_t b = 0; b < cols / 32; ++b) quantize_q8_0_block(row.data() + 32 * b, dr + 34 * b);
            else if (type == SI_TYPE_Q6_K) for (int64_t b = 0; b < cols / 256; ++b) quantize_q6_k_block(row.data() + 256 * b, dr + kQ6KBytes * b);
            else for (int64_t b = 0; b < cols / 256; ++b) quantize_q4_k_block(row.data() + 256 * b, dr + 144 * b);
        }
    }, 8);
    return SI_OK;
}

}  // extern "C"
