/*
 * oracle.c -- CPU restatement of SharpInference's mat-vec numerics.
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, smoke() and the
 * cpu_baseline leg of bench.py. The shipped library never calls it.
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off; no FMA contraction so
 * every product is rounded once, as the reference's `precise` HLSL and the
 * C# scalar code round it).
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* SplitMix64 (Steele, Lea, Flood 2014), used as a counter-based generator:
 * output `index` of the stream seeded with `seed`. */
uint64_t or_splitmix64(uint64_t seed, uint64_t index) {
    uint64_t z = seed + (index + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Element i of the N(0, sigma) stream: pair p = i/2 draws u1 in (0,1] and
 * u2 in [0,1) from outputs 2p and 2p+1; Box-Muller in double precision,
 * even elements take the cosine branch, odd elements the sine branch. */
void or_normal_fill(uint64_t seed, uint64_t offset, int64_t n, float sigma, float *out) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t i = 0; i < n; ++i) {
        uint64_t e = offset + (uint64_t)i;
        uint64_t p = e >> 1;
        double u1 = (double)((or_splitmix64(seed, 2 * p) >> 11) + 1) * 0x1.0p-53;
        double u2 = (double)(or_splitmix64(seed, 2 * p + 1) >> 11) * 0x1.0p-53;
        double r = sqrt(-2.0 * log(u1));
        double z = (e & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
        out[i] = (float)(z * (double)sigma);
    }
}

/* ------------------------------------------------------------------------ */
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        float v = (float)m * 5.9604644775390625e-8f; /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

uint16_t or_f32_to_f16(float f) {
    uint32_t b = f2u(f);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    uint32_t a = b & 0x7fffffffu;
    if (a >= 0x7f800000u) /* Inf / NaN */
        return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? (0x200u | ((a >> 13) & 0x3ffu)) : 0u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to Inf */
    if (a < 0x38800000u) {                                   /* half subnormal range */
        if (a <= 0x33000000u) return sign;                   /* <= 2^-25: ties to even 0 */
        uint32_t mant = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - (a >> 23);
        uint32_t h = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = (a >> 13) - (112u << 10), rem = a & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* ------------------------------------------------------------------------ */
int or_byte_length(uint32_t type, uint64_t elements, uint64_t *bytes) {
    switch (type) {
    case OR_F32: *bytes = elements * 4; return 0;
    case OR_F16: *bytes = elements * 2; return 0;
    case OR_Q8_0:
        if (elements % OR_Q8_0_BLOCK) return -2;
        *bytes = elements / OR_Q8_0_BLOCK * OR_Q8_0_BYTES; return 0;
    case OR_Q4_K:
        if (elements % OR_Q4_K_BLOCK) return -2;
        *bytes = elements / OR_Q4_K_BLOCK * OR_Q4_K_BYTES; return 0;
    case OR_Q6_K:
        if (elements % OR_Q6_K_BLOCK) return -2;
        *bytes = elements / OR_Q6_K_BLOCK * OR_Q6_K_BYTES; return 0;
    default: return -1;
    }
}

/* Q8_0 block: fp16 d, 32 x int8 q; w = d * q. d = absmax / 127 and
 * q = round(x * 127 / absmax), clamped to [-127, 127]. */
void or_quantize_q8_0(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / OR_Q8_0_BLOCK; ++b) {
        const float *v = x + b * OR_Q8_0_BLOCK;
        uint8_t *o = out + b * OR_Q8_0_BYTES;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) { float a = fabsf(v[i]); if (a > amax) amax = a; }
        float d = amax / 127.0f;
        float id = amax > 0.0f ? 127.0f / amax : 0.0f;
        wr16(o, or_f32_to_f16(d));
        for (int i = 0; i < 32; ++i) {
            float q = roundf(v[i] * id);
            if (q > 127.0f) q = 127.0f;
            if (q < -127.0f) q = -127.0f;
            o[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

void or_dequantize_q8_0(const uint8_t *blocks, int64_t n, float *out) {
    for (int64_t b = 0; b < n / OR_Q8_0_BLOCK; ++b) {
        const uint8_t *o = blocks + b * OR_Q8_0_BYTES;
        float d = or_f16_to_f32(rd16(o));
        for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)(int8_t)o[2 + i];
    }
}

/* Q4_K superblock (GGUF layout): fp16 d, fp16 dmin, 12 bytes of packed 6-bit
 * (scale, min) for 8 sub-blocks of 32, then 128 bytes of nibbles. Sub-block s
 * is elements [32s, 32s+32); byte l of chunk j (qs[32j + l]) holds element
 * 64j + l in its low nibble and element 64j + 32 + l in its high nibble.
 * w = (d * sc_s) * q - (dmin * m_s). */
static void q4k_get_scale_min(const uint8_t *sc12, int s, int *sc, int *m) {
    if (s < 4) {
        *sc = sc12[s] & 63;
        *m = sc12[s + 4] & 63;
    } else {
        *sc = (sc12[s + 4] & 0x0f) | ((sc12[s - 4] >> 6) << 4);
        *m = (sc12[s + 4] >> 4) | ((sc12[s] >> 6) << 4);
    }
}

static float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

void or_quantize_q4_k(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / OR_Q4_K_BLOCK; ++b) {
        const float *v = x + b * OR_Q4_K_BLOCK;
        uint8_t *o = out + b * OR_Q4_K_BYTES;
        float scale[8], minv[8], smax = 0.0f, mmax = 0.0f;
        for (int s = 0; s < 8; ++s) {
            float lo = 0.0f, hi = 0.0f;
            for (int i = 0; i < 32; ++i) {
                float t = v[32 * s + i];
                if (t < lo) lo = t;
                if (t > hi) hi = t;
            }
            scale[s] = (hi - lo) / 15.0f;
            minv[s] = -lo;
            if (scale[s] > smax) smax = scale[s];
            if (minv[s] > mmax) mmax = minv[s];
        }
        uint16_t dh = or_f32_to_f16(smax / 63.0f), mh = or_f32_to_f16(mmax / 63.0f);
        float d = or_f16_to_f32(dh), dmin = or_f16_to_f32(mh);
        int sc[8], mn[8];
        for (int s = 0; s < 8; ++s) {
            sc[s] = d > 0.0f ? (int)clampf(roundf(scale[s] / d), 0.0f, 63.0f) : 0;
            if (sc[s] == 0 && scale[s] > 0.0f && d > 0.0f) sc[s] = 1;
            mn[s] = dmin > 0.0f ? (int)clampf(roundf(minv[s] / dmin), 0.0f, 63.0f) : 0;
        }
        wr16(o, dh);
        wr16(o + 2, mh);
        uint8_t *p = o + 4;
        for (int s = 0; s < 4; ++s) {
            p[s] = (uint8_t)((sc[s] & 63) | ((sc[s + 4] >> 4) << 6));
            p[s + 4] = (uint8_t)((mn[s] & 63) | ((mn[s + 4] >> 4) << 6));
            p[s + 8] = (uint8_t)((sc[s + 4] & 15) | ((mn[s + 4] & 15) << 4));
        }
        uint8_t q[256];
        for (int s = 0; s < 8; ++s) {
            float a = d * (float)sc[s], m = dmin * (float)mn[s];
            for (int i = 0; i < 32; ++i)
                q[32 * s + i] = a > 0.0f ? (uint8_t)clampf(roundf((v[32 * s + i] + m) / a), 0.0f, 15.0f) : 0;
        }
        uint8_t *qs = o + 16;
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 32; ++l)
                qs[32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
    }
}

void or_dequantize_q4_k(const uint8_t *blocks, int64_t n, float *out) {
    for (int64_t b = 0; b < n / OR_Q4_K_BLOCK; ++b) {
        const uint8_t *o = blocks + b * OR_Q4_K_BYTES;
        float d = or_f16_to_f32(rd16(o)), dmin = or_f16_to_f32(rd16(o + 2));
        const uint8_t *qs = o + 16;
        float *w = out + b * OR_Q4_K_BLOCK;
        for (int s = 0; s < 8; ++s) {
            int sc, m;
            q4k_get_scale_min(o + 4, s, &sc, &m);
            float a = d * (float)sc, c = dmin * (float)m;
            int j = s >> 1, hi = s & 1;
            for (int l = 0; l < 32; ++l) {
                int q = hi ? (qs[32 * j + l] >> 4) : (qs[32 * j + l] & 15);
                w[32 * s + l] = a * (float)q - c;
            }
        }
    }
}

/* Q6_K superblock (GGUF layout, 210 bytes): ql[128] low four bits, qh[64] high
 * two bits, 16 int8 sub-block scales, fp16 d. Element e = 128h + 32j + l
 * (h < 2, j < 4, l < 32): low bits = ql[64h + l + 32(j & 1)] >> 4(j >> 1),
 * high bits = (qh[32h + l] >> 2j) & 3, q = low | high << 4 in [0, 63];
 * w = (d * scale[e / 16]) * (q - 32). */
static int q6k_code(const uint8_t *o, int e) {
    const int h = e >> 7, j = (e >> 5) & 3, l = e & 31;
    const int low = (o[64 * h + l + 32 * (j & 1)] >> (4 * (j >> 1))) & 15;
    const int high = (o[128 + 32 * h + l] >> (2 * j)) & 3;
    return low | (high << 4);
}

/* Quantiser of this restatement (the format's reader is what parity needs):
 * per 16-element group a scale s = absmax / 31; d = max s / 127 as fp16;
 * scale = round(s / d) in [0, 127] (1 when s > 0 rounds to 0);
 * q = round(x / (d * scale)) + 32 clamped to [0, 63]. */
void or_quantize_q6_k(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / OR_Q6_K_BLOCK; ++b) {
        const float *v = x + b * OR_Q6_K_BLOCK;
        uint8_t *o = out + b * OR_Q6_K_BYTES;
        float gs[16], smax = 0.0f;
        for (int g = 0; g < 16; ++g) {
            float amax = 0.0f;
            for (int i = 0; i < 16; ++i) {
                float t = fabsf(v[16 * g + i]);
                if (t > amax) amax = t;
            }
            gs[g] = amax / 31.0f;
            if (gs[g] > smax) smax = gs[g];
        }
        uint16_t dh = or_f32_to_f16(smax / 127.0f);
        float d = or_f16_to_f32(dh);
        int sc[16];
        for (int g = 0; g < 16; ++g) {
            sc[g] = d > 0.0f ? (int)clampf(roundf(gs[g] / d), 0.0f, 127.0f) : 0;
            if (sc[g] == 0 && gs[g] > 0.0f && d > 0.0f) sc[g] = 1;
        }
        uint8_t q[256];
        for (int e = 0; e < 256; ++e) {
            float a = d * (float)sc[e / 16];
            q[e] = a > 0.0f ? (uint8_t)(clampf(roundf(v[e] / a), -32.0f, 31.0f) + 32.0f) : 32;
        }
        memset(o, 0, OR_Q6_K_BYTES);
        for (int e = 0; e < 256; ++e) {
            const int h = e >> 7, j = (e >> 5) & 3, l = e & 31;
            o[64 * h + l + 32 * (j & 1)] |= (uint8_t)((q[e] & 15) << (4 * (j >> 1)));
            o[128 + 32 * h + l] |= (uint8_t)((q[e] >> 4) << (2 * j));
        }
        for (int g = 0; g < 16; ++g) o[192 + g] = (uint8_t)(int8_t)sc[g];
        wr16(o + 208, dh);
    }
}

void or_dequantize_q6_k(const uint8_t *blocks, int64_t n, float *out) {
    for (int64_t b = 0; b < n / OR_Q6_K_BLOCK; ++b) {
        const uint8_t *o = blocks + b * OR_Q6_K_BYTES;
        float d = or_f16_to_f32(rd16(o + 208));
        float *w = out + b * OR_Q6_K_BLOCK;
        for (int e = 0; e < 256; ++e) {
            float a = d * (float)(int8_t)o[192 + e / 16];
            w[e] = a * (float)(q6k_code(o, e) - 32);
        }
    }
}

int or_dequantize_row(uint32_t type, const void *row, int64_t cols, float *out) {
    switch (type) {
    case OR_F32: memcpy(out, row, (size_t)cols * 4); return 0;
    case OR_F16: {
        const uint8_t *p = (const uint8_t *)row;
        for (int64_t i = 0; i < cols; ++i) out[i] = or_f16_to_f32(rd16(p + 2 * i));
        return 0;
    }
    case OR_Q8_0:
        if (cols % 32) return -2;
        or_dequantize_q8_0((const uint8_t *)row, cols, out); return 0;
    case OR_Q4_K:
        if (cols % 256) return -2;
        or_dequantize_q4_k((const uint8_t *)row, cols, out); return 0;
    case OR_Q6_K:
        if (cols % 256) return -2;
        or_dequantize_q6_k((const uint8_t *)row, cols, out); return 0;
    default: return -1;
    }
}

/* ------------------------------------------------------------------------ */
/* FP32 dot with eight striped lanes (a Vector256<float> accumulation); the
 * summation order of TensorPrimitives.Dot is unspecified by its library. */
static float dot8(const float *a, const float *b, int64_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] += a[i + l] * b[i + l];
    for (int l = 0; i < n; ++i, ++l) acc[l] += a[i] * b[i];
    return ((acc[0] + acc[4]) + (acc[2] + acc[6])) + ((acc[1] + acc[5]) + (acc[3] + acc[7]));
}

static double dot_f64(const float *a, const float *b, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double)a[i] * (double)b[i];
    return s;
}

static uint64_t row_bytes(uint32_t type, int64_t cols) {
    uint64_t b = 0;
    or_byte_length(type, (uint64_t)cols, &b);
    return b;
}

int or_online_cores(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef struct {
    uint32_t wtype;
    const uint8_t *w;
    const float *x;
    float *y;
    double *y64;
    int64_t rows, cols, r0, r1;
    int serial_blocks;
} mv_job;

static void *mv_worker(void *arg) {
    mv_job *j = (mv_job *)arg;
    uint64_t rb = row_bytes(j->wtype, j->cols);
    float *scratch = (float *)malloc((size_t)j->cols * sizeof(float));
    for (int64_t r = j->r0; r < j->r1; ++r) {
        or_dequantize_row(j->wtype, j->w + (uint64_t)r * rb, j->cols, scratch);
        if (j->y64) {
            j->y64[r] = dot_f64(scratch, j->x, j->cols);
        } else if (j->serial_blocks) {
            /* serial branch: bounded 1024-element conversion blocks, FP32
             * sum of block dots (CpuHalfMatrixOperators.cs:15-21,123-137) */
            float sum = 0.0f;
            for (int64_t c = 0; c < j->cols; c += 1024) {
                int64_t len = j->cols - c < 1024 ? j->cols - c : 1024;
                sum += dot8(scratch + c, j->x + c, len);
            }
            j->y[r] = sum;
        } else {
            j->y[r] = dot8(scratch, j->x, j->cols);
        }
    }
    free(scratch);
    return NULL;
}

static int run_matvec(uint32_t wtype, const void *w, const float *x, float *y, double *y64,
                      int64_t rows, int64_t cols, int threads) {
    if (rows <= 0 || cols <= 0 || !w || !x || (!y && !y64)) return -3;
    uint64_t tmp;
    if (or_byte_length(wtype, (uint64_t)cols, &tmp)) return -2;
    /* ParallelRowThreshold = 64, ParallelElementThreshold = 65536
     * (CpuHalfMatrixOperators.cs:8-9) */
    int serial = rows < 64 || rows * cols < 65536;
    if (threads <= 0) threads = or_online_cores();
    if (serial || threads == 1 || rows < threads) threads = 1;
    mv_job *jobs = (mv_job *)calloc((size_t)threads, sizeof(mv_job));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (mv_job){wtype, (const uint8_t *)w, x, y, y64, rows, cols,
                           rows * t / threads, rows * (t + 1) / threads, serial && wtype == OR_F16};
        if (threads > 1) pthread_create(&tids[t], NULL, mv_worker, &jobs[t]);
    }
    if (threads == 1) mv_worker(&jobs[0]);
    else for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
    free(jobs);
    free(tids);
    return 0;
}

int or_matvec(uint32_t wtype, const void *w, const float *x, float *y,
              int64_t rows, int64_t cols, int threads) {
    return run_matvec(wtype, w, x, y, NULL, rows, cols, threads);
}

int or_matvec_f64(uint32_t wtype, const void *w, const float *x, double *y,
                  int64_t rows, int64_t cols, int threads) {
    return run_matvec(wtype, w, x, NULL, y, rows, cols, threads);
}

/* add32 (GpuTierZeroInstruction.cs:316): Neumaier step; a non-finite total
 * clears the correction so Inf/NaN classes survive the final sum. */
static void add32(float *sum, float *correction, float value) {
    volatile float total = *sum + value;
    if (isfinite(total)) {
        float residual = fabsf(*sum) >= fabsf(value) ? (*sum - total) + value : (value - total) + *sum;
        *correction += residual;
    } else {
        *correction = 0.0f;
    }
    *sum = total;
}

static float load_elem(uint32_t type, const void *p, int64_t i) {
    if (type == OR_F16) return or_f16_to_f32(rd16((const uint8_t *)p + 2 * i));
    return ((const float *)p)[i];
}

int or_matvec_cooperative(uint32_t wtype, uint32_t xtype, uint32_t ytype,
                          const void *w, const void *x, void *y,
                          int64_t rows, int64_t cols, int lanes) {
    if ((wtype != OR_F32 && wtype != OR_F16) || (xtype != OR_F32 && xtype != OR_F16) ||
        (ytype != OR_F32 && ytype != OR_F16) || lanes <= 0 || (lanes & (lanes - 1)))
        return -1;
    float *sum = (float *)malloc((size_t)lanes * 4), *cor = (float *)malloc((size_t)lanes * 4);
    for (int64_t r = 0; r < rows; ++r) {
        for (int l = 0; l < lanes; ++l) {
            float s = 0.0f, c = 0.0f;
            for (int64_t j = l; j < cols; j += lanes) {
                volatile float product = load_elem(wtype, w, r * cols + j) * load_elem(xtype, x, j);
                add32(&s, &c, product);
            }
            sum[l] = s;
            cor[l] = c;
        }
        for (int step = lanes / 2; step > 0; step >>= 1)
            for (int l = 0; l < step; ++l) {
                float left = sum[l], residual = cor[l];
                add32(&left, &residual, sum[l + step]);
                add32(&left, &residual, cor[l + step]);
                sum[l] = left;
                cor[l] = residual;
            }
        float result = sum[0] + cor[0];
        if (ytype == OR_F16) wr16((uint8_t *)y + 2 * r, or_f32_to_f16(result));
        else ((float *)y)[r] = result;
    }
    free(sum);
    free(cor);
    return 0;
}

int or_batch_shared_matvec(uint32_t wtype, const void *w, const float *in,
                           const int32_t *control, float *out,
                           int64_t batch, int64_t out_features, int64_t in_features) {
    uint64_t rb;
    if (or_byte_length(wtype, (uint64_t)in_features, &rb)) return -2;
    float *row = (float *)malloc((size_t)in_features * 4);
    int32_t valid = control[1];
    for (int64_t o = 0; o < out_features; ++o) {
        or_dequantize_row(wtype, (const uint8_t *)w + (uint64_t)o * rb, in_features, row);
        for (int64_t b = 0; b < batch; ++b) {
            if (b >= valid) continue;
            float part[64];
            for (int l = 0; l < 64; ++l) {
                float s = 0.0f;
                for (int64_t i = l; i < in_features; i += 64) s += row[i] * in[b * in_features + i];
                part[l] = s;
            }
            for (int step = 32; step > 0; step >>= 1)
                for (int l = 0; l < step; ++l) part[l] += part[l + step];
            out[b * out_features + o] = part[0];
        }
    }
    free(row);
    return 0;
}

int or_matrix_multiply_tr(uint32_t wtype, const float *x, const void *w, float *y,
                          int64_t m, int64_t n, int64_t k, int threads) {
    for (int64_t r = 0; r < m; ++r) {
        int rc = or_matvec(wtype, w, x + r * k, y + r * n, n, k, threads);
        if (rc) return rc;
    }
    return 0;
}
