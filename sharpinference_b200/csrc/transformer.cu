// FP32 transformer instructions of SharpInference (collection
// TransformerFloat32, GpuTransformerInstructionCollection.cs and
// GpuBatchTransformerInstructions.cs) and core.gather-row with quantised
// tables, as sm_100a kernels.
//
// Every kernel is launched with programmatic dependent launch: it lets its
// successor start launching at once (pdl_trigger) and reads its inputs only
// after pdl_wait, so inside the decode graph a GEMV's weight stream overlaps
// the small kernels in front of it. Arithmetic is FP32 with explicit
// round-to-nearest intrinsics where the instruction body fixes an order
// (no contraction into FMA).
//
// Decode attention (transformer.grouped-query-attention) is split over
// tokens: one 8-CTA cluster per key/value head, each CTA an online softmax
// over its share of the cache for all query heads of the group, combined
// through distributed shared memory. No workspace, no atomics.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "device_common.cuh"
#include "si_internal.h"

namespace si::kernels {
namespace {

using namespace si::dev;

constexpr float kNegMax = -3.402823466e+38f;

__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t dsmem_addr(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Remote shared-memory load. Volatile keeps it after the cluster barrier
// (also a volatile asm); without a memory clobber, loads written back to
// back are issued back to back.
__device__ __forceinline__ float dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t dsmem_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
// All threads of all CTAs of the cluster. Every CTA of a cluster is resident
// at once and every thread reaches each call, so the barrier completes.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over the block (blockDim.x a multiple of 32, at most 1024); every
// thread gets the total. `red` holds 33 floats of shared memory.
__device__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

// ---- element access of a table row ----------------------------------------
// Element c of a row in GGUF layout, dequantised exactly as the CPU codecs
// do it: Q8_0 d*q; Q4_K (d*sc)*q - (dmin*m); Q6_K (d*scale)*(q-32).
__device__ __forceinline__ float row_element(uint32_t type, const uint8_t *row, int64_t c) {
    switch (type) {
    case SI_TYPE_Q6_K: {
        const uint8_t *b = row + (c >> 8) * kQ6KBytes;
        const int e = int(c & 255), h = e >> 7, j = (e >> 5) & 3, l = e & 31;
        const int low = (b[64 * h + l + 32 * (j & 1)] >> (4 * (j >> 1))) & 15;
        const int high = (b[128 + 32 * h + l] >> (2 * j)) & 3;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(b[208] | (b[209] << 8))));
        return __fmul_rn(__fmul_rn(d, float(int8_t(b[192 + (e >> 4)]))), float((low | (high << 4)) - 32));
    }
    case SI_TYPE_F32: return reinterpret_cast<const float *>(row)[c];
    case SI_TYPE_F16: return __half2float(reinterpret_cast<const __half *>(row)[c]);
    case SI_TYPE_Q8_0: {
        const uint8_t *b = row + (c >> 5) * kQ8_0Bytes;
        const float d = __half2float(*reinterpret_cast<const __half *>(b));
        return __fmul_rn(d, float(int8_t(b[2 + (c & 31)])));
    }
    default: {  // SI_TYPE_Q4_K
        const uint8_t *b = row + (c >> 8) * kQ4KBytes;
        const float d = __half2float(*reinterpret_cast<const __half *>(b));
        const float dmin = __half2float(*reinterpret_cast<const __half *>(b + 2));
        const uint8_t *sc = b + 4;
        const int e = int(c & 255), s = e >> 5;
        int scale, mn;
        if (s < 4) {
            scale = sc[s] & 63;
            mn = sc[s + 4] & 63;
        } else {
            scale = (sc[s + 4] & 0x0f) | ((sc[s - 4] >> 6) << 4);
            mn = (sc[s + 4] >> 4) | ((sc[s] >> 6) << 4);
        }
        const int q = (b[16 + 32 * (s >> 1) + (e & 31)] >> (4 * (s & 1))) & 15;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, float(scale)), float(q)), __fmul_rn(dmin, float(mn)));
    }
    }
}

// core.gather-row: out = table[index], NaN everywhere for an index outside
// [0, rows) (GpuTierZeroInstruction.cs:397-407).
__global__ void gather_row_kernel(uint32_t type, const uint8_t *table, int64_t rows, int64_t cols, uint64_t row_bytes,
                                  const int32_t *index, float *out) {
    pdl_trigger();
    pdl_wait();
    const int32_t r = *index;
    const bool ok = r >= 0 && r < rows;
    const uint8_t *row = table + (ok ? uint64_t(r) * row_bytes : 0);
    for (int64_t c = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; c < cols; c += int64_t(gridDim.x) * blockDim.x)
        out[c] = ok ? row_element(type, row, c) : __int_as_float(0x7fc00000);
}

// core.gather-row over a list of indices (the prompt's rows of a prefill
// chunk): out[r] = table[indices[r]], a NaN row for an invalid index.
__global__ void gather_rows_quant_kernel(uint32_t type, const uint8_t *table, int64_t rows, int64_t cols,
                                         uint64_t row_bytes, const int32_t *indices, int64_t count, float *out) {
    pdl_trigger();
    pdl_wait();
    const int64_t total = count * cols;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = e / cols, c = e - r * cols;
        const int32_t t = indices[r];
        out[e] = (t >= 0 && t < rows) ? row_element(type, table + uint64_t(t) * row_bytes, c)
                                      : __int_as_float(0x7fc00000);
    }
}

// transformer.embedding-gather-batch: FP16 table rows by index; an index
// outside the table reads 0, as an out-of-range raw-buffer load does under
// Direct3D 12 (GpuTransformerInstructionCollection.cs:184-219).
__global__ void embedding_gather_batch_kernel(const __half *table, int64_t rows, const int32_t *indices, float *out,
                                              int64_t count, int64_t width) {
    pdl_trigger();
    pdl_wait();
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = e / width, col = e - row * width;
        const int64_t t = int64_t(uint32_t(indices[row]));
        out[e] = t < rows ? __half2float(table[t * width + col]) : 0.0f;
    }
}

// transformer.copy-embedding-rows (GpuTransformerInstructionCollection.cs:221-248).
__global__ void copy_rows_kernel(const float *in, float *out, int64_t count) {
    pdl_trigger();
    pdl_wait();
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x)
        out[e] = in[e];
}

// transformer.rms-norm / residual-rms-norm and their batch forms: one CTA
// per row; rows at or beyond control[1] are skipped (batch forms only).
// updated = hidden + residual is stored before the norm reads it back, so
// `updated` may alias `hidden`; a null `updated` (internal callers only)
// recomputes the sum instead of storing it.
constexpr int kRmsHeld = 8;  // elements per thread held in registers (rows <= 8192 at 1024 threads)

template <bool kResidual>
__global__ void __launch_bounds__(1024) rms_norm_kernel(const float *in, const float *residual, const float *weight,
                                                        const int32_t *control, float *updated, float *out,
                                                        int64_t width, float eps) {
    __shared__ float red[33];
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.x;
    if (control && row >= control[1]) return;
    const float *x = in + row * width;
    const float *r = kResidual ? residual + row * width : nullptr;
    float *u = kResidual && updated ? updated + row * width : nullptr;
    float *o = out + row * width;
    // Rows up to kRmsHeld * blockDim elements keep their values and weights in
    // registers: every load is issued before the reduction (one round trip).
    if (width <= int64_t(kRmsHeld) * blockDim.x) {
        float v[kRmsHeld], w[kRmsHeld];
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < kRmsHeld; ++k) {
            const int64_t j = threadIdx.x + int64_t(k) * blockDim.x;
            const bool ok = j < width;
            v[k] = ok ? (kResidual ? __fadd_rn(x[j], r[j]) : x[j]) : 0.0f;
            w[k] = ok ? weight[j] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < kRmsHeld; ++k) {
            const int64_t j = threadIdx.x + int64_t(k) * blockDim.x;
            if (kResidual && u && j < width) u[j] = v[k];
            s = __fadd_rn(s, __fmul_rn(v[k], v[k]));
        }
        s = block_sum(s, red);
        const float scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(s, float(width)), eps));
#pragma unroll
        for (int k = 0; k < kRmsHeld; ++k) {
            const int64_t j = threadIdx.x + int64_t(k) * blockDim.x;
            if (j < width) o[j] = __fmul_rn(__fmul_rn(v[k], scale), w[k]);
        }
        return;
    }
    float s = 0.0f;
    for (int64_t j = threadIdx.x; j < width; j += blockDim.x) {
        float v = x[j];
        if (kResidual) {
            v = __fadd_rn(v, r[j]);
            if (u) u[j] = v;
        }
        s = __fadd_rn(s, __fmul_rn(v, v));
    }
    s = block_sum(s, red);
    const float scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(s, float(width)), eps));
    for (int64_t j = threadIdx.x; j < width; j += blockDim.x) {
        const float v = !kResidual ? x[j] : (u ? u[j] : __fadd_rn(x[j], r[j]));
        o[j] = __fmul_rn(__fmul_rn(v, scale), weight[j]);
    }
}

// transformer.swiglu / batch-swiglu: out = gate / (1 + exp(-gate)) * up with
// gate_up = [gate | up] per row.
__global__ void swiglu_kernel(const float *gate_up, const int32_t *control, float *out, int64_t batch, int64_t width) {
    pdl_trigger();
    pdl_wait();
    const int64_t count = batch * width;
    const int64_t valid = control ? int64_t(control[1]) : batch;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = e / width, col = e - row * width;
        if (row >= valid) continue;
        const float g = gate_up[row * 2 * width + col], up = gate_up[row * 2 * width + width + col];
        out[e] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up);
    }
}

// transformer.scaled-add: out = in + scale * update.
__global__ void scaled_add_kernel(const float *in, const float *update, float *out, int64_t count, float scale) {
    pdl_trigger();
    pdl_wait();
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x)
        out[e] = __fadd_rn(in[e], __fmul_rn(scale, update[e]));
}

// transformer.rope-kv-write / batch-rope-kv-write. Single form: the token
// position is *position and there is one row; batch form: row b is the
// token at control[0] + b, rows b >= control[1] are skipped. Rows whose
// position is outside [0, context) write nothing.
// Multi-stream form (positions non-null): row b is stream b's token at
// positions[b], written into stream b's caches (cache_stride floats apart).
__global__ void rope_kv_kernel(const float *qkv, const int32_t *position, const int32_t *control, const float *freq,
                               float *query, float *key_cache, float *value_cache, int64_t batch, int64_t qsize,
                               int64_t kvsize, int head_size, int rotary, int64_t context, float rope_scale,
                               const int32_t *positions, int64_t cache_stride) {
    pdl_trigger();
    pdl_wait();
    const int64_t width = qsize + 2 * kvsize, count = batch * width;
    const int half = rotary / 2;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = e / width, local = e - row * width;
        int32_t pos;
        int64_t cache_row = 0;
        if (positions) {
            pos = positions[row];
            cache_row = row * cache_stride;
        } else if (control) {
            if (row >= control[1]) continue;
            pos = control[0] + int32_t(row);
        } else {
            pos = *position;
        }
        if (pos < 0 || pos >= context) continue;
        float v = qkv[e];
        const bool is_query = local < qsize, is_key = !is_query && local < qsize + kvsize;
        if (is_query || is_key) {
            const int d = int((is_query ? local : local - qsize) % head_size);
            if (d < rotary) {
                const int ri = d < half ? d : d - half;
                const float other = qkv[d < half ? e + half : e - half];
                const float angle = __fmul_rn(float(pos), freq[ri]);
                const float c = __fmul_rn(cosf(angle), rope_scale), s = __fmul_rn(sinf(angle), rope_scale);
                v = d < half ? __fsub_rn(__fmul_rn(v, c), __fmul_rn(other, s))
                             : __fadd_rn(__fmul_rn(v, c), __fmul_rn(other, s));
            }
            if (is_query) query[row * qsize + local] = v;
            else key_cache[cache_row + int64_t(pos) * kvsize + (local - qsize)] = v;
        } else {
            value_cache[cache_row + int64_t(pos) * kvsize + (local - qsize - kvsize)] = v;
        }
    }
}

// 16-byte asynchronous copies global -> shared (zero-filled when !valid).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    const uint32_t dst = uint32_t(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ---- decode attention --------------------------------------------------------
constexpr int kAttnCluster = 8;

// transformer.rope-kv-write fused into the decode attention (one stream): the
// query and the token's key come from the qkv projection and are rotated on
// the fly with the rope-kv-write arithmetic above; the key and value rows of
// the token are stored into the caches by the CTA whose token range holds the
// position, before it reads them.
struct RopeFuse {
    const float *qkv;   // [query | key | value] of the token
    const float *freq;  // rotary / 2 frequencies
    float *key_cache;   // the caches as written (same buffers the attention reads)
    float *value_cache;
    int64_t qsize, kvsize;
    int rotary;
    float rope_scale;
};

// Element d of one head of qkv after rope (rope_kv_kernel's arithmetic), with
// the scaled cosines / sines of the position's angles in cs[ri], cs[half + ri].
__device__ __forceinline__ float rope_element(const float *head, int d, const float *cs, const RopeFuse &r) {
    const float v = head[d];
    if (d >= r.rotary) return v;
    const int half = r.rotary / 2;
    const int ri = d < half ? d : d - half;
    const float other = head[d < half ? d + half : d - half];
    const float c = cs[ri], sn = cs[half + ri];
    return d < half ? __fsub_rn(__fmul_rn(v, c), __fmul_rn(other, sn)) : __fadd_rn(__fmul_rn(v, c), __fmul_rn(other, sn));
}
// Warps per CTA: 8 for one stream; 4 for several (more clusters fill the
// GPU; measured at 32 Phi-4-14B streams 1198 vs 1025 tok/s, while one
// stream loses with 4: 597 vs 648 tok/s on Phi-4-mini).
constexpr int kAttnWarpsOne = 8, kAttnWarpsMany = 4;

// One cluster of kAttnCluster CTAs per key/value head. Tokens 0..active,
// active = min(max(0, *position), context - 1), are split into contiguous
// per-CTA ranges; inside a CTA each warp takes tiles of kTile tokens and
// keeps an online softmax (running max m, denominator l, weighted values)
// for the G query heads of the group. Lane j holds channels j + 32 i.


// Several streams (a multi-stream session): cluster u serves key/value head
// u % kv_heads of stream u / kv_heads, whose query / output rows are
// q_stride floats apart, caches cache_stride floats apart and whose
// position is position[stream].
template <int NPL, int MAXG, int kTile, int kAttnWarps, bool ROPE>
__global__ void __cluster_dims__(kAttnCluster, 1, 1) __launch_bounds__(kAttnWarps * 32)
    gqa_decode_kernel(const float *query, const float *key_cache, const float *value_cache, const int32_t *position,
                      float *out, int group, int kv_heads, int head_size, int64_t context, float scale,
                      int64_t q_stride, int64_t cache_stride, RopeFuse rf) {
    extern __shared__ float smem[];
    const int G = group, hs = head_size;
    float *w_acc = smem;                                 // [warps][G][hs]
    float *w_m = w_acc + kAttnWarps * G * hs;            // [warps][G]
    float *w_l = w_m + kAttnWarps * G;                   // [warps][G]
    float *c_acc = w_l + kAttnWarps * G;                 // [G][hs]
    float *c_m = c_acc + G * hs;                         // [G]
    float *c_l = c_m + G;                                // [G]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int unit = blockIdx.x / kAttnCluster, kvh = unit % kv_heads, strm = unit / kv_heads;
    query += strm * q_stride;
    out += strm * q_stride;
    key_cache += strm * cache_stride;
    value_cache += strm * cache_stride;
    const uint32_t rank = cta_rank_in_cluster();
    pdl_trigger();
    // Read before the dependency wait: the position (written by an earlier
    // step or a host copy) and every cache row of an earlier token. Only the
    // row at the position is new in this step: written by the preceding
    // rope-kv-write, or (ROPE) taken from this step's qkv.
    const int32_t pos = position[strm];
    int64_t active = pos;
    active = active < 0 ? 0 : (active > context - 1 ? context - 1 : active);
    const int64_t fresh = (pos >= 0 && pos < context) ? int64_t(pos) : -1;
    const int64_t T = active + 1, per = (T + kAttnCluster - 1) / kAttnCluster;
    const int64_t t0 = int64_t(rank) * per, t1 = t0 + per < T ? t0 + per : T;
    const int64_t stride = int64_t(kv_heads) * hs;
    float *rope_cs = c_l + G;  // [rotary]: scaled cos of the half's angles, then scaled sin
    if constexpr (ROPE) {
        const int half = rf.rotary / 2;
        for (int ri = threadIdx.x; ri < half; ri += blockDim.x) {
            const float angle = __fmul_rn(float(pos), rf.freq[ri]);
            rope_cs[ri] = __fmul_rn(cosf(angle), rf.rope_scale);
            rope_cs[half + ri] = __fmul_rn(sinf(angle), rf.rope_scale);
        }
    }
    auto load_tile = [&](int64_t tb, float (&kr)[kTile][NPL], float (&vr)[kTile][NPL], bool skip_fresh) {
#pragma unroll
        for (int u = 0; u < kTile; ++u) {
            const int64_t t = tb + u;
            const bool row_ok = t < t1 && !(skip_fresh && t == fresh);
            const float *kp = key_cache + t * stride + int64_t(kvh) * hs;
            const float *vp = value_cache + t * stride + int64_t(kvh) * hs;
#pragma unroll
            for (int i = 0; i < NPL; ++i) {
                const int d = lane + 32 * i;
                const bool ok = row_ok && d < hs;
                kr[u][i] = ok ? kp[d] : 0.0f;
                vr[u][i] = ok ? vp[d] : 0.0f;
            }
        }
    };
    const int64_t tb0 = t0 + int64_t(warp) * kTile;
    float kr[kTile][NPL], vr[kTile][NPL];
    if (tb0 < t1) load_tile(tb0, kr, vr, true);
    pdl_wait();
    // The new row of this step, in registers: lane channels d = lane + 32 i.
    float kf[NPL], vf[NPL];
    if constexpr (ROPE) {
        __syncthreads();  // the rope table
        const float *kh = rf.qkv + rf.qsize + int64_t(kvh) * hs;
        const float *vh = rf.qkv + rf.qsize + rf.kvsize + int64_t(kvh) * hs;
        const bool mine = fresh >= t0 && fresh < t1;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int d = lane + 32 * i;
            kf[i] = (mine && d < hs) ? rope_element(kh, d, rope_cs, rf) : 0.0f;
            vf[i] = (mine && d < hs) ? vh[d] : 0.0f;
        }
        // the caches keep it for later steps (rope-kv-write writes nothing
        // for a position outside the cache)
        if (mine && warp == 0) {
#pragma unroll
            for (int i = 0; i < NPL; ++i) {
                const int d = lane + 32 * i;
                if (d < hs) {
                    rf.key_cache[fresh * stride + int64_t(kvh) * hs + d] = kf[i];
                    rf.value_cache[fresh * stride + int64_t(kvh) * hs + d] = vf[i];
                }
            }
        }
    }
    float q[MAXG][NPL], acc[MAXG][NPL], m[MAXG], l[MAXG];
#pragma unroll
    for (int g = 0; g < MAXG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int d = lane + 32 * i;
            if constexpr (ROPE)
                q[g][i] = (g < G && d < hs) ? rope_element(rf.qkv + (int64_t(kvh) * G + g) * hs, d, rope_cs, rf)
                                            : 0.0f;
            else
                q[g][i] = (g < G && d < hs) ? query[(int64_t(kvh) * G + g) * hs + d] : 0.0f;
            acc[g][i] = 0.0f;
        }
    }
    for (int64_t tb = tb0; tb < t1; tb += int64_t(kAttnWarps) * kTile) {
        if (tb != tb0) load_tile(tb, kr, vr, false);
        if (fresh >= tb && fresh < tb + kTile && fresh < t1) {
#pragma unroll
            for (int u = 0; u < kTile; ++u) {
                if (tb + u != fresh) continue;
#pragma unroll
                for (int i = 0; i < NPL; ++i) {
                    const int d = lane + 32 * i;
                    if constexpr (ROPE) {
                        kr[u][i] = kf[i];
                        vr[u][i] = vf[i];
                    } else {
                        kr[u][i] = d < hs ? key_cache[fresh * stride + int64_t(kvh) * hs + d] : 0.0f;
                        vr[u][i] = d < hs ? value_cache[fresh * stride + int64_t(kvh) * hs + d] : 0.0f;
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            if (g >= G) break;
            float s[kTile];
            float tile_max = -INFINITY;
#pragma unroll
            for (int u = 0; u < kTile; ++u) {
                float p = 0.0f;
#pragma unroll
                for (int i = 0; i < NPL; ++i) p = __fadd_rn(p, __fmul_rn(q[g][i], kr[u][i]));
                s[u] = __fmul_rn(warp_sum(p), scale);
                if (tb + u < t1) tile_max = fmaxf(tile_max, s[u]);
            }
            const float m_new = fmaxf(m[g], tile_max);
            const float corr = m[g] == -INFINITY ? 0.0f : expf(__fsub_rn(m[g], m_new));
            float lsum = __fmul_rn(l[g], corr);
#pragma unroll
            for (int i = 0; i < NPL; ++i) acc[g][i] = __fmul_rn(acc[g][i], corr);
#pragma unroll
            for (int u = 0; u < kTile; ++u) {
                if (tb + u >= t1) break;
                const float p = expf(__fsub_rn(s[u], m_new));
                lsum = __fadd_rn(lsum, p);
#pragma unroll
                for (int i = 0; i < NPL; ++i) acc[g][i] = __fadd_rn(acc[g][i], __fmul_rn(p, vr[u][i]));
            }
            l[g] = lsum;
            m[g] = m_new;
        }
    }
    // Warp partials -> CTA partial.
#pragma unroll
    for (int g = 0; g < MAXG; ++g) {
        if (g >= G) break;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int d = lane + 32 * i;
            if (d < hs) w_acc[(warp * G + g) * hs + d] = acc[g][i];
        }
        if (lane == 0) {
            w_m[warp * G + g] = m[g];
            w_l[warp * G + g] = l[g];
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * hs; idx += blockDim.x) {
        const int g = idx / hs, d = idx - g * hs;
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, w_m[w * G + g]);
        float A = 0.0f, L = 0.0f;
        if (M != -INFINITY)
            for (int w = 0; w < kAttnWarps; ++w) {
                const float mw = w_m[w * G + g];
                if (mw == -INFINITY) continue;
                const float f = expf(__fsub_rn(mw, M));
                A = __fadd_rn(A, __fmul_rn(w_acc[(w * G + g) * hs + d], f));
                L = __fadd_rn(L, __fmul_rn(w_l[w * G + g], f));
            }
        c_acc[idx] = A;
        if (d == 0) {
            c_m[g] = M;
            c_l[g] = L;
        }
    }
    cluster_sync();
    // CTA partials of the cluster -> output; rank r finishes a slice.
    const int total = G * hs, chunk = (total + kAttnCluster - 1) / kAttnCluster;
    const int lo = int(rank) * chunk, hi = lo + chunk < total ? lo + chunk : total;
    for (int idx = lo + threadIdx.x; idx < hi; idx += blockDim.x) {
        const int g = idx / hs, d = idx - g * hs;
        float mr[kAttnCluster], ar[kAttnCluster], lr[kAttnCluster];
#pragma unroll
        for (int r = 0; r < kAttnCluster; ++r) {  // all 3 x 8 remote loads first
            mr[r] = dsmem_f32(dsmem_addr(c_m + g, uint32_t(r)));
            ar[r] = dsmem_f32(dsmem_addr(c_acc + idx, uint32_t(r)));
            lr[r] = dsmem_f32(dsmem_addr(c_l + g, uint32_t(r)));
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kAttnCluster; ++r) M = fmaxf(M, mr[r]);
        float A = 0.0f, L = 0.0f;
#pragma unroll
        for (int r = 0; r < kAttnCluster; ++r) {
            if (mr[r] == -INFINITY) continue;
            const float f = expf(__fsub_rn(mr[r], M));
            A = __fadd_rn(A, __fmul_rn(ar[r], f));
            L = __fadd_rn(L, __fmul_rn(lr[r], f));
        }
        out[(int64_t(kvh) * G + g) * hs + d] = __fdiv_rn(A, L);
    }
    cluster_sync();  // no CTA leaves while a peer may still read its partials
}

// ---- decode attention with the key/value rows staged in shared memory -------
// One stream. The same cluster of kAttnCluster CTAs per key/value head and the
// same contiguous token ranges as gqa_decode_kernel, but the CTA's cache rows
// are copied into shared memory (cp.async, one warp per row) before the
// dependency wait, and after it every warp works on its own tokens:
//   scores   warp w takes blocks of 32 / MAXG tokens; lane j holds channel
//            quads j (and j + 32 when head_size > 128) of the group's queries
//            in registers and forms the 32 partial dot products (token x
//            query head) of the block, then one reduce-scatter over the lanes
//            (31 shuffles) leaves lane L with the sum of product L;
//   softmax  one warp per query head: running max, rescale, exp, denominator;
//   values   warp w takes tokens w, w + 16, ...; lane j holds channel quads j
//            (and j + 32) of every query head; warp partials summed in warp
//            order.
// The CTA partials (weighted values, max, denominator) go into rank 0's shared
// memory; one cluster-barrier phase later rank 0 forms the per-(CTA, head)
// factors exp(m_r - M) once and merges in rank order. Tokens past the staging
// capacity are taken in further passes (online softmax across passes).
// One stream: 512 threads and up to the 227 KB a CTA may hold (one CTA per
// SM; the kernel is latency-bound). Several streams (thousands of CTAs, a
// throughput problem): 256 threads and at most 113 KB, so two CTAs share an
// SM and one streams its rows while the other computes.
constexpr int kStThreadsOne = 512, kStThreadsMany = 256, kStMaxG = 8;
// CTAs per cluster, i.e. per stream and key/value head (contiguous token
// ranges, partials merged in rank 0): 8 for one stream (short chains); 4 for
// several, so each CTA's fixed phases (prologue, query heads, cluster merge)
// are paid half as often (Phi-4-14B, 32 streams at ~1100 tokens: 130 vs
// 141 us per layer).
constexpr int kStClusterOne = 8, kStClusterMany = 4;
constexpr int kStSmemOne = 227 * 1024, kStSmemMany = 113 * 1024;

struct StLayout {
    int ks, vs, hb, qs, fr, ss, st, cs, sl, slot, total;  // float offsets; total floats
};
// The shared-memory carve-up for G query heads per key/value head, head size
// hs (a multiple of 4), cap staged tokens and a rope table of `rotary`
// floats. Every region starts on a 16-byte boundary.
__host__ __device__ inline StLayout st_layout(int G, int hs, int cap, int rotary, int nw) {
    StLayout L{};
    const int capp = (cap + 31) & ~31;
    int o = 0;
    L.ks = o;  // staged keys [cap][hs]; at the end the warp partials [nw][G][hs]
    o += cap * hs > nw * G * hs ? cap * hs : nw * G * hs;
    L.vs = o;  // staged values [cap][hs]
    o += cap * hs;
    L.hb = o;  // the token's raw q heads, k head, v head
    o += (G + 2) * hs;
    L.qs = o;  // q after rope [G][hs]
    o += G * hs;
    L.fr = o;  // the token's key (after rope) and value [2][hs]
    o += 2 * hs;
    L.ss = o;  // scores, then probabilities [G][capp]; at the end the merge factors [8][8]
    o += G * capp > 64 ? G * capp : 64;
    L.st = o;  // running max [8], denominator [8], rescale [8]
    o += 32;
    L.cs = o;  // rope cos / sin
    o += (rotary + 3) & ~3;
    L.slot = G * hs + 16;  // acc [G][hs], then max at +G*hs, denominator at +G*hs+8
    L.sl = o;              // rank 0: one slot per CTA of the cluster
    o += kAttnCluster * L.slot;
    L.total = o;
    return L;
}

__device__ __forceinline__ void dsmem_st_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Several streams: cluster u serves key/value head u % kv_heads of stream
// u / kv_heads, whose query / output rows are q_stride floats apart, caches
// cache_stride floats apart and whose position is position[stream].
struct StagedAttn {
    const float *query;  // without rope: the query vector
    const float *key_cache, *value_cache;
    const int32_t *position;
    float *out;
    int group, kv_heads, head_size, cap;
    int64_t context, q_stride, cache_stride;
    float scale;
};

// NQ: float4 channel quads per lane in the value pass (head_size <= 32 * 4 NQ).
template <int MAXG, int NQ, bool ROPE, int NT, int CL>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(NT, NT == kStThreadsOne ? 1 : 2)
    gqa_decode_staged_kernel(const StagedAttn a, const RopeFuse rf) {
    constexpr int kStThreads = NT, kStWarps = NT / 32;
    extern __shared__ __align__(16) float sm[];
    const int G = a.group, hs = a.head_size, hs4 = hs >> 2;
    const int cap = a.cap, capp = (cap + 31) & ~31;
    const StLayout L = st_layout(G, hs, cap, ROPE ? rf.rotary : 0, kStWarps);
    float *Ks = sm + L.ks, *Vs = sm + L.vs, *hb = sm + L.hb, *qs = sm + L.qs, *fr = sm + L.fr, *Ss = sm + L.ss,
          *stat = sm + L.st, *cs = sm + L.cs, *slots = sm + L.sl;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int unit = blockIdx.x / CL, kvh = unit % a.kv_heads, strm = unit / a.kv_heads;
    const uint32_t rank = cta_rank_in_cluster();
    // First cluster-barrier phase: arrived here, waited before the first
    // store into rank 0's shared memory (every CTA of the cluster has started).
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
    pdl_trigger();
    // Before the dependency wait: the position and every cache row of an
    // earlier token (written by earlier steps). The row at the position is
    // this step's: from the qkv vector (ROPE) or from the preceding
    // rope-kv-write.
    const int32_t pos = a.position[strm];
    int64_t active = pos;
    active = active < 0 ? 0 : (active > a.context - 1 ? a.context - 1 : active);
    const int64_t fresh = (pos >= 0 && pos < a.context) ? int64_t(pos) : -1;
    const int64_t T = active + 1, per = (T + CL - 1) / CL;
    const int64_t t0 = int64_t(rank) * per, t1 = t0 + per < T ? t0 + per : T;
    const int64_t stride = int64_t(a.kv_heads) * hs;
    const float *kbase = a.key_cache + strm * a.cache_stride + int64_t(kvh) * hs;
    const float *vbase = a.value_cache + strm * a.cache_stride + int64_t(kvh) * hs;
    // rows c0 .. c0 + n - 1 of the CTA's range of one cache into dst, one
    // warp per row, as one copy group (the fresh row is written from
    // registers instead)
    auto stage = [&](float *dst, const float *base, int64_t c0, int n) {
        for (int r = warp; r < n; r += kStWarps) {
            const int64_t t = c0 + r;
            if (t == fresh) continue;
            const float *src = base + t * stride;
            for (int c = lane; c < hs4; c += 32) cp_async16(dst + r * hs + 4 * c, src + 4 * c, true);
        }
        cp_async_commit();
    };
    const int n0 = t1 - t0 < int64_t(cap) ? int(t1 - t0) : cap;  // <= 0: no tokens for this CTA
    if (n0 > 0) {
        stage(Ks, kbase, t0, n0);
        stage(Vs, vbase, t0, n0);
    }
    if (tid < 8) {
        stat[tid] = -INFINITY;
        stat[8 + tid] = 0.0f;
        stat[16 + tid] = 0.0f;
    }
    if constexpr (ROPE) {
        const int half = rf.rotary / 2;
        for (int ri = tid; ri < half; ri += kStThreads) {
            const float angle = __fmul_rn(float(pos), rf.freq[ri]);
            cs[ri] = __fmul_rn(cosf(angle), rf.rope_scale);
            cs[half + ri] = __fmul_rn(sinf(angle), rf.rope_scale);
        }
    }
    pdl_wait();
    const bool mine = fresh >= t0 && fresh < t1;
    {
        // the token's heads, one memory round trip
        const float *qsrc = (ROPE ? rf.qkv : a.query + strm * a.q_stride) + int64_t(kvh) * G * hs;
        float4 *hb4 = reinterpret_cast<float4 *>(hb);
        for (int i = tid; i < G * hs4; i += kStThreads) hb4[i] = *reinterpret_cast<const float4 *>(qsrc + 4 * i);
        if (mine && tid < 2 * hs4) {
            const bool isv = tid >= hs4;
            const int c = isv ? tid - hs4 : tid;
            const float *src;
            if constexpr (ROPE) src = rf.qkv + rf.qsize + (isv ? rf.kvsize : 0) + int64_t(kvh) * hs + 4 * c;
            else src = (isv ? vbase : kbase) + fresh * stride + 4 * c;
            hb4[G * hs4 + tid] = *reinterpret_cast<const float4 *>(src);
        }
    }
    __syncthreads();
    for (int i = tid; i < G * hs; i += kStThreads) {
        if constexpr (ROPE) {
            const int g = i / hs, d = i - g * hs;
            qs[i] = rope_element(hb + g * hs, d, cs, rf);
        } else {
            qs[i] = hb[i];
        }
    }
    if (mine) {
        for (int d = tid; d < hs; d += kStThreads) {
            float kf = hb[G * hs + d];
            if constexpr (ROPE) kf = rope_element(hb + G * hs, d, cs, rf);
            const float vf = hb[(G + 1) * hs + d];
            fr[d] = kf;
            fr[hs + d] = vf;
            if (fresh < t0 + n0) {
                Ks[int(fresh - t0) * hs + d] = kf;
                Vs[int(fresh - t0) * hs + d] = vf;
            }
            if constexpr (ROPE) {  // rope-kv-write's stores (nothing for a position outside the cache)
                rf.key_cache[fresh * stride + int64_t(kvh) * hs + d] = kf;
                rf.value_cache[fresh * stride + int64_t(kvh) * hs + d] = vf;
            }
        }
    }
    __syncthreads();  // qs
    // the group's queries in registers: lane j holds channel quads j + 32 i
    float4 qr[MAXG][NQ], acc[MAXG][NQ];
#pragma unroll
    for (int g = 0; g < MAXG; ++g)
#pragma unroll
        for (int j = 0; j < NQ; ++j) {
            const int c = lane + 32 * j;
            qr[g][j] = (g < G && c < hs4) ? reinterpret_cast<const float4 *>(qs + g * hs)[c]
                                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            acc[g][j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    // Passes of up to cap tokens. Copy groups in commit order: keys and
    // values of pass 0, then per pass the next pass's keys (issued once the
    // scores are done with Ks) and its values (once the value sums are done
    // with Vs), so the next pass's rows stream in under this pass's work.
    for (int64_t c0 = t0; c0 < t1; c0 += cap) {
        const int n = t1 - c0 < int64_t(cap) ? int(t1 - c0) : cap;
        const int64_t c1 = c0 + cap;
        const int n1 = c1 < t1 ? (t1 - c1 < int64_t(cap) ? int(t1 - c1) : cap) : 0;
        cp_async_wait<1>();  // this pass's keys (its values may still be in flight)
        __syncthreads();
        // scores: blocks of TPW tokens per warp, 32 products per block
        constexpr int TPW = 32 / MAXG;
        for (int tb = warp * TPW; tb < n; tb += kStWarps * TPW) {
            float v[32];  // product g * TPW + u
#pragma unroll
            for (int u = 0; u < TPW; ++u) {
                const int t = tb + u < n ? tb + u : n - 1;  // past the end: a repeated row, result unused
                float4 k4[NQ];
#pragma unroll
                for (int j = 0; j < NQ; ++j) {
                    const int c = lane + 32 * j;
                    k4[j] = c < hs4 ? reinterpret_cast<const float4 *>(Ks + t * hs)[c]
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int g = 0; g < MAXG; ++g) {
                    float sc = 0.0f;
#pragma unroll
                    for (int j = 0; j < NQ; ++j) {
                        sc = __fmaf_rn(qr[g][j].x, k4[j].x, sc);
                        sc = __fmaf_rn(qr[g][j].y, k4[j].y, sc);
                        sc = __fmaf_rn(qr[g][j].z, k4[j].z, sc);
                        sc = __fmaf_rn(qr[g][j].w, k4[j].w, sc);
                    }
                    v[g * TPW + u] = sc;
                }
            }
            // reduce-scatter over the lanes: after the level of offset o, a
            // lane keeps the half of the products selected by its bit o
            // (summed with the partner's); lane L ends with product L
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const bool up = (lane & o) != 0;
#pragma unroll
                for (int k = 0; k < o; ++k) {
                    const float send = up ? v[k] : v[k + o];
                    const float keep = up ? v[k + o] : v[k];
                    v[k] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
                }
            }
            const int g = lane / TPW, t = tb + lane % TPW;
            if (g < G && t < n) Ss[g * capp + t] = __fmul_rn(v[0], a.scale);
        }
        __syncthreads();  // Ks is free: the next pass's keys
        if (n1 > 0) {
            stage(Ks, kbase, c1, n1);
            if (fresh >= c1 && fresh < c1 + n1)
                for (int d = tid; d < hs; d += kStThreads) Ks[int(fresh - c1) * hs + d] = fr[d];
        }
        if (warp < G) {
            const int g = warp;
            float mx = -INFINITY;
            for (int t = lane; t < n; t += 32) mx = fmaxf(mx, Ss[g * capp + t]);
            mx = warp_max(mx);
            const float m_old = stat[g], m_new = fmaxf(m_old, mx);
            const float corr = m_old == -INFINITY ? 0.0f : expf(__fsub_rn(m_old, m_new));
            float ls = 0.0f;
            for (int t = lane; t < n; t += 32) {
                const float p = expf(__fsub_rn(Ss[g * capp + t], m_new));
                Ss[g * capp + t] = p;
                ls = __fadd_rn(ls, p);
            }
            ls = warp_sum(ls);
            __syncwarp();
            if (lane == 0) {
                stat[8 + g] = __fadd_rn(__fmul_rn(stat[8 + g], corr), ls);
                stat[g] = m_new;
                stat[16 + g] = corr;
            }
        }
        if (n1 > 0)
            cp_async_wait<1>();  // this pass's values (the next pass's keys may still be in flight)
        else
            cp_async_wait<0>();
        __syncthreads();
        {
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                if (g >= G) break;
                const float corr = stat[16 + g];
#pragma unroll
                for (int j = 0; j < NQ; ++j) {
                    acc[g][j].x = __fmul_rn(acc[g][j].x, corr);
                    acc[g][j].y = __fmul_rn(acc[g][j].y, corr);
                    acc[g][j].z = __fmul_rn(acc[g][j].z, corr);
                    acc[g][j].w = __fmul_rn(acc[g][j].w, corr);
                }
            }
#pragma unroll 2
            for (int t = warp; t < n; t += kStWarps) {
                float4 v4[NQ];
#pragma unroll
                for (int j = 0; j < NQ; ++j) {
                    const int c = lane + 32 * j;
                    v4[j] = c < hs4 ? reinterpret_cast<const float4 *>(Vs + t * hs)[c]
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int g = 0; g < MAXG; ++g) {
                    if (g >= G) break;
                    const float p = Ss[g * capp + t];
#pragma unroll
                    for (int j = 0; j < NQ; ++j) {
                        acc[g][j].x = __fmaf_rn(p, v4[j].x, acc[g][j].x);
                        acc[g][j].y = __fmaf_rn(p, v4[j].y, acc[g][j].y);
                        acc[g][j].z = __fmaf_rn(p, v4[j].z, acc[g][j].z);
                        acc[g][j].w = __fmaf_rn(p, v4[j].w, acc[g][j].w);
                    }
                }
            }
        }
        if (n1 > 0) {
            __syncthreads();  // Vs is free: the next pass's values
            stage(Vs, vbase, c1, n1);
            if (fresh >= c1 && fresh < c1 + n1)
                for (int d = tid; d < hs; d += kStThreads) Vs[int(fresh - c1) * hs + d] = fr[hs + d];
        }
    }
    cp_async_wait<0>();  // a CTA without tokens staged nothing; one with tokens has waited already
    __syncthreads();     // every pass done with Ks: it takes the warp partials now
    float *red = Ks;
    {
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            if (g >= G) break;
#pragma unroll
            for (int j = 0; j < NQ; ++j) {
                const int c = lane + 32 * j;
                if (c < hs4) reinterpret_cast<float4 *>(red + (warp * G + g) * hs)[c] = acc[g][j];
            }
        }
    }
    __syncthreads();
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
    const uint32_t slot0 = dsmem_addr(slots + int(rank) * L.slot, 0);
    for (int i = tid; i < G * hs; i += kStThreads) {
        float A = 0.0f;
#pragma unroll
        for (int w = 0; w < kStWarps; ++w) A = __fadd_rn(A, red[w * G * hs + i]);
        dsmem_st_f32(slot0 + 4u * uint32_t(i), A);
    }
    if (tid < G) {
        dsmem_st_f32(slot0 + 4u * uint32_t(G * hs + tid), stat[tid]);
        dsmem_st_f32(slot0 + 4u * uint32_t(G * hs + 8 + tid), stat[8 + tid]);
    }
    // Second phase: the partials are in rank 0. Ranks 1.. leave (only rank
    // 0's shared memory is read remotely); rank 0 waits and merges.
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
    if (rank != 0) return;
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
    float *fac = Ss;  // [rank][8]: exp(m_r - M) for each query head (0 for a CTA without tokens)
    if (tid < CL * G) {
        const int r = tid / G, g = tid - r * G;
        float M = -INFINITY;
#pragma unroll
        for (int r2 = 0; r2 < CL; ++r2) M = fmaxf(M, slots[r2 * L.slot + G * hs + g]);
        const float mr = slots[r * L.slot + G * hs + g];
        fac[r * 8 + g] = mr == -INFINITY ? 0.0f : expf(__fsub_rn(mr, M));
    }
    __syncthreads();
    for (int i = tid; i < G * hs; i += kStThreads) {
        const int g = i / hs;
        float A = 0.0f, Lsum = 0.0f;
#pragma unroll
        for (int r = 0; r < CL; ++r) {
            const float f = fac[r * 8 + g];
            A = __fadd_rn(A, __fmul_rn(slots[r * L.slot + i], f));
            Lsum = __fadd_rn(Lsum, __fmul_rn(slots[r * L.slot + G * hs + 8 + g], f));
        }
        a.out[strm * a.q_stride + int64_t(kvh) * G * hs + i] = __fdiv_rn(A, Lsum);
    }
}

// ---- unfused attention instructions (single and batch forms) --------------
// transformer.gqa-scores / batch-gqa-scores. Single form (control null):
// active = *position and the token test is the instruction's unsigned
// token <= uint(active). Batch form: rows b < control[1], active =
// control[0] + b and a negative active scores nothing.
__global__ void gqa_scores_kernel(const float *query, const float *key_cache, const int32_t *position,
                                  const int32_t *control, float *scores, int64_t batch, int query_heads, int group,
                                  int kv_heads, int head_size, int64_t context, float scale) {
    pdl_trigger();
    pdl_wait();
    const int64_t count = batch * query_heads * context;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = e / (int64_t(query_heads) * context);
        const int64_t local = e - row * query_heads * context;
        const int head = int(local / context);
        const int64_t token = local - int64_t(head) * context;
        bool take;
        if (control) {
            if (row >= control[1]) continue;
            const int32_t active = control[0] + int32_t(row);
            take = active >= 0 && uint32_t(token) <= uint32_t(active);
        } else {
            take = uint32_t(token) <= uint32_t(*position);
        }
        float s = kNegMax;
        if (take) {
            const int kvh = head / group;
            const float *qp = query + (row * query_heads + head) * head_size;
            const float *kp = key_cache + (token * kv_heads + kvh) * head_size;
            s = 0.0f;
            for (int d = 0; d < head_size; ++d) s = __fadd_rn(s, __fmul_rn(qp[d], kp[d]));
            s = __fmul_rn(s, scale);
        }
        scores[e] = s;
    }
}

// transformer.causal-softmax / batch-causal-softmax: one CTA per (row, head).
__global__ void causal_softmax_kernel(const float *scores, const int32_t *position, const int32_t *control,
                                      float *probs, int heads, int64_t context) {
    __shared__ float red[33];
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.x / heads;
    int32_t active;
    bool valid = true;
    if (control) {
        if (row >= control[1]) return;
        active = control[0] + int32_t(row);
        valid = active >= 0;
    } else {
        active = *position;
    }
    const float *s = scores + int64_t(blockIdx.x) * context;
    float *p = probs + int64_t(blockIdx.x) * context;
    float mx = kNegMax;
    if (valid)
        for (int64_t t = threadIdx.x; uint32_t(t) <= uint32_t(active) && t < context; t += blockDim.x) mx = fmaxf(mx, s[t]);
    // block max
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : kNegMax;
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) red[32] = v;
    }
    __syncthreads();
    const float maximum = red[32];
    __syncthreads();
    float sum = 0.0f;
    if (valid)
        for (int64_t t = threadIdx.x; uint32_t(t) <= uint32_t(active) && t < context; t += blockDim.x)
            sum = __fadd_rn(sum, expf(__fsub_rn(s[t], maximum)));
    const float denominator = block_sum(sum, red);
    for (int64_t t = threadIdx.x; t < context; t += blockDim.x)
        p[t] = valid && uint32_t(t) <= uint32_t(active) ? __fdiv_rn(expf(__fsub_rn(s[t], maximum)), denominator) : 0.0f;
}

// transformer.gqa-values / batch-gqa-values: one thread per output element.
__global__ void gqa_values_kernel(const float *probs, const float *value_cache, const int32_t *position,
                                  const int32_t *control, float *out, int64_t batch, int query_heads, int group,
                                  int kv_heads, int head_size, int64_t context) {
    pdl_trigger();
    pdl_wait();
    const int64_t width = int64_t(query_heads) * head_size, count = batch * width;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = e / width, local = e - row * width;
        const int head = int(local / head_size), d = int(local - int64_t(head) * head_size);
        int32_t active;
        bool valid = true;
        if (control) {
            if (row >= control[1]) continue;
            active = control[0] + int32_t(row);
            valid = active >= 0;
        } else {
            active = *position;
        }
        const int kvh = head / group;
        const float *pp = probs + (row * query_heads + head) * context;
        float s = 0.0f;
        if (valid)
            for (int64_t t = 0; uint32_t(t) <= uint32_t(active) && t < context; ++t)
                s = __fadd_rn(s, __fmul_rn(pp[t], value_cache[(t * kv_heads + kvh) * head_size + d]));
        out[e] = s;
    }
}

// ---- prefill attention ---------------------------------------------------------
// batch-gqa-scores -> batch-causal-softmax -> batch-gqa-values of a prefill
// chunk in one pass, without the [batch, heads, context] score and
// probability buffers: row b (position start + b, b < count) of query head h
// attends cache tokens 0..start + b of key/value head h / group with an
// online softmax (running maximum and denominator per row, the accumulator
// rescaled when the maximum grows). One CTA = kPfRows query rows of one
// head; key/value tiles of kPfKeys tokens are double-buffered in shared
// memory with cp.async. 128 threads as 8 x 16: thread (ty, tx) scores rows
// ty + 8 i against keys tx + 16 j and accumulates rows ty + 8 i, columns
// 4 tx + 64 c of the output. 32-row tiles (not 64) halve the longest CTA of
// the causal triangle, which sets the kernel's time: a 512-token
// Phi-4-mini prefill measured 13.1 ms against 15.1 ms.
constexpr int kPfRows = 32;
constexpr int kPfKeys = 32;
constexpr int kPfThreads = 128;
constexpr int kPfRowStride = kPfThreads / 16;  // rows ty, ty + stride, .. (4 per thread)
static_assert(kPfRows == 4 * kPfRowStride, "four rows per thread");


template <int HS>
__global__ void __launch_bounds__(kPfThreads, HS <= 128 ? 4 : 2)
prefill_attention_kernel(const float *__restrict__ query, const float *__restrict__ key_cache,
                         const float *__restrict__ value_cache, int32_t start, int32_t count, float *__restrict__ out,
                         int query_heads, int group, int kv_heads, float scale) {
    constexpr int QS = HS + 4;       // padded row stride of the query and key tiles
    constexpr int PS = kPfKeys + 4;  // padded row stride of the probability tile
    constexpr int C4 = HS / 64;      // float4 output columns per thread
    constexpr int JK = kPfKeys / 16; // keys per thread per tile
    extern __shared__ __align__(16) float pf_smem[];
    float *qs = pf_smem;                       // [kPfRows][QS]
    float *ks = qs + kPfRows * QS;             // [2][kPfKeys][QS]
    float *vs = ks + 2 * kPfKeys * QS;         // [2][kPfKeys][HS]
    float *ps = vs + 2 * kPfKeys * HS;         // [kPfRows][PS]
    pdl_trigger();
    pdl_wait();
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int head = blockIdx.x, kvh = head / group;
    // heavier (later) row tiles first
    const int row0 = (int(gridDim.y) - 1 - int(blockIdx.y)) * kPfRows;
    const int last_row = min(row0 + kPfRows, count) - 1;
    const int64_t qstride = int64_t(query_heads) * HS, kstride = int64_t(kv_heads) * HS;
    const int nkeys = start + last_row + 1;
    const int tiles = (nkeys + kPfKeys - 1) / kPfKeys;

    auto load_tile = [&](int t, int buf) {
        float *kd = ks + buf * kPfKeys * QS, *vd = vs + buf * kPfKeys * HS;
        for (int e = tid; e < kPfKeys * (HS / 4); e += kPfThreads) {
            const int key = e / (HS / 4), c = (e - key * (HS / 4)) * 4;
            const int token = t * kPfKeys + key;
            const bool valid = token < nkeys;
            const int64_t off = valid ? int64_t(token) * kstride + int64_t(kvh) * HS + c : 0;
            cp_async16(kd + key * QS + c, key_cache + off, valid);
            cp_async16(vd + key * HS + c, value_cache + off, valid);
        }
        cp_async_commit();
    };
    load_tile(0, 0);
    for (int e = tid; e < kPfRows * (HS / 4); e += kPfThreads) {
        const int r = e / (HS / 4), c = (e - r * (HS / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row0 + r < count) v = *reinterpret_cast<const float4 *>(query + int64_t(row0 + r) * qstride +
                                                                      int64_t(head) * HS + c);
        *reinterpret_cast<float4 *>(qs + r * QS + c) = v;
    }

    float acc[4][C4 * 4];
    float mrow[4], lrow[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        mrow[i] = -INFINITY;
        lrow[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < C4 * 4; ++c) acc[i][c] = 0.0f;
    }
    for (int t = 0; t < tiles; ++t) {
        const int buf = t & 1;
        if (t + 1 < tiles) {
            load_tile(t + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *kt = ks + buf * kPfKeys * QS, *vt = vs + buf * kPfKeys * HS;
        float sc[4][JK];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < JK; ++j) sc[i][j] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < HS; d += 4) {
            float4 q[4], k[JK];
#pragma unroll
            for (int i = 0; i < 4; ++i) q[i] = *reinterpret_cast<const float4 *>(qs + (ty + kPfRowStride * i) * QS + d);
#pragma unroll
            for (int j = 0; j < JK; ++j) k[j] = *reinterpret_cast<const float4 *>(kt + (tx + 16 * j) * QS + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < JK; ++j) {
                    sc[i][j] = fmaf(q[i].x, k[j].x, sc[i][j]);
                    sc[i][j] = fmaf(q[i].y, k[j].y, sc[i][j]);
                    sc[i][j] = fmaf(q[i].z, k[j].z, sc[i][j]);
                    sc[i][j] = fmaf(q[i].w, k[j].w, sc[i][j]);
                }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = row0 + ty + kPfRowStride * i;
            const int active = start + row;  // tokens 0..active
            float tile_max = -INFINITY;
#pragma unroll
            for (int j = 0; j < JK; ++j) {
                const int token = t * kPfKeys + tx + 16 * j;
                const bool valid = row < count && token <= active;
                sc[i][j] = valid ? sc[i][j] * scale : -INFINITY;
                tile_max = fmaxf(tile_max, sc[i][j]);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) tile_max = fmaxf(tile_max, __shfl_xor_sync(0xffffffffu, tile_max, o));
            const float m_new = fmaxf(mrow[i], tile_max);
            // all keys of this row masked so far: nothing to rescale or add
            const float alpha = m_new == -INFINITY ? 1.0f : expf(mrow[i] - m_new);
            mrow[i] = m_new;
            lrow[i] *= alpha;
#pragma unroll
            for (int c = 0; c < C4 * 4; ++c) acc[i][c] *= alpha;
#pragma unroll
            for (int j = 0; j < JK; ++j) {
                const float p = sc[i][j] == -INFINITY ? 0.0f : expf(sc[i][j] - m_new);
                lrow[i] += p;
                ps[(ty + kPfRowStride * i) * PS + tx + 16 * j] = p;
            }
        }
        __syncthreads();
#pragma unroll 2
        for (int key = 0; key < kPfKeys; key += 4) {
            float4 p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = *reinterpret_cast<const float4 *>(ps + (ty + kPfRowStride * i) * PS + key);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                for (int c = 0; c < C4; ++c) {
                    const float4 v = *reinterpret_cast<const float4 *>(vt + (key + kk) * HS + 4 * tx + 64 * c);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float pv = kk == 0 ? p[i].x : kk == 1 ? p[i].y : kk == 2 ? p[i].z : p[i].w;
                        acc[i][4 * c + 0] = fmaf(pv, v.x, acc[i][4 * c + 0]);
                        acc[i][4 * c + 1] = fmaf(pv, v.y, acc[i][4 * c + 1]);
                        acc[i][4 * c + 2] = fmaf(pv, v.z, acc[i][4 * c + 2]);
                        acc[i][4 * c + 3] = fmaf(pv, v.w, acc[i][4 * c + 3]);
                    }
                }
            }
        }
        __syncthreads();  // the tile's buffers and the probabilities are rewritten next
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float l = lrow[i];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        const int row = row0 + ty + kPfRowStride * i;
        if (row >= count) continue;
        const float inv = 1.0f / l;
        float *dst = out + int64_t(row) * qstride + int64_t(head) * HS;
#pragma unroll
        for (int c = 0; c < C4; ++c)
            *reinterpret_cast<float4 *>(dst + 4 * tx + 64 * c) =
                make_float4(acc[i][4 * c] * inv, acc[i][4 * c + 1] * inv, acc[i][4 * c + 2] * inv,
                            acc[i][4 * c + 3] * inv);
    }
}

// ---- argmax -----------------------------------------------------------------
constexpr int kArgmaxCluster = 8;
constexpr int kArgmaxThreads = 1024;

// The instruction's merge rule: a candidate replaces the best when greater,
// or equal with a smaller index (GpuTransformerInstructionCollection.cs:697-744).
__device__ __forceinline__ void argmax_merge(float &b, uint32_t &bi, float o, uint32_t oi) {
    if (o > b || (o == b && oi < bi)) {
        b = o;
        bi = oi;
    }
}

// transformer.argmax over one 8-CTA cluster per row (rows n floats apart;
// one row unless a multi-stream session runs one per stream). With `feed`
// set (device-side greedy loop) it also records the token and prepares the
// next step's control: position + 1 and the next prompt token or the
// argmax. With `sfeed` (multi-stream greedy loop) row b records its token
// in stream b's history, and sets stream b's next token and position.
__global__ void __cluster_dims__(kArgmaxCluster, 1, 1) __launch_bounds__(kArgmaxThreads)
    argmax_kernel(const float *in, int64_t n, int32_t *out, DecodeFeed *feed, StreamsFeed *sfeed) {
    __shared__ float sb[32];
    __shared__ uint32_t si[32];
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.x / kArgmaxCluster;
    in += row * n;
    float b = kNegMax;
    uint32_t bi = 0;
    const int64_t stride = int64_t(kArgmaxCluster) * blockDim.x;
    for (int64_t j = (blockIdx.x % kArgmaxCluster) * int64_t(blockDim.x) + threadIdx.x; j < n; j += stride)
        argmax_merge(b, bi, in[j], uint32_t(j));
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, b, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(b, bi, ob, oi);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sb[warp] = b;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        b = lane < int(blockDim.x >> 5) ? sb[lane] : kNegMax;
        bi = lane < int(blockDim.x >> 5) ? si[lane] : 0u;
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, b, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(b, bi, ob, oi);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        sb[0] = b;
        si[0] = bi;
    }
    cluster_sync();
    if (cta_rank_in_cluster() == 0 && threadIdx.x == 0) {
        float best = sb[0];
        uint32_t idx = si[0];
        for (uint32_t r = 1; r < kArgmaxCluster; ++r)
            argmax_merge(best, idx, dsmem_f32(dsmem_addr(sb, r)), dsmem_u32(dsmem_addr(si, r)));
        out[row] = int32_t(idx);
        if (feed) {
            const int32_t pos = feed->control[1], k = pos - feed->base;
            if (k >= 0 && k < feed->capacity) feed->history[k] = int32_t(idx);
            feed->control[1] = pos + 1;
            feed->control[0] = k + 1 < feed->prompt_tokens ? feed->prompt[k + 1] : int32_t(idx);
        }
        if (sfeed) {
            const int32_t pos = sfeed->positions[row], k = pos - sfeed->start[row];
            if (k >= 0 && k < sfeed->capacity) sfeed->history[int64_t(k) * sfeed->streams + row] = int32_t(idx);
            sfeed->positions[row] = pos + 1;
            sfeed->tokens[row] = int32_t(idx);
        }
    }
    cluster_sync();  // rank 0 has read every CTA's candidate
}

// transformer.batch-select-last: out = input row control[1] - 1.
__global__ void select_last_kernel(const float *in, const int32_t *control, float *out, int64_t batch, int64_t width) {
    pdl_trigger();
    pdl_wait();
    const int32_t valid = control[1];
    if (valid <= 0 || valid > batch) return;
    for (int64_t c = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; c < width; c += int64_t(gridDim.x) * blockDim.x)
        out[c] = in[int64_t(valid - 1) * width + c];
}

// transformer.batch-gather-rows: output row b = table row control[0] + b.
__global__ void gather_rows_kernel(const float *table, int64_t rows, const int32_t *control, float *out, int64_t batch,
                                   int64_t width) {
    pdl_trigger();
    pdl_wait();
    const int64_t count = batch * width;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < count; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = e / width, col = e - row * width, src = int64_t(control[0]) + row;
        if (row < control[1] && src >= 0 && src < rows) out[e] = table[src * width + col];
    }
}

// ---- launch helpers -----------------------------------------------------------
int sm_count_cached() { return device_sm_count(); }

int elementwise_grid(int64_t count, int threads) {
    const int64_t blocks = (count + threads - 1) / threads;
    const int64_t cap = int64_t(sm_count_cached()) * 8;
    return int(std::max<int64_t>(1, std::min(blocks, cap)));
}

template <class... KArgs, class... Args>
si_status launch(const char *what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void *stream,
                 Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return SI_OK;
}

}  // namespace

si_status tr_gather_row(uint32_t type, const void *table, int64_t rows, int64_t cols, const int32_t *index, float *out,
                        void *stream) {
    uint64_t row_bytes = 0;
    if (si_status st = byte_length(type, uint64_t(cols), &row_bytes)) return st;
    return launch("core.gather-row", gather_row_kernel, dim3(elementwise_grid(cols, 256)), dim3(256), 0, stream, type,
                  static_cast<const uint8_t *>(table), rows, cols, row_bytes, index, out);
}

si_status tr_gather_rows_quant(uint32_t type, const void *table, int64_t rows, int64_t cols, const int32_t *indices,
                               int64_t count, float *out, void *stream) {
    uint64_t row_bytes = 0;
    if (si_status st = byte_length(type, uint64_t(cols), &row_bytes)) return st;
    return launch("core.gather-row", gather_rows_quant_kernel, dim3(elementwise_grid(count * cols, 256)), dim3(256), 0,
                  stream, type, static_cast<const uint8_t *>(table), rows, cols, row_bytes, indices, count, out);
}

si_status tr_embedding_gather_batch(const uint16_t *table, int64_t rows, const int32_t *indices, float *out,
                                    int64_t batch, int64_t width, void *stream) {
    const int64_t count = batch * width;
    return launch("transformer.embedding-gather-batch", embedding_gather_batch_kernel,
                  dim3(elementwise_grid(count, 256)), dim3(256), 0, stream, reinterpret_cast<const __half *>(table),
                  rows, indices, out, count, width);
}

si_status tr_copy_rows(const float *in, float *out, int64_t count, void *stream) {
    return launch("transformer.copy-embedding-rows", copy_rows_kernel, dim3(elementwise_grid(count, 256)), dim3(256),
                  0, stream, in, out, count);
}

si_status tr_rms_norm(const float *in, const float *residual, const float *weight, const int32_t *control,
                      float *updated, float *out, int64_t batch, int64_t width, float eps, void *stream) {
    // enough threads for kRmsHeld elements each: fewer warps to reduce over
    // (3072-wide rows: 384 threads; Phi-4-mini decode 648 vs 632 tok/s with
    // 1024 threads, 590 with 12 elements per thread)
    const int64_t want = (width + kRmsHeld - 1) / kRmsHeld;
    const int threads = int(std::min<int64_t>(1024, std::max<int64_t>(32, (want + 31) / 32 * 32)));
    if (residual)
        return launch("transformer.residual-rms-norm", rms_norm_kernel<true>, dim3(unsigned(batch)), dim3(threads), 0,
                      stream, in, residual, weight, control, updated, out, width, eps);
    return launch("transformer.rms-norm", rms_norm_kernel<false>, dim3(unsigned(batch)), dim3(threads), 0, stream, in,
                  residual, weight, control, updated, out, width, eps);
}

si_status tr_swiglu(const float *gate_up, const int32_t *control, float *out, int64_t batch, int64_t width,
                    void *stream) {
    // 128-thread CTAs: twice the CTAs of 256 for a decode row (more loads in
    // flight); Phi-4-mini decode 659 vs 648 tok/s with rope-kv-write alike
    return launch("transformer.swiglu", swiglu_kernel, dim3(elementwise_grid(batch * width, 128)), dim3(128), 0,
                  stream, gate_up, control, out, batch, width);
}

si_status tr_scaled_add(const float *in, const float *update, float *out, int64_t count, float scale, void *stream) {
    return launch("transformer.scaled-add", scaled_add_kernel, dim3(elementwise_grid(count, 256)), dim3(256), 0,
                  stream, in, update, out, count, scale);
}

si_status tr_rope_kv_write(const float *qkv, const int32_t *position, const int32_t *control, const float *freq,
                           float *query, float *key_cache, float *value_cache, int64_t batch, int64_t qsize,
                           int64_t kvsize, int head_size, int rotary, int64_t context, float rope_scale,
                           void *stream) {
    const int64_t count = batch * (qsize + 2 * kvsize);
    return launch("transformer.rope-kv-write", rope_kv_kernel, dim3(elementwise_grid(count, 128)), dim3(128), 0,
                  stream, qkv, position, control, freq, query, key_cache, value_cache, batch, qsize, kvsize, head_size,
                  rotary, context, rope_scale, static_cast<const int32_t *>(nullptr), int64_t(0));
}

si_status tr_rope_kv_write_streams(const float *qkv, const int32_t *positions, const float *freq, float *query,
                                   float *key_cache, float *value_cache, int64_t streams, int64_t qsize,
                                   int64_t kvsize, int head_size, int rotary, int64_t context, int64_t cache_stride,
                                   float rope_scale, void *stream) {
    const int64_t count = streams * (qsize + 2 * kvsize);
    return launch("transformer.rope-kv-write", rope_kv_kernel, dim3(elementwise_grid(count, 128)), dim3(128), 0,
                  stream, qkv, static_cast<const int32_t *>(nullptr), static_cast<const int32_t *>(nullptr), freq,
                  query, key_cache, value_cache, streams, qsize, kvsize, head_size, rotary, context, rope_scale,
                  positions, cache_stride);
}

namespace {
template <int NPL, int MAXG, int kTile, int kAttnWarps, bool ROPE = false>
si_status launch_gqa(const float *query, const float *kc, const float *vc, const int32_t *position, float *out,
                     int group, int kv_heads, int head_size, int64_t context, float scale, int streams,
                     int64_t q_stride, int64_t cache_stride, void *stream, const RopeFuse &rf = RopeFuse{}) {
    auto kernel = gqa_decode_kernel<NPL, MAXG, kTile, kAttnWarps, ROPE>;
    const size_t smem = size_t(kAttnWarps * group * head_size + 2 * kAttnWarps * group + group * head_size +
                               2 * group + (ROPE ? rf.rotary : 0)) * sizeof(float);
    if (smem > 48 * 1024) {
        if (const int ae = opt_in_smem(reinterpret_cast<const void *>(kernel), 200 * 1024))
            return fail(SI_ERR_CUDA, "attention shared-memory opt-in failed: %s", cudaGetErrorString(cudaError_t(ae)));
    }
    return launch("transformer.grouped-query-attention", kernel, dim3(unsigned(streams * kv_heads * kAttnCluster)),
                  dim3(kAttnWarps * 32), smem, stream, query, kc, vc, position, out, group, kv_heads, head_size,
                  context, scale, q_stride, cache_stride, rf);
}
}  // namespace

namespace {
// Tokens per staging pass of gqa_decode_staged_kernel<.., NT> for this
// shape (the most a CTA takes at the cache's last position, as far as the
// shared-memory limit of that thread count holds them), or 0 when the shape
// needs the register-tile kernel.
template <int NT, int CL>
int staged_cap(int group, int head_size, int64_t context, int rotary) {
    if (group < 1 || group > kStMaxG || head_size < 4 || head_size > 256 || head_size % 4 != 0) return 0;
    if (group > 4 && head_size > 128) return 0;  // 8 x 2 channel quads of queries and sums: beyond the registers
    const size_t limit = size_t(NT == kStThreadsOne ? kStSmemOne : kStSmemMany);
    int cap = int(std::min<int64_t>((context + CL - 1) / CL, 1024));
    while (cap > 0 && size_t(st_layout(group, head_size, cap, rotary, NT / 32).total) * sizeof(float) > limit)
        cap -= cap > 64 ? 16 : 1;
    return cap;
}

template <bool ROPE, int NT, int CL>
si_status launch_staged(const StagedAttn &a, const RopeFuse &rf, int streams, void *stream) {
    auto kernel = a.head_size > 128 ? gqa_decode_staged_kernel<4, 2, ROPE, NT, CL>
                  : a.group <= 4      ? gqa_decode_staged_kernel<4, 1, ROPE, NT, CL>
                                      : gqa_decode_staged_kernel<kStMaxG, 1, ROPE, NT, CL>;
    const int smem =
        st_layout(a.group, a.head_size, a.cap, ROPE ? rf.rotary : 0, NT / 32).total * int(sizeof(float));
    if (const int ae = opt_in_smem(reinterpret_cast<const void *>(kernel), smem))
        return fail(SI_ERR_CUDA, "attention shared-memory opt-in failed: %s", cudaGetErrorString(cudaError_t(ae)));
    return launch("transformer.grouped-query-attention", kernel,
                  dim3(unsigned(int64_t(streams) * a.kv_heads * CL)), dim3(NT), size_t(smem), stream, a,
                  rf);
}
}  // namespace

si_status tr_attention_decode_rope(const float *qkv, const int32_t *position, const float *freq, float *kc, float *vc,
                                   float *out, int query_heads, int kv_heads, int head_size, int rotary,
                                   int64_t context, float rope_scale, void *stream) {
    const int group = query_heads / kv_heads;
    const float scale = 1.0f / sqrtf(float(head_size));
    const int npl = (head_size + 31) / 32;
    const int64_t qsize = int64_t(query_heads) * head_size, kvsize = int64_t(kv_heads) * head_size;
    const RopeFuse rf{qkv, freq, kc, vc, qsize, kvsize, rotary, rope_scale};
    if (const int cap = staged_cap<kStThreadsOne, kStClusterOne>(group, head_size, context, rotary))
        return launch_staged<true, kStThreadsOne, kStClusterOne>(
            StagedAttn{nullptr, kc, vc, position, out, group, kv_heads, head_size, cap, context, 0, 0, scale}, rf, 1,
            stream);
#define SI_GQA_R(NPL, MAXG, TILE)                                                                               \
    launch_gqa<NPL, MAXG, TILE, kAttnWarpsOne, true>(qkv, kc, vc, position, out, group, kv_heads, head_size,      \
                                                     context, scale, 1, qsize, 0, stream, rf)
    if (group <= 4) {
        if (npl <= 1) return SI_GQA_R(1, 4, 8);
        if (npl <= 2) return SI_GQA_R(2, 4, 8);
        if (npl <= 4) return SI_GQA_R(4, 4, 8);
        return SI_GQA_R(8, 4, 4);
    }
    if (npl <= 1) return SI_GQA_R(1, 8, 8);
    if (npl <= 2) return SI_GQA_R(2, 8, 4);
    if (npl <= 4) return SI_GQA_R(4, 8, 4);
    return SI_GQA_R(8, 8, 2);
#undef SI_GQA_R
}

si_status tr_attention_decode(const float *query, const float *kc, const float *vc, const int32_t *position, float *out,
                              int query_heads, int kv_heads, int head_size, int64_t context, void *stream) {
    return tr_attention_decode_streams(query, kc, vc, position, out, 1, query_heads, kv_heads, head_size, context, 0,
                                       stream);
}

si_status tr_attention_decode_streams(const float *query, const float *kc, const float *vc, const int32_t *position,
                                      float *out, int streams, int query_heads, int kv_heads, int head_size,
                                      int64_t context, int64_t cache_stride, void *stream) {
    const int group = query_heads / kv_heads;
    const float scale = 1.0f / sqrtf(float(head_size));
    const int npl = (head_size + 31) / 32;
    const int64_t q_stride = int64_t(query_heads) * head_size;
    if (streams == 1) {
        if (const int cap = staged_cap<kStThreadsOne, kStClusterOne>(group, head_size, context, 0))
            return launch_staged<false, kStThreadsOne, kStClusterOne>(
                StagedAttn{query, kc, vc, position, out, group, kv_heads, head_size, cap, context, 0, 0, scale},
                RopeFuse{}, 1, stream);
    } else if (const int cap = staged_cap<kStThreadsMany, kStClusterMany>(group, head_size, context, 0)) {
        return launch_staged<false, kStThreadsMany, kStClusterMany>(StagedAttn{query, kc, vc, position, out, group, kv_heads,
                                                               head_size, cap, context, q_stride, cache_stride, scale},
                                                    RopeFuse{}, streams, stream);
    }
#define SI_GQA(NPL, MAXG, TILE)                                                                                \
    (streams > 1 ? launch_gqa<NPL, MAXG, TILE, kAttnWarpsMany>(query, kc, vc, position, out, group, kv_heads,      \
                                                               head_size, context, scale, streams, q_stride,      \
                                                               cache_stride, stream)                              \
                 : launch_gqa<NPL, MAXG, TILE, kAttnWarpsOne>(query, kc, vc, position, out, group, kv_heads,       \
                                                              head_size, context, scale, streams, q_stride,       \
                                                              cache_stride, stream))
    if (group <= 4) {
        if (npl <= 1) return SI_GQA(1, 4, 8);
        if (npl <= 2) return SI_GQA(2, 4, 8);
        if (npl <= 4) return SI_GQA(4, 4, 8);
        return SI_GQA(8, 4, 4);
    }
    if (npl <= 1) return SI_GQA(1, 8, 8);
    if (npl <= 2) return SI_GQA(2, 8, 4);
    if (npl <= 4) return SI_GQA(4, 8, 4);
    return SI_GQA(8, 8, 2);
#undef SI_GQA
}

si_status tr_gqa_scores(const float *query, const float *kc, const int32_t *position, const int32_t *control,
                        float *scores, int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context,
                        void *stream) {
    const int64_t count = batch * query_heads * context;
    return launch("transformer.gqa-scores", gqa_scores_kernel, dim3(elementwise_grid(count, 256)), dim3(256), 0,
                  stream, query, kc, position, control, scores, batch, query_heads, query_heads / kv_heads, kv_heads,
                  head_size, context, 1.0f / sqrtf(float(head_size)));
}

namespace {
template <int HS>
si_status launch_prefill_attention(const float *query, const float *kc, const float *vc, int32_t start, int32_t count,
                                   float *out, int query_heads, int kv_heads, void *stream) {
    constexpr size_t smem = size_t(kPfRows * (HS + 4) + 2 * kPfKeys * (HS + 4) + 2 * kPfKeys * HS +
                                   kPfRows * (kPfKeys + 4)) * sizeof(float);
    if (const int ae = opt_in_smem(reinterpret_cast<const void *>(prefill_attention_kernel<HS>), int(smem)))
        return fail(SI_ERR_CUDA, "prefill attention shared-memory opt-in failed: %s",
                    cudaGetErrorString(cudaError_t(ae)));
    const dim3 grid(unsigned(query_heads), unsigned((count + kPfRows - 1) / kPfRows));
    return launch("transformer.batch-grouped-query-attention", prefill_attention_kernel<HS>, grid, dim3(kPfThreads),
                  smem, stream, query, kc, vc, start, count, out, query_heads, query_heads / kv_heads, kv_heads,
                  1.0f / sqrtf(float(HS)));
}
}  // namespace

bool tr_prefill_attention_supported(int head_size) {
    return head_size == 64 || head_size == 128 || head_size == 192 || head_size == 256;
}

si_status tr_prefill_attention(const float *query, const float *kc, const float *vc, int32_t start, int32_t count,
                               float *out, int query_heads, int kv_heads, int head_size, int64_t context,
                               void *stream) {
    if (count <= 0) return SI_OK;
    if ((int64_t(count) + kPfRows - 1) / kPfRows > 65535)
        return fail(SI_ERR_UNSUPPORTED, "prefill attention takes at most %d rows per call", 65535 * kPfRows);
    if (start < 0 || int64_t(start) + count > context)
        return fail(SI_ERR_INVALID_ARGUMENT, "prefill rows [%d, %d) outside the context of %lld", start,
                    start + count, (long long)context);
    for (const void *p : {static_cast<const void *>(query), static_cast<const void *>(kc),
                          static_cast<const void *>(vc), static_cast<const void *>(out)})
        if (reinterpret_cast<uintptr_t>(p) % 16)
            return fail(SI_ERR_INVALID_ARGUMENT, "prefill attention buffers must be 16-byte aligned");
    switch (head_size) {
    case 64: return launch_prefill_attention<64>(query, kc, vc, start, count, out, query_heads, kv_heads, stream);
    case 128: return launch_prefill_attention<128>(query, kc, vc, start, count, out, query_heads, kv_heads, stream);
    case 192: return launch_prefill_attention<192>(query, kc, vc, start, count, out, query_heads, kv_heads, stream);
    case 256: return launch_prefill_attention<256>(query, kc, vc, start, count, out, query_heads, kv_heads, stream);
    default: return fail(SI_ERR_UNSUPPORTED, "prefill attention supports head sizes 64, 128, 192 and 256");
    }
}

si_status tr_causal_softmax(const float *scores, const int32_t *position, const int32_t *control, float *probs,
                            int64_t batch, int heads, int64_t context, void *stream) {
    return launch("transformer.causal-softmax", causal_softmax_kernel, dim3(unsigned(batch * heads)), dim3(256), 0,
                  stream, scores, position, control, probs, heads, context);
}

si_status tr_gqa_values(const float *probs, const float *vc, const int32_t *position, const int32_t *control,
                        float *out, int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context,
                        void *stream) {
    const int64_t count = batch * query_heads * head_size;
    return launch("transformer.gqa-values", gqa_values_kernel, dim3(elementwise_grid(count, 256)), dim3(256), 0,
                  stream, probs, vc, position, control, out, batch, query_heads, query_heads / kv_heads, kv_heads,
                  head_size, context);
}

si_status tr_argmax(const float *in, int64_t n, int32_t *out, DecodeFeed *feed, void *stream) {
    return launch("transformer.argmax", argmax_kernel, dim3(kArgmaxCluster), dim3(kArgmaxThreads), 0, stream, in, n,
                  out, feed, static_cast<StreamsFeed *>(nullptr));
}

si_status tr_argmax_rows(const float *in, int64_t rows, int64_t n, int32_t *out, StreamsFeed *sfeed, void *stream) {
    return launch("transformer.argmax", argmax_kernel, dim3(unsigned(rows * kArgmaxCluster)), dim3(kArgmaxThreads), 0,
                  stream, in, n, out, static_cast<DecodeFeed *>(nullptr), sfeed);
}

si_status tr_select_last(const float *in, const int32_t *control, float *out, int64_t batch, int64_t width,
                         void *stream) {
    return launch("transformer.batch-select-last", select_last_kernel, dim3(elementwise_grid(width, 256)), dim3(256),
                  0, stream, in, control, out, batch, width);
}

si_status tr_gather_rows(const float *table, int64_t rows, const int32_t *control, float *out, int64_t batch,
                         int64_t width, void *stream) {
    return launch("transformer.batch-gather-rows", gather_rows_kernel, dim3(elementwise_grid(batch * width, 256)),
                  dim3(256), 0, stream, table, rows, control, out, batch, width);
}

}  // namespace si::kernels
