// Persistent decode step: the whole Phi-4 decode program of one token
// (Phi4D3D12TextSession.cs:866-920) as one cooperative launch, one CTA per
// SM. The program becomes a list of phases separated by grid-wide arrival
// counters:
//
//   gather    hidden = token_embedding[token] (+ per-CTA sums of squares)
//   per layer:
//     GEMV    qkv = W_qkv rms(hidden)              (norm scale from the sums)
//     ATTN    per (kv head, token chunk): rope of q / k, the key and value
//             rows of the token stored, an online softmax over the chunk
//     COMBINE attention = the chunks' partials merged
//     GEMV    after = hidden + W_o attention        (+ sums of squares)
//     GEMV    gate_up = W_up rms(after)
//     GEMV    hidden = after + W_down swiglu(gate_up) (+ sums of squares)
//   GEMV      logits = token_embedding rms(hidden)  (+ per-CTA best row)
//   ARGMAX    next token (CTA 0)
//
// Every projection's weights stream through one shared-memory ring: the
// producer warp issues the tiles (16 rows x up to 16 superblocks, one bulk
// copy per row) of all GEMV phases in program order and never waits for an
// activation, so the weight stream runs ahead across phase boundaries while
// the compute warps wait for the previous phase. Sixteen compute warps run
// the phases (the tensor-core GEMV of gemv_core.cuh, one superblock column
// each); the reducer warp sums the column partials of every row in a fixed
// order, adds the residual, stores the row and keeps the row statistics.
//
// Every wait is bounded: the grid barrier polls with a time limit and on
// expiry sets the device error word and an abort flag that makes all later
// waits return at once; the ring's mbarrier waits are bounded as in the
// stand-alone GEMV. The launch is cooperative (all CTAs co-resident).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "device_common.cuh"
#include "gemv_core.cuh"
#include "si_internal.h"

namespace si::dev {
namespace {

constexpr int kSC = 16;                   // compute warps
constexpr int kSThreads = (kSC + 2) * 32; // + producer warp kSC, reducer warp kSC + 1
constexpr int kSRows = 16;                // rows per weight tile
constexpr int kSAttnTile = 2;             // tokens per warp step of the attention phase
constexpr int kSMaxG = 4;                 // query heads per key/value head
constexpr int kSNpl = 4;                  // head channels per lane (head_size <= 128)
constexpr int kStageVec = 4;              // float4 per thread when a GEMV input is staged: K <= 8192
constexpr uint32_t kErrStepBarrierTimeout = 32u;
constexpr uint64_t kStepWaitLimitNs = 1000000000ull;  // 1 s per grid barrier

enum : int { kPhGather = 0, kPhGemv = 1, kPhAttention = 2, kPhCombine = 3, kPhArgmax = 4 };

struct StepPhase {
    int kind;
    int mode;        // GEMV input: 0 as is, 1 x * s * norm (s from `stats`), 2 swiglu of [gate | up]
    int rows;
    int nsb;         // superblocks of a full row (K / 256)
    int kchunks;     // K chunks per row tile (1 or 2)
    int nsb_tile;    // superblocks per chunk
    int row_tiles;
    int layer;       // attention: the layer's caches
    uint32_t row_bytes, chunk_bytes, row_stride;
    int argmax;      // track the best row (vocabulary projection)
    const uint8_t *w;
    const float *x;
    const float *norm;
    const float *stats;  // mode 1: per-CTA partial sums of squares of x (gridDim entries)
    float *y;
    const float *resid;  // y = resid + W x when non-null
    float *stats_out;    // per-CTA sum of squares of the stored rows (null: none)
};

struct StepParams {
    const StepPhase *phases;
    int num_phases;
    int stages;
    uint32_t stage_bytes;
    uint32_t attn_smem_off;  // offsets into dynamic shared memory
    uint32_t part_off, bars_off, scratch_off;
    // model
    int hidden, qh, kvh, hs, rotary, group, attn_chunks, vocab;
    int64_t context;
    float eps, rope_scale, attn_scale;
    const float *freq;
    float *const *key_cache;
    float *const *value_cache;
    const float *qkv;
    float *attention;
    float *ws_acc, *ws_m, *ws_l;  // [items][group][hs], [items][group]
    const uint8_t *embedding;
    uint32_t embedding_type;
    uint64_t embedding_row_bytes;
    float *hidden_out;
    float *gather_stats;
    float *amax_val;
    uint32_t *amax_idx;
    int32_t *control;
    int32_t *next_token;
    kernels::DecodeFeed *feed;
    unsigned long long *bar;  // arrivals, zeroed before every launch
    uint32_t *abort;          // nonzero: every later wait returns at once
    // Optional phase trace (null: off), zeroed before every launch: for
    // CTAs 0, 1 and the last, per phase 8 entries at
    // trace[(slot * num_phases + phase) * 8]: %globaltimer after the grid
    // wait, after the compute warps' work, after the arrival; then the ns
    // compute warp 0 waited on full / pempty, the producer on empty and the
    // reducer on pfull; entry 7: GEMV phases, the %globaltimer when the
    // tiles start (input staged and loaded).
    unsigned long long *trace;
};

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Barrier 1: the compute warps. Barrier 2: compute warps + reducer (phase end).
__device__ __forceinline__ void compute_sync() { named_sync(1, kSC * 32); }
__device__ __forceinline__ void phase_end_sync() { named_sync(2, (kSC + 1) * 32); }

// Waits until `target` arrivals (all CTAs finished the earlier phases), or
// the abort flag, or the time limit (which raises the abort flag).
__device__ void grid_wait(const StepParams &P, unsigned long long target) {
    if (threadIdx.x == 0 && !*reinterpret_cast<volatile uint32_t *>(P.abort)) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t polls = 0;
        while (ld_acquire_u64(P.bar) < target) {
            if (*reinterpret_cast<volatile uint32_t *>(P.abort)) break;
            if (++polls > kMaxPolls || globaltimer_ns() - t0 > kStepWaitLimitNs) {
                atomicOr(&g_error_word, kErrStepBarrierTimeout);
                atomicExch(P.abort, 1u);
                break;
            }
        }
    }
    compute_sync();
}

__device__ __forceinline__ float table_element(uint32_t type, const uint8_t *row, int64_t c) {
    switch (type) {
    case SI_TYPE_F32: return reinterpret_cast<const float *>(row)[c];
    case SI_TYPE_F16: return __half2float(reinterpret_cast<const __half *>(row)[c]);
    case SI_TYPE_Q8_0: {
        const uint8_t *b = row + (c >> 5) * kQ8_0Bytes;
        return __fmul_rn(__half2float(*reinterpret_cast<const __half *>(b)), float(int8_t(b[2 + (c & 31)])));
    }
    default: {
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

// Sum of the gridDim per-CTA partials in one fixed order (every warp of
// every CTA derives the same value).
// All loads are issued before the first add (one round trip); gridDim.x <= 32 * kMaxGridSlices.
constexpr int kMaxGridSlices = 5;
__device__ __forceinline__ float sum_partials(const float *stats, int lane) {
    float v[kMaxGridSlices];
#pragma unroll
    for (int j = 0; j < kMaxGridSlices; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < int(gridDim.x) ? __ldcg(stats + i) : 0.0f;
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxGridSlices; ++j) s = __fadd_rn(s, v[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    return s;
}

__device__ __forceinline__ void argmax_merge(float &b, uint32_t &bi, float o, uint32_t oi) {
    if (o > b || (o == b && oi < bi)) {
        b = o;
        bi = oi;
    }
}

// ---- compute-warp phases ---------------------------------------------------------
__device__ void gather_phase(const StepParams &P, float *red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int32_t tok = *reinterpret_cast<volatile int32_t *>(P.control);
    const bool ok = tok >= 0 && tok < P.vocab;
    const uint8_t *row = P.embedding + (ok ? uint64_t(tok) * P.embedding_row_bytes : 0);
    const int per = (P.hidden + int(gridDim.x) - 1) / int(gridDim.x);
    const int e0 = int(blockIdx.x) * per, e1 = min(P.hidden, e0 + per);
    float ss = 0.0f;
    for (int e = e0 + tid; e < e1; e += kSC * 32) {
        const float v = ok ? table_element(P.embedding_type, row, e) : __int_as_float(0x7fc00000);
        P.hidden_out[e] = v;
        ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) red[warp] = ss;
    compute_sync();
    if (tid == 0) {
        float t = 0.0f;
        for (int w = 0; w < kSC; ++w) t = __fadd_rn(t, red[w]);
        P.gather_stats[blockIdx.x] = t;
    }
}

__device__ __forceinline__ float rope_value(const float *head, int d, int rotary, int32_t pos, const float *freq,
                                            float rope_scale) {
    const float v = __ldcg(head + d);
    if (d >= rotary) return v;
    const int half = rotary >> 1, ri = d < half ? d : d - half;
    const float other = __ldcg(head + (d < half ? d + half : d - half));
    const float angle = __fmul_rn(float(pos), freq[ri]);
    const float c = __fmul_rn(cosf(angle), rope_scale), s = __fmul_rn(sinf(angle), rope_scale);
    return d < half ? __fsub_rn(__fmul_rn(v, c), __fmul_rn(other, s)) : __fadd_rn(__fmul_rn(v, c), __fmul_rn(other, s));
}

// One (kv head, token chunk) item per CTA: rope of the group's query heads,
// the token's key / value rows stored by the CTA that owns the token, an
// online softmax per warp over tiles of kSAttnTile tokens, the CTA's
// partial (max, denominator, weighted values) to the workspace.
__device__ void attention_phase(const StepParams &P, const StepPhase &f, float *sm) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = P.group, hs = P.hs, chunks = P.attn_chunks;
    const int item = int(blockIdx.x);
    const bool busy = item < P.kvh * chunks;
    const int h = busy ? item / chunks : 0, c = busy ? item % chunks : 0;
    const int32_t pos = *reinterpret_cast<volatile int32_t *>(P.control + 1);
    const int64_t T = int64_t(pos) + 1, per = (T + chunks - 1) / chunks;
    const int64_t t0 = int64_t(c) * per, t1 = t0 + per < T ? t0 + per : T;
    float *kc = P.key_cache[f.layer], *vc = P.value_cache[f.layer];
    const int64_t stride = int64_t(P.kvh) * hs;
    const int64_t qsize = int64_t(P.qh) * hs;
    float *w_acc = sm;                            // [kSC][G][hs]
    float *w_m = w_acc + kSC * G * hs;            // [kSC][G]
    float *w_l = w_m + kSC * G;                   // [kSC][G]
    float *qs = w_l + kSC * G;                    // [G][hs] rotated query heads
    // One pass (one round trip): the group's query heads rotated into shared
    // memory; the CTA that owns the token also rotates its key and stores
    // the key / value rows.
    const bool owner = busy && t0 <= int64_t(pos) && int64_t(pos) < t1;
    const float *kin = P.qkv + qsize + int64_t(h) * hs;
    const int n1 = busy ? G * hs + (owner ? 2 * hs : 0) : 0;
    for (int i = tid; i < n1; i += kSC * 32) {
        if (i < G * hs) {
            const int g = i / hs, d = i - g * hs;
            qs[i] = rope_value(P.qkv + (int64_t(h) * G + g) * hs, d, P.rotary, pos, P.freq, P.rope_scale);
        } else if (i < G * hs + hs) {
            const int d = i - G * hs;
            kc[int64_t(pos) * stride + int64_t(h) * hs + d] = rope_value(kin, d, P.rotary, pos, P.freq, P.rope_scale);
        } else {
            const int d = i - G * hs - hs;
            vc[int64_t(pos) * stride + int64_t(h) * hs + d] = __ldcg(kin + stride + d);
        }
    }
    compute_sync();  // the token's rows and the rotated queries are read below
    float acc[kSMaxG][kSNpl], m[kSMaxG], l[kSMaxG];
#pragma unroll
    for (int g = 0; g < kSMaxG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < kSNpl; ++i) acc[g][i] = 0.0f;
    }
    if (busy) {
        for (int64_t tb = t0 + int64_t(warp) * kSAttnTile; tb < t1; tb += int64_t(kSC) * kSAttnTile) {
            float kr[kSAttnTile][kSNpl], vr[kSAttnTile][kSNpl];
#pragma unroll
            for (int u = 0; u < kSAttnTile; ++u) {
                const int64_t t = tb + u;
                const float *kp = kc + t * stride + int64_t(h) * hs;
                const float *vp = vc + t * stride + int64_t(h) * hs;
#pragma unroll
                for (int i = 0; i < kSNpl; ++i) {
                    const int d = lane + 32 * i;
                    const bool okk = t < t1 && d < hs;
                    kr[u][i] = okk ? __ldcg(kp + d) : 0.0f;
                    vr[u][i] = okk ? __ldcg(vp + d) : 0.0f;
                }
            }
#pragma unroll
            for (int g = 0; g < kSMaxG; ++g) {
                if (g >= G) break;
                float sc[kSAttnTile];
                float tmax = -INFINITY;
#pragma unroll
                for (int u = 0; u < kSAttnTile; ++u) {
                    float p = 0.0f;
#pragma unroll
                    for (int i = 0; i < kSNpl; ++i) {
                        const int d = lane + 32 * i;
                        p = __fadd_rn(p, __fmul_rn(d < hs ? qs[g * hs + d] : 0.0f, kr[u][i]));
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, o));
                    sc[u] = __fmul_rn(p, P.attn_scale);
                    if (tb + u < t1) tmax = fmaxf(tmax, sc[u]);
                }
                const float mn = fmaxf(m[g], tmax);
                const float corr = m[g] == -INFINITY ? 0.0f : expf(__fsub_rn(m[g], mn));
                float ls = __fmul_rn(l[g], corr);
#pragma unroll
                for (int i = 0; i < kSNpl; ++i) acc[g][i] = __fmul_rn(acc[g][i], corr);
#pragma unroll
                for (int u = 0; u < kSAttnTile; ++u) {
                    if (tb + u >= t1) break;
                    const float p = expf(__fsub_rn(sc[u], mn));
                    ls = __fadd_rn(ls, p);
#pragma unroll
                    for (int i = 0; i < kSNpl; ++i) acc[g][i] = __fadd_rn(acc[g][i], __fmul_rn(p, vr[u][i]));
                }
                l[g] = ls;
                m[g] = mn;
            }
        }
    }
#pragma unroll
    for (int g = 0; g < kSMaxG; ++g) {
        if (g >= G) break;
#pragma unroll
        for (int i = 0; i < kSNpl; ++i) {
            const int d = lane + 32 * i;
            if (d < hs) w_acc[(warp * G + g) * hs + d] = acc[g][i];
        }
        if (lane == 0) {
            w_m[warp * G + g] = m[g];
            w_l[warp * G + g] = l[g];
        }
    }
    compute_sync();
    if (busy) {
        for (int idx = tid; idx < G * hs; idx += kSC * 32) {
            const int g = idx / hs, d = idx - g * hs;
            float M = -INFINITY;
            for (int w = 0; w < kSC; ++w) M = fmaxf(M, w_m[w * G + g]);
            float A = 0.0f, L = 0.0f;
            if (M != -INFINITY)
                for (int w = 0; w < kSC; ++w) {
                    const float mw = w_m[w * G + g];
                    if (mw == -INFINITY) continue;
                    const float e = expf(__fsub_rn(mw, M));
                    A = __fadd_rn(A, __fmul_rn(w_acc[(w * G + g) * hs + d], e));
                    L = __fadd_rn(L, __fmul_rn(w_l[w * G + g], e));
                }
            P.ws_acc[(int64_t(item) * G + g) * hs + d] = A;
            if (d == 0) {
                P.ws_m[item * G + g] = M;
                P.ws_l[item * G + g] = L;
            }
        }
    }
    compute_sync();  // the scratch is reused by the next phase
}

// attention[e] for this CTA's slice: the chunks of its kv head merged, one
// warp per element, the chunks spread over the lanes (one round trip).
constexpr int kMaxChunkSlices = 5;  // chunks <= 32 * kMaxChunkSlices
__device__ void combine_phase(const StepParams &P) {
    const int G = P.group, hs = P.hs, chunks = P.attn_chunks;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int Q = P.qh * hs, per = (Q + int(gridDim.x) - 1) / int(gridDim.x);
    const int e0 = int(blockIdx.x) * per, e1 = min(Q, e0 + per);
    for (int e = e0 + warp; e < e1; e += kSC) {
        const int head = e / hs, d = e - head * hs, h = head / G, g = head - h * G;
        float mc[kMaxChunkSlices], lc[kMaxChunkSlices], ac[kMaxChunkSlices];
#pragma unroll
        for (int j = 0; j < kMaxChunkSlices; ++j) {
            const int c = lane + 32 * j, it = h * chunks + c;
            const bool ok = c < chunks;
            mc[j] = ok ? __ldcg(P.ws_m + it * G + g) : -INFINITY;
            lc[j] = ok ? __ldcg(P.ws_l + it * G + g) : 0.0f;
            ac[j] = ok ? __ldcg(P.ws_acc + (int64_t(it) * G + g) * hs + d) : 0.0f;
        }
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < kMaxChunkSlices; ++j) M = fmaxf(M, mc[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float A = 0.0f, L = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxChunkSlices; ++j) {
            if (mc[j] == -INFINITY) continue;
            const float w = expf(__fsub_rn(mc[j], M));
            A = __fadd_rn(A, __fmul_rn(ac[j], w));
            L = __fadd_rn(L, __fmul_rn(lc[j], w));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            A = __fadd_rn(A, __shfl_xor_sync(0xffffffffu, A, o));
            L = __fadd_rn(L, __shfl_xor_sync(0xffffffffu, L, o));
        }
        if (lane == 0) P.attention[e] = __fdiv_rn(A, L);
    }
}

__device__ void argmax_phase(const StepParams &P) {
    if (blockIdx.x != 0 || threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    float b = -3.402823466e+38f;
    uint32_t bi = 0;
    for (int i = lane; i < int(gridDim.x); i += 32) argmax_merge(b, bi, __ldcg(P.amax_val + i), __ldcg(P.amax_idx + i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, b, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(b, bi, ob, oi);
    }
    if (lane == 0) {
        *P.next_token = int32_t(bi);
        if (kernels::DecodeFeed *feed = P.feed) {
            const int32_t pos = feed->control[1], k = pos - feed->base;
            if (k >= 0 && k < feed->capacity) feed->history[k] = int32_t(bi);
            feed->control[1] = pos + 1;
            feed->control[0] = k + 1 < feed->prompt_tokens ? feed->prompt[k + 1] : int32_t(bi);
        }
    }
}

__device__ __forceinline__ unsigned long long *trace_row(const StepParams &P, int ph) {
    if (!P.trace) return nullptr;
    const int slot = blockIdx.x == 0 ? 0 : (blockIdx.x == 1 ? 1 : (blockIdx.x == gridDim.x - 1 ? 2 : -1));
    return slot < 0 ? nullptr : P.trace + (size_t(slot) * P.num_phases + ph) * 8;
}

template <class Path>
struct GemvCursor {
    int s = 0, it = 0;
    uint32_t ring_phase = 0;
};

// The compute warps' part of a GEMV phase: x fragments of this warp's
// superblock column(s), then every (row tile, chunk) of this CTA from the ring.
template <class Path>
__device__ void gemv_compute(const StepParams &P, const StepPhase &f, uint8_t *smem, GemvCursor<Path> &cur,
                             uint8_t *scratch, unsigned long long *trace) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.bars_off);
    uint64_t *empty = full + P.stages;
    uint64_t *pfull = empty + P.stages;
    uint64_t *pempty = pfull + 2;
    float *part = reinterpret_cast<float *>(smem + P.part_off);  // [2][kSC][kSRows]
    const bool active = warp < f.nsb_tile;
    const int64_t K = int64_t(f.nsb) * 256;
    const bool aborted = *reinterpret_cast<volatile uint32_t *>(P.abort) != 0;
    // The input of each of this warp's superblock columns, transformed
    // (mode 1: x * s * norm with s from the producing phase's sums of
    // squares; mode 2: swiglu of [gate | up]), goes through a per-warp
    // shared-memory buffer: every global load of the warp is issued before
    // any is used (one round trip), then the fragments are built from the
    // buffer as the load paths do from memory.
    float *wbuf = reinterpret_cast<float *>(smem + P.attn_smem_off) + warp * 256;
    typename Path::State st0, st1;
    if (active && !aborted) {
        float4 a[2 * 2], b[2 * 2];
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int64_t i = int64_t(c * f.nsb_tile + warp) * 256 + 8 * lane + 4 * j;
                const bool ok = c < f.kchunks;
                a[2 * c + j] = ok ? __ldcg(reinterpret_cast<const float4 *>(f.x + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
                b[2 * c + j] = ok && f.mode != 0
                                   ? __ldcg(reinterpret_cast<const float4 *>((f.mode == 2 ? f.x + K : f.norm) + i))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        float scale = 1.0f;
        if (f.mode == 1) scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sum_partials(f.stats, lane), float(K)), P.eps));
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            if (c >= f.kchunks) break;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float4 x4 = a[2 * c + j], y4 = b[2 * c + j];
                float4 v = x4;
                if (f.mode == 2)
                    v = make_float4(XSrc<2, 1>::swish_mul(x4.x, y4.x), XSrc<2, 1>::swish_mul(x4.y, y4.y),
                                    XSrc<2, 1>::swish_mul(x4.z, y4.z), XSrc<2, 1>::swish_mul(x4.w, y4.w));
                else if (f.mode == 1)
                    v = make_float4(__fmul_rn(__fmul_rn(x4.x, scale), y4.x), __fmul_rn(__fmul_rn(x4.y, scale), y4.y),
                                    __fmul_rn(__fmul_rn(x4.z, scale), y4.z), __fmul_rn(__fmul_rn(x4.w, scale), y4.w));
                *reinterpret_cast<float4 *>(wbuf + 8 * lane + 4 * j) = v;
            }
            __syncwarp();
            const XSrc<0, 2> X{wbuf, nullptr, nullptr, 1.0f, 256};
            Path::load(X, 0, lane, c == 0 ? st0 : st1, scratch, 0, 1);
            __syncwarp();  // the buffer is rewritten for the next chunk
        }
    }
    if (trace) trace[7] = globaltimer_ns();
    const int g = lane >> 2, t = lane & 3, mq = lane >> 3;
    const uint32_t off_ldsm = uint32_t((mq & 1) * 8 + (lane & 7)) * f.row_stride + uint32_t(mq >> 1) * 16u +
                              Path::kQsOffset + Path::kColBytes * uint32_t(warp);
    const uint32_t off_g = uint32_t(g) * f.row_stride + Path::kColBytes * uint32_t(warp);
    const uint32_t off_g8 = uint32_t(g + 8) * f.row_stride + Path::kColBytes * uint32_t(warp);
    uint8_t *ring = smem;
    for (int rt = int(blockIdx.x); rt < f.row_tiles; rt += int(gridDim.x)) {
        for (int c = 0; c < f.kchunks; ++c, ++cur.it) {
            const int b = cur.it & 1;
            const uint64_t w0 = trace ? globaltimer_ns() : 0;
            mbar_wait(&full[cur.s], cur.ring_phase, kErrFullBarrierTimeout);
            const uint64_t w1 = trace ? globaltimer_ns() : 0;
            const uint8_t *stage = ring + size_t(cur.s) * P.stage_bytes;
            if (cur.it >= 2) mbar_wait(&pempty[b], ((cur.it >> 1) - 1) & 1, kErrEpilogueTimeout);
            if (trace) trace[3] += w1 - w0, trace[4] += globaltimer_ns() - w1;
            float *pw = part + (b * kSC + warp) * kSRows;
            if (active && !aborted) {
                float2 v = Path::rows16(smem_u32(stage) + off_ldsm, stage + off_g, stage + off_g8, lane,
                                        c == 0 ? st0 : st1, scratch);
                v.x += __shfl_xor_sync(0xffffffffu, v.x, 1);
                v.y += __shfl_xor_sync(0xffffffffu, v.y, 1);
                v.x += __shfl_xor_sync(0xffffffffu, v.x, 2);
                v.y += __shfl_xor_sync(0xffffffffu, v.y, 2);
                if (t == 0) {
                    pw[g] = v.x;
                    pw[g + 8] = v.y;
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[cur.s]);
                mbar_arrive(&pfull[b]);
            }
            if (++cur.s == P.stages) cur.s = 0, cur.ring_phase ^= 1u;
        }
    }
}

template <class Path>
__global__ void __launch_bounds__(kSThreads, 1) decode_step_kernel(const StepParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.bars_off);
    uint64_t *empty = full + P.stages;
    uint64_t *pfull = empty + P.stages;
    uint64_t *pempty = pfull + 2;
    float *part = reinterpret_cast<float *>(smem + P.part_off);
    float *red = reinterpret_cast<float *>(smem + P.attn_smem_off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < P.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kSC);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&pfull[b], kSC);
            mbar_init(&pempty[b], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kSC) {
        // Producer: the weight tiles of every GEMV phase, in program order.
        int s = 0, it = 0;
        uint32_t ring_phase = 0;
        for (int ph = 0; ph < P.num_phases; ++ph) {
            const StepPhase &f = P.phases[ph];
            if (f.kind != kPhGemv) continue;
            for (int rt = int(blockIdx.x); rt < f.row_tiles; rt += int(gridDim.x)) {
                const int r0 = rt * kSRows, nrows = min(kSRows, f.rows - r0);
                for (int c = 0; c < f.kchunks; ++c, ++it) {
                    const uint64_t w0 = P.trace ? globaltimer_ns() : 0;
                    if (it >= P.stages) mbar_wait(&empty[s], ring_phase ^ 1u, kErrEmptyBarrierTimeout);
                    if (unsigned long long *tr = lane == 0 ? trace_row(P, ph) : nullptr) tr[5] += globaltimer_ns() - w0;
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], uint32_t(nrows) * f.chunk_bytes);
                    __syncwarp();
                    uint8_t *dst = smem + size_t(s) * P.stage_bytes;
                    for (int r = lane; r < nrows; r += 32)
                        bulk_copy_g2s(dst + size_t(r) * f.row_stride,
                                      f.w + size_t(r0 + r) * f.row_bytes + size_t(c) * f.chunk_bytes, f.chunk_bytes,
                                      &full[s]);
                    if (++s == P.stages) s = 0, ring_phase ^= 1u;
                }
            }
        }
        return;
    }
    if (warp == kSC + 1) {
        // Reducer: fixed-order sum of the column partials of each row, the
        // residual added, the row stored, statistics kept.
        int it = 0;
        for (int ph = 0; ph < P.num_phases; ++ph) {
            const StepPhase &f = P.phases[ph];
            if (f.kind == kPhArgmax) break;
            if (f.kind == kPhGemv) {
                float ss = 0.0f, best = -3.402823466e+38f;
                uint32_t best_i = 0;
                for (int rt = int(blockIdx.x); rt < f.row_tiles; rt += int(gridDim.x)) {
                    float a = 0.0f;
                    const int row = rt * kSRows + lane;
                    // the residual of the row, loaded while the partials are computed
                    const float rv = (f.resid && lane < kSRows && row < f.rows) ? __ldcg(f.resid + row) : 0.0f;
                    for (int c = 0; c < f.kchunks; ++c, ++it) {
                        const int b = it & 1;
                        const uint64_t w0 = P.trace ? globaltimer_ns() : 0;
                        mbar_wait(&pfull[b], (it >> 1) & 1, kErrEpilogueTimeout);
                        if (unsigned long long *tr = lane == 0 ? trace_row(P, ph) : nullptr) tr[6] += globaltimer_ns() - w0;
                        if (lane < kSRows) {
                            const float *pb = part + b * kSC * kSRows + lane;
                            for (int w = 0; w < f.nsb_tile; ++w) a += pb[w * kSRows];
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&pempty[b]);
                    }
                    if (lane < kSRows && row < f.rows) {
                        const float v = f.resid ? __fadd_rn(rv, a) : a;
                        f.y[row] = v;
                        ss = __fadd_rn(ss, __fmul_rn(v, v));
                        if (f.argmax) argmax_merge(best, best_i, v, uint32_t(row));
                    }
                }
                if (f.stats_out) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
                    if (lane == 0) f.stats_out[blockIdx.x] = ss;
                }
                if (f.argmax) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
                        const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                        argmax_merge(best, best_i, ob, oi);
                    }
                    if (lane == 0) {
                        P.amax_val[blockIdx.x] = best;
                        P.amax_idx[blockIdx.x] = best_i;
                    }
                }
                __threadfence();
            }
            phase_end_sync();
        }
        return;
    }
    // Compute warps.
    GemvCursor<Path> cur;
    uint8_t *scratch = smem + P.scratch_off + size_t(warp) * Path::kScratchBytes;
    const int tslot = blockIdx.x == 0 ? 0 : (blockIdx.x == 1 ? 1 : (blockIdx.x == gridDim.x - 1 ? 2 : -1));
    unsigned long long *trace = (P.trace && tslot >= 0 && threadIdx.x == 0) ? P.trace + size_t(tslot) * P.num_phases * 8
                                                                            : nullptr;
    for (int ph = 0; ph < P.num_phases; ++ph) {
        const StepPhase &f = P.phases[ph];
        if (ph > 0) grid_wait(P, (unsigned long long)ph * gridDim.x);
        if (trace) trace[ph * 8 + 0] = globaltimer_ns();
        switch (f.kind) {
        case kPhGather: gather_phase(P, red); break;
        case kPhAttention: attention_phase(P, f, red); break;
        case kPhCombine: combine_phase(P); break;
        case kPhArgmax: argmax_phase(P); break;
        default: gemv_compute<Path>(P, f, smem, cur, scratch, trace ? trace + ph * 8 : nullptr);
        }
        if (trace) trace[ph * 8 + 1] = globaltimer_ns();
        if (f.kind == kPhArgmax) break;
        __threadfence();
        phase_end_sync();
        if (threadIdx.x == 0) atomicAdd(P.bar, 1ull);
        if (trace) trace[ph * 8 + 2] = globaltimer_ns();
    }
}

}  // namespace
}  // namespace si::dev

namespace si::kernels {

struct DecodeStep {
    dev::StepParams params{};
    std::vector<void *> allocations;
    size_t smem = 0;
    int grid = 0;
    uint32_t weight_type = 0;
};

namespace {

template <class T>
si_status dalloc(DecodeStep *st, size_t count, T **out) {
    void *p = nullptr;
    const cudaError_t e = cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 16));
    if (e != cudaSuccess) return cuda_error(int(e), "cudaMalloc");
    st->allocations.push_back(p);
    cudaMemset(p, 0, std::max<size_t>(count * sizeof(T), 16));
    *out = static_cast<T *>(p);
    return SI_OK;
}

// GEMV phase geometry: K split into chunks of at most 16 superblocks.
bool gemv_phase(dev::StepPhase &f, const void *w, int rows, int64_t cols, uint32_t col_bytes) {
    if (cols % 256 || cols > int64_t(dev::kStageVec) * 4 * dev::kSC * 32) return false;
    const int nsb = int(cols / 256);
    const int kchunks = (nsb + 15) / 16;
    if (kchunks > 2 || nsb % kchunks) return false;
    if (reinterpret_cast<uintptr_t>(w) & 15u) return false;
    f.kind = dev::kPhGemv;
    f.w = static_cast<const uint8_t *>(w);
    f.rows = rows;
    f.nsb = nsb;
    f.kchunks = kchunks;
    f.nsb_tile = nsb / kchunks;
    f.row_tiles = (rows + dev::kSRows - 1) / dev::kSRows;
    f.row_bytes = col_bytes * uint32_t(nsb);
    f.chunk_bytes = col_bytes * uint32_t(f.nsb_tile);
    // Row pitch / 16 odd: ldmatrix's 8 row addresses hit 8 distinct bank quads.
    f.row_stride = f.chunk_bytes + (((f.chunk_bytes / 16) % 2 == 0) ? 16u : 32u);
    return true;
}

}  // namespace

si_status decode_step_create(const DecodeStepModel &m, DecodeStep **out) {
    *out = nullptr;
    // The persistent step covers Q4_K weights and token embedding, groups of
    // at most four query heads, heads of at most 128 channels.
    if (m.weight_type != SI_TYPE_Q4_K || m.embedding_type != SI_TYPE_Q4_K) return SI_ERR_UNSUPPORTED;
    const int G = m.query_heads / m.kv_heads;
    if (G > dev::kSMaxG || m.head_size > 32 * dev::kSNpl || m.head_size % 4) return SI_ERR_UNSUPPORTED;
    int dev_id = 0, sms = 0;
    cudaGetDevice(&dev_id);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev_id);
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev_id);
    if (!coop || sms <= 0) return SI_ERR_UNSUPPORTED;
    using Path = dev::I8Path;
    const uint32_t CB = Path::kColBytes;
    const int64_t H = m.hidden, KV = int64_t(m.kv_heads) * m.head_size, QKV = H + 2 * KV, F = m.intermediate;

    auto *st = new DecodeStep();
    st->weight_type = m.weight_type;
    auto fail_free = [&](si_status s) {
        decode_step_destroy(st);
        return s;
    };
    dev::StepParams &P = st->params;
    std::vector<dev::StepPhase> ph;
    float *stats_hidden = nullptr, *stats_after = nullptr;
    if (si_status s = dalloc(st, size_t(sms), &stats_hidden)) return fail_free(s);
    if (si_status s = dalloc(st, size_t(sms), &stats_after)) return fail_free(s);
    uint32_t max_stride = 0;
    {
        dev::StepPhase g{};
        g.kind = dev::kPhGather;
        ph.push_back(g);
    }
    for (int l = 0; l < m.layers; ++l) {
        dev::StepPhase f{};
        if (!gemv_phase(f, m.w_qkv[l], int(QKV), H, CB)) return fail_free(SI_ERR_UNSUPPORTED);
        f.mode = 1, f.x = m.act_hidden, f.norm = m.attn_norm[l], f.stats = stats_hidden, f.y = m.act_qkv;
        ph.push_back(f);
        dev::StepPhase a{};
        a.kind = dev::kPhAttention;
        a.layer = l;
        ph.push_back(a);
        dev::StepPhase cmb{};
        cmb.kind = dev::kPhCombine;
        ph.push_back(cmb);
        dev::StepPhase o{};
        if (!gemv_phase(o, m.w_out[l], int(H), H, CB)) return fail_free(SI_ERR_UNSUPPORTED);
        o.x = m.act_attention, o.y = m.act_after, o.resid = m.act_hidden, o.stats_out = stats_after;
        ph.push_back(o);
        dev::StepPhase u{};
        if (!gemv_phase(u, m.w_up[l], int(2 * F), H, CB)) return fail_free(SI_ERR_UNSUPPORTED);
        u.mode = 1, u.x = m.act_after, u.norm = m.ffn_norm[l], u.stats = stats_after, u.y = m.act_gate_up;
        ph.push_back(u);
        dev::StepPhase dn{};
        if (!gemv_phase(dn, m.w_down[l], int(H), F, CB)) return fail_free(SI_ERR_UNSUPPORTED);
        dn.mode = 2, dn.x = m.act_gate_up, dn.y = m.act_hidden, dn.resid = m.act_after, dn.stats_out = stats_hidden;
        ph.push_back(dn);
    }
    {
        dev::StepPhase v{};
        if (!gemv_phase(v, m.embedding, m.vocab, H, CB)) return fail_free(SI_ERR_UNSUPPORTED);
        v.mode = 1, v.x = m.act_hidden, v.norm = m.output_norm, v.stats = stats_hidden, v.y = m.act_logits, v.argmax = 1;
        ph.push_back(v);
        dev::StepPhase am{};
        am.kind = dev::kPhArgmax;
        ph.push_back(am);
    }
    for (const auto &f : ph)
        if (f.kind == dev::kPhGemv) max_stride = std::max(max_stride, f.row_stride);

    // Shared memory: ring | attention scratch (also the gather's reduction) |
    // column partials | mbarriers | per-warp load scratch.
    const uint32_t stage_bytes = (uint32_t(dev::kSRows) * max_stride + 127u) / 128u * 128u;
    // attention: per-warp partials + rotated queries; GEMV phases with a
    // transformed input stage that vector (K floats) in the same area.
    const uint32_t attn_bytes = std::max(uint32_t(dev::kSC * G * m.head_size + 2 * dev::kSC * G + G * m.head_size) * 4u,
                                         uint32_t(std::max(H, F)) * 4u);
    const uint32_t part_bytes = 2u * dev::kSC * dev::kSRows * 4u;
    const uint32_t scratch_bytes = dev::kSC * Path::kScratchBytes;
    const uint32_t fixed = attn_bytes + part_bytes + scratch_bytes + 1024u;
    const uint32_t budget = 227u * 1024u;
    if (fixed + 2 * stage_bytes > budget) return fail_free(SI_ERR_UNSUPPORTED);
    int stages = int(std::min<uint32_t>(8u, (budget - fixed) / stage_bytes));
    if (const char *e = std::getenv("SI_DECODE_STAGES")) stages = std::max(2, std::min(stages, std::atoi(e)));
    uint32_t off = uint32_t(stages) * stage_bytes;
    P.attn_smem_off = off;
    off += (attn_bytes + 127u) / 128u * 128u;
    P.part_off = off;
    off += part_bytes;
    P.bars_off = off;
    off += uint32_t(2 * stages + 4) * 8u;
    off = (off + 15u) / 16u * 16u;
    P.scratch_off = off;
    off += scratch_bytes;
    st->smem = off;
    P.stages = stages;
    P.stage_bytes = stage_bytes;

    // Attention work split: a chunk of the tokens per CTA, chunks per head
    // so that the items fill the grid.
    const int chunks = std::min(32 * dev::kMaxChunkSlices, std::max(1, sms / m.kv_heads));
    if (sms > 32 * dev::kMaxGridSlices) return fail_free(SI_ERR_UNSUPPORTED);
    P.attn_chunks = chunks;
    const int items = m.kv_heads * chunks;
    if (si_status s = dalloc(st, size_t(items) * G * m.head_size, &P.ws_acc)) return fail_free(s);
    if (si_status s = dalloc(st, size_t(items) * G, &P.ws_m)) return fail_free(s);
    if (si_status s = dalloc(st, size_t(items) * G, &P.ws_l)) return fail_free(s);
    if (si_status s = dalloc(st, size_t(sms), &P.amax_val)) return fail_free(s);
    if (si_status s = dalloc(st, size_t(sms), &P.amax_idx)) return fail_free(s);
    unsigned long long *sync = nullptr;
    if (si_status s = dalloc(st, 2, &sync)) return fail_free(s);
    P.bar = sync;
    P.abort = reinterpret_cast<uint32_t *>(sync + 1);
    float **caches = nullptr;
    if (si_status s = dalloc(st, size_t(2 * m.layers), &caches)) return fail_free(s);
    std::vector<float *> host_caches(size_t(2 * m.layers));
    for (int l = 0; l < m.layers; ++l) {
        host_caches[size_t(l)] = m.key_cache[l];
        host_caches[size_t(m.layers + l)] = m.value_cache[l];
    }
    cudaMemcpy(caches, host_caches.data(), host_caches.size() * sizeof(float *), cudaMemcpyHostToDevice);
    P.key_cache = caches;
    P.value_cache = caches + m.layers;
    dev::StepPhase *table = nullptr;
    if (si_status s = dalloc(st, ph.size(), &table)) return fail_free(s);
    cudaMemcpy(table, ph.data(), ph.size() * sizeof(dev::StepPhase), cudaMemcpyHostToDevice);
    P.phases = table;
    P.num_phases = int(ph.size());
    P.hidden = m.hidden;
    P.qh = m.query_heads;
    P.kvh = m.kv_heads;
    P.hs = m.head_size;
    P.rotary = m.rotary_size;
    P.group = G;
    P.vocab = m.vocab;
    P.context = m.context;
    P.eps = m.epsilon;
    P.rope_scale = m.rope_scale;
    P.attn_scale = 1.0f / sqrtf(float(m.head_size));
    P.freq = m.freq;
    P.qkv = m.act_qkv;
    P.attention = m.act_attention;
    P.embedding = static_cast<const uint8_t *>(m.embedding);
    P.embedding_type = m.embedding_type;
    byte_length(m.embedding_type, uint64_t(H), &P.embedding_row_bytes);
    P.hidden_out = m.act_hidden;
    P.gather_stats = stats_hidden;
    P.control = m.control;
    P.next_token = m.next_token;
    if (m.trace) {
        if (si_status s = dalloc(st, size_t(3) * ph.size() * 8, &P.trace)) return fail_free(s);
        *m.trace = P.trace;
        *m.trace_entries = uint64_t(3) * ph.size() * 8;
    }

    auto kernel = dev::decode_step_kernel<Path>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(st->smem)) != cudaSuccess) {
        cudaGetLastError();
        return fail_free(SI_ERR_UNSUPPORTED);
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, dev::kSThreads, st->smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return fail_free(SI_ERR_UNSUPPORTED);
    }
    st->grid = sms;
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_free(cuda_error(int(e), "decode step setup"));
    *out = st;
    return SI_OK;
}

si_status decode_step_launch(DecodeStep *st, DecodeFeed *feed, void *stream) {
    auto s = static_cast<cudaStream_t>(stream);
    dev::StepParams P = st->params;
    P.feed = feed;
    if (cudaError_t e = cudaMemsetAsync(P.bar, 0, 16, s); e != cudaSuccess)
        return cuda_error(int(e), "decode step barrier reset");
    if (P.trace)
        if (cudaError_t e = cudaMemsetAsync(P.trace, 0, size_t(3) * P.num_phases * 8 * 8, s); e != cudaSuccess)
            return cuda_error(int(e), "decode step trace reset");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(st->grid));
    cfg.blockDim = dim3(unsigned(dev::kSThreads));
    cfg.dynamicSmemBytes = st->smem;
    cfg.stream = s;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, dev::decode_step_kernel<dev::I8Path>, P);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "decode step launch failed: %s", cudaGetErrorString(e));
    return SI_OK;
}

void decode_step_destroy(DecodeStep *st) {
    if (!st) return;
    for (void *p : st->allocations) cudaFree(p);
    delete st;
}

si_status take_error_decode_step(int device, uint32_t *code) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return fail(SI_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    uint32_t v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, dev::g_error_word, sizeof v);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(dev::g_error_word, &zero, sizeof zero);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return fail(SI_ERR_CUDA, "device error word: %s", cudaGetErrorString(e));
    *code |= v;
    return SI_OK;
}

}  // namespace si::kernels
