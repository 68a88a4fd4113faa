// Internal helpers shared by the host-side translation units of
// libsharpinfer_cuda: error reporting, type geometry, argument checks.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/sharpinfer_cuda.h"

namespace si {

// Thread-local last-error message; every failing entry point sets it.
si_status fail(si_status status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();
const std::string &last_error();

constexpr int kQ8_0Block = 32;
constexpr int kQ8_0Bytes = 34;
constexpr int kQ4KBlock = 256;
constexpr int kQ4KBytes = 144;
constexpr int kQ6KBytes = 210;

inline bool known_type(uint32_t t) {
    return t == SI_TYPE_F32 || t == SI_TYPE_F16 || t == SI_TYPE_Q8_0 || t == SI_TYPE_Q4_K || t == SI_TYPE_Q6_K;
}

inline const char *type_name(uint32_t t) {
    switch (t) {
    case SI_TYPE_F32: return "F32";
    case SI_TYPE_F16: return "F16";
    case SI_TYPE_Q8_0: return "Q8_0";
    case SI_TYPE_Q4_K: return "Q4_K";
    case SI_TYPE_Q6_K: return "Q6_K";
    default: return "unknown";
    }
}

// Bytes of `elements` elements; returns SI_ERR_INVALID_DATA when a block
// type's count is not a multiple of its block, SI_ERR_UNSUPPORTED for an
// unknown type (GgufModelFile.cs:301-331 throws the same way).
si_status byte_length(uint32_t type, uint64_t elements, uint64_t *bytes);

// IEEE binary16 <-> binary32 (round to nearest even).
float half_to_float(uint16_t h);
uint16_t float_to_half(float f);

// The tensor [ptr, ptr + bytes) lies inside one device allocation of the
// current device (SI_ERR_INVALID_ARGUMENT naming `port` otherwise).
si_status device_range(const char *port, const void *ptr, uint64_t bytes);
bool ranges_overlap(const void *a, uint64_t an, const void *b, uint64_t bn);
// Maps a cudaError_t onto si_status with the runtime's message.
si_status cuda_error(int error, const char *what);

// This rank's arena of a peer group (si_peer_group_create), the group's
// size and rank, and the arena's data bytes (before the 4 KB of state).
uint8_t *peer_group_arena(si_peer_group *g, int *nranks, int *rank, uint64_t *data_bytes);
namespace kernels { struct PeerGather; }
// The exchange descriptor of a peer GEMV whose output rows land at row
// row_base of the float vector at output_offset in every rank's arena.
si_status peer_gather_desc(si_peer_group *g, uint64_t output_offset, int64_t row_base, int64_t rows,
                           kernels::PeerGather *out);
// Publish-only exchange of kind `kind` (0..3): the producer descriptor, and
// this rank's counts / epoch of that kind for the consumer's wait.
si_status peer_gather_desc_nowait(si_peer_group *g, uint64_t output_offset, int64_t row_base, int64_t rows, int kind,
                                  kernels::PeerGather *out);
si_status peer_counts(si_peer_group *g, int kind, const unsigned long long **counts, const uint32_t **epoch);

// Per-device launch state (launch_state.cpp). Kernel attributes and the SM
// count are properties of a device; one process may drive several devices
// from several threads, so both are kept per device behind a lock.
constexpr int kMaxDevices = 64;
int current_device();
// Streaming multiprocessors of the current device.
int device_sm_count();
// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device (once per device and kernel); returns the cudaError_t value.
int opt_in_smem(const void *kernel, int bytes);

}  // namespace si

// Launch wrappers implemented in the .cu files (host side of each kernel).
namespace si::kernels {
si_status matvec_dense(uint32_t wtype, const void *w, uint32_t xtype, const void *x,
                       uint32_t ytype, void *y, int64_t rows, int64_t cols, void *stream);
si_status matvec_quant(uint32_t wtype, const void *w, const float *x, float *y,
                       int64_t rows, int64_t cols, void *stream);
si_status shared_weight_matvec(uint32_t wtype, const void *w, const float *x, const int32_t *control,
                               float *y, int64_t m, int64_t n, int64_t k, void *stream);
si_status batch_shared_matvec(uint32_t wtype, const void *w, const float *in,
                              const int32_t *control, float *out, int64_t batch,
                              int64_t out_features, int64_t in_features, void *stream);
si_status gemm_workspace_bytes(uint32_t wtype, int64_t m, int64_t n, int64_t k, uint64_t *bytes);
si_status gemm_tn(uint32_t wtype, const float *x, const void *w, float *y, int64_t m, int64_t n,
                  int64_t k, void *workspace, uint64_t workspace_bytes, void *stream);
// Few-row tcgen05 GEMM (gemm_skinny.cu): Y = X W^T for any m with BN = 16,
// 32 or 64 input rows per tile, no workspace; rows t >= control[1] are not
// written when control is non-null. SI_ERR_UNSUPPORTED (nothing launched)
// when gemm_skinny_supported is false.
bool gemm_skinny_supported(uint32_t wtype, const void *w, const float *x, int64_t m, int64_t n, int64_t k);
si_status gemm_skinny(uint32_t wtype, const void *w, const float *x, const int32_t *control, float *y, int64_t m,
                      int64_t n, int64_t k, void *stream);
si_status take_error_gemm_skinny(int device, uint32_t *code);
// Few-row GEMM with the dequantised weights in tensor memory (gemm_fewrow.cu):
// Q4_K / Q8_0, 1..32 input rows, k a multiple of 256, 16-byte aligned weight
// rows and X; rows t >= control[1] are not written.
bool gemm_fewrow_supported(uint32_t wtype, const void *w, const float *x, int64_t m, int64_t n, int64_t k);
si_status gemm_fewrow(uint32_t wtype, const void *w, const float *x, const int32_t *control, float *y, int64_t m,
                      int64_t n, int64_t k, void *stream);
si_status take_error_gemm_fewrow(int device, uint32_t *code);
si_status take_error_gemv(int device, uint32_t *code);
si_status take_error_gemm(int device, uint32_t *code);
si_status take_error_gemv_mma(int device, uint32_t *code);
// Row-sharded output exchange of a fused GEMV (see si_rowshard_matvec_peer).
constexpr int kMaxPeerRanks = 8;
struct PeerGather {
    float *ys[kMaxPeerRanks];         // every rank's output vector, as mapped in this process
    uint32_t *flags[kMaxPeerRanks];   // every rank's flag array [nranks]
    uint32_t *ticket;                 // this rank's CTA ticket counter
    uint32_t *epoch;                  // this rank's call counter
    int nranks;                       // 0: not a sharded call
    int rank;
    int64_t row_base;                 // global index of this rank's first row
    // Publish-only exchange (no wait at the producer): every CTA adds the rows
    // it stored to counts[q][rank] of every rank q (after a system-scope
    // fence), and the launch's last CTA advances this rank's kind_epoch; the
    // consumer waits for the counts (GemvFusion::wait_*).
    int nowait;
    unsigned long long *counts[kMaxPeerRanks];
    uint32_t *kind_epoch;
};
// control/token: batch-shared use, y is written only when token < control[1].
si_status matvec_quant_mma(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                           void *stream, const PeerGather *peer = nullptr, const int32_t *control = nullptr,
                           int token = 0);
// Neighbours of a decode-program GEMV fused into it (batch 1, one GPU):
//  in_mode 1: the input is rms-normed on the fly (transformer.rms-norm with
//             weight norm_w and epsilon eps: rows = (W (x * norm_w)) / rms(x));
//  in_mode 2: the input is transformer.swiglu of x = [gate | up] (K floats each);
//  in_mode 3: the input is the residual stream after a K-split exchange,
//             x + parts[0] + ... + parts[nparts-1] (rank order, part_stride
//             floats apart), rms-normed as in mode 1; CTA 0 stores that sum
//             to h_out when h_out is given;
//  resid:     y[r] = resid[r] + (W x)[r] (the residual add; resid may be y).
// peer: the output rows go to every rank's arena (PeerGather) instead of y.
struct GemvFusion {
    int in_mode = 0;
    const float *norm_w = nullptr;
    float eps = 0.0f;
    const float *resid = nullptr;
    const float *parts = nullptr;
    int nparts = 0;
    int64_t part_stride = 0;
    float *h_out = nullptr;
    // Consumer of a publish-only exchange: before reading x / parts, wait
    // until every rank's count reached (*wait_epoch) * wait_rows.
    const unsigned long long *wait_counts = nullptr;
    const uint32_t *wait_epoch = nullptr;
    int wait_ranks = 0;
    int64_t wait_rows = 0;
};
si_status matvec_quant_fused(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                             const GemvFusion &f, void *stream, const PeerGather *peer = nullptr);
// The launch shape matvec_quant_mma picks, and one GEMV with an explicit shape
// (si_gemv_default_plan / si_matvec_quant_planned).
si_status gemv_default_plan(uint32_t wtype, int64_t rows, int64_t cols, si_gemv_plan *plan);
si_status matvec_quant_planned(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                               const si_gemv_plan &plan, void *stream);
// Q4_K batch on the tensor cores, eight input rows per launch; SI_ERR_UNSUPPORTED
// when the shape or alignment needs another kernel (nothing launched then).
si_status matvec_q4k_batched(const void *w, const float *x, float *y, int64_t m, int64_t rows, int64_t cols,
                             void *stream, const int32_t *control);
// ---- transformer instructions (transformer.cu) ------------------------------
// Device-side greedy loop state read by the argmax kernel after each decode
// step: it stores the step's token in history[position - base] and writes
// the next step's control = (next token, position + 1), where the next token
// is prompt[k + 1] while prompt tokens remain, else the argmax.
struct DecodeFeed {
    int32_t *control;       // [token, position] read by the decode step
    const int32_t *prompt;  // prompt tokens, prompt[0] at position `base`
    int32_t *history;       // argmax of every step, `capacity` entries
    int32_t base;
    int32_t prompt_tokens;
    int32_t capacity;
    int32_t pad;
};
// Multi-stream greedy loop state read by the per-row argmax: row b stores
// its token in history[(positions[b] - start[b]) * streams + b] (when
// within `capacity` steps), then sets tokens[b] = the token and
// positions[b] += 1 for the next step.
struct StreamsFeed {
    int32_t *tokens;
    int32_t *positions;
    const int32_t *start;
    int32_t *history;
    int32_t capacity;
    int32_t streams;
};
si_status tr_gather_row(uint32_t type, const void *table, int64_t rows, int64_t cols, const int32_t *index, float *out,
                        void *stream);
// core.gather-row for `count` indices at once (rows of a prefill chunk).
si_status tr_gather_rows_quant(uint32_t type, const void *table, int64_t rows, int64_t cols, const int32_t *indices,
                               int64_t count, float *out, void *stream);
si_status tr_embedding_gather_batch(const uint16_t *table, int64_t rows, const int32_t *indices, float *out,
                                    int64_t batch, int64_t width, void *stream);
si_status tr_copy_rows(const float *in, float *out, int64_t count, void *stream);
// residual == nullptr: rms-norm; otherwise residual-rms-norm (updated written).
// control == nullptr: every row; otherwise rows < control[1].
si_status tr_rms_norm(const float *in, const float *residual, const float *weight, const int32_t *control,
                      float *updated, float *out, int64_t batch, int64_t width, float eps, void *stream);
si_status tr_swiglu(const float *gate_up, const int32_t *control, float *out, int64_t batch, int64_t width,
                    void *stream);
si_status tr_scaled_add(const float *in, const float *update, float *out, int64_t count, float scale, void *stream);
// control == nullptr: single form at *position; otherwise the batch form.
si_status tr_rope_kv_write(const float *qkv, const int32_t *position, const int32_t *control, const float *freq,
                           float *query, float *key_cache, float *value_cache, int64_t batch, int64_t qsize,
                           int64_t kvsize, int head_size, int rotary, int64_t context, float rope_scale, void *stream);
si_status tr_attention_decode(const float *query, const float *kc, const float *vc, const int32_t *position, float *out,
                              int query_heads, int kv_heads, int head_size, int64_t context, void *stream);
// transformer.rope-kv-write followed by transformer.grouped-query-attention
// (one stream), as one kernel: q and the token's k rotated from qkv, the k / v
// rows stored into the caches at *position, then the attention.
si_status tr_attention_decode_rope(const float *qkv, const int32_t *position, const float *freq, float *kc, float *vc,
                                   float *out, int query_heads, int kv_heads, int head_size, int rotary,
                                   int64_t context, float rope_scale, void *stream);
si_status tr_gqa_scores(const float *query, const float *kc, const int32_t *position, const int32_t *control,
                        float *scores, int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context,
                        void *stream);
si_status tr_causal_softmax(const float *scores, const int32_t *position, const int32_t *control, float *probs,
                            int64_t batch, int heads, int64_t context, void *stream);
si_status tr_gqa_values(const float *probs, const float *vc, const int32_t *position, const int32_t *control,
                        float *out, int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context,
                        void *stream);
// batch-gqa-scores -> batch-causal-softmax -> batch-gqa-values fused for
// the rows [start, start + count) of a prefill chunk (head sizes for which
// tr_prefill_attention_supported is true).
bool tr_prefill_attention_supported(int head_size);
si_status tr_prefill_attention(const float *query, const float *kc, const float *vc, int32_t start, int32_t count,
                               float *out, int query_heads, int kv_heads, int head_size, int64_t context,
                               void *stream);
si_status tr_argmax(const float *in, int64_t n, int32_t *out, DecodeFeed *feed, void *stream);
// argmax of each of `rows` rows of n floats into out[row].
si_status tr_argmax_rows(const float *in, int64_t rows, int64_t n, int32_t *out, StreamsFeed *sfeed, void *stream);
// Multi-stream decode forms: row b is stream b's token at positions[b];
// stream b's caches start cache_stride floats after stream b - 1's.
si_status tr_rope_kv_write_streams(const float *qkv, const int32_t *positions, const float *freq, float *query,
                                   float *key_cache, float *value_cache, int64_t streams, int64_t qsize,
                                   int64_t kvsize, int head_size, int rotary, int64_t context, int64_t cache_stride,
                                   float rope_scale, void *stream);
si_status tr_attention_decode_streams(const float *query, const float *kc, const float *vc, const int32_t *positions,
                                      float *out, int streams, int query_heads, int kv_heads, int head_size,
                                      int64_t context, int64_t cache_stride, void *stream);
si_status tr_select_last(const float *in, const int32_t *control, float *out, int64_t batch, int64_t width,
                         void *stream);
si_status tr_gather_rows(const float *table, int64_t rows, const int32_t *control, float *out, int64_t batch,
                         int64_t width, void *stream);
}  // namespace si::kernels
