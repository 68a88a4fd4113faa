// Phi-4 text decoder session on CUDA: the decode program that
// Phi4D3D12TextSession.Build assembles from core.* and transformer.*
// instructions (Phi4D3D12TextSession.cs:307-920), recorded once into a CUDA
// graph and replayed per token. ForwardToken semantics (one host round trip
// per token) and a device-resident greedy loop (the argmax kernel writes the
// next step's control) share the same recorded step.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <tuple>
#include <utility>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "si_internal.h"

using si::fail;
namespace k = si::kernels;

struct si_decoder {
    int device = 0;
    cudaStream_t stream = nullptr;
    si_decoder_config cfg{};
    struct Slot {
        void *ptr;
        uint64_t bytes;
    };
    std::vector<void *> allocations;
    std::unordered_map<std::string, Slot> slots;
    // Resolved slot pointers.
    const void *embedding = nullptr;
    const float *output_norm = nullptr;
    std::vector<const float *> attn_norm, ffn_norm;
    std::vector<const void *> w_qkv, w_out, w_up, w_down;
    // GGUF type of every layer's projection weights (one type for all of them
    // unless the session was created with per-slot types, as a Q4_K_M file has)
    std::vector<uint32_t> t_qkv, t_out, t_up, t_down;
    std::vector<float *> key_cache, value_cache;
    float *freq = nullptr;
    int32_t *control = nullptr, *next_token = nullptr, *prompt = nullptr, *history = nullptr;
    k::DecodeFeed *feed = nullptr;
    float *hidden = nullptr, *after = nullptr, *normalized = nullptr, *qkv = nullptr, *query = nullptr,
          *attention = nullptr, *projected = nullptr, *gate_up = nullptr, *activated = nullptr, *down = nullptr,
          *logits = nullptr;
    // Pinned host staging: [0,1] control, [2] next token, then the feed
    // descriptor, then prompt / history staging of `context` entries each.
    int32_t *pinned = nullptr;
    k::DecodeFeed *pinned_feed = nullptr;
    int32_t *pinned_prompt = nullptr, *pinned_history = nullptr;
    cudaGraphExec_t step_exec = nullptr, feed_exec = nullptr;

    // Row-sharded session (si_decoder_create_sharded): the peer group, this
    // rank's arena (the five projection outputs live there, gathered by the
    // peer GEMV) and the vocabulary projection's rows of token_embedding.
    si_peer_group *group = nullptr;
    uint8_t *arena = nullptr;
    const void *w_vocab = nullptr;
    // Which projections are split by rows (qkv, attn_output, ffn_up,
    // ffn_down, vocabulary); the others are replicated and run whole on
    // every rank, their outputs written into the rank's own arena.
    enum { kQkv, kOut, kUp, kDown, kVocab };
    bool sharded[5] = {false, false, false, false, false};
    // The projection outputs of even / odd layers (arena regions).
    float *par_qkv[2] = {}, *par_out[2] = {}, *par_up[2] = {}, *par_down[2] = {};
    // Tensor-parallel session (si_decoder_create_tensor_parallel): this rank's
    // partition, the residual stream in two local buffers, and the exchange
    // descriptors of the out / down partial sums and the vocabulary rows.
    bool tp = false;
    si_tp_partition part{};
    float *res_a = nullptr, *res_b = nullptr;
    float *o_parts = nullptr, *down_parts = nullptr;  // [nranks][hidden] in this rank's arena
    k::PeerGather pg_out{}, pg_down{}, pg_vocab{};
    // this rank's counts / epochs of the publish-only out (0) and down (1) exchanges
    const unsigned long long *o_counts = nullptr, *d_counts = nullptr;
    const uint32_t *o_epoch = nullptr, *d_epoch = nullptr;
    // Multi-stream session (si_decoder_create_streams): `streams` rows per
    // step, stream b's caches at rows b * context of each layer's cache;
    // per-stream tokens / positions / greedy-loop state on the device.
    int32_t streams = 1;
    int32_t *st_tokens = nullptr, *st_positions = nullptr, *st_start = nullptr, *st_next = nullptr,
            *st_history = nullptr;
    k::StreamsFeed *st_feed = nullptr;
    int32_t *pinned_st = nullptr;  // host staging: tokens, positions, next, history
    cudaGraphExec_t streams_exec = nullptr, streams_feed_exec = nullptr;
    // Prompt prefill in chunks of up to kPrefillRows rows (buffers allocated
    // by the first prefill call): the chunk's activations, one (start,
    // count) control pair per chunk, the split-operand GEMM workspace.
    struct Prefill {
        float *hidden, *after, *normalized, *qkv, *query, *attention, *projected, *gate_up, *activated, *down;
        int32_t *control;
        void *workspace;
        uint64_t workspace_bytes;
    } pf{};
    bool pf_ready = false;
    int32_t position = 0;
    std::mutex lock;  // session calls are serialised, as the executor's are
};

namespace {

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

si_status cuda(cudaError_t e, const char *what) { return si::cuda_error(int(e), what); }

si_status alloc_slot(si_decoder *d, const std::string &name, uint64_t bytes, void **out) {
    void *p = nullptr;
    if (si_status st = cuda(cudaMalloc(&p, bytes), "cudaMalloc")) return st;
    d->allocations.push_back(p);
    if (si_status st = cuda(cudaMemset(p, 0, bytes), "cudaMemset")) return st;
    d->slots[name] = {p, bytes};
    *out = p;
    return SI_OK;
}

template <class T>
si_status alloc_typed(si_decoder *d, const std::string &name, uint64_t bytes, T **out) {
    void *p = nullptr;
    si_status st = alloc_slot(d, name, bytes, &p);
    *out = static_cast<T *>(p);
    return st;
}

si_status fill_ones(float *p, int64_t n) {
    std::vector<float> ones(size_t(n), 1.0f);
    return cuda(cudaMemcpy(p, ones.data(), size_t(n) * 4, cudaMemcpyHostToDevice), "cudaMemcpy");
}

void destroy(si_decoder *d) {
    DeviceScope scope(d->device);
    if (d->stream) cudaStreamSynchronize(d->stream);
    if (d->step_exec) cudaGraphExecDestroy(d->step_exec);
    if (d->feed_exec) cudaGraphExecDestroy(d->feed_exec);
    if (d->streams_exec) cudaGraphExecDestroy(d->streams_exec);
    if (d->streams_feed_exec) cudaGraphExecDestroy(d->streams_feed_exec);
    if (d->pinned_st) cudaFreeHost(d->pinned_st);
    for (void *p : d->allocations) cudaFree(p);
    if (d->pinned) cudaFreeHost(d->pinned);
    if (d->stream) cudaStreamDestroy(d->stream);
    delete d;
}

si_status project(uint32_t type, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                  cudaStream_t s) {
    if (type == SI_TYPE_Q8_0 || type == SI_TYPE_Q4_K || type == SI_TYPE_Q6_K)
        return k::matvec_quant(type, w, x, y, rows, cols, s);
    return k::matvec_dense(type, w, SI_TYPE_F32, x, SI_TYPE_F32, y, rows, cols, s);
}

// A projection of the session: the whole mat-vec, or in a row-sharded
// session this rank's rows with the output stored into every rank's arena
// (y lies in the arena; its offset is the same on every rank).
si_status project_rows(si_decoder *d, int kind, uint32_t type, const void *w, const float *x, float *y, int64_t rows,
                       int64_t cols) {
    if (!d->group || !d->sharded[kind]) return project(type, w, x, y, rows, cols, d->stream);
    const uint64_t offset = uint64_t(reinterpret_cast<uint8_t *>(y) - d->arena);
    return si_rowshard_matvec_peer(d->group, type, w, x, offset, rows, cols, d->stream);
}

// Arena layout of a row-sharded session: the qkv, attention-output,
// gate_up and down vectors twice (even and odd layers) and the logits, each
// 256-byte aligned. A rank enters a peer GEMV only after every rank has
// finished its previous peer GEMV, i.e. after every rank has consumed what
// it read before that call; with two copies per layer-repeated region (and
// gate_up split whenever anything is), a region is overwritten only after
// its previous content has been consumed on every rank.
struct ArenaLayout {
    uint64_t qkv[2], out[2], up[2], down[2], logits, data_bytes;
};

ArenaLayout arena_layout(const si_decoder_config &c) {
    const uint64_t H = uint64_t(c.hidden), QKV = H + 2 * uint64_t(c.kv_heads) * uint64_t(c.head_size);
    auto al = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
    ArenaLayout a{};
    uint64_t o = 0;
    for (int par = 0; par < 2; ++par) {
        a.qkv[par] = o, o += al(QKV * 4);
        a.out[par] = o, o += al(H * 4);
        a.up[par] = o, o += al(2 * uint64_t(c.intermediate) * 4);
        a.down[par] = o, o += al(H * 4);
    }
    a.logits = o, o += al(uint64_t(c.vocab) * 4);
    a.data_bytes = o;
    return a;
}

// The decode program one instruction per launch (Phi4D3D12TextSession.cs:866-920).
// Fusing rope-kv-write into the attention launch measured slower (1.69 vs
// 1.59 ms per token): the one-wave rope kernel is another window in which
// the next GEMV streams its weights.
// Measured on B200 (Phi-4-mini, position ~600): 1.69-1.75 ms per token.
// A variant with the norms, swiglu and rope fused into the neighbouring
// kernels (five launches per layer) measured 2.02 ms: back-to-back GEMVs
// each need every SM's shared memory, so a GEMV could no longer stream its
// weights during the previous kernel the way it does during a one-CTA norm.
si_status record_step_unfused(si_decoder *d, k::DecodeFeed *feed) {
    const si_decoder_config &c = d->cfg;
    const int64_t H = c.hidden, KV = int64_t(c.kv_heads) * c.head_size, QKV = H + 2 * KV, F = c.intermediate;
    cudaStream_t s = d->stream;
    int32_t *position = d->control + 1;
    if (si_status st = k::tr_gather_row(c.embedding_type, d->embedding, c.vocab, H, d->control, d->hidden, s)) return st;
    if (si_status st = k::tr_rms_norm(d->hidden, nullptr, d->attn_norm[0], nullptr, nullptr, d->normalized, 1, H,
                                      c.epsilon, s))
        return st;
    for (int l = 0; l < c.layers; ++l) {
        // row-sharded: this layer's copy of the projection outputs
        float *qkv = d->group ? d->par_qkv[l & 1] : d->qkv, *projected = d->group ? d->par_out[l & 1] : d->projected;
        float *gate_up = d->group ? d->par_up[l & 1] : d->gate_up, *down = d->group ? d->par_down[l & 1] : d->down;
        if (si_status st = project_rows(d, si_decoder::kQkv, d->t_qkv[l], d->w_qkv[l], d->normalized, qkv, QKV, H)) return st;
        if (si_status st = k::tr_rope_kv_write(qkv, position, nullptr, d->freq, d->query, d->key_cache[l],
                                               d->value_cache[l], 1, H, KV, c.head_size, c.rotary_size, c.context,
                                               c.rope_scale, s))
            return st;
        if (si_status st = k::tr_attention_decode(d->query, d->key_cache[l], d->value_cache[l], position, d->attention,
                                                  c.query_heads, c.kv_heads, c.head_size, c.context, s))
            return st;
        if (si_status st = project_rows(d, si_decoder::kOut, d->t_out[l], d->w_out[l], d->attention, projected, H, H)) return st;
        if (si_status st = k::tr_rms_norm(d->hidden, projected, d->ffn_norm[l], nullptr, d->after, d->normalized, 1,
                                          H, c.epsilon, s))
            return st;
        if (si_status st = project_rows(d, si_decoder::kUp, d->t_up[l], d->w_up[l], d->normalized, gate_up, 2 * F, H)) return st;
        if (si_status st = k::tr_swiglu(gate_up, nullptr, d->activated, 1, F, s)) return st;
        if (si_status st = project_rows(d, si_decoder::kDown, d->t_down[l], d->w_down[l], d->activated, down, H, F)) return st;
        const float *next_norm = l + 1 < c.layers ? d->attn_norm[l + 1] : d->output_norm;
        if (si_status st = k::tr_rms_norm(d->after, down, next_norm, nullptr, d->hidden, d->normalized, 1, H,
                                          c.epsilon, s))
            return st;
    }
    if (si_status st = project_rows(d, si_decoder::kVocab, c.embedding_type, d->w_vocab, d->normalized, d->logits, c.vocab, H)) return st;
    return k::tr_argmax(d->logits, c.vocab, d->next_token, feed, s);
}

// The decode program with each small instruction fused into a neighbouring
// launch, five launches per layer (one GPU, Q4_K / Q8_0 projections):
//   qkv GEMV        rms-norm(hidden, attn_norm) fused into its input load
//   attention       rope-kv-write fused in (q and k rotated from qkv, the
//                   token's k / v rows stored into the caches)
//   out GEMV        residual add in its epilogue: hidden += W_o attention
//   gate_up GEMV    rms-norm(hidden, ffn_norm) fused into its input load
//   down GEMV       swiglu(gate_up) fused into its input load, residual add:
//                   hidden += W_down swiglu(gate_up)
// then the vocabulary GEMV with rms-norm(hidden, output_norm) and argmax.
// The residual stream lives in `hidden` (updated in place); the reference's
// separate after / normalized / activated vectors are never materialised.
// The arithmetic is the instructions' own except for the order of two
// roundings: the norm scale 1/rms multiplies each output row instead of each
// input element (W (x * s * w) = s * (W (x * w))).
bool fused_step_supported(const si_decoder *d) {
    const si_decoder_config &c = d->cfg;
    const auto quant = [](uint32_t t) { return t == SI_TYPE_Q4_K || t == SI_TYPE_Q8_0; };
    for (int l = 0; l < c.layers; ++l)
        if (!quant(d->t_qkv[l]) || !quant(d->t_out[l]) || !quant(d->t_up[l]) || !quant(d->t_down[l])) return false;
    return !d->group && d->streams == 1 && quant(c.embedding_type) && c.hidden % 256 == 0 &&
           c.intermediate % 256 == 0 && c.rotary_size % 2 == 0;
}

si_status record_step_fused(si_decoder *d, k::DecodeFeed *feed) {
    const si_decoder_config &c = d->cfg;
    const int64_t H = c.hidden, KV = int64_t(c.kv_heads) * c.head_size, QKV = H + 2 * KV, F = c.intermediate;
    cudaStream_t s = d->stream;
    int32_t *position = d->control + 1;
    auto gemv = [&](const void *w, const float *x, float *y, int64_t rows, int64_t cols, int in_mode,
                    const float *norm, const float *resid, uint32_t type) -> si_status {
        k::GemvFusion f;
        f.in_mode = in_mode;
        f.norm_w = norm;
        f.eps = c.epsilon;
        f.resid = resid;
        const si_status st = k::matvec_quant_fused(type, w, x, y, rows, cols, f, s);
        if (st == SI_ERR_UNSUPPORTED)
            return fail(SI_ERR_UNSUPPORTED, "fused decode step: no tensor-core GEMV for [%lld, %lld]", (long long)rows,
                        (long long)cols);
        return st;
    };
    if (si_status st = k::tr_gather_row(c.embedding_type, d->embedding, c.vocab, H, d->control, d->hidden, s)) return st;
    for (int l = 0; l < c.layers; ++l) {
        if (si_status st = gemv(d->w_qkv[l], d->hidden, d->qkv, QKV, H, 1, d->attn_norm[l], nullptr, d->t_qkv[l]))
            return st;
        if (si_status st = k::tr_attention_decode_rope(d->qkv, position, d->freq, d->key_cache[l], d->value_cache[l],
                                                       d->attention, c.query_heads, c.kv_heads, c.head_size,
                                                       c.rotary_size, c.context, c.rope_scale, s))
            return st;
        if (si_status st = gemv(d->w_out[l], d->attention, d->hidden, H, H, 0, nullptr, d->hidden, d->t_out[l]))
            return st;
        if (si_status st = gemv(d->w_up[l], d->hidden, d->gate_up, 2 * F, H, 1, d->ffn_norm[l], nullptr, d->t_up[l]))
            return st;
        if (si_status st = gemv(d->w_down[l], d->gate_up, d->hidden, H, F, 2, nullptr, d->hidden, d->t_down[l]))
            return st;
    }
    if (si_status st = gemv(d->w_vocab, d->hidden, d->logits, c.vocab, H, 1, d->output_norm, nullptr, c.embedding_type))
        return st;
    return k::tr_argmax(d->logits, c.vocab, d->next_token, feed, s);
}

// One decode step on d->stream: the persistent step's launch, the fused
// program (five launches per layer) or the program instruction by
// instruction (nine launches per layer); every launch programmatically
// dependent on the previous one.
si_status record_step_tp(si_decoder *d, k::DecodeFeed *feed);

si_status record_step(si_decoder *d, k::DecodeFeed *feed) {
    if (d->tp) return record_step_tp(d, feed);
    if (fused_step_supported(d)) return record_step_fused(d, feed);
    return record_step_unfused(d, feed);
}

si_status build_graph(si_decoder *d, k::DecodeFeed *feed, cudaGraphExec_t *out) {
    if (si_status st = cuda(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture"))
        return st;
    const si_status rec = record_step(d, feed);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(d->stream, &g);
    if (rec != SI_OK) {
        if (g) cudaGraphDestroy(g);
        return rec;
    }
    if (e != cudaSuccess) return cuda(e, "cudaStreamEndCapture");
    const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return cuda(ie, "cudaGraphInstantiate");
}

// Prefill chunk rows: two tcgen05 GEMM tiles of input rows (N = 256 each).
// Measured against 256-row chunks on a 512-token Phi-4-mini prompt: 15.4 vs
// 19.7 ms (half the chunks: half the X splits, reductions and launches).
constexpr int64_t kPrefillRows = 512;

si_status ensure_prefill(si_decoder *d) {
    if (d->pf_ready) return SI_OK;
    const si_decoder_config &c = d->cfg;
    const int64_t H = c.hidden, KV = int64_t(c.kv_heads) * c.head_size, QKV = H + 2 * KV, F = c.intermediate;
    const int64_t R = kPrefillRows;
    auto &P = d->pf;
    struct A {
        const char *name;
        float **dst;
        int64_t n;
    } acts[] = {{"batch_hidden", &P.hidden, R * H},       {"batch_hidden_after_attention", &P.after, R * H},
                {"batch_normalized", &P.normalized, R * H}, {"batch_qkv", &P.qkv, R * QKV},
                {"batch_query", &P.query, R * H},         {"batch_attention", &P.attention, R * H},
                {"batch_projected", &P.projected, R * H}, {"batch_gate_up", &P.gate_up, R * 2 * F},
                {"batch_activated", &P.activated, R * F}, {"batch_down", &P.down, R * H}};
    for (const A &a : acts)
        if (si_status st = alloc_typed(d, a.name, uint64_t(a.n) * 4, a.dst)) return st;
    const int64_t chunks = (c.context + R - 1) / R;
    if (si_status st = alloc_typed(d, "prefill_control", uint64_t(chunks) * 8, &P.control)) return st;
    uint64_t ws = 0;
    for (auto [n, kk] : {std::pair<int64_t, int64_t>{QKV, H}, {H, H}, {2 * F, H}, {H, F}})
        for (int64_t rows = 64; rows <= R; rows += 64) {  // the split count depends on the rows
            uint64_t b = 0;
            for (uint32_t t : {d->t_qkv[0], d->t_out[0], d->t_up[0], d->t_down[0], uint32_t(SI_TYPE_Q4_K),
                               uint32_t(SI_TYPE_Q8_0)}) {
                k::gemm_workspace_bytes(t, rows, n, kk, &b);
                ws = std::max(ws, b);
            }
            ws = std::max(ws, b);
        }
    if (ws) {
        void *p = nullptr;
        if (si_status st = alloc_slot(d, "gemm_workspace", ws, &p)) return st;
        P.workspace = p;
        P.workspace_bytes = ws;
    }
    d->pf_ready = true;
    return SI_OK;
}

// Y[rows, n] = X[rows, k] W^T: the tcgen05 GEMM from 64 rows, the batch
// GEMV below that.
si_status batch_project(si_decoder *d, uint32_t type, const void *w, const float *x, float *y, int64_t rows, int64_t n,
                        int64_t k) {
    return k::gemm_tn(type, x, w, y, rows, n, k, d->pf.workspace, d->pf.workspace_bytes, d->stream);
}

// The prefill program of one chunk (Phi4D3D12TextSession.cs:1018-1155) on
// rows [start, start + rows) whose hidden rows are already in pf.hidden:
// batch instructions with control = (start, rows), the three attention
// instructions fused, and after the last chunk select-last -> vocabulary
// projection -> argmax into next_token.
si_status prefill_chunk(si_decoder *d, const int32_t *control, int32_t start, int32_t rows, bool last,
                        int64_t cache_offset) {
    const si_decoder_config &c = d->cfg;
    const int64_t H = c.hidden, KV = int64_t(c.kv_heads) * c.head_size, QKV = H + 2 * KV, F = c.intermediate;
    auto &P = d->pf;
    cudaStream_t s = d->stream;
    if (si_status st = k::tr_rms_norm(P.hidden, nullptr, d->attn_norm[0], control, nullptr, P.normalized, rows, H,
                                      c.epsilon, s))
        return st;
    for (int l = 0; l < c.layers; ++l) {
        if (si_status st = batch_project(d, d->t_qkv[l], d->w_qkv[l], P.normalized, P.qkv, rows, QKV, H)) return st;
        float *kc = d->key_cache[l] + cache_offset, *vc = d->value_cache[l] + cache_offset;
        if (si_status st = k::tr_rope_kv_write(P.qkv, nullptr, control, d->freq, P.query, kc, vc, rows, H, KV,
                                               c.head_size, c.rotary_size, c.context,
                                               c.rope_scale, s))
            return st;
        if (si_status st = k::tr_prefill_attention(P.query, kc, vc, start, rows,
                                                   P.attention, c.query_heads, c.kv_heads, c.head_size, c.context, s))
            return st;
        if (si_status st = batch_project(d, d->t_out[l], d->w_out[l], P.attention, P.projected, rows, H, H)) return st;
        if (si_status st = k::tr_rms_norm(P.hidden, P.projected, d->ffn_norm[l], control, P.after, P.normalized, rows,
                                          H, c.epsilon, s))
            return st;
        if (si_status st = batch_project(d, d->t_up[l], d->w_up[l], P.normalized, P.gate_up, rows, 2 * F, H)) return st;
        if (si_status st = k::tr_swiglu(P.gate_up, control, P.activated, rows, F, s)) return st;
        if (si_status st = batch_project(d, d->t_down[l], d->w_down[l], P.activated, P.down, rows, H, F)) return st;
        const float *next_norm = l + 1 < c.layers ? d->attn_norm[l + 1] : d->output_norm;
        if (si_status st = k::tr_rms_norm(P.after, P.down, next_norm, control, P.hidden, P.normalized, rows, H,
                                          c.epsilon, s))
            return st;
    }
    if (!last) return SI_OK;
    if (si_status st = k::tr_select_last(P.normalized, control, d->normalized, rows, H, s)) return st;
    if (si_status st = project_rows(d, si_decoder::kVocab, c.embedding_type, d->w_vocab, d->normalized, d->logits, c.vocab, H)) return st;
    return k::tr_argmax(d->logits, c.vocab, d->next_token, nullptr, s);
}

// Prefill of `count` rows from the session position: token ids (gathered
// from token_embedding) or ready embedding rows from the host.
// `start0`: the first row's position; `cache_offset`: floats from each
// layer's cache base to the stream's cache (0 for a single-stream session).
si_status prefill(si_decoder *d, const int32_t *tokens, const float *embeddings, int32_t count, int32_t start0,
                  int64_t cache_offset, int32_t *next_token) {
    const si_decoder_config &c = d->cfg;
    const int64_t H = c.hidden;
    if (si_status st = ensure_prefill(d)) return st;
    cudaStream_t s = d->stream;
    const int32_t chunks = int32_t((count + kPrefillRows - 1) / kPrefillRows);
    std::vector<int32_t> pairs(size_t(chunks) * 2);
    for (int32_t i = 0; i < chunks; ++i) {
        pairs[size_t(2 * i)] = start0 + int32_t(i * kPrefillRows);
        pairs[size_t(2 * i + 1)] = int32_t(std::min<int64_t>(kPrefillRows, count - i * kPrefillRows));
    }
    if (si_status st = cuda(cudaMemcpyAsync(d->pf.control, pairs.data(), pairs.size() * 4, cudaMemcpyHostToDevice, s),
                            "upload"))
        return st;
    if (tokens) {
        std::memcpy(d->pinned_prompt, tokens, size_t(count) * 4);
        if (si_status st = cuda(cudaMemcpyAsync(d->prompt, d->pinned_prompt, size_t(count) * 4,
                                                cudaMemcpyHostToDevice, s), "upload"))
            return st;
    }
    for (int32_t i = 0; i < chunks; ++i) {
        const int32_t start = pairs[size_t(2 * i)], rows = pairs[size_t(2 * i + 1)];
        const int64_t first = int64_t(i) * kPrefillRows;
        if (tokens) {
            if (si_status st = k::tr_gather_rows_quant(c.embedding_type, d->embedding, c.vocab, H, d->prompt + first,
                                                       rows, d->pf.hidden, s))
                return st;
        } else if (si_status st = cuda(cudaMemcpyAsync(d->pf.hidden, embeddings + first * H, size_t(rows) * H * 4,
                                                       cudaMemcpyHostToDevice, s), "upload")) {
            return st;
        }
        if (si_status st = prefill_chunk(d, d->pf.control + 2 * i, start, rows, i + 1 == chunks, cache_offset))
            return st;
    }
    if (si_status st = cuda(cudaMemcpyAsync(d->pinned + 2, d->next_token, 4, cudaMemcpyDeviceToHost, s), "readback"))
        return st;
    if (si_status st = cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize")) return st;
    *next_token = d->pinned[2];
    return SI_OK;
}

// One decode step of every stream of a multi-stream session: the decode
// program with each instruction over `streams` rows -- the projections as
// the few-row tcgen05 GEMM (each weight read once per step for all
// streams), rope-kv-write and attention at each stream's own position and
// cache, argmax per row.
si_status record_step_streams(si_decoder *d, k::StreamsFeed *sfeed) {
    const si_decoder_config &c = d->cfg;
    const int64_t H = c.hidden, KV = int64_t(c.kv_heads) * c.head_size, QKV = H + 2 * KV, F = c.intermediate;
    const int64_t B = d->streams, stride = c.context * KV;
    cudaStream_t s = d->stream;
    auto proj = [&](uint32_t type, const void *w, const float *x, float *y, int64_t rows, int64_t cols) {
        return k::shared_weight_matvec(type, w, x, nullptr, y, B, rows, cols, s);
    };
    if (si_status st = k::tr_gather_rows_quant(c.embedding_type, d->embedding, c.vocab, H, d->st_tokens, B, d->hidden,
                                               s))
        return st;
    if (si_status st = k::tr_rms_norm(d->hidden, nullptr, d->attn_norm[0], nullptr, nullptr, d->normalized, B, H,
                                      c.epsilon, s))
        return st;
    for (int l = 0; l < c.layers; ++l) {
        if (si_status st = proj(d->t_qkv[l], d->w_qkv[l], d->normalized, d->qkv, QKV, H)) return st;
        if (si_status st = k::tr_rope_kv_write_streams(d->qkv, d->st_positions, d->freq, d->query, d->key_cache[l],
                                                       d->value_cache[l], B, H, KV, c.head_size, c.rotary_size,
                                                       c.context, stride, c.rope_scale, s))
            return st;
        if (si_status st = k::tr_attention_decode_streams(d->query, d->key_cache[l], d->value_cache[l],
                                                          d->st_positions, d->attention, int(B), c.query_heads,
                                                          c.kv_heads, c.head_size, c.context, stride, s))
            return st;
        if (si_status st = proj(d->t_out[l], d->w_out[l], d->attention, d->projected, H, H)) return st;
        if (si_status st = k::tr_rms_norm(d->hidden, d->projected, d->ffn_norm[l], nullptr, d->after, d->normalized, B,
                                          H, c.epsilon, s))
            return st;
        if (si_status st = proj(d->t_up[l], d->w_up[l], d->normalized, d->gate_up, 2 * F, H)) return st;
        if (si_status st = k::tr_swiglu(d->gate_up, nullptr, d->activated, B, F, s)) return st;
        if (si_status st = proj(d->t_down[l], d->w_down[l], d->activated, d->down, H, F)) return st;
        const float *next_norm = l + 1 < c.layers ? d->attn_norm[l + 1] : d->output_norm;
        if (si_status st = k::tr_rms_norm(d->after, d->down, next_norm, nullptr, d->hidden, d->normalized, B, H,
                                          c.epsilon, s))
            return st;
    }
    if (si_status st = proj(c.embedding_type, d->embedding, d->normalized, d->logits, c.vocab, H)) return st;
    return k::tr_argmax_rows(d->logits, B, c.vocab, d->st_next, sfeed, s);
}

si_status build_streams_graph(si_decoder *d, k::StreamsFeed *sfeed, cudaGraphExec_t *out) {
    if (si_status st = cuda(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture"))
        return st;
    const si_status rec = record_step_streams(d, sfeed);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(d->stream, &g);
    if (rec != SI_OK) {
        if (g) cudaGraphDestroy(g);
        return rec;
    }
    if (e != cudaSuccess) return cuda(e, "cudaStreamEndCapture");
    const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return cuda(ie, "cudaGraphInstantiate");
}

// Host-side checks of a multi-stream call: every stream's token in the
// vocabulary and positions [p, p + steps) inside the context.
si_status check_streams(si_decoder *d, const int32_t *tokens, const int32_t *positions, int32_t steps) {
    if (d->streams < 2) return fail(SI_ERR_INVALID_ARGUMENT, "not a multi-stream session");
    for (int32_t b = 0; b < d->streams; ++b) {
        if (tokens[b] < 0 || tokens[b] >= d->cfg.vocab)
            return fail(SI_ERR_INVALID_ARGUMENT, "stream %d: token %d outside the vocabulary", b, tokens[b]);
        if (positions[b] < 0 || int64_t(positions[b]) + steps > d->cfg.context)
            return fail(SI_ERR_INVALID_ARGUMENT,
                        "stream %d: positions %d..%d exceed the GPU KV cache capacity of %lld tokens", b,
                        positions[b], positions[b] + steps - 1, (long long)d->cfg.context);
    }
    return SI_OK;
}

si_status upload_streams(si_decoder *d, const int32_t *tokens, const int32_t *positions, bool start) {
    const size_t B = size_t(d->streams);
    cudaStream_t s = d->stream;
    std::memcpy(d->pinned_st, tokens, B * 4);
    std::memcpy(d->pinned_st + B, positions, B * 4);
    if (si_status st = cuda(cudaMemcpyAsync(d->st_tokens, d->pinned_st, B * 4, cudaMemcpyHostToDevice, s), "upload"))
        return st;
    if (si_status st = cuda(cudaMemcpyAsync(d->st_positions, d->pinned_st + B, B * 4, cudaMemcpyHostToDevice, s),
                            "upload"))
        return st;
    if (start)
        return cuda(cudaMemcpyAsync(d->st_start, d->pinned_st + B, B * 4, cudaMemcpyHostToDevice, s), "upload");
    return SI_OK;
}

si_status validate(const si_decoder_config *c) {
    if (!c) return fail(SI_ERR_INVALID_ARGUMENT, "null config");
    if (c->layers <= 0 || c->hidden <= 0 || c->query_heads <= 0 || c->kv_heads <= 0 || c->head_size <= 0 ||
        c->rotary_size <= 0 || c->intermediate <= 0 || c->vocab <= 0 || c->context <= 0 || c->context > INT32_MAX)
        return fail(SI_ERR_INVALID_ARGUMENT, "decoder dimensions must be positive");
    if (int64_t(c->query_heads) * c->head_size != c->hidden)
        return fail(SI_ERR_ADAPTATION, "query_heads * head_size (%d * %d) must equal hidden (%d)", c->query_heads,
                    c->head_size, c->hidden);
    if (c->query_heads % c->kv_heads) return fail(SI_ERR_ADAPTATION, "Query heads must be divisible by key/value heads.");
    if (c->query_heads / c->kv_heads > 8 || c->head_size > 256)
        return fail(SI_ERR_UNSUPPORTED, "attention supports up to 8 query heads per key/value head and head_size <= 256");
    if (c->rotary_size > c->head_size || c->rotary_size % 2)
        return fail(SI_ERR_ADAPTATION, "Invalid query, cache, head, or rotary dimensions.");
    if (!(std::isfinite(c->epsilon) && c->epsilon > 0) || !(std::isfinite(c->rope_scale) && c->rope_scale > 0) ||
        !(std::isfinite(c->rope_base) && c->rope_base > 0))
        return fail(SI_ERR_ADAPTATION, "epsilon, rope_base and rope_scale must be finite and positive");
    if (!si::known_type(c->weight_type) || !si::known_type(c->embedding_type))
        return fail(SI_ERR_UNSUPPORTED, "unsupported weight type");
    uint64_t b;
    for (int64_t cols : {int64_t(c->hidden), int64_t(c->intermediate)})
        if (si_status st = si::byte_length(c->weight_type, uint64_t(cols), &b)) return st;
    return si::byte_length(c->embedding_type, uint64_t(c->hidden), &b);
}


// slot_types: null, or one GGUF type per slot of si_decoder_slot order
// (token_embedding, output_norm, then per layer attn_norm, ffn_norm, qkv,
// attn_output, ffn_up, ffn_down): the projections' own types.
si_status create(int device, const si_decoder_config *c, si_peer_group *group, int32_t streams,
                 uint64_t shard_min_bytes, si_decoder **out, const uint32_t *slot_types = nullptr) {
    auto *d = new si_decoder();
    d->device = device;
    d->cfg = *c;
    d->streams = streams;
    const uint64_t B = uint64_t(streams);
    auto cleanup = [&](si_status st) {
        destroy(d);
        return st;
    };
    if (si_status st = cuda(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "cudaStreamCreate"))
        return cleanup(st);
    const int64_t H = c->hidden, KV = int64_t(c->kv_heads) * c->head_size, QKV = H + 2 * KV, F = c->intermediate;
    uint64_t rb_h = 0, rb_f = 0, rb_e = 0;
    si::byte_length(c->weight_type, uint64_t(H), &rb_h);
    si::byte_length(c->weight_type, uint64_t(F), &rb_f);
    si::byte_length(c->embedding_type, uint64_t(H), &rb_e);
    int nranks = 1, rank = 0;
    uint64_t data_bytes = 0;
    if (group) {
        d->group = group;
        d->arena = si::peer_group_arena(group, &nranks, &rank, &data_bytes);
    }
    // A projection is split by rows when its weight bytes reach
    // shard_min_bytes; rows of it held by this rank (all of them otherwise).
    if (group) {
        const uint64_t bytes[5] = {rb_h * uint64_t(QKV), rb_h * uint64_t(H), rb_h * uint64_t(2 * F),
                                   rb_f * uint64_t(H), rb_e * uint64_t(c->vocab)};
        bool any = false;
        for (int kind = 0; kind < 5; ++kind) any |= d->sharded[kind] = bytes[kind] >= shard_min_bytes;
        // a layer-repeated peer call in every layer, so that the vocabulary
        // projection is never the only one (its logits region has one copy)
        if (any) d->sharded[si_decoder::kUp] = true;
    }
    auto shard = [&](int kind, int64_t rows, int64_t *begin) {
        int64_t b = 0, n = rows, per = rows;
        if (group && d->sharded[kind]) si_rowshard_plan(rows, nranks, rank, &b, &n, &per);
        if (begin) *begin = b;
        return n;
    };
    void *p = nullptr;
    // The whole table on every rank: gather-row reads any token's row.
    if (si_status st = alloc_slot(d, "token_embedding", rb_e * uint64_t(c->vocab), &p)) return cleanup(st);
    d->embedding = p;
    {
        int64_t vocab_begin = 0;
        shard(si_decoder::kVocab, c->vocab, &vocab_begin);
        d->w_vocab = static_cast<const uint8_t *>(p) + uint64_t(vocab_begin) * rb_e;
    }

    float *f = nullptr;
    if (si_status st = alloc_typed(d, "output_norm", H * 4, &f)) return cleanup(st);
    if (si_status st = fill_ones(f, H)) return cleanup(st);
    d->output_norm = f;
    for (int l = 0; l < c->layers; ++l) {
        const std::string L = std::to_string(l);
        if (si_status st = alloc_typed(d, "attn_norm_" + L, H * 4, &f)) return cleanup(st);
        if (si_status st = fill_ones(f, H)) return cleanup(st);
        d->attn_norm.push_back(f);
        if (si_status st = alloc_typed(d, "ffn_norm_" + L, H * 4, &f)) return cleanup(st);
        if (si_status st = fill_ones(f, H)) return cleanup(st);
        d->ffn_norm.push_back(f);
        const uint32_t *lt = slot_types ? slot_types + 2 + 6 * l : nullptr;
        const uint32_t tq = lt ? lt[2] : c->weight_type, to = lt ? lt[3] : c->weight_type,
                       tu = lt ? lt[4] : c->weight_type, td = lt ? lt[5] : c->weight_type;
        d->t_qkv.push_back(tq), d->t_out.push_back(to), d->t_up.push_back(tu), d->t_down.push_back(td);
        auto rb = [](uint32_t t, int64_t cols) {
            uint64_t b = 0;
            si::byte_length(t, uint64_t(cols), &b);
            return b;
        };
        if (si_status st = alloc_slot(d, "qkv_weight_" + L, rb(tq, H) * uint64_t(shard(si_decoder::kQkv, QKV, nullptr)), &p))
            return cleanup(st);
        d->w_qkv.push_back(p);
        if (si_status st = alloc_slot(d, "attn_output_weight_" + L, rb(to, H) * uint64_t(shard(si_decoder::kOut, H, nullptr)), &p))
            return cleanup(st);
        d->w_out.push_back(p);
        if (si_status st = alloc_slot(d, "ffn_up_weight_" + L, rb(tu, H) * uint64_t(shard(si_decoder::kUp, 2 * F, nullptr)), &p))
            return cleanup(st);
        d->w_up.push_back(p);
        if (si_status st = alloc_slot(d, "ffn_down_weight_" + L, rb(td, F) * uint64_t(shard(si_decoder::kDown, H, nullptr)), &p))
            return cleanup(st);
        d->w_down.push_back(p);
        if (si_status st = alloc_typed(d, "key_cache_" + L, B * uint64_t(c->context) * KV * 4, &f)) return cleanup(st);
        d->key_cache.push_back(f);
        if (si_status st = alloc_typed(d, "value_cache_" + L, B * uint64_t(c->context) * KV * 4, &f))
            return cleanup(st);
        d->value_cache.push_back(f);
    }
    // rope_frequencies initializer (Phi4D3D12TextSession.cs:394-398).
    if (si_status st = alloc_typed(d, "rope_frequencies", uint64_t(c->rotary_size / 2) * 4, &d->freq)) return cleanup(st);
    {
        std::vector<float> fr(size_t(c->rotary_size / 2));
        for (int i = 0; i < c->rotary_size / 2; ++i)
            fr[size_t(i)] = 1.0f / std::pow(c->rope_base, 2.0f * float(i) / float(c->rotary_size));
        if (si_status st = cuda(cudaMemcpy(d->freq, fr.data(), fr.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy"))
            return cleanup(st);
    }
    struct A {
        const char *name;
        float **dst;
        int64_t n;
    } acts[] = {{"hidden", &d->hidden, H},         {"hidden_after_attention", &d->after, H},
                {"normalized", &d->normalized, H}, {"qkv", &d->qkv, QKV},
                {"query", &d->query, H},           {"attention", &d->attention, H},
                {"projected", &d->projected, H},   {"gate_up", &d->gate_up, 2 * F},
                {"activated", &d->activated, F},   {"down", &d->down, H},
                {"logits", &d->logits, c->vocab}};
    const ArenaLayout lay = arena_layout(*c);
    for (const A &a : acts) {
        // Row-sharded: the projection outputs are the arena's vectors.
        const std::string name = a.name;
        uint64_t off = UINT64_MAX;
        if (group) {
            if (name == "qkv") off = lay.qkv[0];
            else if (name == "projected") off = lay.out[0];
            else if (name == "gate_up") off = lay.up[0];
            else if (name == "down") off = lay.down[0];
            else if (name == "logits") off = lay.logits;
        }
        if (off != UINT64_MAX) {
            *a.dst = reinterpret_cast<float *>(d->arena + off);
            d->slots[name] = {d->arena + off, uint64_t(a.n) * 4};
        } else if (si_status st = alloc_typed(d, a.name, B * uint64_t(a.n) * 4, a.dst)) {
            return cleanup(st);
        }
    }
    if (group) {
        for (int par = 0; par < 2; ++par) {
            d->par_qkv[par] = reinterpret_cast<float *>(d->arena + lay.qkv[par]);
            d->par_out[par] = reinterpret_cast<float *>(d->arena + lay.out[par]);
            d->par_up[par] = reinterpret_cast<float *>(d->arena + lay.up[par]);
            d->par_down[par] = reinterpret_cast<float *>(d->arena + lay.down[par]);
        }
    }
    if (streams > 1) {
        const uint64_t cap = uint64_t(c->context);
        if (si_status st = alloc_typed(d, "stream_tokens", B * 4, &d->st_tokens)) return cleanup(st);
        if (si_status st = alloc_typed(d, "stream_positions", B * 4, &d->st_positions)) return cleanup(st);
        if (si_status st = alloc_typed(d, "stream_start", B * 4, &d->st_start)) return cleanup(st);
        if (si_status st = alloc_typed(d, "stream_next", B * 4, &d->st_next)) return cleanup(st);
        if (si_status st = alloc_typed(d, "stream_history", B * cap * 4, &d->st_history)) return cleanup(st);
        if (si_status st = alloc_typed(d, "stream_feed", sizeof(k::StreamsFeed), &d->st_feed)) return cleanup(st);
        const k::StreamsFeed feed{d->st_tokens, d->st_positions, d->st_start, d->st_history, int32_t(cap), streams};
        if (si_status st = cuda(cudaMemcpy(d->st_feed, &feed, sizeof feed, cudaMemcpyHostToDevice), "cudaMemcpy"))
            return cleanup(st);
        if (si_status st = cuda(cudaMallocHost(reinterpret_cast<void **>(&d->pinned_st), (3 * B + B * cap) * 4),
                                "cudaMallocHost"))
            return cleanup(st);
    }
    if (si_status st = alloc_typed(d, "control", 8, &d->control)) return cleanup(st);
    if (si_status st = alloc_typed(d, "next_token", 4, &d->next_token)) return cleanup(st);
    if (si_status st = alloc_typed(d, "prompt", uint64_t(c->context) * 4, &d->prompt)) return cleanup(st);
    if (si_status st = alloc_typed(d, "history", uint64_t(c->context) * 4, &d->history)) return cleanup(st);
    if (si_status st = alloc_typed(d, "feed", sizeof(k::DecodeFeed), &d->feed)) return cleanup(st);
    const size_t pinned_bytes = 64 + sizeof(k::DecodeFeed) + 2 * size_t(c->context) * 4;
    if (si_status st = cuda(cudaMallocHost(reinterpret_cast<void **>(&d->pinned), pinned_bytes), "cudaMallocHost"))
        return cleanup(st);
    d->pinned_feed = reinterpret_cast<k::DecodeFeed *>(reinterpret_cast<uint8_t *>(d->pinned) + 64);
    d->pinned_prompt = reinterpret_cast<int32_t *>(d->pinned_feed + 1);
    d->pinned_history = d->pinned_prompt + c->context;
    if (si_status st = cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize")) return cleanup(st);
    *out = d;
    return SI_OK;
}

// ---- tensor-parallel session ------------------------------------------------
// Megatron-style pairing of the decode program over the ranks of a peer
// group, one GPU each:
//   qkv       rows of this rank's key/value heads (their query, key and value
//             rows), input = rms-norm of the residual stream
//   attention this rank's heads only (rope-kv-write fused, local caches)
//   out       K-parallel: W_o[:, this rank's query-head columns] times the
//             local attention output; the partial vector goes to every
//             rank's arena (the exchange is fused into the GEMV)
//   gate_up   rows of this rank's slice of the intermediate (its gate rows
//             and the matching up rows), input = rms-norm of (residual +
//             the out partials of every rank, in rank order)
//   down      K-parallel over the same slice, swiglu fused into its input,
//             partial vector exchanged like out's
// and the vocabulary projection row-sharded over the ranks (rows gathered
// into every arena) after the final norm, then argmax on every rank. Two
// exchanges per layer; every rank sums the partials in the same order, so
// every rank holds bit-identical residual streams and picks the same token.
// The out and down exchanges are publish-only: the producing GEMV stores its
// partial rows into every arena, fences, and adds its row count to every
// rank's count of that exchange; it does not wait for the peers. The
// consuming GEMV (gate_up after out; the next qkv, or the vocabulary GEMV,
// after down) waits for every rank's count after its weight prefetch.
// Region reuse: rank A writes the out partials of layer l + 1 into rank B's
// arena only after A's qkv of layer l + 1 saw B's down count of layer l,
// which B publishes from its down GEMV of layer l; that GEMV stores after
// its dependency wait, i.e. after B's gate_up of layer l — the reader of the
// out partials of layer l — completed. Likewise A writes the down partials
// of layer l + 1 only after A's gate_up of layer l + 1 saw B's out count of
// layer l + 1, published after B's qkv of layer l + 1, the reader of the
// down partials of layer l, completed. The vocabulary rows keep the full
// handshake, so every token ends with all ranks in step.
struct TpLayout {
    uint64_t o_parts, down_parts, logits, data_bytes;
};

TpLayout tp_layout(const si_decoder_config &c, int nranks) {
    auto al = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
    TpLayout t{};
    uint64_t o = 0;
    t.o_parts = o, o += al(uint64_t(nranks) * uint64_t(c.hidden) * 4);
    t.down_parts = o, o += al(uint64_t(nranks) * uint64_t(c.hidden) * 4);
    t.logits = o, o += al(uint64_t(c.vocab) * 4);
    t.data_bytes = o;
    return t;
}

// Contiguous split of `units` over n ranks, the first units % n ranks one more.
void split_units(int64_t units, int n, int r, int64_t *begin, int64_t *count) {
    const int64_t base = units / n, extra = units % n;
    *count = base + (r < extra ? 1 : 0);
    *begin = r * base + std::min<int64_t>(r, extra);
}

si_status tp_plan(const si_decoder_config &c, int n, int r, si_tp_partition *p) {
    if (n < 1 || r < 0 || r >= n) return fail(SI_ERR_INVALID_ARGUMENT, "rank %d of %d ranks", r, n);
    if (c.kv_heads < n)
        return fail(SI_ERR_UNSUPPORTED, "%d key/value heads cannot be split over %d ranks", c.kv_heads, n);
    const int G = c.query_heads / c.kv_heads;
    int64_t b = 0, cnt = 0;
    split_units(c.kv_heads, n, r, &b, &cnt);
    p->kv_head_begin = int32_t(b), p->kv_heads = int32_t(cnt);
    p->query_head_begin = int32_t(b * G), p->query_heads = int32_t(cnt * G);
    // the intermediate in 256-element units: the down GEMV's K slice is whole superblocks
    if (c.intermediate % 256) return fail(SI_ERR_UNSUPPORTED, "intermediate %d is not a multiple of 256", c.intermediate);
    split_units(c.intermediate / 256, n, r, &b, &cnt);
    if (cnt == 0) return fail(SI_ERR_UNSUPPORTED, "intermediate %d leaves rank %d without rows", c.intermediate, r);
    p->ffn_begin = b * 256, p->ffn_rows = cnt * 256;
    int64_t per = 0;
    if (si_status st = si_rowshard_plan(c.vocab, n, r, &b, &cnt, &per)) return st;
    if (per * (n - 1) >= c.vocab) return fail(SI_ERR_UNSUPPORTED, "vocabulary %d leaves a rank without rows", c.vocab);
    p->vocab_begin = b, p->vocab_rows = cnt;
    // the out projection's K slice (this rank's query-head columns) is whole superblocks too
    for (int q = 0; q < n; ++q) {
        int64_t kb, kc;
        split_units(c.kv_heads, n, q, &kb, &kc);
        if ((kb * G * c.head_size) % 256 || (kc * G * c.head_size) % 256)
            return fail(SI_ERR_UNSUPPORTED,
                        "the out projection's column slice of rank %d (%lld query heads of %d) is not a multiple of "
                        "256 columns", q, (long long)(kc * G), c.head_size);
    }
    return SI_OK;
}

si_status record_step_tp(si_decoder *d, k::DecodeFeed *feed) {
    const si_decoder_config &c = d->cfg;
    const si_tp_partition &P = d->part;
    const int64_t H = c.hidden, hs = c.head_size;
    const int64_t qkv_local = int64_t(P.query_heads + 2 * P.kv_heads) * hs, q_cols = int64_t(P.query_heads) * hs;
    const int nranks = d->pg_out.nranks;
    cudaStream_t s = d->stream;
    int32_t *position = d->control + 1;
    auto gemv = [&](uint32_t type, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                    const k::GemvFusion &f, const k::PeerGather *peer) -> si_status {
        const si_status st = k::matvec_quant_fused(type, w, x, y, rows, cols, f, s, peer);
        if (st == SI_ERR_UNSUPPORTED)
            return fail(SI_ERR_UNSUPPORTED, "tensor-parallel step: no tensor-core GEMV for [%lld, %lld]",
                        (long long)rows, (long long)cols);
        return st;
    };
    // the GEMV input: rms-norm of (x + parts[0] + ... + parts[nparts-1]), that sum stored to h_out;
    // the parts of the publish-only exchanges are read once every rank's count has arrived
    auto norm_of = [&](const float *parts, int nparts, const float *norm, float *h_out) {
        k::GemvFusion f;
        f.in_mode = 3;
        f.norm_w = norm;
        f.eps = c.epsilon;
        f.parts = parts;
        f.nparts = nparts;
        f.part_stride = H;
        f.h_out = h_out;
        if (nparts > 0) {
            f.wait_counts = parts == d->o_parts ? d->o_counts : d->d_counts;
            f.wait_epoch = parts == d->o_parts ? d->o_epoch : d->d_epoch;
            f.wait_ranks = nparts;
            f.wait_rows = H;
        }
        return f;
    };
    if (si_status st = k::tr_gather_row(c.embedding_type, d->embedding, c.vocab, H, d->control, d->res_b, s)) return st;
    for (int l = 0; l < c.layers; ++l) {
        // residual stream: res_b (+ the previous layer's down partials) -> res_a
        if (si_status st = gemv(d->t_qkv[l], d->w_qkv[l], d->res_b, d->qkv, qkv_local, H,
                                norm_of(d->down_parts, l ? nranks : 0, d->attn_norm[l], d->res_a), nullptr))
            return st;
        if (si_status st = k::tr_attention_decode_rope(d->qkv, position, d->freq, d->key_cache[l], d->value_cache[l],
                                                       d->attention, P.query_heads, P.kv_heads, c.head_size,
                                                       c.rotary_size, c.context, c.rope_scale, s))
            return st;
        if (si_status st = gemv(d->t_out[l], d->w_out[l], d->attention, nullptr, H, q_cols, k::GemvFusion{}, &d->pg_out))
            return st;
        // residual stream: res_a + the out partials -> res_b
        if (si_status st = gemv(d->t_up[l], d->w_up[l], d->res_a, d->gate_up, 2 * P.ffn_rows, H,
                                norm_of(d->o_parts, nranks, d->ffn_norm[l], d->res_b), nullptr))
            return st;
        k::GemvFusion sw;
        sw.in_mode = 2;
        if (si_status st = gemv(d->t_down[l], d->w_down[l], d->gate_up, nullptr, H, P.ffn_rows, sw, &d->pg_down))
            return st;
    }
    if (si_status st = gemv(c.embedding_type, d->w_vocab, d->res_b, nullptr, P.vocab_rows, H,
                            norm_of(d->down_parts, nranks, d->output_norm, nullptr), &d->pg_vocab))
        return st;
    return k::tr_argmax(d->logits, c.vocab, d->next_token, feed, s);
}

si_status create_tp(int device, const si_decoder_config *c, si_peer_group *group, si_decoder **out) {
    auto *d = new si_decoder();
    d->device = device;
    d->cfg = *c;
    d->tp = true;
    d->group = group;
    auto cleanup = [&](si_status st) {
        destroy(d);
        return st;
    };
    int nranks = 1, rank = 0;
    uint64_t data_bytes = 0;
    d->arena = si::peer_group_arena(group, &nranks, &rank, &data_bytes);
    if (si_status st = tp_plan(*c, nranks, rank, &d->part)) return cleanup(st);
    const si_tp_partition &P = d->part;
    const TpLayout lay = tp_layout(*c, nranks);
    if (data_bytes < lay.data_bytes)
        return cleanup(fail(SI_ERR_INVALID_ARGUMENT, "the peer group's arenas hold %llu data bytes, the session needs %llu",
                            (unsigned long long)data_bytes, (unsigned long long)lay.data_bytes));
    if (si_status st = cuda(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "cudaStreamCreate"))
        return cleanup(st);
    const int64_t H = c->hidden, hs = c->head_size, F = P.ffn_rows;
    const int64_t qkv_local = int64_t(P.query_heads + 2 * P.kv_heads) * hs, q_cols = int64_t(P.query_heads) * hs;
    const int64_t kv_local = int64_t(P.kv_heads) * hs;
    auto rb = [](uint32_t t, int64_t cols) {
        uint64_t b = 0;
        si::byte_length(t, uint64_t(cols), &b);
        return b;
    };
    void *p = nullptr;
    if (si_status st = alloc_slot(d, "token_embedding", rb(c->embedding_type, H) * uint64_t(c->vocab), &p))
        return cleanup(st);
    d->embedding = p;
    d->w_vocab = static_cast<const uint8_t *>(p) + uint64_t(P.vocab_begin) * rb(c->embedding_type, H);
    float *f = nullptr;
    if (si_status st = alloc_typed(d, "output_norm", H * 4, &f)) return cleanup(st);
    if (si_status st = fill_ones(f, H)) return cleanup(st);
    d->output_norm = f;
    const uint32_t t = c->weight_type;
    for (int l = 0; l < c->layers; ++l) {
        const std::string L = std::to_string(l);
        if (si_status st = alloc_typed(d, "attn_norm_" + L, H * 4, &f)) return cleanup(st);
        if (si_status st = fill_ones(f, H)) return cleanup(st);
        d->attn_norm.push_back(f);
        if (si_status st = alloc_typed(d, "ffn_norm_" + L, H * 4, &f)) return cleanup(st);
        if (si_status st = fill_ones(f, H)) return cleanup(st);
        d->ffn_norm.push_back(f);
        d->t_qkv.push_back(t), d->t_out.push_back(t), d->t_up.push_back(t), d->t_down.push_back(t);
        // this rank's rows: its query heads, then its key heads, then its value heads
        if (si_status st = alloc_slot(d, "qkv_weight_" + L, rb(t, H) * uint64_t(qkv_local), &p)) return cleanup(st);
        d->w_qkv.push_back(p);
        // every row, this rank's query-head columns
        if (si_status st = alloc_slot(d, "attn_output_weight_" + L, rb(t, q_cols) * uint64_t(H), &p)) return cleanup(st);
        d->w_out.push_back(p);
        // this rank's gate rows, then the matching up rows
        if (si_status st = alloc_slot(d, "ffn_up_weight_" + L, rb(t, H) * uint64_t(2 * F), &p)) return cleanup(st);
        d->w_up.push_back(p);
        // every row, this rank's intermediate columns
        if (si_status st = alloc_slot(d, "ffn_down_weight_" + L, rb(t, F) * uint64_t(H), &p)) return cleanup(st);
        d->w_down.push_back(p);
        if (si_status st = alloc_typed(d, "key_cache_" + L, uint64_t(c->context) * kv_local * 4, &f)) return cleanup(st);
        d->key_cache.push_back(f);
        if (si_status st = alloc_typed(d, "value_cache_" + L, uint64_t(c->context) * kv_local * 4, &f))
            return cleanup(st);
        d->value_cache.push_back(f);
    }
    if (si_status st = alloc_typed(d, "rope_frequencies", uint64_t(c->rotary_size / 2) * 4, &d->freq)) return cleanup(st);
    {
        std::vector<float> fr(size_t(c->rotary_size / 2));
        for (int i = 0; i < c->rotary_size / 2; ++i)
            fr[size_t(i)] = 1.0f / std::pow(c->rope_base, 2.0f * float(i) / float(c->rotary_size));
        if (si_status st = cuda(cudaMemcpy(d->freq, fr.data(), fr.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy"))
            return cleanup(st);
    }
    if (si_status st = alloc_typed(d, "hidden", H * 4, &d->res_b)) return cleanup(st);
    if (si_status st = alloc_typed(d, "hidden_after_attention", H * 4, &d->res_a)) return cleanup(st);
    if (si_status st = alloc_typed(d, "qkv", uint64_t(qkv_local) * 4, &d->qkv)) return cleanup(st);
    if (si_status st = alloc_typed(d, "attention", uint64_t(q_cols) * 4, &d->attention)) return cleanup(st);
    if (si_status st = alloc_typed(d, "gate_up", uint64_t(2 * F) * 4, &d->gate_up)) return cleanup(st);
    d->o_parts = reinterpret_cast<float *>(d->arena + lay.o_parts);
    d->down_parts = reinterpret_cast<float *>(d->arena + lay.down_parts);
    d->logits = reinterpret_cast<float *>(d->arena + lay.logits);
    d->slots["logits"] = {d->logits, uint64_t(c->vocab) * 4};
    // out / down: publish-only exchanges (the next GEMV waits for them); the vocabulary rows: full handshake
    if (si_status st = si::peer_gather_desc_nowait(group, lay.o_parts, int64_t(rank) * H, H, 0, &d->pg_out))
        return cleanup(st);
    if (si_status st = si::peer_counts(group, 0, &d->o_counts, &d->o_epoch)) return cleanup(st);
    if (si_status st = si::peer_counts(group, 1, &d->d_counts, &d->d_epoch)) return cleanup(st);
    if (si_status st = si::peer_gather_desc_nowait(group, lay.down_parts, int64_t(rank) * H, H, 1, &d->pg_down))
        return cleanup(st);
    if (si_status st = si::peer_gather_desc(group, lay.logits, P.vocab_begin, P.vocab_rows, &d->pg_vocab))
        return cleanup(st);
    if (si_status st = alloc_typed(d, "control", 8, &d->control)) return cleanup(st);
    if (si_status st = alloc_typed(d, "next_token", 4, &d->next_token)) return cleanup(st);
    if (si_status st = alloc_typed(d, "prompt", uint64_t(c->context) * 4, &d->prompt)) return cleanup(st);
    if (si_status st = alloc_typed(d, "history", uint64_t(c->context) * 4, &d->history)) return cleanup(st);
    if (si_status st = alloc_typed(d, "feed", sizeof(k::DecodeFeed), &d->feed)) return cleanup(st);
    const size_t pinned_bytes = 64 + sizeof(k::DecodeFeed) + 2 * size_t(c->context) * 4;
    if (si_status st = cuda(cudaMallocHost(reinterpret_cast<void **>(&d->pinned), pinned_bytes), "cudaMallocHost"))
        return cleanup(st);
    d->pinned_feed = reinterpret_cast<k::DecodeFeed *>(reinterpret_cast<uint8_t *>(d->pinned) + 64);
    d->pinned_prompt = reinterpret_cast<int32_t *>(d->pinned_feed + 1);
    d->pinned_history = d->pinned_prompt + c->context;
    if (si_status st = cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize")) return cleanup(st);
    *out = d;
    return SI_OK;
}

si_status ensure_graphs(si_decoder *d) {
    if (!d->step_exec)
        if (si_status st = build_graph(d, nullptr, &d->step_exec)) return st;
    if (!d->feed_exec)
        if (si_status st = build_graph(d, d->feed, &d->feed_exec)) return st;
    return SI_OK;
}

// One decode step on the stream: the recorded graph.
si_status run_step(si_decoder *d, bool with_feed) {
    return cuda(cudaGraphLaunch(with_feed ? d->feed_exec : d->step_exec, d->stream), "cudaGraphLaunch");
}

si_status slot_range(si_decoder *d, const char *name, uint64_t offset, uint64_t bytes, uint8_t **p) {
    if (!name) return fail(SI_ERR_INVALID_ARGUMENT, "null slot name");
    auto it = d->slots.find(name);
    if (it == d->slots.end()) return fail(SI_ERR_INVALID_ARGUMENT, "No slot named '%s'.", name);
    if (offset > it->second.bytes || bytes > it->second.bytes - offset)
        return fail(SI_ERR_INVALID_ARGUMENT, "slot '%s': %llu bytes at offset %llu exceed its %llu bytes", name,
                    (unsigned long long)bytes, (unsigned long long)offset, (unsigned long long)it->second.bytes);
    *p = static_cast<uint8_t *>(it->second.ptr) + offset;
    return SI_OK;
}

}  // namespace

extern "C" {

si_status si_decoder_create(int device, const si_decoder_config *config, si_decoder **out) {
    if (!out) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (si_status st = validate(config)) return st;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(SI_ERR_NO_DEVICE, "no CUDA device is available");
    }
    if (device < 0 || device >= n) return fail(SI_ERR_INVALID_ARGUMENT, "device %d out of range [0,%d)", device, n);
    DeviceScope scope(device);
    return create(device, config, nullptr, 1, 0, out);
}

si_status si_decoder_create_typed(int device, const si_decoder_config *config, const uint32_t *slot_types,
                                  int32_t slot_count, si_decoder **out) {
    if (!out || !slot_types) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (si_status st = validate(config)) return st;
    const si_decoder_config &c = *config;
    if (slot_count != 2 + 6 * c.layers)
        return fail(SI_ERR_INVALID_ARGUMENT, "%d slot types given, the session has %d slots", slot_count,
                    2 + 6 * c.layers);
    if (slot_types[0] != c.embedding_type)
        return fail(SI_ERR_INVALID_ARGUMENT, "token_embedding type %u differs from the configuration's %u",
                    slot_types[0], c.embedding_type);
    for (int i = 0; i < slot_count; ++i) {
        const int r = i < 2 ? i : (i - 2) % 6;  // 1, 0, 1 = norms
        const bool norm = i == 1 || (i >= 2 && r < 2);
        if (norm && slot_types[i] != SI_TYPE_F32)
            return fail(SI_ERR_UNSUPPORTED, "norm slot %d must be F32 (GGUF type 0), got %u", i, slot_types[i]);
        if (!norm && !si::known_type(slot_types[i]))
            return fail(SI_ERR_UNSUPPORTED, "slot %d: GGUF tensor type '%u' is not supported.", i, slot_types[i]);
        if (!norm && i >= 2) {
            uint64_t b;
            if (si_status st = si::byte_length(slot_types[i], uint64_t(r == 5 ? c.intermediate : c.hidden), &b))
                return st;
        }
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(SI_ERR_NO_DEVICE, "no CUDA device is available");
    }
    if (device < 0 || device >= n) return fail(SI_ERR_INVALID_ARGUMENT, "device %d out of range [0,%d)", device, n);
    DeviceScope scope(device);
    return create(device, config, nullptr, 1, 0, out, slot_types);
}

si_status si_decoder_arena_bytes(const si_decoder_config *config, uint64_t *bytes) {
    if (!bytes) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    if (si_status st = validate(config)) return st;
    *bytes = arena_layout(*config).data_bytes + 4096;
    return SI_OK;
}

si_status si_decoder_create_sharded(int device, const si_decoder_config *config, si_peer_group *group,
                                    uint64_t shard_min_bytes, si_decoder **out) {
    if (!out || !group) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (si_status st = validate(config)) return st;
    const si_decoder_config &c = *config;
    for (uint32_t t : {c.weight_type, c.embedding_type})
        if (t != SI_TYPE_Q4_K && t != SI_TYPE_Q8_0)
            return fail(SI_ERR_UNSUPPORTED, "a row-sharded session takes Q4_K or Q8_0 weights");
    int nranks = 1, rank = 0;
    uint64_t data_bytes = 0;
    si::peer_group_arena(group, &nranks, &rank, &data_bytes);
    const ArenaLayout lay = arena_layout(c);
    if (data_bytes < lay.data_bytes)
        return fail(SI_ERR_INVALID_ARGUMENT, "the peer group's arenas hold %llu data bytes, the session needs %llu",
                    (unsigned long long)data_bytes, (unsigned long long)lay.data_bytes);
    const int64_t H = c.hidden, QKV = H + 2 * int64_t(c.kv_heads) * c.head_size;
    for (int64_t rows : {QKV, H, 2 * int64_t(c.intermediate), int64_t(c.vocab)}) {
        int64_t b, n, per;
        if (si_status st = si_rowshard_plan(rows, nranks, rank, &b, &n, &per)) return st;
        if (per * (nranks - 1) >= rows)
            return fail(SI_ERR_UNSUPPORTED, "%lld rows leave a rank of %d without rows", (long long)rows, nranks);
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(SI_ERR_NO_DEVICE, "no CUDA device is available");
    }
    if (device < 0 || device >= n) return fail(SI_ERR_INVALID_ARGUMENT, "device %d out of range [0,%d)", device, n);
    DeviceScope scope(device);
    return create(device, config, group, 1, shard_min_bytes, out);
}

si_status si_tp_partition_plan(const si_decoder_config *config, int32_t nranks, int32_t rank, si_tp_partition *out) {
    if (!out) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    if (si_status st = validate(config)) return st;
    return tp_plan(*config, nranks, rank, out);
}

si_status si_decoder_tp_arena_bytes(const si_decoder_config *config, int32_t nranks, uint64_t *bytes) {
    if (!bytes || nranks < 1) return fail(SI_ERR_INVALID_ARGUMENT, "null argument or no ranks");
    if (si_status st = validate(config)) return st;
    *bytes = tp_layout(*config, nranks).data_bytes + 4096;  // + the peer group's state
    return SI_OK;
}

si_status si_decoder_create_tensor_parallel(int device, const si_decoder_config *config, si_peer_group *group,
                                            si_decoder **out) {
    if (!out || !group) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (si_status st = validate(config)) return st;
    const si_decoder_config &c = *config;
    for (uint32_t t : {c.weight_type, c.embedding_type})
        if (t != SI_TYPE_Q4_K && t != SI_TYPE_Q8_0)
            return fail(SI_ERR_UNSUPPORTED, "a tensor-parallel session takes Q4_K or Q8_0 weights");
    if (c.hidden % 256) return fail(SI_ERR_UNSUPPORTED, "hidden %d is not a multiple of 256", c.hidden);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(SI_ERR_NO_DEVICE, "no CUDA device is available");
    }
    if (device < 0 || device >= n) return fail(SI_ERR_INVALID_ARGUMENT, "device %d out of range [0,%d)", device, n);
    DeviceScope scope(device);
    return create_tp(device, config, group, out);
}

si_status si_decoder_destroy(si_decoder *decoder) {
    if (decoder) destroy(decoder);
    return SI_OK;
}

si_status si_decoder_slot(si_decoder *d, const char *name, void **device_pointer, uint64_t *bytes) {
    if (!d || !device_pointer || !bytes) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    uint8_t *p = nullptr;
    if (si_status st = slot_range(d, name, 0, 0, &p)) return st;
    *device_pointer = p;
    *bytes = d->slots[name].bytes;
    return SI_OK;
}

si_status si_decoder_upload(si_decoder *d, const char *name, uint64_t offset, const void *host, uint64_t bytes) {
    if (!d || (!host && bytes)) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->lock);
    uint8_t *p = nullptr;
    if (si_status st = slot_range(d, name, offset, bytes, &p)) return st;
    DeviceScope scope(d->device);
    if (si_status st = cuda(cudaMemcpyAsync(p, host, bytes, cudaMemcpyHostToDevice, d->stream), "cudaMemcpyAsync"))
        return st;
    return cuda(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
}

si_status si_decoder_read(si_decoder *d, const char *name, uint64_t offset, void *host, uint64_t bytes) {
    if (!d || (!host && bytes)) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->lock);
    uint8_t *p = nullptr;
    if (si_status st = slot_range(d, name, offset, bytes, &p)) return st;
    DeviceScope scope(d->device);
    if (si_status st = cuda(cudaMemcpyAsync(host, p, bytes, cudaMemcpyDeviceToHost, d->stream), "cudaMemcpyAsync"))
        return st;
    return cuda(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
}

si_status si_decoder_stream(si_decoder *d, void **stream) {
    if (!d || !stream) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *stream = d->stream;
    return SI_OK;
}

si_status si_decoder_forward_token(si_decoder *d, int32_t token, int32_t *next_token) {
    if (!d || !next_token) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->lock);
    if (token < 0 || token >= d->cfg.vocab)
        return fail(SI_ERR_INVALID_ARGUMENT, "token %d outside the vocabulary of %d", token, d->cfg.vocab);
    if (d->position >= d->cfg.context)
        return fail(SI_ERR_INVALID_ARGUMENT, "The GPU KV cache capacity of %lld tokens has been reached.",
                    (long long)d->cfg.context);
    DeviceScope scope(d->device);
    if (si_status st = ensure_graphs(d)) return st;
    d->pinned[0] = token;
    d->pinned[1] = d->position;
    if (si_status st = cuda(cudaMemcpyAsync(d->control, d->pinned, 8, cudaMemcpyHostToDevice, d->stream), "upload"))
        return st;
    if (si_status st = run_step(d, false)) return st;
    if (si_status st = cuda(cudaMemcpyAsync(d->pinned + 2, d->next_token, 4, cudaMemcpyDeviceToHost, d->stream),
                            "readback"))
        return st;
    if (si_status st = cuda(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize")) return st;
    ++d->position;
    *next_token = d->pinned[2];
    return SI_OK;
}

si_status si_decoder_generate(si_decoder *d, const int32_t *prompt, int32_t prompt_tokens, int32_t steps,
                              int32_t *tokens) {
    if (!d || !prompt || !tokens) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->lock);
    if (prompt_tokens <= 0 || steps < 0) return fail(SI_ERR_INVALID_ARGUMENT, "prompt_tokens must be positive, steps >= 0");
    const int64_t n = int64_t(prompt_tokens) + steps;
    if (d->position + n > d->cfg.context)
        return fail(SI_ERR_INVALID_ARGUMENT, "The GPU KV cache capacity of %lld tokens has been reached.",
                    (long long)d->cfg.context);
    for (int32_t i = 0; i < prompt_tokens; ++i)
        if (prompt[i] < 0 || prompt[i] >= d->cfg.vocab)
            return fail(SI_ERR_INVALID_ARGUMENT, "prompt token %d (%d) outside the vocabulary", i, prompt[i]);
    DeviceScope scope(d->device);
    if (si_status st = ensure_graphs(d)) return st;
    std::memcpy(d->pinned_prompt, prompt, size_t(prompt_tokens) * 4);
    *d->pinned_feed = k::DecodeFeed{d->control, d->prompt, d->history, d->position, prompt_tokens, int32_t(n), 0};
    d->pinned[0] = prompt[0];
    d->pinned[1] = d->position;
    cudaStream_t s = d->stream;
    if (si_status st = cuda(cudaMemcpyAsync(d->prompt, d->pinned_prompt, size_t(prompt_tokens) * 4,
                                            cudaMemcpyHostToDevice, s), "upload"))
        return st;
    if (si_status st = cuda(cudaMemcpyAsync(d->feed, d->pinned_feed, sizeof(k::DecodeFeed), cudaMemcpyHostToDevice, s),
                            "upload"))
        return st;
    if (si_status st = cuda(cudaMemcpyAsync(d->control, d->pinned, 8, cudaMemcpyHostToDevice, s), "upload")) return st;
    for (int64_t i = 0; i < n; ++i)
        if (si_status st = run_step(d, true)) return st;
    if (si_status st = cuda(cudaMemcpyAsync(d->pinned_history, d->history, size_t(n) * 4, cudaMemcpyDeviceToHost, s),
                            "readback"))
        return st;
    if (si_status st = cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize")) return st;
    std::memcpy(tokens, d->pinned_history, size_t(n) * 4);
    d->position += int32_t(n);
    return SI_OK;
}

si_status si_decoder_prefill(si_decoder *d, const int32_t *prompt, int32_t prompt_tokens, int32_t *next_token) {
    if (!d || !prompt || !next_token) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    if (prompt_tokens <= 0) return fail(SI_ERR_INVALID_ARGUMENT, "prompt_tokens must be positive");
    {
        std::lock_guard<std::mutex> g(d->lock);
        if (d->position + int64_t(prompt_tokens) > d->cfg.context)
            return fail(SI_ERR_INVALID_ARGUMENT, "The GPU KV cache capacity of %lld tokens has been reached.",
                        (long long)d->cfg.context);
        for (int32_t i = 0; i < prompt_tokens; ++i)
            if (prompt[i] < 0 || prompt[i] >= d->cfg.vocab)
                return fail(SI_ERR_INVALID_ARGUMENT, "prompt token %d (%d) outside the vocabulary", i, prompt[i]);
        if (!d->group && k::tr_prefill_attention_supported(d->cfg.head_size)) {
            DeviceScope scope(d->device);
            if (si_status st = prefill(d, prompt, nullptr, prompt_tokens, d->position, 0, next_token)) return st;
            d->position += prompt_tokens;
            return SI_OK;
        }
    }
    // Head sizes the fused prefill attention does not cover, and row-sharded
    // sessions: the decode program once per prompt token.
    std::vector<int32_t> history(static_cast<size_t>(prompt_tokens));
    if (si_status st = si_decoder_generate(d, prompt, prompt_tokens, 0, history.data())) return st;
    *next_token = history.back();
    return SI_OK;
}

si_status si_decoder_prefill_embeddings(si_decoder *d, const float *embeddings, int32_t rows, int32_t *next_token) {
    if (!d || !embeddings || !next_token) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    if (rows <= 0) return fail(SI_ERR_INVALID_ARGUMENT, "rows must be positive");
    std::lock_guard<std::mutex> g(d->lock);
    if (d->position + int64_t(rows) > d->cfg.context)
        return fail(SI_ERR_INVALID_ARGUMENT, "The GPU KV cache capacity of %lld tokens has been reached.",
                    (long long)d->cfg.context);
    if (!k::tr_prefill_attention_supported(d->cfg.head_size))
        return fail(SI_ERR_UNSUPPORTED, "prefill attention supports head sizes 64, 128, 192 and 256");
    if (d->group) return fail(SI_ERR_UNSUPPORTED, "embedding prefill is not available in a row-sharded session");
    DeviceScope scope(d->device);
    if (si_status st = prefill(d, nullptr, embeddings, rows, d->position, 0, next_token)) return st;
    d->position += rows;
    return SI_OK;
}

si_status si_decoder_create_streams(int device, const si_decoder_config *config, int32_t streams,
                                    si_decoder **out) {
    if (!out) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (streams < 1 || streams > 1024) return fail(SI_ERR_INVALID_ARGUMENT, "streams must be 1..1024");
    if (si_status st = validate(config)) return st;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(SI_ERR_NO_DEVICE, "no CUDA device is available");
    }
    if (device < 0 || device >= n) return fail(SI_ERR_INVALID_ARGUMENT, "device %d out of range [0,%d)", device, n);
    DeviceScope scope(device);
    return create(device, config, nullptr, streams, 0, out);
}


si_status si_decoder_step_streams(si_decoder *d, const int32_t *tokens, const int32_t *positions,
                                  int32_t *next_tokens) {
    if (!d || !tokens || !positions || !next_tokens) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->lock);
    if (si_status st = check_streams(d, tokens, positions, 1)) return st;
    DeviceScope scope(d->device);
    if (!d->streams_exec)
        if (si_status st = build_streams_graph(d, nullptr, &d->streams_exec)) return st;
    const size_t B = size_t(d->streams);
    cudaStream_t s = d->stream;
    if (si_status st = upload_streams(d, tokens, positions, false)) return st;
    if (si_status st = cuda(cudaGraphLaunch(d->streams_exec, s), "cudaGraphLaunch")) return st;
    if (si_status st = cuda(cudaMemcpyAsync(d->pinned_st + 2 * B, d->st_next, B * 4, cudaMemcpyDeviceToHost, s),
                            "readback"))
        return st;
    if (si_status st = cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize")) return st;
    std::memcpy(next_tokens, d->pinned_st + 2 * B, B * 4);
    return SI_OK;
}

si_status si_decoder_generate_streams(si_decoder *d, const int32_t *tokens, const int32_t *positions, int32_t steps,
                                      int32_t *out) {
    if (!d || !tokens || !positions || !out) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    if (steps < 1) return fail(SI_ERR_INVALID_ARGUMENT, "steps must be positive");
    std::lock_guard<std::mutex> g(d->lock);
    if (si_status st = check_streams(d, tokens, positions, steps)) return st;
    DeviceScope scope(d->device);
    if (!d->streams_feed_exec)
        if (si_status st = build_streams_graph(d, d->st_feed, &d->streams_feed_exec)) return st;
    const size_t B = size_t(d->streams);
    cudaStream_t s = d->stream;
    if (si_status st = upload_streams(d, tokens, positions, true)) return st;
    for (int32_t i = 0; i < steps; ++i)
        if (si_status st = cuda(cudaGraphLaunch(d->streams_feed_exec, s), "cudaGraphLaunch")) return st;
    if (si_status st = cuda(cudaMemcpyAsync(d->pinned_st + 3 * B, d->st_history, size_t(steps) * B * 4,
                                            cudaMemcpyDeviceToHost, s),
                            "readback"))
        return st;
    if (si_status st = cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize")) return st;
    std::memcpy(out, d->pinned_st + 3 * B, size_t(steps) * B * 4);
    return SI_OK;
}

si_status si_decoder_prefill_stream(si_decoder *d, int32_t stream, const int32_t *prompt, int32_t prompt_tokens,
                                    int32_t start, int32_t *next_token) {
    if (!d || !prompt || !next_token) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(d->lock);
    if (stream < 0 || stream >= d->streams)
        return fail(SI_ERR_INVALID_ARGUMENT, "stream %d outside [0, %d)", stream, d->streams);
    if (prompt_tokens <= 0 || start < 0)
        return fail(SI_ERR_INVALID_ARGUMENT, "prompt_tokens must be positive and start >= 0");
    if (int64_t(start) + prompt_tokens > d->cfg.context)
        return fail(SI_ERR_INVALID_ARGUMENT, "The GPU KV cache capacity of %lld tokens has been reached.",
                    (long long)d->cfg.context);
    for (int32_t i = 0; i < prompt_tokens; ++i)
        if (prompt[i] < 0 || prompt[i] >= d->cfg.vocab)
            return fail(SI_ERR_INVALID_ARGUMENT, "prompt token %d (%d) outside the vocabulary", i, prompt[i]);
    if (d->group || !k::tr_prefill_attention_supported(d->cfg.head_size))
        return fail(SI_ERR_UNSUPPORTED, "stream prefill needs the fused prefill attention (head size 64/128/192/256)");
    DeviceScope scope(d->device);
    const int64_t offset = int64_t(stream) * d->cfg.context * int64_t(d->cfg.kv_heads) * d->cfg.head_size;
    return prefill(d, prompt, nullptr, prompt_tokens, start, offset, next_token);
}

si_status si_decoder_reset(si_decoder *d) {
    if (!d) return fail(SI_ERR_INVALID_ARGUMENT, "null decoder");
    std::lock_guard<std::mutex> g(d->lock);
    d->position = 0;
    return SI_OK;
}

si_status si_decoder_position(si_decoder *d, int32_t *position) {
    if (!d || !position) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *position = d->position;
    return SI_OK;
}

}  // extern "C"
