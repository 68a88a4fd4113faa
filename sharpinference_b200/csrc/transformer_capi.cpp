// C ABI of the transformer instructions: the shape checks each
// instruction's Generate performs in the reference (throwing
// InstructionAdaptationException -> SI_ERR_ADAPTATION), pointer checks
// against the device allocations, then the kernels of transformer.cu.
#include <cmath>
#include <cstdint>
#include <initializer_list>
#include <tuple>

#include "si_internal.h"

using namespace si;

namespace {

constexpr uint64_t F = sizeof(float);

si_status adapt(const char *op, const char *msg) { return fail(SI_ERR_ADAPTATION, "%s: %s", op, msg); }

bool positive_finite(float v) { return std::isfinite(v) && v > 0.0f; }

// Each (port, pointer, bytes) must be device memory of the current device.
si_status ports(std::initializer_list<std::tuple<const char *, const void *, uint64_t>> list) {
    for (const auto &[name, ptr, bytes] : list)
        if (si_status st = device_range(name, ptr, bytes)) return st;
    return SI_OK;
}

si_status attention_shape(const char *op, int32_t query_heads, int32_t kv_heads, int32_t head_size, int64_t context) {
    if (query_heads <= 0 || kv_heads <= 0 || head_size <= 0 || context <= 0)
        return adapt(op, "dimensions must be positive.");
    if (query_heads % kv_heads) return adapt(op, "Query heads must be divisible by key/value heads.");
    if (int64_t(context) * kv_heads * head_size > (int64_t(1) << 40)) return adapt(op, "cache too large.");
    return SI_OK;
}

}  // namespace

extern "C" {

si_status si_gather_row(uint32_t table_type, const void *table, int64_t rows, int64_t cols, const int32_t *index,
                        float *output, void *stream) {
    if (rows <= 0 || cols <= 0) return adapt("core.gather-row", "invalid table/index shapes.");
    if (!known_type(table_type)) return fail(SI_ERR_UNSUPPORTED, "GGUF tensor type '%u' is not supported.", table_type);
    uint64_t row_bytes = 0;
    if (si_status st = byte_length(table_type, uint64_t(cols), &row_bytes)) return st;
    if (si_status st = ports({{"table", table, row_bytes * uint64_t(rows)}, {"index", index, 4},
                              {"output", output, uint64_t(cols) * F}}))
        return st;
    return kernels::tr_gather_row(table_type, table, rows, cols, index, output, stream);
}

si_status si_rms_norm(const float *input, const float *weight, float *output, int64_t count, float epsilon,
                      void *stream) {
    if (count <= 0) return adapt("transformer.rms-norm", "count must be positive.");
    if (!positive_finite(epsilon)) return adapt("transformer.rms-norm", "Attribute 'epsilon' must be finite and positive.");
    if (si_status st = ports({{"input", input, count * F}, {"weight", weight, count * F}, {"output", output, count * F}}))
        return st;
    return kernels::tr_rms_norm(input, nullptr, weight, nullptr, nullptr, output, 1, count, epsilon, stream);
}

si_status si_residual_rms_norm(const float *hidden, const float *residual, const float *weight, float *updated,
                               float *output, int64_t count, float epsilon, void *stream) {
    if (count <= 0) return adapt("transformer.residual-rms-norm", "count must be positive.");
    if (!positive_finite(epsilon))
        return adapt("transformer.residual-rms-norm", "Attribute 'epsilon' must be finite and positive.");
    if (si_status st = ports({{"hidden", hidden, count * F}, {"residual", residual, count * F},
                              {"weight", weight, count * F}, {"updated", updated, count * F},
                              {"output", output, count * F}}))
        return st;
    return kernels::tr_rms_norm(hidden, residual, weight, nullptr, updated, output, 1, count, epsilon, stream);
}

si_status si_swiglu(const float *gate_up, float *output, int64_t count, void *stream) {
    if (count <= 0) return adapt("transformer.swiglu", "count must be positive.");
    if (si_status st = ports({{"gate_up", gate_up, 2 * count * F}, {"output", output, count * F}})) return st;
    return kernels::tr_swiglu(gate_up, nullptr, output, 1, count, stream);
}

si_status si_scaled_add(const float *input, const float *update, float *output, int64_t count, float scale,
                        void *stream) {
    if (count <= 0) return adapt("transformer.scaled-add", "count must be positive.");
    if (!positive_finite(scale)) return adapt("transformer.scaled-add", "Attribute 'scale' must be finite and positive.");
    if (si_status st = ports({{"input", input, count * F}, {"update", update, count * F}, {"output", output, count * F}}))
        return st;
    return kernels::tr_scaled_add(input, update, output, count, scale, stream);
}

static si_status rope_shape(const char *op, int64_t query_size, int32_t kv_heads, int32_t head_size,
                            int32_t rotary_size, int64_t context, float rope_scale) {
    if (query_size <= 0 || kv_heads <= 0 || head_size <= 0 || rotary_size <= 0 || context <= 0)
        return adapt(op, "Invalid query, cache, head, or rotary dimensions.");
    if (rotary_size > head_size || rotary_size % 2 || query_size % head_size)
        return adapt(op, "Invalid query, cache, head, or rotary dimensions.");
    if (!positive_finite(rope_scale)) return adapt(op, "Attribute 'rope_scale' must be finite and positive.");
    return SI_OK;
}

si_status si_rope_kv_write(const float *qkv, const int32_t *position, const float *frequencies, float *query,
                           float *key_cache, float *value_cache, int64_t query_size, int32_t kv_heads,
                           int32_t head_size, int32_t rotary_size, int64_t context, float rope_scale, void *stream) {
    const char *op = "transformer.rope-kv-write";
    if (si_status st = rope_shape(op, query_size, kv_heads, head_size, rotary_size, context, rope_scale)) return st;
    const int64_t kv = int64_t(kv_heads) * head_size;
    if (si_status st = ports({{"qkv", qkv, (query_size + 2 * kv) * F}, {"position", position, 4},
                              {"frequencies", frequencies, uint64_t(rotary_size / 2) * F},
                              {"query", query, query_size * F}, {"key_cache", key_cache, context * kv * F},
                              {"value_cache", value_cache, context * kv * F}}))
        return st;
    return kernels::tr_rope_kv_write(qkv, position, nullptr, frequencies, query, key_cache, value_cache, 1, query_size,
                                     kv, head_size, rotary_size, context, rope_scale, stream);
}

si_status si_grouped_query_attention(const float *query, const float *key_cache, const float *value_cache,
                                     const int32_t *position, float *output, int32_t query_heads, int32_t kv_heads,
                                     int32_t head_size, int64_t context, void *stream) {
    const char *op = "transformer.grouped-query-attention";
    if (si_status st = attention_shape(op, query_heads, kv_heads, head_size, context)) return st;
    if (head_size > 256) return fail(SI_ERR_UNSUPPORTED, "%s: head_size %d above 256.", op, head_size);
    if (query_heads / kv_heads > 8) return fail(SI_ERR_UNSUPPORTED, "%s: more than 8 query heads per key/value head.", op);
    const uint64_t q = uint64_t(query_heads) * head_size * F, cache = uint64_t(context) * kv_heads * head_size * F;
    if (si_status st = ports({{"query", query, q}, {"key_cache", key_cache, cache}, {"value_cache", value_cache, cache},
                              {"position", position, 4}, {"output", output, q}}))
        return st;
    return kernels::tr_attention_decode(query, key_cache, value_cache, position, output, query_heads, kv_heads,
                                        head_size, context, stream);
}

si_status si_rope_grouped_query_attention(const float *qkv, const int32_t *position, const float *frequencies,
                                          float *key_cache, float *value_cache, float *output, int32_t query_heads,
                                          int32_t kv_heads, int32_t head_size, int32_t rotary_size, int64_t context,
                                          float rope_scale, void *stream) {
    const char *op = "transformer.grouped-query-attention";
    if (si_status st = attention_shape(op, query_heads, kv_heads, head_size, context)) return st;
    const int64_t qsize = int64_t(query_heads) * head_size;
    if (si_status st = rope_shape("transformer.rope-kv-write", qsize, kv_heads, head_size, rotary_size, context,
                                  rope_scale))
        return st;
    if (head_size > 256) return fail(SI_ERR_UNSUPPORTED, "%s: head_size %d above 256.", op, head_size);
    if (query_heads / kv_heads > 8) return fail(SI_ERR_UNSUPPORTED, "%s: more than 8 query heads per key/value head.", op);
    const int64_t kv = int64_t(kv_heads) * head_size;
    if (si_status st = ports({{"qkv", qkv, (qsize + 2 * kv) * F}, {"position", position, 4},
                              {"frequencies", frequencies, uint64_t(rotary_size / 2) * F},
                              {"key_cache", key_cache, context * kv * F}, {"value_cache", value_cache, context * kv * F},
                              {"output", output, qsize * F}}))
        return st;
    return kernels::tr_attention_decode_rope(qkv, position, frequencies, key_cache, value_cache, output, query_heads,
                                             kv_heads, head_size, rotary_size, context, rope_scale, stream);
}

si_status si_gqa_scores(const float *query, const float *key_cache, const int32_t *position, float *scores,
                        int32_t query_heads, int32_t kv_heads, int32_t head_size, int64_t context, void *stream) {
    if (si_status st = attention_shape("transformer.gqa-scores", query_heads, kv_heads, head_size, context)) return st;
    if (si_status st = ports({{"query", query, uint64_t(query_heads) * head_size * F},
                              {"key_cache", key_cache, uint64_t(context) * kv_heads * head_size * F},
                              {"position", position, 4}, {"scores", scores, uint64_t(query_heads) * context * F}}))
        return st;
    return kernels::tr_gqa_scores(query, key_cache, position, nullptr, scores, 1, query_heads, kv_heads, head_size,
                                  context, stream);
}

si_status si_causal_softmax(const float *scores, const int32_t *position, float *probabilities, int32_t heads,
                            int64_t context, void *stream) {
    if (heads <= 0 || context <= 0) return adapt("transformer.causal-softmax", "Softmax requires matching rank-two tensors.");
    const uint64_t bytes = uint64_t(heads) * context * F;
    if (si_status st = ports({{"scores", scores, bytes}, {"position", position, 4}, {"probabilities", probabilities, bytes}}))
        return st;
    return kernels::tr_causal_softmax(scores, position, nullptr, probabilities, 1, heads, context, stream);
}

si_status si_gqa_values(const float *probabilities, const float *value_cache, const int32_t *position, float *output,
                        int32_t query_heads, int32_t kv_heads, int32_t head_size, int64_t context, void *stream) {
    if (si_status st = attention_shape("transformer.gqa-values", query_heads, kv_heads, head_size, context)) return st;
    if (si_status st = ports({{"probabilities", probabilities, uint64_t(query_heads) * context * F},
                              {"value_cache", value_cache, uint64_t(context) * kv_heads * head_size * F},
                              {"position", position, 4}, {"output", output, uint64_t(query_heads) * head_size * F}}))
        return st;
    return kernels::tr_gqa_values(probabilities, value_cache, position, nullptr, output, 1, query_heads, kv_heads,
                                  head_size, context, stream);
}

si_status si_argmax(const float *input, int64_t count, int32_t *output, void *stream) {
    if (count <= 0 || count > INT32_MAX) return adapt("transformer.argmax", "input must have 1..2^31-1 elements.");
    if (si_status st = ports({{"input", input, uint64_t(count) * F}, {"output", output, 4}})) return st;
    return kernels::tr_argmax(input, count, output, nullptr, stream);
}

si_status si_embedding_gather_batch(const uint16_t *table, int64_t rows, const int32_t *indices, float *output,
                                    int64_t batch, int64_t width, void *stream) {
    if (rows <= 0 || batch <= 0 || width <= 0) return adapt("transformer.embedding-gather-batch", "dimensions must be positive.");
    if (si_status st = ports({{"table", table, uint64_t(rows) * width * 2}, {"indices", indices, uint64_t(batch) * 4},
                              {"output", output, uint64_t(batch) * width * F}}))
        return st;
    return kernels::tr_embedding_gather_batch(table, rows, indices, output, batch, width, stream);
}

si_status si_copy_embedding_rows(const float *input, float *output, int64_t output_rows, int64_t rows, int64_t width,
                                 int64_t output_start, void *stream) {
    const char *op = "transformer.copy-embedding-rows";
    if (rows <= 0) return fail(SI_ERR_ADAPTATION, "%s: Attribute 'rows' must be positive.", op);
    if (output_start < 0) return fail(SI_ERR_ADAPTATION, "%s: Attribute 'output_start' must be non-negative.", op);
    if (width <= 0 || output_start + rows > output_rows) return adapt(op, "rows do not fit the output.");
    if (si_status st = ports({{"input", input, uint64_t(rows) * width * F},
                              {"output", output, uint64_t(output_rows) * width * F}}))
        return st;
    return kernels::tr_copy_rows(input, output + output_start * width, rows * width, stream);
}

// ---- batch forms ------------------------------------------------------------
si_status si_batch_rms_norm(const float *input, const float *weight, const int32_t *control, float *output,
                            int64_t batch, int64_t width, float epsilon, void *stream) {
    const char *op = "transformer.batch-rms-norm";
    if (batch <= 0 || width <= 0) return adapt(op, "'input' dimensions must be positive.");
    if (batch > 65535) return fail(SI_ERR_UNSUPPORTED, "%s: batch above 65535.", op);
    if (!positive_finite(epsilon)) return adapt(op, "Attribute 'epsilon' must be finite and positive.");
    const uint64_t m = uint64_t(batch) * width * F;
    if (si_status st = ports({{"input", input, m}, {"weight", weight, width * F}, {"control", control, 8}, {"output", output, m}}))
        return st;
    return kernels::tr_rms_norm(input, nullptr, weight, control, nullptr, output, batch, width, epsilon, stream);
}

si_status si_batch_residual_rms_norm(const float *hidden, const float *residual, const float *weight,
                                     const int32_t *control, float *updated, float *output, int64_t batch,
                                     int64_t width, float epsilon, void *stream) {
    const char *op = "transformer.batch-residual-rms-norm";
    if (batch <= 0 || width <= 0) return adapt(op, "'hidden' dimensions must be positive.");
    if (batch > 65535) return fail(SI_ERR_UNSUPPORTED, "%s: batch above 65535.", op);
    if (!positive_finite(epsilon)) return adapt(op, "Attribute 'epsilon' must be finite and positive.");
    const uint64_t m = uint64_t(batch) * width * F;
    if (si_status st = ports({{"hidden", hidden, m}, {"residual", residual, m}, {"weight", weight, width * F},
                              {"control", control, 8}, {"updated", updated, m}, {"output", output, m}}))
        return st;
    return kernels::tr_rms_norm(hidden, residual, weight, control, updated, output, batch, width, epsilon, stream);
}

si_status si_batch_swiglu(const float *gate_up, const int32_t *control, float *output, int64_t batch, int64_t width,
                          void *stream) {
    if (batch <= 0 || width <= 0) return adapt("transformer.batch-swiglu", "Expected gate_up [B,2I] and output [B,I].");
    if (si_status st = ports({{"gate_up", gate_up, uint64_t(batch) * 2 * width * F}, {"control", control, 8},
                              {"output", output, uint64_t(batch) * width * F}}))
        return st;
    return kernels::tr_swiglu(gate_up, control, output, batch, width, stream);
}

si_status si_batch_rope_kv_write(const float *qkv, const int32_t *control, const float *frequencies, float *query,
                                 float *key_cache, float *value_cache, int64_t batch, int64_t query_size,
                                 int32_t kv_heads, int32_t head_size, int32_t rotary_size, int64_t context,
                                 float rope_scale, void *stream) {
    const char *op = "transformer.batch-rope-kv-write";
    if (batch <= 0) return adapt(op, "'qkv' dimensions must be positive.");
    if (si_status st = rope_shape(op, query_size, kv_heads, head_size, rotary_size, context, rope_scale)) return st;
    const int64_t kv = int64_t(kv_heads) * head_size;
    if (si_status st = ports({{"qkv", qkv, uint64_t(batch) * (query_size + 2 * kv) * F}, {"control", control, 8},
                              {"frequencies", frequencies, uint64_t(rotary_size / 2) * F},
                              {"query", query, uint64_t(batch) * query_size * F},
                              {"key_cache", key_cache, context * kv * F}, {"value_cache", value_cache, context * kv * F}}))
        return st;
    return kernels::tr_rope_kv_write(qkv, nullptr, control, frequencies, query, key_cache, value_cache, batch,
                                     query_size, kv, head_size, rotary_size, context, rope_scale, stream);
}

si_status si_batch_gqa_scores(const float *query, const float *key_cache, const int32_t *control, float *scores,
                              int64_t batch, int32_t query_heads, int32_t kv_heads, int32_t head_size,
                              int64_t context, void *stream) {
    const char *op = "transformer.batch-gqa-scores";
    if (batch <= 0) return adapt(op, "'query' dimensions must be positive.");
    if (si_status st = attention_shape(op, query_heads, kv_heads, head_size, context)) return st;
    if (si_status st = ports({{"query", query, uint64_t(batch) * query_heads * head_size * F},
                              {"key_cache", key_cache, uint64_t(context) * kv_heads * head_size * F},
                              {"control", control, 8}, {"scores", scores, uint64_t(batch) * query_heads * context * F}}))
        return st;
    return kernels::tr_gqa_scores(query, key_cache, nullptr, control, scores, batch, query_heads, kv_heads, head_size,
                                  context, stream);
}

si_status si_batch_causal_softmax(const float *scores, const int32_t *control, float *probabilities, int64_t batch,
                                  int32_t heads, int64_t context, void *stream) {
    const char *op = "transformer.batch-causal-softmax";
    if (batch <= 0 || heads <= 0 || context <= 0) return adapt(op, "'scores' dimensions must be positive.");
    if (batch * heads > 0x7fffffff) return fail(SI_ERR_UNSUPPORTED, "%s: too many rows.", op);
    const uint64_t bytes = uint64_t(batch) * heads * context * F;
    if (si_status st = ports({{"scores", scores, bytes}, {"control", control, 8}, {"probabilities", probabilities, bytes}}))
        return st;
    return kernels::tr_causal_softmax(scores, nullptr, control, probabilities, batch, heads, context, stream);
}

si_status si_batch_gqa_values(const float *probabilities, const float *value_cache, const int32_t *control,
                              float *output, int64_t batch, int32_t query_heads, int32_t kv_heads, int32_t head_size,
                              int64_t context, void *stream) {
    const char *op = "transformer.batch-gqa-values";
    if (batch <= 0) return adapt(op, "Incompatible probability, value cache, and output shapes.");
    if (si_status st = attention_shape(op, query_heads, kv_heads, head_size, context)) return st;
    if (si_status st = ports({{"probabilities", probabilities, uint64_t(batch) * query_heads * context * F},
                              {"value_cache", value_cache, uint64_t(context) * kv_heads * head_size * F},
                              {"control", control, 8}, {"output", output, uint64_t(batch) * query_heads * head_size * F}}))
        return st;
    return kernels::tr_gqa_values(probabilities, value_cache, nullptr, control, output, batch, query_heads, kv_heads,
                                  head_size, context, stream);
}

si_status si_batch_grouped_query_attention(const float *query, const float *key_cache, const float *value_cache,
                                           int32_t start, int32_t count, float *output, int32_t query_heads,
                                           int32_t kv_heads, int32_t head_size, int64_t context, void *stream) {
    const char *op = "transformer.batch-grouped-query-attention";
    if (count <= 0) return adapt(op, "count must be positive.");
    if (si_status st = attention_shape(op, query_heads, kv_heads, head_size, context)) return st;
    if (!kernels::tr_prefill_attention_supported(head_size))
        return fail(SI_ERR_UNSUPPORTED, "%s supports head sizes 64, 128, 192 and 256", op);
    const uint64_t width = uint64_t(query_heads) * head_size;
    if (si_status st = ports({{"query", query, uint64_t(count) * width * F},
                              {"key_cache", key_cache, uint64_t(context) * kv_heads * head_size * F},
                              {"value_cache", value_cache, uint64_t(context) * kv_heads * head_size * F},
                              {"output", output, uint64_t(count) * width * F}}))
        return st;
    return kernels::tr_prefill_attention(query, key_cache, value_cache, start, count, output, query_heads, kv_heads,
                                         head_size, context, stream);
}

si_status si_batch_select_last(const float *input, const int32_t *control, float *output, int64_t batch,
                               int64_t width, void *stream) {
    if (batch <= 0 || width <= 0) return adapt("transformer.batch-select-last", "Expected input [B,H] and output [H].");
    if (si_status st = ports({{"input", input, uint64_t(batch) * width * F}, {"control", control, 8},
                              {"output", output, uint64_t(width) * F}}))
        return st;
    return kernels::tr_select_last(input, control, output, batch, width, stream);
}

si_status si_batch_gather_rows(const float *table, int64_t rows, const int32_t *control, float *output,
                               int64_t batch, int64_t width, void *stream) {
    if (rows <= 0 || batch <= 0 || width <= 0)
        return adapt("transformer.batch-gather-rows", "Expected table [N,H] and output [B,H].");
    if (si_status st = ports({{"table", table, uint64_t(rows) * width * F}, {"control", control, 8},
                              {"output", output, uint64_t(batch) * width * F}}))
        return st;
    return kernels::tr_gather_rows(table, rows, control, output, batch, width, stream);
}

}  // extern "C"
