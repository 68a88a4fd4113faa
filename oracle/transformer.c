/*
 * transformer.c -- CPU restatement of SharpInference's FP32 transformer
 * instructions (collection TransformerFloat32) and of the Phi-4 decode
 * program built from them. TEST INFRASTRUCTURE ONLY: the checker for the
 * CUDA kernels in tests/, smoke() and bench.py's cpu_baseline leg. Nothing
 * in the shipped library links or calls this code.
 *
 * Each function restates one instruction body of
 *   src/SharpInference.Instructions.D3D12/GpuTransformerInstructionCollection.cs
 *   src/SharpInference.Instructions.D3D12/GpuBatchTransformerInstructions.cs
 * with the same 64-lane partial sums and shared-memory tree merges where the
 * instruction has them (a "group" of 64 lanes, gpu.groupIndex = lane), the
 * same masks, clamps and sentinel values. HLSL exp/cos/sin/rsqrt are
 * restated with the C library's expf/cosf/sinf and 1/sqrtf; the HLSL
 * intrinsics are not bit-specified, so parity with them is tolerance-based.
 *
 * Parity pins: the known answers of GpuTransformerInstructionTests.cs
 * (residual-rms-norm, swiglu, scaled-add, batch-rms-norm, batch-gather-rows,
 * batch attention with its KV-cache contents) are fixtures in tests/golden/.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

#define LANES 64
#define NEG_MAX (-3.402823466e+38f)

/* Shared-memory tree of the instruction bodies:
 * for(step=32;step>0;step>>=1) if(lane<step) r[lane]+=r[lane+step]; */
static float tree_sum(float *r) {
    for (int step = LANES / 2; step > 0; step >>= 1)
        for (int l = 0; l < step; ++l) r[l] += r[l + step];
    return r[0];
}

static float tree_max(float *r) {
    for (int step = LANES / 2; step > 0; step >>= 1)
        for (int l = 0; l < step; ++l) r[l] = fmaxf(r[l], r[l + step]);
    return r[0];
}

/* transformer.rms-norm (GpuTransformerInstructionCollection.cs:323-368). */
void or_rms_norm(const float *in, const float *weight, float *out, int64_t n, float eps) {
    float r[LANES];
    for (int l = 0; l < LANES; ++l) {
        float s = 0.0f;
        for (int64_t j = l; j < n; j += LANES) s += in[j] * in[j];
        r[l] = s;
    }
    const float scale = 1.0f / sqrtf(tree_sum(r) / (float)n + eps);
    for (int64_t j = 0; j < n; ++j) out[j] = in[j] * scale * weight[j];
}

/* transformer.residual-rms-norm (GpuTransformerInstructionCollection.cs:370-417):
 * updated = hidden + residual; output = rms-norm(updated) * weight. */
void or_residual_rms_norm(const float *hidden, const float *residual, const float *weight, float *updated,
                          float *out, int64_t n, float eps) {
    float r[LANES];
    for (int l = 0; l < LANES; ++l) {
        float s = 0.0f;
        for (int64_t j = l; j < n; j += LANES) {
            const float v = hidden[j] + residual[j];
            updated[j] = v;
            s += v * v;
        }
        r[l] = s;
    }
    const float scale = 1.0f / sqrtf(tree_sum(r) / (float)n + eps);
    for (int64_t j = 0; j < n; ++j) out[j] = updated[j] * scale * weight[j];
}

/* transformer.swiglu (GpuTransformerInstructionCollection.cs:419-443):
 * gate is the first half of gate_up, up the second. */
void or_swiglu(const float *gate_up, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const float gate = gate_up[i], up = gate_up[i + n];
        out[i] = gate / (1.0f + expf(-gate)) * up;
    }
}

/* transformer.scaled-add (GpuTransformerInstructionCollection.cs:151-182). */
void or_scaled_add(const float *in, const float *update, float *out, int64_t n, float scale) {
    for (int64_t i = 0; i < n; ++i) out[i] = in[i] + scale * update[i];
}

/* core.gather-row (GpuTierZeroInstruction.cs:397-407): row `index` of the
 * table, or NaN everywhere for an index outside [0, rows). */
int or_gather_row(uint32_t table_type, const void *table, int64_t rows, int64_t cols, int32_t index, float *out) {
    if (index < 0 || index >= rows) {
        const uint32_t nan_bits = 0x7fc00000u;
        float nan;
        memcpy(&nan, &nan_bits, 4);
        for (int64_t c = 0; c < cols; ++c) out[c] = nan;
        return 0;
    }
    uint64_t row_bytes = 0;
    if (or_byte_length(table_type, (uint64_t)cols, &row_bytes)) return -1;
    return or_dequantize_row(table_type, (const uint8_t *)table + (uint64_t)index * row_bytes, cols, out);
}

/* One rotated element of the rope-kv-write bodies: element d of a head,
 * its pair partner `other`, the angle token * frequency[d mod half]. */
static float rope_value(float value, float other, int d, int half, int32_t token, const float *freq,
                        float rope_scale) {
    const int ri = d < half ? d : d - half;
    const float angle = (float)token * freq[ri];
    const float c = cosf(angle) * rope_scale, s = sinf(angle) * rope_scale;
    return d < half ? value * c - other * s : value * c + other * s;
}

/* transformer.rope-kv-write (GpuTransformerInstructionCollection.cs:445-543):
 * rotates the first rotary_size channels of every query and key head
 * (pairs (d, d + rotary/2)), writes query and the key/value rows of the
 * cache at `position`; nothing is written when position is outside
 * [0, context). qkv = [query | key | value]. */
void or_rope_kv_write(const float *qkv, int32_t position, const float *freq, float *query, float *key_cache,
                      float *value_cache, int64_t query_size, int64_t kv_size, int head_size, int rotary_size,
                      int64_t context, float rope_scale) {
    if (position < 0 || position >= context) return;
    const int half = rotary_size / 2;
    for (int64_t i = 0; i < query_size + 2 * kv_size; ++i) {
        if (i < query_size) {
            const int d = (int)(i % head_size);
            float v = qkv[i];
            if (d < rotary_size) v = rope_value(v, qkv[d < half ? i + half : i - half], d, half, position, freq, rope_scale);
            query[i] = v;
        } else if (i < query_size + kv_size) {
            const int64_t local = i - query_size;
            const int d = (int)(local % head_size);
            float v = qkv[i];
            if (d < rotary_size) v = rope_value(v, qkv[d < half ? i + half : i - half], d, half, position, freq, rope_scale);
            key_cache[(int64_t)position * kv_size + local] = v;
        } else {
            const int64_t local = i - query_size - kv_size;
            value_cache[(int64_t)position * kv_size + local] = qkv[i];
        }
    }
}

/* transformer.grouped-query-attention (GpuTransformerInstructionCollection.cs:46-148):
 * per query head one 64-lane group; tokens 0..active with
 * active = min(max(0, position), context - 1); scores scaled by
 * 1/sqrt(head_size); max and denominator by 64-lane partials + tree;
 * output channel = sum_t p_t v_t / denominator (tokens in order). */
void or_grouped_query_attention(const float *query, const float *key_cache, const float *value_cache,
                                int32_t position, float *out, int query_heads, int kv_heads, int head_size,
                                int64_t context) {
    const float scale = 1.0f / sqrtf((float)head_size);
    int64_t active = position < 0 ? 0 : position;
    if (active > context - 1) active = context - 1;
    float *scores = (float *)malloc((size_t)(active + 1) * sizeof(float));
    float r[LANES];
    const int group = query_heads / kv_heads;
    for (int head = 0; head < query_heads; ++head) {
        const int kvh = head / group;
        for (int l = 0; l < LANES; ++l) {
            float local_max = NEG_MAX;
            for (int64_t t = l; t <= active; t += LANES) {
                float s = 0.0f;
                for (int c = 0; c < head_size; ++c)
                    s += query[head * head_size + c] * key_cache[(t * kv_heads + kvh) * head_size + c];
                s *= scale;
                scores[t] = s;
                local_max = fmaxf(local_max, s);
            }
            r[l] = local_max;
        }
        const float maximum = tree_max(r);
        for (int l = 0; l < LANES; ++l) {
            float local = 0.0f;
            for (int64_t t = l; t <= active; t += LANES) {
                const float p = expf(scores[t] - maximum);
                scores[t] = p;
                local += p;
            }
            r[l] = local;
        }
        const float denominator = tree_sum(r);
        for (int c = 0; c < head_size; ++c) {
            float v = 0.0f;
            for (int64_t t = 0; t <= active; ++t)
                v += scores[t] * value_cache[(t * kv_heads + kvh) * head_size + c];
            out[head * head_size + c] = v / denominator;
        }
    }
    free(scores);
}

/* transformer.gqa-scores (GpuTransformerInstructionCollection.cs:545-594):
 * scores [query_heads, context]; tokens with token <= (uint)position get the
 * scaled dot product, the rest -FLT_MAX. The comparison is unsigned, as in
 * the instruction, so a negative position scores every token. */
void or_gqa_scores(const float *query, const float *key_cache, int32_t position, float *scores, int query_heads,
                   int kv_heads, int head_size, int64_t context) {
    const float scale = 1.0f / sqrtf((float)head_size);
    const int group = query_heads / kv_heads;
    for (int head = 0; head < query_heads; ++head)
        for (int64_t t = 0; t < context; ++t) {
            float s = NEG_MAX;
            if ((uint32_t)t <= (uint32_t)position) {
                const int kvh = head / group;
                s = 0.0f;
                for (int d = 0; d < head_size; ++d)
                    s += query[head * head_size + d] * key_cache[(t * kv_heads + kvh) * head_size + d];
                s *= scale;
            }
            scores[head * context + t] = s;
        }
}

/* Causal softmax of one score row over tokens token <= (uint)active and
 * token < context (GpuTransformerInstructionCollection.cs:596-654). */
static void softmax_row(const float *scores, float *probs, int64_t active, int valid, int64_t context) {
    float r[LANES];
    for (int l = 0; l < LANES; ++l) {
        float m = NEG_MAX;
        if (valid)
            for (int64_t t = l; (uint32_t)t <= (uint32_t)active && t < context; t += LANES) m = fmaxf(m, scores[t]);
        r[l] = m;
    }
    const float maximum = tree_max(r);
    for (int l = 0; l < LANES; ++l) {
        float s = 0.0f;
        if (valid)
            for (int64_t t = l; (uint32_t)t <= (uint32_t)active && t < context; t += LANES) s += expf(scores[t] - maximum);
        r[l] = s;
    }
    const float denominator = tree_sum(r);
    for (int64_t t = 0; t < context; ++t)
        probs[t] = valid && (uint32_t)t <= (uint32_t)active ? expf(scores[t] - maximum) / denominator : 0.0f;
}

/* transformer.causal-softmax (GpuTransformerInstructionCollection.cs:596-654). */
void or_causal_softmax(const float *scores, int32_t position, float *probs, int heads, int64_t context) {
    for (int h = 0; h < heads; ++h) softmax_row(scores + h * context, probs + h * context, position, 1, context);
}

/* transformer.gqa-values (GpuTransformerInstructionCollection.cs:656-695). */
void or_gqa_values(const float *probs, const float *value_cache, int32_t position, float *out, int query_heads,
                   int kv_heads, int head_size, int64_t context) {
    const int group = query_heads / kv_heads;
    for (int head = 0; head < query_heads; ++head)
        for (int d = 0; d < head_size; ++d) {
            const int kvh = head / group;
            float s = 0.0f;
            for (int64_t t = 0; (uint32_t)t <= (uint32_t)position && t < context; ++t)
                s += probs[head * context + t] * value_cache[(t * kv_heads + kvh) * head_size + d];
            out[head * head_size + d] = s;
        }
}

/* transformer.argmax (GpuTransformerInstructionCollection.cs:697-744):
 * 64 lanes keep (best, index) starting from (-FLT_MAX, 0); a value replaces
 * the best when greater, or equal with a smaller index; the tree merges with
 * the same rule. NaN never wins; if nothing exceeds -FLT_MAX the answer is 0. */
int32_t or_argmax(const float *in, int64_t n) {
    float best[LANES];
    uint32_t idx[LANES];
    for (int l = 0; l < LANES; ++l) {
        float b = NEG_MAX;
        uint32_t bi = 0;
        for (int64_t j = l; j < n; j += LANES) {
            const float v = in[j];
            if (v > b || (v == b && (uint32_t)j < bi)) {
                b = v;
                bi = (uint32_t)j;
            }
        }
        best[l] = b;
        idx[l] = bi;
    }
    for (int step = LANES / 2; step > 0; step >>= 1)
        for (int l = 0; l < step; ++l) {
            const float o = best[l + step];
            const uint32_t oi = idx[l + step];
            if (o > best[l] || (o == best[l] && oi < idx[l])) {
                best[l] = o;
                idx[l] = oi;
            }
        }
    return (int32_t)idx[0];
}

/* ------------------------------------------------------------------------ */
/* Batch forms (GpuBatchTransformerInstructions.cs). control = (start,
 * validCount); rows b >= validCount are left untouched. */

/* transformer.batch-rms-norm (GpuBatchTransformerInstructions.cs:101-157). */
void or_batch_rms_norm(const float *in, const float *weight, const int32_t *control, float *out, int64_t batch,
                       int64_t width, float eps) {
    for (int64_t b = 0; b < batch && b < control[1]; ++b) or_rms_norm(in + b * width, weight, out + b * width, width, eps);
}

/* transformer.batch-residual-rms-norm (GpuBatchTransformerInstructions.cs:159-222). */
void or_batch_residual_rms_norm(const float *hidden, const float *residual, const float *weight,
                                const int32_t *control, float *updated, float *out, int64_t batch, int64_t width,
                                float eps) {
    for (int64_t b = 0; b < batch && b < control[1]; ++b)
        or_residual_rms_norm(hidden + b * width, residual + b * width, weight, updated + b * width, out + b * width,
                             width, eps);
}

/* transformer.batch-swiglu (GpuBatchTransformerInstructions.cs:281-318). */
void or_batch_swiglu(const float *gate_up, const int32_t *control, float *out, int64_t batch, int64_t width) {
    for (int64_t b = 0; b < batch && b < control[1]; ++b) or_swiglu(gate_up + b * 2 * width, out + b * width, width);
}

/* transformer.batch-rope-kv-write (GpuBatchTransformerInstructions.cs:320-413):
 * row b is the token at position control[0] + b. */
void or_batch_rope_kv_write(const float *qkv, const int32_t *control, const float *freq, float *query,
                            float *key_cache, float *value_cache, int64_t batch, int64_t query_size,
                            int64_t kv_size, int head_size, int rotary_size, int64_t context, float rope_scale) {
    const int64_t width = query_size + 2 * kv_size;
    for (int64_t b = 0; b < batch && b < control[1]; ++b)
        or_rope_kv_write(qkv + b * width, control[0] + (int32_t)b, freq, query + b * query_size, key_cache,
                         value_cache, query_size, kv_size, head_size, rotary_size, context, rope_scale);
}

/* transformer.batch-gqa-scores (GpuBatchTransformerInstructions.cs:415-473):
 * row b attends through position active = control[0] + b; a negative
 * active leaves every score at -FLT_MAX. */
void or_batch_gqa_scores(const float *query, const float *key_cache, const int32_t *control, float *scores,
                         int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context) {
    const float scale = 1.0f / sqrtf((float)head_size);
    const int group = query_heads / kv_heads;
    for (int64_t b = 0; b < batch && b < control[1]; ++b) {
        const int32_t active = control[0] + (int32_t)b;
        for (int head = 0; head < query_heads; ++head)
            for (int64_t t = 0; t < context; ++t) {
                float s = NEG_MAX;
                if (active >= 0 && (uint32_t)t <= (uint32_t)active) {
                    const int kvh = head / group;
                    s = 0.0f;
                    for (int d = 0; d < head_size; ++d)
                        s += query[(b * query_heads + head) * head_size + d] *
                             key_cache[(t * kv_heads + kvh) * head_size + d];
                    s *= scale;
                }
                scores[(b * query_heads + head) * context + t] = s;
            }
    }
}

/* transformer.batch-causal-softmax (GpuBatchTransformerInstructions.cs:475-551). */
void or_batch_causal_softmax(const float *scores, const int32_t *control, float *probs, int64_t batch, int heads,
                             int64_t context) {
    for (int64_t b = 0; b < batch && b < control[1]; ++b) {
        const int32_t active = control[0] + (int32_t)b;
        for (int h = 0; h < heads; ++h) {
            const int64_t base = (b * heads + h) * context;
            softmax_row(scores + base, probs + base, active, active >= 0, context);
        }
    }
}

/* transformer.batch-gqa-values (GpuBatchTransformerInstructions.cs:553-611). */
void or_batch_gqa_values(const float *probs, const float *value_cache, const int32_t *control, float *out,
                         int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context) {
    const int group = query_heads / kv_heads;
    const int64_t width = (int64_t)query_heads * head_size;
    for (int64_t b = 0; b < batch && b < control[1]; ++b) {
        const int32_t active = control[0] + (int32_t)b;
        for (int head = 0; head < query_heads; ++head)
            for (int d = 0; d < head_size; ++d) {
                const int kvh = head / group;
                float s = 0.0f;
                if (active >= 0)
                    for (int64_t t = 0; (uint32_t)t <= (uint32_t)active && t < context; ++t)
                        s += probs[(b * query_heads + head) * context + t] *
                             value_cache[(t * kv_heads + kvh) * head_size + d];
                out[b * width + head * head_size + d] = s;
            }
    }
}

/* transformer.batch-select-last (GpuBatchTransformerInstructions.cs:613-641). */
void or_batch_select_last(const float *in, const int32_t *control, float *out, int64_t batch, int64_t width) {
    const int32_t valid = control[1];
    if (valid > 0 && valid <= batch) memcpy(out, in + (int64_t)(valid - 1) * width, (size_t)width * 4);
}

/* transformer.batch-gather-rows (GpuBatchTransformerInstructions.cs:643-679):
 * output row b = table row control[0] + b for b < validCount when that row
 * exists. */
void or_batch_gather_rows(const float *table, int64_t rows, const int32_t *control, float *out, int64_t batch,
                          int64_t width) {
    for (int64_t b = 0; b < batch; ++b) {
        const int64_t src = (int64_t)control[0] + b;
        if (b < control[1] && src >= 0 && src < rows) memcpy(out + b * width, table + src * width, (size_t)width * 4);
    }
}

/* ------------------------------------------------------------------------ */
/* The Phi-4 decode program (Phi4D3D12TextSession.cs:866-920), one token:
 *   hidden = gather-row(token_embedding, token); normalized = rms(hidden, attn_norm_0)
 *   per layer: qkv = W_qkv normalized; rope-kv-write; attention = gqa(query, caches)
 *              projected = W_o attention
 *              (hidden_after, normalized) = residual-rms(hidden, projected, ffn_norm)
 *              gate_up = W_up normalized; activated = swiglu(gate_up)
 *              down = W_down activated
 *              (hidden, normalized) = residual-rms(hidden_after, down, next norm)
 *   logits = token_embedding normalized; next = argmax(logits)
 * Weight slots in `w`: [0] token_embedding, [1] output_norm, then per layer
 * attn_norm, ffn_norm, qkv, attn_output, ffn_up, ffn_down. Caches are
 * [layers][context][kv_heads][head_size]. */
int or_decoder_step(const or_decoder_config *cfg, const void *const *w, const float *freq, float *key_cache,
                    float *value_cache, int32_t token, int32_t position, float *logits, int32_t *next_token,
                    int threads) {
    return or_decoder_step_typed(cfg, w, NULL, freq, key_cache, value_cache, token, position, logits, next_token,
                                 threads);
}

/* The same program with a GGUF type per slot (`types` in the order of `w`,
 * NULL: cfg's weight_type for every projection), as a mixed-type file holds. */
int or_decoder_step_typed(const or_decoder_config *cfg, const void *const *w, const uint32_t *types,
                          const float *freq, float *key_cache, float *value_cache, int32_t token, int32_t position,
                          float *logits, int32_t *next_token, int threads) {
    const int64_t H = cfg->hidden, Q = (int64_t)cfg->query_heads * cfg->head_size,
                  KV = (int64_t)cfg->kv_heads * cfg->head_size, F = cfg->intermediate;
    if (Q != H) return -3;
    float *hidden = (float *)malloc((size_t)H * 4), *after = (float *)malloc((size_t)H * 4),
          *normalized = (float *)malloc((size_t)H * 4), *qkv = (float *)malloc((size_t)(Q + 2 * KV) * 4),
          *query = (float *)malloc((size_t)Q * 4), *attention = (float *)malloc((size_t)H * 4),
          *projected = (float *)malloc((size_t)H * 4), *gate_up = (float *)malloc((size_t)(2 * F) * 4),
          *activated = (float *)malloc((size_t)F * 4), *down = (float *)malloc((size_t)H * 4);
    int rc = or_gather_row(cfg->embedding_type, w[0], cfg->vocab, H, token, hidden);
    if (!rc) or_rms_norm(hidden, (const float *)w[2], normalized, H, cfg->epsilon);
    const int64_t layer_cache = cfg->context * KV;
    for (int l = 0; l < cfg->layers && !rc; ++l) {
        const void *const *lw = w + 2 + 6 * l;
        const uint32_t *lt = types ? types + 2 + 6 * l : NULL;
        const uint32_t tq = lt ? lt[2] : cfg->weight_type, to = lt ? lt[3] : cfg->weight_type,
                       tu = lt ? lt[4] : cfg->weight_type, td = lt ? lt[5] : cfg->weight_type;
        float *kc = key_cache + l * layer_cache, *vc = value_cache + l * layer_cache;
        if ((rc = or_matvec(tq, lw[2], normalized, qkv, Q + 2 * KV, H, threads))) break;
        or_rope_kv_write(qkv, position, freq, query, kc, vc, Q, KV, cfg->head_size, cfg->rotary_size, cfg->context,
                         cfg->rope_scale);
        or_grouped_query_attention(query, kc, vc, position, attention, cfg->query_heads, cfg->kv_heads,
                                   cfg->head_size, cfg->context);
        if ((rc = or_matvec(to, lw[3], attention, projected, H, Q, threads))) break;
        or_residual_rms_norm(hidden, projected, (const float *)lw[1], after, normalized, H, cfg->epsilon);
        if ((rc = or_matvec(tu, lw[4], normalized, gate_up, 2 * F, H, threads))) break;
        or_swiglu(gate_up, activated, F);
        if ((rc = or_matvec(td, lw[5], activated, down, H, F, threads))) break;
        const float *next_norm = l == cfg->layers - 1 ? (const float *)w[1] : (const float *)w[2 + 6 * (l + 1)];
        or_residual_rms_norm(after, down, next_norm, hidden, normalized, H, cfg->epsilon);
    }
    if (!rc) rc = or_matvec(cfg->embedding_type, w[0], normalized, logits, cfg->vocab, H, threads);
    if (!rc) *next_token = or_argmax(logits, cfg->vocab);
    free(hidden); free(after); free(normalized); free(qkv); free(query);
    free(attention); free(projected); free(gate_up); free(activated); free(down);
    return rc;
}

/* RoPE frequencies of the decode program (Phi4D3D12TextSession.cs:394-398):
 * f_i = 1 / base^(2i / rotary_size), i < rotary_size / 2. */
void or_rope_frequencies(float base, int rotary_size, float *out) {
    for (int i = 0; i < rotary_size / 2; ++i) out[i] = 1.0f / powf(base, 2.0f * (float)i / (float)rotary_size);
}

/* transformer.embedding-gather-batch (GpuTransformerInstructionCollection.cs:184-219):
 * output row r = FP16 table row indices[r]. The instruction loads without a
 * bounds check; out-of-range raw-buffer loads read 0 under Direct3D 12, so
 * an index outside [0, rows) yields zeros here. */
void or_embedding_gather_batch(const uint16_t *table, int64_t rows, const int32_t *indices, float *out,
                               int64_t batch, int64_t width) {
    for (int64_t r = 0; r < batch; ++r)
        for (int64_t c = 0; c < width; ++c) {
            const int64_t t = (int64_t)(uint32_t)indices[r];
            out[r * width + c] = t < rows ? or_f16_to_f32(table[t * width + c]) : 0.0f;
        }
}

/* transformer.copy-embedding-rows (GpuTransformerInstructionCollection.cs:221-248):
 * output[output_start * width + e] = input[e] for e < rows * width. */
void or_copy_embedding_rows(const float *in, float *out, int64_t rows, int64_t width, int64_t output_start) {
    memcpy(out + output_start * width, in, (size_t)(rows * width) * 4);
}
