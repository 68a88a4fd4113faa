/*
 * oracle.h -- CPU restatement of SharpInference's mat-vec / matrix-multiply
 * numerics, used ONLY as test infrastructure (the checker in tests/, the
 * smoke() check and bench.py's cpu_baseline leg). Nothing in the shipped
 * library links, loads or calls this code.
 *
 * Parity status
 *   - Dense FP32/FP16 mat-vec (cooperative Neumaier form and the CPU Dot form)
 *     is pinned against the known answers in the reference's own tests
 *     (GpuMatVecTests.cs:13-67, CpuVmMixedWeightsTests.cs:62-104,
 *     GpuTransformerInstructionTests.cs:280-324); the fixtures live in
 *     tests/golden/ with the script that writes them.
 *   - Q8_0 / Q4_K / Q6_K: the reference has no quantized arithmetic
 *     (GgufModelFile.cs:314-320 throws for the K-quants). The block layouts
 *     follow the published GGUF format; dequantisation is exact FP32
 *     arithmetic. The dequantisers are pinned bit for bit to an independent
 *     implementation, gguf-py 0.19.0 (`gguf.quants.dequantize`, llama.cpp's
 *     Python package), on the BASELINE workloads' blocks and on random valid
 *     blocks (tests/test_gguf_reference_codecs.py); the Q8_0 quantiser is
 *     pinned to gguf-py's too. Kernel and oracle consume identical bytes.
 *   - TensorPrimitives.Dot (System.Numerics.Tensors 10.0.0) does not specify
 *     its SIMD summation order, so bitwise parity with the CPU path is
 *     unpinned; the restatement uses an 8-lane FP32 accumulation.
 */
#ifndef SI_ORACLE_H
#define SI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type ids (GgufModelFile.cs:24-46). */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q6_K = 14 };

/* Block geometry: Q8_0 34 B / 32 elements (GgufModelFile.cs:318),
 * Q4_K 144 B / 256 elements (absent from the reference; GGUF format). */
#define OR_Q8_0_BLOCK 32
#define OR_Q8_0_BYTES 34
#define OR_Q4_K_BLOCK 256
#define OR_Q4_K_BYTES 144
/* Q6_K 210 B / 256 elements (GGUF format; the reference's table stops at Q8_1). */
#define OR_Q6_K_BLOCK 256
#define OR_Q6_K_BYTES 210

/* ---- seeded synthetic inputs ------------------------------------------ */
uint64_t or_splitmix64(uint64_t seed, uint64_t index);
void or_normal_fill(uint64_t seed, uint64_t offset, int64_t n, float sigma, float *out);

/* ---- IEEE binary16 ------------------------------------------------------ */
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);

/* ---- byte lengths (GgufModelFile.GetByteLength, GgufModelFile.cs:301-331) */
int or_byte_length(uint32_t type, uint64_t elements, uint64_t *bytes);

/* ---- block codecs ------------------------------------------------------- */
void or_quantize_q8_0(const float *x, int64_t n, uint8_t *out);
void or_dequantize_q8_0(const uint8_t *blocks, int64_t n, float *out);
void or_quantize_q4_k(const float *x, int64_t n, uint8_t *out);
void or_dequantize_q4_k(const uint8_t *blocks, int64_t n, float *out);
void or_quantize_q6_k(const float *x, int64_t n, uint8_t *out);
void or_dequantize_q6_k(const uint8_t *blocks, int64_t n, float *out);
/* Dequantise one row of `cols` elements of any supported type. */
int or_dequantize_row(uint32_t type, const void *row, int64_t cols, float *out);

/* ---- mat-vec ------------------------------------------------------------ */
/* CpuHalfMatrixOperators.MatVec semantics (CpuHalfMatrixOperators.cs:11-43):
 * per row, convert/dequantise into an FP32 scratch row, FP32 dot with x.
 * Rows run in parallel on `threads` threads (0 = all online cores). */
int or_matvec(uint32_t wtype, const void *w, const float *x, float *y,
              int64_t rows, int64_t cols, int threads);
/* Same, double accumulation over the dequantised FP32 weights. */
int or_matvec_f64(uint32_t wtype, const void *w, const float *x, double *y,
                  int64_t rows, int64_t cols, int threads);
/* The D3D12 cooperative mat-vec (GpuTierZeroInstruction.cs:44-90): `lanes`
 * lanes per row stride the columns, per-lane Neumaier (sum, correction)
 * (add32, GpuTierZeroInstruction.cs:316), then a shared-memory tree merge.
 * xtype/ytype are OR_F32 or OR_F16 (FP16 output rounds to nearest even). */
int or_matvec_cooperative(uint32_t wtype, uint32_t xtype, uint32_t ytype,
                          const void *w, const void *x, void *y,
                          int64_t rows, int64_t cols, int lanes);

/* transformer.batch-shared-matvec (GpuBatchTransformerInstructions.cs:224-275):
 * out[b,o] = sum_i W[o,i] in[b,i] for b < control[1]; rows b >= control[1]
 * are left untouched. 64-lane plain FP32 partial sums and tree merge. */
int or_batch_shared_matvec(uint32_t wtype, const void *w, const float *in,
                           const int32_t *control, float *out,
                           int64_t batch, int64_t out_features, int64_t in_features);

/* core.matrix-multiply with transpose_right = true
 * (CpuInstructionNumerics.MatrixMultiply, CpuInstructionNumerics.cs:61-82):
 * Y[M,N] = X[M,K] W[N,K]^T as one mat-vec per row of X. */
int or_matrix_multiply_tr(uint32_t wtype, const float *x, const void *w, float *y,
                          int64_t m, int64_t n, int64_t k, int threads);

int or_online_cores(void);

/* ---- transformer instructions (oracle/transformer.c) -------------------- */
void or_rms_norm(const float *in, const float *weight, float *out, int64_t n, float eps);
void or_residual_rms_norm(const float *hidden, const float *residual, const float *weight, float *updated,
                          float *out, int64_t n, float eps);
void or_swiglu(const float *gate_up, float *out, int64_t n);
void or_scaled_add(const float *in, const float *update, float *out, int64_t n, float scale);
int or_gather_row(uint32_t table_type, const void *table, int64_t rows, int64_t cols, int32_t index, float *out);
void or_rope_kv_write(const float *qkv, int32_t position, const float *freq, float *query, float *key_cache,
                      float *value_cache, int64_t query_size, int64_t kv_size, int head_size, int rotary_size,
                      int64_t context, float rope_scale);
void or_grouped_query_attention(const float *query, const float *key_cache, const float *value_cache,
                                int32_t position, float *out, int query_heads, int kv_heads, int head_size,
                                int64_t context);
void or_gqa_scores(const float *query, const float *key_cache, int32_t position, float *scores, int query_heads,
                   int kv_heads, int head_size, int64_t context);
void or_causal_softmax(const float *scores, int32_t position, float *probs, int heads, int64_t context);
void or_gqa_values(const float *probs, const float *value_cache, int32_t position, float *out, int query_heads,
                   int kv_heads, int head_size, int64_t context);
int32_t or_argmax(const float *in, int64_t n);
void or_batch_rms_norm(const float *in, const float *weight, const int32_t *control, float *out, int64_t batch,
                       int64_t width, float eps);
void or_batch_residual_rms_norm(const float *hidden, const float *residual, const float *weight,
                                const int32_t *control, float *updated, float *out, int64_t batch, int64_t width,
                                float eps);
void or_batch_swiglu(const float *gate_up, const int32_t *control, float *out, int64_t batch, int64_t width);
void or_batch_rope_kv_write(const float *qkv, const int32_t *control, const float *freq, float *query,
                            float *key_cache, float *value_cache, int64_t batch, int64_t query_size,
                            int64_t kv_size, int head_size, int rotary_size, int64_t context, float rope_scale);
void or_batch_gqa_scores(const float *query, const float *key_cache, const int32_t *control, float *scores,
                         int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context);
void or_batch_causal_softmax(const float *scores, const int32_t *control, float *probs, int64_t batch, int heads,
                             int64_t context);
void or_batch_gqa_values(const float *probs, const float *value_cache, const int32_t *control, float *out,
                         int64_t batch, int query_heads, int kv_heads, int head_size, int64_t context);
void or_batch_select_last(const float *in, const int32_t *control, float *out, int64_t batch, int64_t width);
void or_batch_gather_rows(const float *table, int64_t rows, const int32_t *control, float *out, int64_t batch,
                          int64_t width);
void or_embedding_gather_batch(const uint16_t *table, int64_t rows, const int32_t *indices, float *out,
                               int64_t batch, int64_t width);
void or_copy_embedding_rows(const float *in, float *out, int64_t rows, int64_t width, int64_t output_start);

/* ---- Phi-4 decode program (Phi4D3D12TextSession.cs:866-920) ------------- */
typedef struct or_decoder_config {
    int32_t layers, hidden, query_heads, kv_heads, head_size, rotary_size, intermediate, vocab;
    int64_t context;
    float epsilon, rope_base, rope_scale;
    uint32_t weight_type;     /* linear projections */
    uint32_t embedding_type;  /* token_embedding (tied vocabulary projection) */
} or_decoder_config;
void or_rope_frequencies(float base, int rotary_size, float *out);
int or_decoder_step(const or_decoder_config *cfg, const void *const *w, const float *freq, float *key_cache,
                    float *value_cache, int32_t token, int32_t position, float *logits, int32_t *next_token,
                    int threads);
int or_decoder_step_typed(const or_decoder_config *cfg, const void *const *w, const uint32_t *types,
                          const float *freq, float *key_cache, float *value_cache, int32_t token, int32_t position,
                          float *logits, int32_t *next_token, int threads);

#ifdef __cplusplus
}
#endif
#endif
