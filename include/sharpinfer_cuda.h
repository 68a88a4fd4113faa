/*
 * sharpinfer_cuda.h -- C ABI of libsharpinfer_cuda, the CUDA (sm_100a)
 * backend for SharpInference's mat-vec / matrix-multiply instructions.
 *
 * Every entry point returns an si_status and never aborts the process; the
 * message for the last failure on the calling thread is returned by
 * si_last_error(). Status codes map onto the exception types the reference
 * raises for the same condition (see si_status).
 *
 * Reference interfaces each group replaces are cited as
 * path:line inside JohnMasen/SharpInference/src.
 *
 * Tensor element types use the GGUF type ids of
 * SharpInference.Gguf/GgufModelFile.cs:24-46 (F32 = 0, F16 = 1, Q8_0 = 8,
 * Q4_K = 12). Quantized weights are the raw GGUF block bytes, row-major:
 * row r of a [rows, cols] matrix starts at r * si_row_bytes(type, cols).
 */
#ifndef SHARPINFER_CUDA_H
#define SHARPINFER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SI_ABI_VERSION 1

typedef enum si_status {
    SI_OK = 0,
    SI_ERR_INVALID_ARGUMENT = 1, /* ArgumentException / ArgumentOutOfRangeException */
    SI_ERR_UNSUPPORTED = 2,      /* NotSupportedException (unknown type, no implementation) */
    SI_ERR_ADAPTATION = 3,       /* InstructionAdaptationException (signature / config mismatch) */
    SI_ERR_INVALID_DATA = 4,     /* InvalidDataException (bad program, bad block count) */
    SI_ERR_CUDA = 5,             /* CUDA runtime error (device removed, launch failure) */
    SI_ERR_OUT_OF_MEMORY = 6,
    SI_ERR_NCCL = 7,
    SI_ERR_TIMEOUT = 8,          /* bounded device-side or host-side wait expired */
    SI_ERR_NO_DEVICE = 9
} si_status;

typedef enum si_type {
    SI_TYPE_F32 = 0,
    SI_TYPE_F16 = 1,
    SI_TYPE_Q8_0 = 8,
    SI_TYPE_Q4_K = 12,
    SI_TYPE_I32 = 26 /* control ports only (GgufModelTensorType.Int32) */
} si_type;

/* Execution configurations of core.mat-vec
 * (GpuMatVecExecution.cs:8-10 serial-matvec / cooperative-matvec, plus the
 * CUDA quantized implementations). SI_MATVEC_DEFAULT picks per type. */
typedef enum si_matvec_config {
    SI_MATVEC_DEFAULT = 0,
    SI_MATVEC_COOPERATIVE = 1, /* "cooperative-matvec": Neumaier per lane + merge (F32/F16 weights) */
    SI_MATVEC_QUANT_STAGED = 2 /* "cuda-gemv-staged": TMA bulk row staging (Q8_0 / Q4_K) */
} si_matvec_config;

/* ---------------------------------------------------------------------- */
/* Library / error state                                                  */
/* ---------------------------------------------------------------------- */
int si_abi_version(void);
/* Copies the calling thread's last error message (NUL-terminated). */
si_status si_last_error(char *buffer, size_t capacity);
si_status si_device_count(int *count);

/* ---------------------------------------------------------------------- */
/* GGUF formats (host only, no GPU needed)                                */
/* ---------------------------------------------------------------------- */
/* GgufModelFile.GetByteLength (SharpInference.Gguf/GgufModelFile.cs:301-331),
 * extended with Q4_K (144 B / 256 elements). A block type whose element
 * count is not a multiple of its block gives SI_ERR_INVALID_DATA; an unknown
 * type gives SI_ERR_UNSUPPORTED, as the reference throws. */
si_status si_tensor_byte_length(uint32_t type, const uint64_t *dims, int rank, uint64_t *bytes);
/* Byte length of one row of `cols` elements. */
si_status si_row_bytes(uint32_t type, int64_t cols, uint64_t *bytes);
/* Host block codecs. Quantizers are deterministic; dequantisation is exact
 * FP32 arithmetic: Q8_0 w = d*q; Q4_K w = (d*sc)*q - (dmin*m).
 * No reference counterpart (the reference has no quantized arithmetic). */
si_status si_quantize(uint32_t type, const float *src, int64_t count, void *dst);
si_status si_dequantize(uint32_t type, const void *src, int64_t count, float *dst);
/* Seeded N(0, sigma) generator (SplitMix64 counter + Box-Muller) shared by
 * tests and benchmarks so CPU and GPU paths see identical bytes. `threads`
 * <= 0 uses all online cores. */
si_status si_synth_normal(uint64_t seed, uint64_t offset, int64_t count, float sigma,
                          float *dst, int threads);
/* Generate + quantize a [rows, cols] weight matrix in one pass (same values
 * as si_synth_normal followed by si_quantize). */
si_status si_synth_weights(uint32_t type, uint64_t seed, int64_t rows, int64_t cols, float sigma,
                           void *dst, int threads);
/* Rows [row_begin, row_begin + rows) of the same matrix (a row shard). */
si_status si_synth_weight_rows(uint32_t type, uint64_t seed, int64_t row_begin, int64_t rows, int64_t cols,
                               float sigma, void *dst, int threads);

/* ---------------------------------------------------------------------- */
/* Kernel entry points on caller-owned device memory                      */
/* `stream` is a cudaStream_t (NULL = legacy default stream). Calls are   */
/* asynchronous; argument errors are reported before anything launches.  */
/* ---------------------------------------------------------------------- */
/* core.mat-vec: y[r] = sum_c W[r,c] * x[c]
 * (TierZeroOperationContracts.cs:113-115,161; GpuTierZeroInstruction.cs:44-90;
 *  CpuInstructionNumerics.MatVec, CpuInstructionNumerics.cs:16-23).
 * weight_type: F32, F16 (cooperative Neumaier), Q8_0, Q4_K (staged GEMV).
 * input_type / output_type: F32 or F16 (F16 only with F32/F16 weights, the
 * [f16,f16]->f16 signature of the T0 FP16 collection). */
si_status si_matvec(uint32_t weight_type, const void *weight,
                    uint32_t input_type, const void *input,
                    uint32_t output_type, void *output,
                    int64_t rows, int64_t cols, uint32_t config, void *stream);

/* transformer.batch-shared-matvec
 * (GpuBatchTransformerInstructions.cs:224-279): for b < control[1],
 * out[b,o] = sum_i W[o,i] * in[b,i]; rows b >= control[1] are not written.
 * `control` is a device pointer to int32[2] = (start, validCount), read on
 * the device. Weight F16, Q8_0 or Q4_K; input/output F32. */
si_status si_batch_shared_matvec(uint32_t weight_type, const void *weight,
                                 const float *input, const int32_t *control, float *output,
                                 int64_t batch, int64_t out_features, int64_t in_features,
                                 void *stream);

/* core.matrix-multiply with transpose_left=false, transpose_right=true
 * (TierZeroOperationContracts.cs:172-179; CpuInstructionNumerics.cs:61-82):
 * Y[m,n] = sum_k X[m,k] * W[n,k]. X, Y F32; W F32, F16, Q8_0 or Q4_K.
 * `workspace` is caller-owned device scratch of at least
 * si_matrix_multiply_workspace_bytes(...) bytes (may be NULL when that is 0). */
si_status si_matrix_multiply_workspace_bytes(uint32_t weight_type, int64_t m, int64_t n, int64_t k,
                                             uint64_t *bytes);
si_status si_matrix_multiply(uint32_t weight_type, const float *x, const void *weight, float *y,
                             int64_t m, int64_t n, int64_t k,
                             void *workspace, uint64_t workspace_bytes, void *stream);

/* Same operation, for callers that cannot allocate device memory: hosts
 * whose own pool owns every device byte, and loops that must not hit
 * cudaMalloc/cudaFree (they can synchronise the whole device). No counterpart
 * in the reference. Allocates nothing: the scratch is a fixed 64 MiB array
 * that every GPU loading this library holds until exit; calls needing more
 * (4*m*k bytes on the tensor-core path) get SI_ERR_INVALID_ARGUMENT. The
 * first call on a device looks the array up (cudaGetSymbolAddress), so make
 * it before any stream capture. All calls share the array: calls that
 * overlap on the GPU race, so serialise them. */
si_status si_matrix_multiply_static_workspace(uint32_t weight_type, const float *x, const void *weight, float *y,
                                              int64_t m, int64_t n, int64_t k, void *stream);

/* Device error word written by bounded device-side waits (a timed-out
 * mbarrier wait sets it instead of trapping). Reading clears it. */
si_status si_device_error_take(int device, uint32_t *code);

/* ---------------------------------------------------------------------- */
/* Multi-GPU row sharding (no counterpart in the reference, which runs on  */
/* one device): rank r of n owns weight rows [r*per, min((r+1)*per, rows))  */
/* with per = ceil(rows / n); the output slices are all-gathered.          */
/* ---------------------------------------------------------------------- */
typedef struct si_comm si_comm;
si_status si_rowshard_plan(int64_t rows, int nranks, int rank, int64_t *row_begin, int64_t *row_count,
                           int64_t *rows_per_rank);
/* 128-byte NCCL unique id, created on one rank and shared with the others. */
si_status si_comm_unique_id(uint8_t *id, size_t capacity);
/* Joins the communicator; returns SI_ERR_TIMEOUT after `timeout_ms` when a
 * rank never joins (the half-built communicator is aborted, nothing hangs). */
si_status si_comm_create(int device, int nranks, int rank, const uint8_t *id, int timeout_ms, si_comm **out);
si_status si_comm_destroy(si_comm *comm);
/* GEMV of this rank's weight rows (weight_shard = its row_count rows) into
 * output_full[rank*per ...], then an in-place all-gather so every rank holds
 * output_full[0 .. n*per) (the first `rows` entries are y). Both run on
 * `stream`; output_full must hold n*per floats. */
si_status si_rowshard_matvec_allgather(si_comm *comm, uint32_t weight_type, const void *weight_shard,
                                       const float *input, float *output_full, int64_t rows, int64_t cols,
                                       void *stream);

/* Fused alternative (no collective launch): row-sharded GEMV whose kernel
 * stores every output row straight into all ranks' "arenas" over NVLink peer
 * memory. An arena is a device buffer per rank, exported with
 * si_ipc_export, mapped by every other rank with si_ipc_open (CUDA IPC, one
 * process per GPU), at least 4 KB + the output vectors; its last 4 KB hold
 * the group's flags. Create the group on every rank, then synchronise the
 * ranks (host barrier) before the first call. si_rowshard_matvec_peer: rank r
 * computes its rows (si_rowshard_plan; every rank must get at least one row)
 * and, when the call completes in stream order, every rank's arena holds the
 * whole y[rows] at byte `output_offset` (16-byte aligned). The kernel's last
 * CTA waits, bounded by 2 s, for every rank's rows; a rank that never
 * arrives sets bit 16 of the device error word instead of hanging. Two
 * consecutive calls must use different output offsets (a rank can run one
 * call ahead of another). Q4_K and Q8_0 weights on the tensor-core path. */
typedef struct si_peer_group si_peer_group;
si_status si_ipc_export(const void *device_ptr, uint8_t *handle, size_t capacity);  /* 64-byte handle */
si_status si_ipc_open(int device, const uint8_t *handle, void **ptr);
si_status si_ipc_close(int device, void *ptr);
/* arena_addrs[q]: rank q's arena as mapped in this process (this rank's own
 * buffer at q = rank); every arena has arena_bytes bytes. */
si_status si_peer_group_create(int device, int nranks, int rank, const uint64_t *arena_addrs, uint64_t arena_bytes,
                               si_peer_group **out);
si_status si_peer_group_destroy(si_peer_group *group);
si_status si_rowshard_matvec_peer(si_peer_group *group, uint32_t weight_type, const void *weight_shard,
                                  const float *input, uint64_t output_offset, int64_t rows, int64_t cols,
                                  void *stream);

/* ---------------------------------------------------------------------- */
/* Executor: device buffers per slot, uploads/readbacks and stream        */
/* (D3D12VmExecutor.cs:283-361,452-482 Upload / Readback / Execute /     */
/*  ExecuteWithTransfers / MeasureGpuMicroseconds; D3D12VmResourcePool).  */
/* ---------------------------------------------------------------------- */
typedef struct si_context si_context;
typedef struct si_buffer si_buffer;

si_status si_context_create(int device, si_context **out);
si_status si_context_destroy(si_context *ctx);
/* The context's stream (cudaStream_t) for interop. */
si_status si_context_stream(si_context *ctx, void **stream);
si_status si_context_synchronize(si_context *ctx);
/* Number of kernel launches (submissions) the context has issued. */
si_status si_context_submission_count(si_context *ctx, uint64_t *count);

si_status si_buffer_create(si_context *ctx, uint64_t bytes, si_buffer **out);
si_status si_buffer_destroy(si_context *ctx, si_buffer *buffer);
si_status si_buffer_device_pointer(si_buffer *buffer, void **pointer, uint64_t *bytes);
/* Synchronous upload / readback at a byte offset (Upload/Readback). */
si_status si_buffer_upload(si_context *ctx, si_buffer *buffer, uint64_t offset,
                           const void *src, uint64_t bytes);
si_status si_buffer_readback(si_context *ctx, si_buffer *buffer, uint64_t offset,
                             void *dst, uint64_t bytes);
/* Asynchronous variants on the context stream (src/dst should be pinned). */
si_status si_buffer_upload_async(si_context *ctx, si_buffer *buffer, uint64_t offset,
                                 const void *src, uint64_t bytes);
si_status si_buffer_readback_async(si_context *ctx, si_buffer *buffer, uint64_t offset,
                                   void *dst, uint64_t bytes);
si_status si_host_alloc_pinned(uint64_t bytes, void **out);
si_status si_host_free_pinned(void *ptr);

/* Instruction dispatch on executor buffers. Tensor arguments are
 * (buffer, byte offset) pairs, mirroring VmArgument.ByteOffset
 * (SharpInference.Vm/VmProgram.cs:45). */
si_status si_ctx_matvec(si_context *ctx, uint32_t weight_type, si_buffer *weight, uint64_t weight_offset,
                        uint32_t input_type, si_buffer *input, uint64_t input_offset,
                        uint32_t output_type, si_buffer *output, uint64_t output_offset,
                        int64_t rows, int64_t cols, uint32_t config);
si_status si_ctx_batch_shared_matvec(si_context *ctx, uint32_t weight_type,
                                     si_buffer *weight, uint64_t weight_offset,
                                     si_buffer *input, uint64_t input_offset,
                                     si_buffer *control, uint64_t control_offset,
                                     si_buffer *output, uint64_t output_offset,
                                     int64_t batch, int64_t out_features, int64_t in_features);
/* Uses a context-owned workspace grown on demand. */
si_status si_ctx_matrix_multiply(si_context *ctx, uint32_t weight_type,
                                 si_buffer *x, uint64_t x_offset,
                                 si_buffer *weight, uint64_t weight_offset,
                                 si_buffer *y, uint64_t y_offset,
                                 int64_t m, int64_t n, int64_t k);

/* Recorded submissions: everything issued on the context stream between
 * si_graph_begin and si_graph_end (async uploads/readbacks from pinned
 * memory, instruction dispatches, row-shard collectives) is captured once
 * and replayed by si_graph_launch -- the counterpart of the pre-recorded
 * command list D3D12VmExecutor.ExecuteWithTransfers submits per call
 * (D3D12VmExecutor.cs:298-361). Synchronous uploads/readbacks are not
 * allowed while capturing. */
typedef struct si_graph si_graph;
si_status si_graph_begin(si_context *ctx);
si_status si_graph_end(si_context *ctx, si_graph **out);
si_status si_graph_launch(si_context *ctx, si_graph *graph);
si_status si_graph_destroy(si_graph *graph);

/* ---------------------------------------------------------------------- */
/* Instruction registry (InstructionCollection.cs:146-218)                */
/* ---------------------------------------------------------------------- */
/* Resolves (collection GUID, instruction name) for target "cuda". Returns
 * SI_ERR_UNSUPPORTED when no CUDA implementation exists, as
 * InstructionRegistry.Resolve throws NotSupportedException. */
si_status si_instruction_resolve(const char *collection_id, const char *name, int *instruction_id);
/* Validates a signature: port element types in port order and an execution
 * configuration name ("" = none). SI_ERR_ADAPTATION mirrors
 * InstructionAdaptationException. */
si_status si_instruction_validate(int instruction_id, const uint32_t *port_types, int port_count,
                                  const char *configuration);

/* ---------------------------------------------------------------------- */
/* Transformer instructions (collection TransformerFloat32,               */
/* GpuTransformerInstructionCollection.cs:8-33) and core.gather-row       */
/* ---------------------------------------------------------------------- */
/* Device pointers, FP32 tensors, enqueued on `stream` (NULL = legacy
 * default stream). Shape checks return SI_ERR_ADAPTATION as the
 * instruction's Generate throws InstructionAdaptationException; pointers
 * are checked against their device allocations. `position` and `control`
 * live in device memory, so one recorded graph serves every decode step.
 * Batch forms take control = (start position, validCount): rows
 * b >= validCount are left untouched (GpuBatchTransformerInstructions.cs:78-82). */

/* core.gather-row (GpuTierZeroInstruction.cs:397-407; Phi4D3D12TextSession.cs:510-516):
 * output[c] = table[*index, c] dequantised to FP32 (table F32, F16, Q8_0 or
 * Q4_K in GGUF layout), NaN in every element for an index outside [0, rows). */
si_status si_gather_row(uint32_t table_type, const void *table, int64_t rows, int64_t cols, const int32_t *index,
                        float *output, void *stream);
/* transformer.rms-norm (GpuTransformerInstructionCollection.cs:323-368). */
si_status si_rms_norm(const float *input, const float *weight, float *output, int64_t count, float epsilon,
                      void *stream);
/* transformer.residual-rms-norm (GpuTransformerInstructionCollection.cs:370-417):
 * updated = hidden + residual; output = updated * rsqrt(mean(updated^2) + eps) * weight. */
si_status si_residual_rms_norm(const float *hidden, const float *residual, const float *weight, float *updated,
                               float *output, int64_t count, float epsilon, void *stream);
/* transformer.swiglu (GpuTransformerInstructionCollection.cs:419-443): gate_up = [gate | up],
 * output[i] = gate / (1 + exp(-gate)) * up, count = output length. */
si_status si_swiglu(const float *gate_up, float *output, int64_t count, void *stream);
/* transformer.scaled-add (GpuTransformerInstructionCollection.cs:151-182); scale > 0 and finite. */
si_status si_scaled_add(const float *input, const float *update, float *output, int64_t count, float scale,
                        void *stream);
/* transformer.rope-kv-write (GpuTransformerInstructionCollection.cs:445-543): qkv = [query |
 * key | value]; rotates the first rotary_size channels of every query/key head (pairs d,
 * d + rotary/2, angle = position * frequencies[d mod rotary/2], cos/sin scaled by rope_scale),
 * writes query and the cache rows [context, kv_heads, head_size] at *position; nothing is
 * written for a position outside [0, context). */
si_status si_rope_kv_write(const float *qkv, const int32_t *position, const float *frequencies, float *query,
                           float *key_cache, float *value_cache, int64_t query_size, int32_t kv_heads,
                           int32_t head_size, int32_t rotary_size, int64_t context, float rope_scale, void *stream);
/* transformer.grouped-query-attention (GpuTransformerInstructionCollection.cs:46-148): causal
 * attention of one query over cache tokens 0..min(max(0,*position), context-1), query head h
 * reading kv head h / (query_heads / kv_heads), scores scaled by 1/sqrt(head_size). */
si_status si_grouped_query_attention(const float *query, const float *key_cache, const float *value_cache,
                                     const int32_t *position, float *output, int32_t query_heads, int32_t kv_heads,
                                     int32_t head_size, int64_t context, void *stream);
/* transformer.gqa-scores / causal-softmax / gqa-values
 * (GpuTransformerInstructionCollection.cs:545-695): the unfused attention, scores and
 * probabilities [query_heads, context]; token t takes part when (uint)t <= (uint)*position. */
si_status si_gqa_scores(const float *query, const float *key_cache, const int32_t *position, float *scores,
                        int32_t query_heads, int32_t kv_heads, int32_t head_size, int64_t context, void *stream);
si_status si_causal_softmax(const float *scores, const int32_t *position, float *probabilities, int32_t heads,
                            int64_t context, void *stream);
si_status si_gqa_values(const float *probabilities, const float *value_cache, const int32_t *position, float *output,
                        int32_t query_heads, int32_t kv_heads, int32_t head_size, int64_t context, void *stream);
/* transformer.argmax (GpuTransformerInstructionCollection.cs:697-744): the smallest index of
 * the largest value; NaN never wins; 0 when no value exceeds -FLT_MAX. */
si_status si_argmax(const float *input, int64_t count, int32_t *output, void *stream);
/* transformer.embedding-gather-batch (GpuTransformerInstructionCollection.cs:184-219): output
 * row r = FP16 table row indices[r] as FP32; an index outside the table gives zeros. */
si_status si_embedding_gather_batch(const uint16_t *table, int64_t rows, const int32_t *indices, float *output,
                                    int64_t batch, int64_t width, void *stream);
/* transformer.copy-embedding-rows (GpuTransformerInstructionCollection.cs:221-280):
 * output[output_start * width + e] = input[e], e < rows * width. */
si_status si_copy_embedding_rows(const float *input, float *output, int64_t output_rows, int64_t rows,
                                 int64_t width, int64_t output_start, void *stream);
/* Batch forms (GpuBatchTransformerInstructions.cs:101-679). */
si_status si_batch_rms_norm(const float *input, const float *weight, const int32_t *control, float *output,
                            int64_t batch, int64_t width, float epsilon, void *stream);
si_status si_batch_residual_rms_norm(const float *hidden, const float *residual, const float *weight,
                                     const int32_t *control, float *updated, float *output, int64_t batch,
                                     int64_t width, float epsilon, void *stream);
si_status si_batch_swiglu(const float *gate_up, const int32_t *control, float *output, int64_t batch, int64_t width,
                          void *stream);
/* Row b is the token at position control[0] + b. */
si_status si_batch_rope_kv_write(const float *qkv, const int32_t *control, const float *frequencies, float *query,
                                 float *key_cache, float *value_cache, int64_t batch, int64_t query_size,
                                 int32_t kv_heads, int32_t head_size, int32_t rotary_size, int64_t context,
                                 float rope_scale, void *stream);
si_status si_batch_gqa_scores(const float *query, const float *key_cache, const int32_t *control, float *scores,
                              int64_t batch, int32_t query_heads, int32_t kv_heads, int32_t head_size,
                              int64_t context, void *stream);
si_status si_batch_causal_softmax(const float *scores, const int32_t *control, float *probabilities, int64_t batch,
                                  int32_t heads, int64_t context, void *stream);
si_status si_batch_gqa_values(const float *probabilities, const float *value_cache, const int32_t *control,
                              float *output, int64_t batch, int32_t query_heads, int32_t kv_heads, int32_t head_size,
                              int64_t context, void *stream);
/* batch-gqa-scores -> batch-causal-softmax -> batch-gqa-values in one pass
 * (the prefill chunk's attention, GpuBatchTransformerInstructions.cs:320-551
 * composed): query [count, query_heads * head_size] holds rows at positions
 * start .. start + count - 1; row b attends cache tokens 0..start + b.
 * 0 <= start, start + count <= context; head_size 64, 128, 192 or 256
 * (SI_ERR_UNSUPPORTED otherwise); buffers 16-byte aligned. */
si_status si_batch_grouped_query_attention(const float *query, const float *key_cache, const float *value_cache,
                                           int32_t start, int32_t count, float *output, int32_t query_heads,
                                           int32_t kv_heads, int32_t head_size, int64_t context, void *stream);
/* output = input row control[1] - 1 when 0 < control[1] <= batch. */
si_status si_batch_select_last(const float *input, const int32_t *control, float *output, int64_t batch,
                               int64_t width, void *stream);
/* output row b = table row control[0] + b for b < control[1] when that row exists. */
si_status si_batch_gather_rows(const float *table, int64_t rows, const int32_t *control, float *output,
                               int64_t batch, int64_t width, void *stream);

/* ---------------------------------------------------------------------- */
/* Phi-4 text decoder session (Phi4D3D12TextSession.cs)                   */
/* ---------------------------------------------------------------------- */
/* The decode program of Phi4D3D12TextSession.Build (:307-920) as one CUDA
 * graph per token: gather-row, rms-norm, then per layer qkv mat-vec,
 * rope-kv-write, grouped-query-attention, output mat-vec, residual-rms-norm,
 * gate_up mat-vec, swiglu, down mat-vec, residual-rms-norm; vocabulary
 * mat-vec over the tied token_embedding and argmax. Weights keep their GGUF
 * bytes; KV caches are FP32 [context, kv_heads, head_size] per layer
 * (:420-425). query_heads * head_size must equal hidden. */
typedef struct si_decoder_config {
    int32_t layers, hidden, query_heads, kv_heads, head_size, rotary_size, intermediate, vocab;
    int64_t context;          /* maximumContext */
    float epsilon;            /* phi3.attention.layer_norm_rms_epsilon */
    float rope_base;          /* phi3.rope.freq_base */
    float rope_scale;         /* phi3.rope.scaling.attn_factor */
    uint32_t weight_type;     /* qkv / attn_output / ffn_up / ffn_down: F16, F32, Q8_0 or Q4_K */
    uint32_t embedding_type;  /* token_embedding (gathered and used as the vocabulary projection) */
} si_decoder_config;
typedef struct si_decoder si_decoder;
si_status si_decoder_create(int device, const si_decoder_config *config, si_decoder **out);
si_status si_decoder_destroy(si_decoder *decoder);
/* Row-sharded session on one rank of a peer group (config 5: Phi-4-14B
 * weights row-sharded over 2/4/8 GPUs with the outputs all-gathered). Each
 * projection slot (qkv, attn_output, ffn_up, ffn_down) holds only this
 * rank's rows (si_rowshard_plan; upload those rows), and runs as
 * si_rowshard_matvec_peer, whose kernel stores the rank's output rows into
 * every rank's arena over NVLink; the vocabulary projection uses this
 * rank's rows of token_embedding (uploaded whole: gather-row reads any
 * row). Norms, rope, attention, swiglu, argmax and the KV cache are
 * replicated, so every rank computes the same tokens. The group's arenas
 * need si_decoder_arena_bytes(config) bytes; every rank must make the same
 * session calls in the same order. Q4_K or Q8_0 weights; the persistent
 * step and the batched prefill are not used (prefill runs the decode
 * program per token). */
si_status si_decoder_arena_bytes(const si_decoder_config *config, uint64_t *bytes);
si_status si_decoder_create_sharded(int device, const si_decoder_config *config, si_peer_group *group,
                                    si_decoder **out);
/* Slots by the reference's names (Phi4D3D12TextSession.cs:391-425, 427-446):
 * token_embedding, output_norm, attn_norm_L, ffn_norm_L, qkv_weight_L,
 * attn_output_weight_L, ffn_up_weight_L, ffn_down_weight_L, rope_frequencies
 * (filled from rope_base at creation), key_cache_L, value_cache_L, hidden,
 * hidden_after_attention, normalized, qkv, query, attention, projected,
 * gate_up, activated, down, logits, next_token, control. */
si_status si_decoder_slot(si_decoder *decoder, const char *name, void **device_pointer, uint64_t *bytes);
si_status si_decoder_upload(si_decoder *decoder, const char *name, uint64_t offset, const void *host, uint64_t bytes);
si_status si_decoder_read(si_decoder *decoder, const char *name, uint64_t offset, void *host, uint64_t bytes);
si_status si_decoder_stream(si_decoder *decoder, void **stream);
/* ForwardToken (Phi4D3D12TextSession.cs:212-227): upload (token, position),
 * run the decode graph, read back the argmax; position advances by one.
 * SI_ERR_INVALID_ARGUMENT for a token outside the vocabulary or a full cache. */
si_status si_decoder_forward_token(si_decoder *decoder, int32_t token, int32_t *next_token);
/* Device-resident greedy loop: feeds prompt[0..prompt_tokens) and then its
 * own argmax for `steps` more positions, without host round trips between
 * tokens. tokens[k] = argmax after the k-th forward (prompt_tokens + steps
 * entries); position advances by prompt_tokens + steps. */
si_status si_decoder_generate(si_decoder *decoder, const int32_t *prompt, int32_t prompt_tokens, int32_t steps,
                              int32_t *tokens);
/* Batched prompt prefill (the prefill_fused_16 program,
 * Phi4D3D12TextSession.cs:267-286 and :1018-1155): the prompt in chunks of
 * up to 256 rows with control = (position, rows) per chunk; projections as
 * GEMMs, batch rope-kv-write, the batch scores / causal-softmax / values
 * instructions fused into one attention pass, batch residual norms; after
 * the last chunk select-last, vocabulary mat-vec and argmax. *next_token =
 * the prediction after the last prompt token; position advances by
 * prompt_tokens. Head sizes other than 64/128/192/256 run the decode
 * program once per token instead. */
si_status si_decoder_prefill(si_decoder *decoder, const int32_t *prompt, int32_t prompt_tokens, int32_t *next_token);
/* PrefillFusedEmbeddings (Phi4D3D12TextSession.cs:267-286): the same
 * program on `rows` ready FP32 embedding rows [rows, hidden] from host
 * memory instead of gathered token rows. */
si_status si_decoder_prefill_embeddings(si_decoder *decoder, const float *embeddings, int32_t rows,
                                        int32_t *next_token);
si_status si_decoder_reset(si_decoder *decoder);  /* Reset(): position = 0 */
si_status si_decoder_position(si_decoder *decoder, int32_t *position);

/* ---------------------------------------------------------------------- */
/* GGUF model files (GgufModelFile.cs)                                    */
/* ---------------------------------------------------------------------- */
/* si_gguf_open parses a GGUF v3 file as GgufModelFile.Open does
 * (GgufModelFile.cs:57-160) and maps it read-only; SI_ERR_INVALID_DATA for
 * a malformed file (InvalidDataException), SI_ERR_UNSUPPORTED for an
 * unknown tensor type (NotSupportedException). Tensor data pointers point
 * into the mapping and stay valid until si_gguf_close; their bytes are
 * uploaded unchanged (Phi4D3D12TextSession.cs:56-57). Tensor types are GGUF
 * ids (GgufModelTensorType, GgufModelFile.cs:24-46); byte lengths follow
 * GetByteLength (:301-331) plus the K-quant superblocks (Q2_K..Q8_K). */
typedef struct si_gguf si_gguf;
si_status si_gguf_open(const char *path, si_gguf **out);
si_status si_gguf_close(si_gguf *file);
si_status si_gguf_tensor_count(si_gguf *file, int64_t *count);
si_status si_gguf_find_tensor(si_gguf *file, const char *name, int64_t *index);
/* dims: 8 entries (unused ones 0), in file order (fastest dimension first). */
si_status si_gguf_tensor_info(si_gguf *file, int64_t index, char *name, size_t name_capacity, uint32_t *type,
                              int32_t *rank, uint64_t *dims, uint64_t *bytes, const void **data);
/* Metadata in file order; type = GgufMetadataType (:7-22); arrays report
 * their element type and count. */
si_status si_gguf_metadata_count(si_gguf *file, int64_t *count);
si_status si_gguf_metadata_key(si_gguf *file, int64_t index, char *key, size_t capacity, uint32_t *type,
                               uint32_t *element_type, uint64_t *count);
/* Numeric and Bool values as double (GetMetadata<T>'s conversion). */
si_status si_gguf_metadata_number(si_gguf *file, const char *key, double *value);
si_status si_gguf_metadata_string(si_gguf *file, const char *key, char *buffer, size_t capacity, size_t *length);
/* Arrays of fixed-size elements: a pointer to the packed little-endian
 * elements in the mapping; String arrays: count and element type only. */
si_status si_gguf_metadata_array(si_gguf *file, const char *key, uint32_t *element_type, uint64_t *count,
                                 const void **data);

#ifdef __cplusplus
}
#endif
#endif
