// C ABI of libsharpinfer_cuda: argument validation (the checks the
// reference performs when it binds and launches an instruction), pointer
// range checks against the CUDA allocation that holds each tensor, the
// executor (context / buffers / stream), and the instruction registry.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "si_internal.h"

struct si_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    uint64_t submissions = 0;
    void *workspace = nullptr;
    uint64_t workspace_bytes = 0;
    std::mutex lock;  // executor calls are serialised (D3D12VmExecutor.cs:285,307,457)
};

struct si_graph {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    si_context *owner = nullptr;
};

struct si_buffer {
    void *ptr = nullptr;
    uint64_t bytes = 0;
    si_context *owner = nullptr;
};

namespace si {
namespace {

using GetRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

// cuMemGetAddressRange through the runtime's driver entry point, so the
// library does not link libcuda directly.
GetRangeFn address_range_fn() {
    static GetRangeFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<GetRangeFn>(p);
    }();
    return fn;
}

// The tensor [ptr, ptr + bytes) must lie inside one device allocation of the
// current device. Host pointers, freed memory and short buffers are refused
// here instead of faulting the GPU.
si_status check_device_range(const char *port, const void *ptr, uint64_t bytes) {
    if (!ptr) return fail(SI_ERR_INVALID_ARGUMENT, "port '%s': null pointer", port);
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        cudaGetLastError();
        return fail(SI_ERR_INVALID_ARGUMENT, "port '%s': not a CUDA pointer", port);
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
        return fail(SI_ERR_INVALID_ARGUMENT, "port '%s': pointer is not device memory", port);
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr.device != dev)
        return fail(SI_ERR_INVALID_ARGUMENT, "port '%s': pointer belongs to device %d, current device is %d", port,
                    attr.device, dev);
    if (GetRangeFn fn = address_range_fn()) {
        CUdeviceptr base = 0;
        size_t size = 0;
        if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) == CUDA_SUCCESS) {
            const uint64_t off = uint64_t(reinterpret_cast<uintptr_t>(ptr) - base);
            if (off + bytes > size)
                return fail(SI_ERR_INVALID_ARGUMENT,
                            "port '%s': %llu bytes at offset %llu exceed the %llu-byte allocation", port,
                            (unsigned long long)bytes, (unsigned long long)off, (unsigned long long)size);
        }
    }
    return SI_OK;
}

bool overlaps(const void *a, uint64_t an, const void *b, uint64_t bn) {
    const auto pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
    return pa < pb + bn && pb < pa + an;
}

uint64_t elem_size(uint32_t t) { return t == SI_TYPE_F16 ? 2 : 4; }

si_status validate_matvec(uint32_t wtype, const void *w, uint32_t xtype, const void *x, uint32_t ytype,
                          const void *y, int64_t rows, int64_t cols, uint32_t config, bool check_ptrs) {
    if (rows <= 0 || cols <= 0)
        return fail(SI_ERR_INVALID_ARGUMENT, "Mixed matvec requires [rows,columns] x [columns] -> [rows].");
    // GpuMatVecExecution.Groups: rows beyond 32-bit thread indexing of a
    // 64-lane group are rejected (GpuMatVecExecution.cs:15-17).
    if (uint64_t(rows) > 0xFFFFFFFFull / 64)
        return fail(SI_ERR_INVALID_ARGUMENT, "Cooperative MatVec exceeds 32-bit thread indexing.");
    if (!known_type(wtype)) return fail(SI_ERR_UNSUPPORTED, "GGUF tensor type '%u' is not supported.", wtype);
    const bool quant = wtype == SI_TYPE_Q8_0 || wtype == SI_TYPE_Q4_K || wtype == SI_TYPE_Q6_K;
    if ((xtype != SI_TYPE_F32 && xtype != SI_TYPE_F16) || (ytype != SI_TYPE_F32 && ytype != SI_TYPE_F16))
        return fail(SI_ERR_ADAPTATION, "core.mat-vec: input and output must be F32 or F16.");
    if (quant && (xtype != SI_TYPE_F32 || ytype != SI_TYPE_F32))
        return fail(SI_ERR_ADAPTATION, "core.mat-vec: %s weights take an F32 input and produce an F32 output.",
                    type_name(wtype));
    if (config == SI_MATVEC_COOPERATIVE && quant)
        return fail(SI_ERR_ADAPTATION, "Unsupported CUDA execution configuration 'cooperative-matvec' for %s.",
                    type_name(wtype));
    if (config == SI_MATVEC_QUANT_STAGED && !quant)
        return fail(SI_ERR_ADAPTATION, "Unsupported CUDA execution configuration 'cuda-gemv-staged' for %s.",
                    type_name(wtype));
    if (config > SI_MATVEC_QUANT_STAGED) return fail(SI_ERR_ADAPTATION, "Unknown execution configuration %u.", config);
    uint64_t rb;
    if (si_status st = byte_length(wtype, uint64_t(cols), &rb)) return st;
    if (rows > 0 && rb > UINT64_MAX / uint64_t(rows)) return fail(SI_ERR_INVALID_ARGUMENT, "weight size overflows");
    const uint64_t wbytes = rb * uint64_t(rows), xbytes = uint64_t(cols) * elem_size(xtype),
                   ybytes = uint64_t(rows) * elem_size(ytype);
    if (!w || !x || !y) return fail(SI_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (overlaps(y, ybytes, w, wbytes) || overlaps(y, ybytes, x, xbytes))
        return fail(SI_ERR_UNSUPPORTED, "core.mat-vec: output aliases an input.");
    if (check_ptrs) {
        if (si_status st = check_device_range("weight", w, wbytes)) return st;
        if (si_status st = check_device_range("input", x, xbytes)) return st;
        if (si_status st = check_device_range("output", y, ybytes)) return st;
    }
    return SI_OK;
}

si_status run_matvec(uint32_t wtype, const void *w, uint32_t xtype, const void *x, uint32_t ytype, void *y,
                     int64_t rows, int64_t cols, void *stream) {
    if (wtype == SI_TYPE_Q8_0 || wtype == SI_TYPE_Q4_K || wtype == SI_TYPE_Q6_K)
        return kernels::matvec_quant(wtype, w, static_cast<const float *>(x), static_cast<float *>(y), rows, cols,
                                     stream);
    return kernels::matvec_dense(wtype, w, xtype, x, ytype, y, rows, cols, stream);
}

si_status validate_shared(const char *op, uint32_t wtype, const void *w, const float *x, const int32_t *control,
                          const float *y, int64_t m, int64_t n, int64_t k, bool check_ptrs) {
    if (m <= 0 || n <= 0 || k <= 0)
        return fail(SI_ERR_ADAPTATION, "%s: expected weight [O,I], input [B,I], and output [B,O].", op);
    if (!known_type(wtype)) return fail(SI_ERR_UNSUPPORTED, "GGUF tensor type '%u' is not supported.", wtype);
    if (m > 65535LL * 32) return fail(SI_ERR_INVALID_ARGUMENT, "%s: too many input rows (%lld).", op, (long long)m);
    uint64_t rb;
    if (si_status st = byte_length(wtype, uint64_t(k), &rb)) return st;
    const uint64_t wbytes = rb * uint64_t(n), xbytes = uint64_t(m) * uint64_t(k) * 4,
                   ybytes = uint64_t(m) * uint64_t(n) * 4;
    if (!w || !x || !y) return fail(SI_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (overlaps(y, ybytes, w, wbytes) || overlaps(y, ybytes, x, xbytes) ||
        (control && overlaps(y, ybytes, control, 8)))
        return fail(SI_ERR_UNSUPPORTED, "%s: output aliases an input.", op);
    if (check_ptrs) {
        if (si_status st = check_device_range("weight", w, wbytes)) return st;
        if (si_status st = check_device_range("input", x, xbytes)) return st;
        if (si_status st = check_device_range("output", y, ybytes)) return st;
        if (control)
            if (si_status st = check_device_range("control", control, 8)) return st;
    }
    return SI_OK;
}

si_status cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return SI_OK;
    if (e == cudaErrorMemoryAllocation) return fail(SI_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
        return fail(SI_ERR_NO_DEVICE, "%s: %s", what, cudaGetErrorString(e));
    return fail(SI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

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

si_status buffer_range(si_context *ctx, si_buffer *b, uint64_t off, uint64_t bytes, const char *port, void **p) {
    if (!b) return fail(SI_ERR_INVALID_ARGUMENT, "port '%s': null buffer", port);
    if (b->owner != ctx) return fail(SI_ERR_INVALID_ARGUMENT, "port '%s': buffer belongs to another context", port);
    if (off > b->bytes || bytes > b->bytes - off)
        return fail(SI_ERR_INVALID_ARGUMENT, "port '%s': %llu bytes at offset %llu exceed the %llu-byte slot", port,
                    (unsigned long long)bytes, (unsigned long long)off, (unsigned long long)b->bytes);
    *p = static_cast<uint8_t *>(b->ptr) + off;
    return SI_OK;
}

// ---- instruction registry --------------------------------------------------
// Collection ids of InstructionCollectionIds (InstructionCollection.cs:6-12).
constexpr const char *kTierZeroFloat32 = "00000000-0000-0000-0000-000000000000";
constexpr const char *kTierZeroFloat16 = "00000000-0000-0000-0000-000000000001";
constexpr const char *kTransformerFloat32 = "824d0f9c-16c7-46d8-b49d-0f91d6a4ec83";

enum InstructionId { kMatVec32 = 1, kMatVec16 = 2, kMatrixMultiply = 3, kBatchSharedMatVec = 4, kGatherRow = 5,
                     kTransformerBase = 16 };

// Port element types of the FP32 transformer instructions, in port order
// (GpuTransformerInstructionCollection.cs, GpuBatchTransformerInstructions.cs):
// f = F32, i = Int32, h = F16.
struct TransformerSignature {
    const char *name;
    const char *ports;
};
constexpr TransformerSignature kTransformer[] = {
    {"transformer.rms-norm", "fff"},
    {"transformer.residual-rms-norm", "fffff"},
    {"transformer.swiglu", "ff"},
    {"transformer.rope-kv-write", "fiffff"},
    {"transformer.gqa-scores", "ffif"},
    {"transformer.causal-softmax", "fif"},
    {"transformer.gqa-values", "ffif"},
    {"transformer.grouped-query-attention", "fffif"},
    {"transformer.argmax", "fi"},
    {"transformer.scaled-add", "fff"},
    {"transformer.embedding-gather-batch", "hif"},
    {"transformer.copy-embedding-rows", "ff"},
    {"transformer.batch-rms-norm", "ffif"},
    {"transformer.batch-residual-rms-norm", "fffiff"},
    {"transformer.batch-swiglu", "fif"},
    {"transformer.batch-rope-kv-write", "fiffff"},
    {"transformer.batch-gqa-scores", "ffif"},
    {"transformer.batch-causal-softmax", "fif"},
    {"transformer.batch-gqa-values", "ffif"},
    {"transformer.batch-select-last", "fif"},
    {"transformer.batch-gather-rows", "fif"},
};
constexpr int kTransformerCount = int(sizeof(kTransformer) / sizeof(kTransformer[0]));

bool iequal(const char *a, const char *b) {
    for (; *a && *b; ++a, ++b)
        if (std::tolower(static_cast<unsigned char>(*a)) != std::tolower(static_cast<unsigned char>(*b))) return false;
    return *a == *b;
}

}  // namespace

// Shared with the other host translation units (si_internal.h).
si_status device_range(const char *port, const void *ptr, uint64_t bytes) {
    return check_device_range(port, ptr, bytes);
}
bool ranges_overlap(const void *a, uint64_t an, const void *b, uint64_t bn) { return overlaps(a, an, b, bn); }
si_status cuda_error(int error, const char *what) { return cuda_status(static_cast<cudaError_t>(error), what); }

}  // namespace si

using namespace si;

extern "C" {

si_status si_device_count(int *count) {
    if (!count) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? SI_OK : cuda_status(e, "cudaGetDeviceCount");
    }
    *count = n;
    return SI_OK;
}

si_status si_matvec(uint32_t weight_type, const void *weight, uint32_t input_type, const void *input,
                    uint32_t output_type, void *output, int64_t rows, int64_t cols, uint32_t config, void *stream) {
    if (si_status st = validate_matvec(weight_type, weight, input_type, input, output_type, output, rows, cols, config,
                                       true))
        return st;
    return run_matvec(weight_type, weight, input_type, input, output_type, output, rows, cols, stream);
}

si_status si_gemv_default_plan(uint32_t weight_type, int64_t rows, int64_t cols, si_gemv_plan *plan) {
    if (!plan) return fail(SI_ERR_INVALID_ARGUMENT, "null plan");
    if (rows <= 0 || cols <= 0) return fail(SI_ERR_INVALID_ARGUMENT, "rows and cols must be positive");
    const si_status st = kernels::gemv_default_plan(weight_type, rows, cols, plan);
    if (st == SI_ERR_UNSUPPORTED)
        return fail(SI_ERR_UNSUPPORTED, "no tensor-core GEMV shape for %s [%lld, %lld]", type_name(weight_type),
                    (long long)rows, (long long)cols);
    return st;
}

si_status si_matvec_quant_planned(uint32_t weight_type, const void *weight, const float *input, float *output,
                                  int64_t rows, int64_t cols, const si_gemv_plan *plan, void *stream) {
    if (!plan) return fail(SI_ERR_INVALID_ARGUMENT, "null plan");
    if (weight_type != SI_TYPE_Q8_0 && weight_type != SI_TYPE_Q4_K)
        return fail(SI_ERR_ADAPTATION, "planned GEMV: weight must be Q8_0 or Q4_K.");
    if (si_status st = validate_matvec(weight_type, weight, SI_TYPE_F32, input, SI_TYPE_F32, output, rows, cols,
                                       SI_MATVEC_DEFAULT, true))
        return st;
    return kernels::matvec_quant_planned(weight_type, weight, input, output, rows, cols, *plan, stream);
}

si_status si_batch_shared_matvec(uint32_t weight_type, const void *weight, const float *input, const int32_t *control,
                                 float *output, int64_t batch, int64_t out_features, int64_t in_features,
                                 void *stream) {
    if (!control) return fail(SI_ERR_INVALID_ARGUMENT, "transformer.batch-shared-matvec requires a control tensor.");
    if (weight_type == SI_TYPE_F32)
        return fail(SI_ERR_ADAPTATION, "transformer.batch-shared-matvec: weight must be F16, Q8_0 or Q4_K.");
    if (si_status st = validate_shared("transformer.batch-shared-matvec", weight_type, weight, input, control, output,
                                       batch, out_features, in_features, true))
        return st;
    return kernels::batch_shared_matvec(weight_type, weight, input, control, output, batch, out_features, in_features,
                                        stream);
}

si_status si_matrix_multiply_workspace_bytes(uint32_t weight_type, int64_t m, int64_t n, int64_t k, uint64_t *bytes) {
    if (!bytes) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    if (m <= 0 || n <= 0 || k <= 0) return fail(SI_ERR_INVALID_ARGUMENT, "Incompatible matrix multiplication dimensions.");
    if (!known_type(weight_type)) return fail(SI_ERR_UNSUPPORTED, "GGUF tensor type '%u' is not supported.", weight_type);
    return kernels::gemm_workspace_bytes(weight_type, m, n, k, bytes);
}

si_status si_matrix_multiply(uint32_t weight_type, const float *x, const void *weight, float *y, int64_t m, int64_t n,
                             int64_t k, void *workspace, uint64_t workspace_bytes, void *stream) {
    if (si_status st = validate_shared("core.matrix-multiply", weight_type, weight, x, nullptr, y, m, n, k, true))
        return st;
    uint64_t need = 0;
    if (si_status st = kernels::gemm_workspace_bytes(weight_type, m, n, k, &need)) return st;
    if (workspace_bytes < need)
        return fail(SI_ERR_INVALID_ARGUMENT, "core.matrix-multiply: workspace of %llu bytes, %llu required",
                    (unsigned long long)workspace_bytes, (unsigned long long)need);
    if (need) {
        if (si_status st = check_device_range("workspace", workspace, need)) return st;
        if (overlaps(workspace, need, y, uint64_t(m) * n * 4) || overlaps(workspace, need, x, uint64_t(m) * k * 4))
            return fail(SI_ERR_UNSUPPORTED, "core.matrix-multiply: workspace aliases a tensor.");
    }
    return kernels::gemm_tn(weight_type, x, weight, y, m, n, k, workspace, workspace_bytes, stream);
}

si_status si_device_error_take(int device, uint32_t *code) {
    if (!code) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *code = 0;
    if (si_status st = kernels::take_error_gemv(device, code)) return st;
    if (si_status st = kernels::take_error_gemv_mma(device, code)) return st;
    if (si_status st = kernels::take_error_gemm_skinny(device, code)) return st;
    if (si_status st = kernels::take_error_gemm_fewrow(device, code)) return st;
    return kernels::take_error_gemm(device, code);
}

// ---- executor ----------------------------------------------------------------
si_status si_context_create(int device, si_context **out) {
    if (!out) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(SI_ERR_NO_DEVICE, "no CUDA device is available");
    }
    if (device < 0 || device >= n) return fail(SI_ERR_INVALID_ARGUMENT, "device %d out of range [0,%d)", device, n);
    DeviceScope scope(device);
    auto *ctx = new si_context();
    ctx->device = device;
    if (si_status st = cuda_status(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking), "cudaStreamCreate")) {
        delete ctx;
        return st;
    }
    *out = ctx;
    return SI_OK;
}

si_status si_context_destroy(si_context *ctx) {
    if (!ctx) return SI_OK;
    DeviceScope scope(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->workspace) cudaFree(ctx->workspace);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return SI_OK;
}

si_status si_context_stream(si_context *ctx, void **stream) {
    if (!ctx || !stream) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *stream = ctx->stream;
    return SI_OK;
}

si_status si_context_synchronize(si_context *ctx) {
    if (!ctx) return fail(SI_ERR_INVALID_ARGUMENT, "null context");
    DeviceScope scope(ctx->device);
    return cuda_status(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
}

si_status si_context_submission_count(si_context *ctx, uint64_t *count) {
    if (!ctx || !count) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *count = ctx->submissions;
    return SI_OK;
}

si_status si_buffer_create(si_context *ctx, uint64_t bytes, si_buffer **out) {
    if (!ctx || !out || bytes == 0) return fail(SI_ERR_INVALID_ARGUMENT, "buffer requires a context and bytes > 0");
    DeviceScope scope(ctx->device);
    void *p = nullptr;
    if (si_status st = cuda_status(cudaMalloc(&p, bytes), "cudaMalloc")) return st;
    auto *b = new si_buffer();
    b->ptr = p;
    b->bytes = bytes;
    b->owner = ctx;
    *out = b;
    return SI_OK;
}

si_status si_buffer_destroy(si_context *ctx, si_buffer *buffer) {
    if (!buffer) return SI_OK;
    if (buffer->owner != ctx) return fail(SI_ERR_INVALID_ARGUMENT, "buffer belongs to another context");
    DeviceScope scope(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(buffer->ptr);
    delete buffer;
    return SI_OK;
}

si_status si_buffer_device_pointer(si_buffer *buffer, void **pointer, uint64_t *bytes) {
    if (!buffer || !pointer) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *pointer = buffer->ptr;
    if (bytes) *bytes = buffer->bytes;
    return SI_OK;
}

static si_status copy(si_context *ctx, si_buffer *b, uint64_t off, void *host, uint64_t bytes, bool upload, bool sync) {
    if (!ctx) return fail(SI_ERR_INVALID_ARGUMENT, "null context");
    if (!host && bytes) return fail(SI_ERR_INVALID_ARGUMENT, "null host pointer");
    void *dev = nullptr;
    if (si_status st = buffer_range(ctx, b, off, bytes, upload ? "upload" : "readback", &dev)) return st;
    if (!bytes) return SI_OK;
    std::lock_guard<std::mutex> g(ctx->lock);
    DeviceScope scope(ctx->device);
    cudaError_t e = upload ? cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, ctx->stream)
                           : cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess && sync) e = cudaStreamSynchronize(ctx->stream);
    return cuda_status(e, upload ? "upload" : "readback");
}

si_status si_buffer_upload(si_context *ctx, si_buffer *buffer, uint64_t offset, const void *src, uint64_t bytes) {
    return copy(ctx, buffer, offset, const_cast<void *>(src), bytes, true, true);
}
si_status si_buffer_readback(si_context *ctx, si_buffer *buffer, uint64_t offset, void *dst, uint64_t bytes) {
    return copy(ctx, buffer, offset, dst, bytes, false, true);
}
si_status si_buffer_upload_async(si_context *ctx, si_buffer *buffer, uint64_t offset, const void *src, uint64_t bytes) {
    return copy(ctx, buffer, offset, const_cast<void *>(src), bytes, true, false);
}
si_status si_buffer_readback_async(si_context *ctx, si_buffer *buffer, uint64_t offset, void *dst, uint64_t bytes) {
    return copy(ctx, buffer, offset, dst, bytes, false, false);
}

si_status si_host_alloc_pinned(uint64_t bytes, void **out) {
    if (!out || !bytes) return fail(SI_ERR_INVALID_ARGUMENT, "pinned allocation requires bytes > 0");
    return cuda_status(cudaHostAlloc(out, bytes, cudaHostAllocPortable), "cudaHostAlloc");
}

si_status si_host_free_pinned(void *ptr) {
    if (!ptr) return SI_OK;
    return cuda_status(cudaFreeHost(ptr), "cudaFreeHost");
}

si_status si_ctx_matvec(si_context *ctx, uint32_t weight_type, si_buffer *weight, uint64_t weight_offset,
                        uint32_t input_type, si_buffer *input, uint64_t input_offset, uint32_t output_type,
                        si_buffer *output, uint64_t output_offset, int64_t rows, int64_t cols, uint32_t config) {
    if (!ctx) return fail(SI_ERR_INVALID_ARGUMENT, "null context");
    if (rows <= 0 || cols <= 0)
        return fail(SI_ERR_INVALID_ARGUMENT, "Mixed matvec requires [rows,columns] x [columns] -> [rows].");
    uint64_t rb;
    if (si_status st = byte_length(weight_type, uint64_t(cols), &rb)) return st;
    void *w = nullptr, *x = nullptr, *y = nullptr;
    if (si_status st = buffer_range(ctx, weight, weight_offset, rb * uint64_t(rows), "weight", &w)) return st;
    if (si_status st = buffer_range(ctx, input, input_offset, uint64_t(cols) * elem_size(input_type), "input", &x))
        return st;
    if (si_status st = buffer_range(ctx, output, output_offset, uint64_t(rows) * elem_size(output_type), "output", &y))
        return st;
    if (si_status st = validate_matvec(weight_type, w, input_type, x, output_type, y, rows, cols, config, false))
        return st;
    std::lock_guard<std::mutex> g(ctx->lock);
    DeviceScope scope(ctx->device);
    const si_status st = run_matvec(weight_type, w, input_type, x, output_type, y, rows, cols, ctx->stream);
    if (st == SI_OK) ++ctx->submissions;
    return st;
}

si_status si_ctx_batch_shared_matvec(si_context *ctx, uint32_t weight_type, si_buffer *weight, uint64_t weight_offset,
                                     si_buffer *input, uint64_t input_offset, si_buffer *control,
                                     uint64_t control_offset, si_buffer *output, uint64_t output_offset, int64_t batch,
                                     int64_t out_features, int64_t in_features) {
    if (!ctx) return fail(SI_ERR_INVALID_ARGUMENT, "null context");
    if (batch <= 0 || out_features <= 0 || in_features <= 0)
        return fail(SI_ERR_ADAPTATION, "Expected weight [O,I], input [B,I], and output [B,O].");
    if (weight_type == SI_TYPE_F32)
        return fail(SI_ERR_ADAPTATION, "transformer.batch-shared-matvec: weight must be F16, Q8_0 or Q4_K.");
    uint64_t rb;
    if (si_status st = byte_length(weight_type, uint64_t(in_features), &rb)) return st;
    void *w = nullptr, *x = nullptr, *c = nullptr, *y = nullptr;
    if (si_status st = buffer_range(ctx, weight, weight_offset, rb * uint64_t(out_features), "weight", &w)) return st;
    if (si_status st = buffer_range(ctx, input, input_offset, uint64_t(batch) * in_features * 4, "input", &x)) return st;
    if (si_status st = buffer_range(ctx, control, control_offset, 8, "control", &c)) return st;
    if (si_status st = buffer_range(ctx, output, output_offset, uint64_t(batch) * out_features * 4, "output", &y))
        return st;
    if (si_status st = validate_shared("transformer.batch-shared-matvec", weight_type, w, static_cast<float *>(x),
                                       static_cast<int32_t *>(c), static_cast<float *>(y), batch, out_features,
                                       in_features, false))
        return st;
    std::lock_guard<std::mutex> g(ctx->lock);
    DeviceScope scope(ctx->device);
    const si_status st =
        kernels::batch_shared_matvec(weight_type, w, static_cast<const float *>(x), static_cast<const int32_t *>(c),
                                     static_cast<float *>(y), batch, out_features, in_features, ctx->stream);
    if (st == SI_OK) ++ctx->submissions;
    return st;
}

si_status si_ctx_matrix_multiply(si_context *ctx, uint32_t weight_type, si_buffer *x, uint64_t x_offset,
                                 si_buffer *weight, uint64_t weight_offset, si_buffer *y, uint64_t y_offset, int64_t m,
                                 int64_t n, int64_t k) {
    if (!ctx) return fail(SI_ERR_INVALID_ARGUMENT, "null context");
    if (m <= 0 || n <= 0 || k <= 0) return fail(SI_ERR_INVALID_ARGUMENT, "Incompatible matrix multiplication dimensions.");
    uint64_t rb;
    if (si_status st = byte_length(weight_type, uint64_t(k), &rb)) return st;
    void *px = nullptr, *pw = nullptr, *py = nullptr;
    if (si_status st = buffer_range(ctx, x, x_offset, uint64_t(m) * k * 4, "left", &px)) return st;
    if (si_status st = buffer_range(ctx, weight, weight_offset, rb * uint64_t(n), "right", &pw)) return st;
    if (si_status st = buffer_range(ctx, y, y_offset, uint64_t(m) * n * 4, "output", &py)) return st;
    if (si_status st = validate_shared("core.matrix-multiply", weight_type, pw, static_cast<float *>(px), nullptr,
                                       static_cast<float *>(py), m, n, k, false))
        return st;
    uint64_t need = 0;
    if (si_status st = kernels::gemm_workspace_bytes(weight_type, m, n, k, &need)) return st;
    std::lock_guard<std::mutex> g(ctx->lock);
    DeviceScope scope(ctx->device);
    if (need > ctx->workspace_bytes) {
        cudaStreamSynchronize(ctx->stream);
        if (ctx->workspace) cudaFree(ctx->workspace);
        ctx->workspace = nullptr;
        ctx->workspace_bytes = 0;
        if (si_status st = cuda_status(cudaMalloc(&ctx->workspace, need), "workspace cudaMalloc")) return st;
        ctx->workspace_bytes = need;
    }
    const si_status st = kernels::gemm_tn(weight_type, static_cast<const float *>(px), pw, static_cast<float *>(py), m,
                                          n, k, ctx->workspace, ctx->workspace_bytes, ctx->stream);
    if (st == SI_OK) ++ctx->submissions;
    return st;
}

// ---- recorded submissions (CUDA graphs) ----------------------------------------
si_status si_graph_begin(si_context *ctx) {
    if (!ctx) return fail(SI_ERR_INVALID_ARGUMENT, "null context");
    DeviceScope scope(ctx->device);
    return cuda_status(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
}

si_status si_graph_end(si_context *ctx, si_graph **out) {
    if (!ctx || !out) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    DeviceScope scope(ctx->device);
    cudaGraph_t g = nullptr;
    if (si_status st = cuda_status(cudaStreamEndCapture(ctx->stream, &g), "cudaStreamEndCapture")) return st;
    cudaGraphExec_t exec = nullptr;
    if (si_status st = cuda_status(cudaGraphInstantiate(&exec, g, 0), "cudaGraphInstantiate")) {
        cudaGraphDestroy(g);
        return st;
    }
    auto *graph = new si_graph();
    graph->graph = g;
    graph->exec = exec;
    graph->owner = ctx;
    *out = graph;
    return SI_OK;
}

si_status si_graph_launch(si_context *ctx, si_graph *graph) {
    if (!ctx || !graph || graph->owner != ctx) return fail(SI_ERR_INVALID_ARGUMENT, "graph belongs to another context");
    std::lock_guard<std::mutex> g(ctx->lock);
    DeviceScope scope(ctx->device);
    const si_status st = cuda_status(cudaGraphLaunch(graph->exec, ctx->stream), "cudaGraphLaunch");
    if (st == SI_OK) ++ctx->submissions;
    return st;
}

si_status si_graph_destroy(si_graph *graph) {
    if (!graph) return SI_OK;
    if (graph->exec) cudaGraphExecDestroy(graph->exec);
    if (graph->graph) cudaGraphDestroy(graph->graph);
    delete graph;
    return SI_OK;
}

// ---- instruction registry ------------------------------------------------------
si_status si_instruction_resolve(const char *collection_id, const char *name, int *instruction_id) {
    if (!collection_id || !name || !instruction_id || !*name)
        return fail(SI_ERR_INVALID_ARGUMENT, "collection id and instruction name are required");
    const bool t0f32 = iequal(collection_id, kTierZeroFloat32), t0f16 = iequal(collection_id, kTierZeroFloat16),
               tr = iequal(collection_id, kTransformerFloat32);
    if (!t0f32 && !t0f16 && !tr)
        return fail(SI_ERR_UNSUPPORTED, "Instruction collection '%s' is not installed.", collection_id);
    int id = 0;
    if ((t0f32 || t0f16) && std::strcmp(name, "core.mat-vec") == 0) id = t0f32 ? kMatVec32 : kMatVec16;
    else if (t0f32 && std::strcmp(name, "core.matrix-multiply") == 0) id = kMatrixMultiply;
    else if (tr && std::strcmp(name, "transformer.batch-shared-matvec") == 0) id = kBatchSharedMatVec;
    else if (t0f32 && std::strcmp(name, "core.gather-row") == 0) id = kGatherRow;
    else if (tr)
        for (int i = 0; i < kTransformerCount; ++i)
            if (std::strcmp(name, kTransformer[i].name) == 0) id = kTransformerBase + i;
    if (!id) return fail(SI_ERR_UNSUPPORTED, "No cuda implementation for '%s/%s'.", collection_id, name);
    *instruction_id = id;
    return SI_OK;
}

si_status si_instruction_validate(int instruction_id, const uint32_t *t, int n, const char *configuration) {
    if (!t && n) return fail(SI_ERR_INVALID_ARGUMENT, "null port types");
    const char *cfg = configuration ? configuration : "";
    auto quant = [](uint32_t v) { return v == SI_TYPE_Q8_0 || v == SI_TYPE_Q4_K || v == SI_TYPE_Q6_K; };
    switch (instruction_id) {
    case kMatVec32:
    case kMatVec16: {
        // ports: matrix|weight, input, output
        bool ok = n == 3;
        if (ok && instruction_id == kMatVec32)
            ok = (t[0] == SI_TYPE_F32 || t[0] == SI_TYPE_F16 || quant(t[0])) && t[1] == SI_TYPE_F32 &&
                 t[2] == SI_TYPE_F32;
        else if (ok)
            ok = t[0] == SI_TYPE_F16 && t[1] == SI_TYPE_F16 && t[2] == SI_TYPE_F16;
        if (!ok) return fail(SI_ERR_ADAPTATION, "core.mat-vec: no supported parameter/precision signature.");
        if (!*cfg) return SI_OK;
        if (std::strcmp(cfg, "cooperative-matvec") == 0 && !quant(t[0])) return SI_OK;
        if (std::strcmp(cfg, "cuda-gemv-staged") == 0 && quant(t[0])) return SI_OK;
        return fail(SI_ERR_ADAPTATION, "Unsupported CUDA execution configuration '%s'.", cfg);
    }
    case kMatrixMultiply: {
        const bool ok = n == 3 && t[0] == SI_TYPE_F32 &&
                        (t[1] == SI_TYPE_F32 || t[1] == SI_TYPE_F16 || quant(t[1])) && t[2] == SI_TYPE_F32;
        if (!ok) return fail(SI_ERR_ADAPTATION, "core.matrix-multiply: no supported parameter/precision signature.");
        if (!*cfg || std::strcmp(cfg, "cuda-gemm") == 0) return SI_OK;
        return fail(SI_ERR_ADAPTATION, "Unsupported CUDA execution configuration '%s'.", cfg);
    }
    case kBatchSharedMatVec: {
        const bool ok = n == 4 && (t[0] == SI_TYPE_F16 || quant(t[0])) && t[1] == SI_TYPE_F32 &&
                        t[2] == SI_TYPE_I32 && t[3] == SI_TYPE_F32;
        if (!ok)
            return fail(SI_ERR_ADAPTATION, "transformer.batch-shared-matvec: no supported parameter/precision signature.");
        if (!*cfg) return SI_OK;
        return fail(SI_ERR_ADAPTATION, "Unsupported CUDA execution configuration '%s'.", cfg);
    }
    case kGatherRow: {
        // table, index, output: [f32|f16|q8_0|q4_k, Int32] -> [f32] (TierZeroOperationContracts.cs:159)
        const bool ok = n == 3 && (t[0] == SI_TYPE_F32 || t[0] == SI_TYPE_F16 || quant(t[0])) &&
                        t[1] == SI_TYPE_I32 && t[2] == SI_TYPE_F32;
        if (!ok) return fail(SI_ERR_ADAPTATION, "core.gather-row: no supported parameter/precision signature.");
        if (!*cfg) return SI_OK;
        return fail(SI_ERR_ADAPTATION, "Unsupported CUDA execution configuration '%s'.", cfg);
    }
    default: {
        const int i = instruction_id - kTransformerBase;
        if (i < 0 || i >= kTransformerCount) return fail(SI_ERR_UNSUPPORTED, "unknown instruction id %d", instruction_id);
        const char *ports = kTransformer[i].ports;
        bool ok = int(std::strlen(ports)) == n;
        for (int p = 0; ok && p < n; ++p) {
            const uint32_t want = ports[p] == 'f' ? SI_TYPE_F32 : ports[p] == 'i' ? SI_TYPE_I32 : SI_TYPE_F16;
            ok = t[p] == want;
        }
        if (!ok) return fail(SI_ERR_ADAPTATION, "%s: no supported parameter/precision signature.", kTransformer[i].name);
        if (!*cfg) return SI_OK;
        return fail(SI_ERR_ADAPTATION, "Unsupported CUDA execution configuration '%s'.", cfg);
    }
    }
}

}  // extern "C"
