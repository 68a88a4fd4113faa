// P/Invoke layer over libsharpinfer_cuda (include/sharpinfer_cuda.h): the
// only place managed code touches the native library. Every entry returns a
// status; Check maps it to the exception type the reference raises for the
// same condition (ArgumentException, NotSupportedException,
// InstructionAdaptationException, InvalidDataException).
//
// Not built in this repository (no .NET toolchain in the image); compiled as
// part of SharpInference.Backends.CudaVm next to SharpInference.Backends.D3D12Vm.
using System.Runtime.InteropServices;

namespace SharpInference.Backends.CudaVm;

internal static unsafe partial class SharpInferCuda
{
    private const string Lib = "sharpinfer_cuda"; // libsharpinfer_cuda.so

    public const int AbiVersion = 1;

    public enum Status
    {
        Ok = 0, InvalidArgument = 1, Unsupported = 2, Adaptation = 3, InvalidData = 4,
        Cuda = 5, OutOfMemory = 6, Nccl = 7, Timeout = 8, NoDevice = 9,
    }

    /// <summary>GGUF tensor type ids (GgufModelFile.cs:24-46) used for every port type.</summary>
    public enum TensorType : uint { F32 = 0, F16 = 1, Q8_0 = 8, Q4_K = 12, Q6_K = 14, I32 = 26 }

    [LibraryImport(Lib)] public static partial int si_abi_version();
    [LibraryImport(Lib)] public static partial Status si_last_error(byte* buffer, nuint capacity);
    [LibraryImport(Lib)] public static partial Status si_device_count(out int count);
    [LibraryImport(Lib)] public static partial Status si_tensor_byte_length(uint type, ulong* dims, int rank, out ulong bytes);

    // executor level (D3D12VmExecutor.cs:283-700)
    [LibraryImport(Lib)] public static partial Status si_context_create(int device, out nint ctx);
    [LibraryImport(Lib)] public static partial Status si_context_destroy(nint ctx);
    [LibraryImport(Lib)] public static partial Status si_context_stream(nint ctx, out nint stream);
    [LibraryImport(Lib)] public static partial Status si_context_synchronize(nint ctx);
    [LibraryImport(Lib)] public static partial Status si_context_submission_count(nint ctx, out ulong count);
    [LibraryImport(Lib)] public static partial Status si_buffer_create(nint ctx, ulong bytes, out nint buffer);
    [LibraryImport(Lib)] public static partial Status si_buffer_destroy(nint ctx, nint buffer);
    [LibraryImport(Lib)] public static partial Status si_buffer_device_pointer(nint buffer, out nint pointer, out ulong bytes);
    [LibraryImport(Lib)] public static partial Status si_buffer_upload(nint ctx, nint buffer, ulong offset, void* src, ulong bytes);
    [LibraryImport(Lib)] public static partial Status si_buffer_readback(nint ctx, nint buffer, ulong offset, void* dst, ulong bytes);
    [LibraryImport(Lib)] public static partial Status si_buffer_upload_async(nint ctx, nint buffer, ulong offset, void* src, ulong bytes);
    [LibraryImport(Lib)] public static partial Status si_buffer_readback_async(nint ctx, nint buffer, ulong offset, void* dst, ulong bytes);
    [LibraryImport(Lib)] public static partial Status si_host_alloc_pinned(ulong bytes, out nint pointer);
    [LibraryImport(Lib)] public static partial Status si_host_free_pinned(nint pointer);
    [LibraryImport(Lib)] public static partial Status si_graph_begin(nint ctx);
    [LibraryImport(Lib)] public static partial Status si_graph_end(nint ctx, out nint graph);
    [LibraryImport(Lib)] public static partial Status si_graph_launch(nint ctx, nint graph);
    [LibraryImport(Lib)] public static partial Status si_graph_destroy(nint graph);

    // T0 instructions on executor buffers: (buffer, byte offset) per port (VmArgument.ByteOffset)
    [LibraryImport(Lib)] public static partial Status si_ctx_matvec(nint ctx, uint weightType, nint weight, ulong weightOffset,
        uint inputType, nint input, ulong inputOffset, uint outputType, nint output, ulong outputOffset,
        long rows, long cols, uint config);
    [LibraryImport(Lib)] public static partial Status si_ctx_batch_shared_matvec(nint ctx, uint weightType,
        nint weight, ulong weightOffset, nint input, ulong inputOffset, nint control, ulong controlOffset,
        nint output, ulong outputOffset, long batch, long outFeatures, long inFeatures);
    [LibraryImport(Lib)] public static partial Status si_ctx_matrix_multiply(nint ctx, uint weightType,
        nint x, ulong xOffset, nint weight, ulong weightOffset, nint y, ulong yOffset, long m, long n, long k);

    // transformer instructions on device pointers, enqueued on the context stream
    [LibraryImport(Lib)] public static partial Status si_gather_row(uint tableType, nint table, long rows, long cols, nint index, nint output, nint stream);
    [LibraryImport(Lib)] public static partial Status si_rms_norm(nint input, nint weight, nint output, long count, float epsilon, nint stream);
    [LibraryImport(Lib)] public static partial Status si_residual_rms_norm(nint hidden, nint residual, nint weight, nint updated,
        nint output, long count, float epsilon, nint stream);
    [LibraryImport(Lib)] public static partial Status si_swiglu(nint gateUp, nint output, long count, nint stream);
    [LibraryImport(Lib)] public static partial Status si_scaled_add(nint input, nint update, nint output, long count, float scale, nint stream);
    [LibraryImport(Lib)] public static partial Status si_rope_kv_write(nint qkv, nint position, nint frequencies, nint query,
        nint keyCache, nint valueCache, long querySize, int kvHeads, int headSize, int rotarySize, long context,
        float ropeScale, nint stream);
    [LibraryImport(Lib)] public static partial Status si_grouped_query_attention(nint query, nint keyCache, nint valueCache,
        nint position, nint output, int queryHeads, int kvHeads, int headSize, long context, nint stream);
    // transformer.rope-kv-write followed by transformer.grouped-query-attention in one launch
    // (Phi4D3D12TextSession.cs:873-916 dispatches the two in turn).
    [LibraryImport(Lib)] public static partial Status si_rope_grouped_query_attention(nint qkv, nint position,
        nint frequencies, nint keyCache, nint valueCache, nint output, int queryHeads, int kvHeads, int headSize,
        int rotarySize, long context, float ropeScale, nint stream);
    [LibraryImport(Lib)] public static partial Status si_argmax(nint input, long count, nint output, nint stream);

    // registry (InstructionCollection.cs:146-218)
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial Status si_instruction_resolve(string collectionId, string name, out int instructionId);
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial Status si_instruction_validate(int instructionId, uint* portTypes, int portCount, string configuration);

    public static string LastError()
    {
        var buffer = stackalloc byte[1024];
        si_last_error(buffer, 1024);
        return Marshal.PtrToStringUTF8((nint)buffer) ?? string.Empty;
    }

    /// <summary>Throws the reference's exception type for a failing status.</summary>
    public static void Check(Status status, Func<string, Exception>? adaptation = null)
    {
        if (status == Status.Ok) return;
        var message = LastError();
        if (message.Length == 0) message = status.ToString();
        throw status switch
        {
            Status.InvalidArgument => new ArgumentException(message),
            Status.Unsupported => new NotSupportedException(message),
            Status.Adaptation => adaptation?.Invoke(message) ?? new InvalidOperationException(message),
            Status.InvalidData => new InvalidDataException(message),
            Status.OutOfMemory => new OutOfMemoryException(message),
            Status.Timeout => new TimeoutException(message),
            _ => new InvalidOperationException($"{status}: {message}"),
        };
    }
}
