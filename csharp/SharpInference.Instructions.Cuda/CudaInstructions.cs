// Instruction collections for target "cuda": the same collection ids,
// instruction names, port names and FP32 precision profile as the D3D12 and
// CPU collections (InstructionCollection.cs:6-24; TierZeroInstruction.cs;
// GpuTransformerInstructionCollection.cs:8-33), with the quantised weight
// signatures added ([q8_0|q4_k|q6_k, f32] -> f32). The native library's
// registry (si_instruction_resolve / si_instruction_validate) is the
// authority on what exists and which signatures bind; this provider exposes
// it through IInstructionCollectionProvider.
//
// Source only here: built as SharpInference.Instructions.Cuda against the
// reference's SharpInference.Instructions and SharpInference.Graphs.
using SharpInference.Backends.CudaVm;
using SharpInference.Graphs;

namespace SharpInference.Instructions.Cuda;

public static class CudaInstructionTarget
{
    /// <summary>Target "cuda", next to InstructionTarget.Cpu and InstructionTarget.Direct3D12.</summary>
    public static readonly InstructionTarget Cuda = new("cuda");
}

/// <summary>Counterpart of D3D12InstructionExecutionConfiguration (InstructionExecutionConfiguration.cs:36-40).</summary>
public sealed record CudaInstructionExecutionConfiguration : InstructionExecutionConfiguration
{
    public CudaInstructionExecutionConfiguration(InstructionImplementationId implementation) : base(implementation) { }
    public override InstructionTarget Target => CudaInstructionTarget.Cuda;

    /// <summary>Dense mat-vec with the reference's Neumaier lanes and merge (GpuMatVecExecution.cs:8-10).</summary>
    public static readonly CudaInstructionExecutionConfiguration CooperativeMatVec = new(new("cooperative-matvec"));
    /// <summary>Quantised mat-vec on the SIMT staged kernel instead of the tensor-core GEMV.</summary>
    public static readonly CudaInstructionExecutionConfiguration QuantStaged = new(new("cuda-gemv-staged"));
    /// <summary>The tcgen05 prefill GEMM behind core.matrix-multiply.</summary>
    public static readonly CudaInstructionExecutionConfiguration Gemm = new(new("cuda-gemm"));
}

public sealed class CudaInstructionCollectionProvider : IInstructionCollectionProvider
{
    public IReadOnlyList<InstructionCollectionDescription> QueryInstructionCollection() =>
    [
        new(InstructionCollectionIds.TierZeroFloat32, "CUDA tier-zero FP32", 0, CudaInstructionTarget.Cuda),
        new(InstructionCollectionIds.TierZeroFloat16, "CUDA tier-zero FP16", 0, CudaInstructionTarget.Cuda),
        new(InstructionCollectionIds.TransformerFloat32, "CUDA transformer FP32", 0, CudaInstructionTarget.Cuda),
    ];

    public IReadOnlyList<Instruction> QueryInstruction(Guid collectionId, string instructionName)
    {
        ArgumentException.ThrowIfNullOrWhiteSpace(instructionName);
        var status = SharpInferCuda.si_instruction_resolve(collectionId.ToString("D"), instructionName, out var id);
        if (status == SharpInferCuda.Status.Unsupported) return [];
        SharpInferCuda.Check(status);
        return [new CudaInstruction(collectionId, instructionName, id)];
    }
}

/// <summary>One native instruction. Signatures list the port types the native registry binds.</summary>
public sealed class CudaInstruction : Instruction
{
    private static readonly KernelPrecisionProfile Fp32 = new(GraphElementType.Float32, GraphElementType.Float32);

    internal CudaInstruction(Guid collectionId, string name, int nativeId)
    {
        CollectionId = collectionId;
        Name = name;
        NativeId = nativeId;
        Signatures = CreateSignatures(collectionId, name);
    }

    public override Guid CollectionId { get; }
    public override string Name { get; }
    public override InstructionTarget Target => CudaInstructionTarget.Cuda;
    public override IReadOnlyList<InstructionSignature> Signatures { get; }
    public override IReadOnlyList<InstructionIndexBound> IndexBounds =>
        Name == "core.gather-row" ? [new("index", "table", 0)] : [];
    /// <summary>Id returned by si_instruction_resolve; the executor dispatches on it.</summary>
    public int NativeId { get; }

    protected override void ValidateExecutionConfiguration(InstructionExecutionConfiguration? configuration)
    {
        if (configuration is null) return;
        if (configuration is not CudaInstructionExecutionConfiguration)
            throw new InstructionAdaptationException(CollectionId, Name, "Execution configuration has a different target.");
    }

    protected override InstructionRecording GenerateConfigured(InstructionParameter[] parameters,
        InstructionExecutionConfiguration? configuration)
    {
        var tensors = parameters.OfType<InstructionTensorParameter>().ToArray();
        unsafe
        {
            var types = stackalloc uint[tensors.Length];
            for (var i = 0; i < tensors.Length; i++) types[i] = (uint)ToNative(tensors[i].Tensor.ElementType);
            SharpInferCuda.Check(SharpInferCuda.si_instruction_validate(NativeId, types, tensors.Length,
                configuration?.Implementation.Value ?? string.Empty),
                message => new InstructionAdaptationException(CollectionId, Name, message));
        }
        // The CUDA backend launches native kernels, not generated source: the
        // recording names the native instruction and its bound ports.
        var ports = string.Join(",", tensors.Select(t => $"{t.Name}={t.Source}+{t.ByteOffset}"));
        return new InstructionRecording($"cuda:{NativeId}:{Name}:{configuration?.Implementation.Value}:{ports}");
    }

    protected override InstructionRecording Generate(InstructionParameter[] parameters) =>
        GenerateConfigured(parameters, null);

    internal static SharpInferCuda.TensorType ToNative(GraphElementType type) => type switch
    {
        GraphElementType.Float32 => SharpInferCuda.TensorType.F32,
        GraphElementType.Float16 => SharpInferCuda.TensorType.F16,
        GraphElementType.Int32 => SharpInferCuda.TensorType.I32,
        GraphElementType.Q8_0 => SharpInferCuda.TensorType.Q8_0,
        GraphElementType.Q4_K => SharpInferCuda.TensorType.Q4_K,
        GraphElementType.Q6_K => SharpInferCuda.TensorType.Q6_K,
        _ => throw new NotSupportedException($"Element type {type} has no CUDA tensor type."),
    };

    private static InstructionPort R(string name, GraphElementType type) => new(name, type, GraphResourceAccess.Read);
    private static InstructionPort W(string name, GraphElementType type) => new(name, type, GraphResourceAccess.Write);

    private static IReadOnlyList<InstructionSignature> CreateSignatures(Guid collection, string name)
    {
        const GraphElementType f32 = GraphElementType.Float32, f16 = GraphElementType.Float16,
            i32 = GraphElementType.Int32;
        GraphElementType[] quant = [GraphElementType.Q8_0, GraphElementType.Q4_K, GraphElementType.Q6_K];
        var list = new List<InstructionPort[]>();
        if (name == "core.mat-vec" && collection == InstructionCollectionIds.TierZeroFloat16)
            list.Add([R("matrix", f16), R("input", f16), W("output", f16)]);
        else if (name == "core.mat-vec")
            foreach (var weight in new[] { f32, f16 }.Concat(quant))
            {
                list.Add([R("matrix", weight), R("input", f32), W("output", f32)]);
                list.Add([R("weight", weight), R("input", f32), W("output", f32)]);
            }
        else if (name == "core.matrix-multiply")
            foreach (var right in new[] { f32, f16 }.Concat(quant))
                list.Add([R("left", f32), R("right", right), W("output", f32)]);
        else if (name == "core.gather-row")
            foreach (var table in new[] { f32, f16 }.Concat(quant))
                list.Add([R("table", table), R("index", i32), W("output", f32)]);
        else if (name == "transformer.batch-shared-matvec")
            foreach (var weight in new[] { f16 }.Concat(quant))
                list.Add([R("weight", weight), R("input", f32), R("control", i32), W("output", f32)]);
        // the transformer.* instructions keep their D3D12 port lists
        // (GpuTransformerInstructionCollection.cs); the native registry checks them
        string[] attributes = name == "core.matrix-multiply" ? ["transpose_left", "transpose_right"] : [];
        return list.Select(ports => new InstructionSignature(ports, attributes, Fp32)).ToArray();
    }
}
