// VmOperator -> native launch, one case per instruction the CUDA collections
// provide. Ports are bound by name exactly as the reference's instructions
// name them (TierZeroOperationContracts.cs; GpuTransformerInstructionCollection.cs;
// GpuBatchTransformerInstructions.cs), shapes come from the bound slots'
// VmTensor dimensions and scalar attributes from VmOperator.Attributes.
using System.Globalization;
using SharpInference.Instructions;
using SharpInference.Vm;
using static SharpInference.Backends.CudaVm.SharpInferCuda;

namespace SharpInference.Backends.CudaVm;

internal static class CudaVmDispatch
{
    public static void Launch(CudaVmExecutor exe, VmOperator op, IReadOnlyDictionary<string, (int Slot, ulong Offset)> ports)
    {
        (int Slot, ulong Offset) Port(string name) => ports.TryGetValue(name, out var p) ? p
            : throw new InvalidDataException($"{op.InstructionName}: port '{name}' is not bound.");
        nint Ptr(string name) { var p = Port(name); return exe.DevicePointer(p.Slot, p.Offset); }
        VmTensor T(string name) => exe.Tensor(Port(name).Slot);
        float F(string name) => float.Parse(op.Attributes[name], CultureInfo.InvariantCulture);
        int I(string name) => int.Parse(op.Attributes[name], CultureInfo.InvariantCulture);
        uint Type(VmTensor t) => (uint)ToNative(t.ElementType);
        var s = exe.Stream;

        switch (op.InstructionName)
        {
            case "core.mat-vec":
            {
                var w = ports.ContainsKey("weight") ? "weight" : "matrix";
                var (ws, wo) = Port(w);
                var (xs, xo) = Port("input");
                var (ys, yo) = Port("output");
                var cfg = op.ExecutionConfiguration?.Implementation.Value switch
                {
                    null => 0u, "cooperative-matvec" => 1u, "cuda-gemv-staged" => 2u,
                    var other => throw new InstructionAdaptationException(op.InstructionCollectionId, op.InstructionName,
                        $"Unsupported CUDA execution configuration '{other}'."),
                };
                var wt = T(w);
                Check(si_ctx_matvec(exe.Context, Type(wt), exe.Buffer(ws), wo, Type(T("input")), exe.Buffer(xs), xo,
                    Type(T("output")), exe.Buffer(ys), yo, wt.Dimensions[0], wt.Dimensions[1], cfg));
                break;
            }
            case "core.matrix-multiply":
            {
                if (op.Attributes.GetValueOrDefault("transpose_left") == "true" || op.Attributes.GetValueOrDefault("transpose_right") != "true")
                    throw new NotSupportedException("core.matrix-multiply on CUDA: transpose_left=false, transpose_right=true.");
                var (xs, xo) = Port("left");
                var (ws, wo) = Port("right");
                var (ys, yo) = Port("output");
                var x = T("left");
                var w = T("right");
                Check(si_ctx_matrix_multiply(exe.Context, Type(w), exe.Buffer(xs), xo, exe.Buffer(ws), wo, exe.Buffer(ys), yo,
                    x.Dimensions[0], w.Dimensions[0], w.Dimensions[1]));
                break;
            }
            case "transformer.batch-shared-matvec":
            {
                var (ws, wo) = Port("weight");
                var (xs, xo) = Port("input");
                var (cs, co) = Port("control");
                var (ys, yo) = Port("output");
                var w = T("weight");
                Check(si_ctx_batch_shared_matvec(exe.Context, Type(w), exe.Buffer(ws), wo, exe.Buffer(xs), xo, exe.Buffer(cs), co,
                    exe.Buffer(ys), yo, T("input").Dimensions[0], w.Dimensions[0], w.Dimensions[1]));
                break;
            }
            case "core.gather-row":
            {
                var table = T("table");
                Check(si_gather_row(Type(table), Ptr("table"), table.Dimensions[0], table.Dimensions[1], Ptr("index"),
                    Ptr("output"), s));
                break;
            }
            case "transformer.rms-norm":
                Check(si_rms_norm(Ptr("input"), Ptr("weight"), Ptr("output"), (long)T("input").ElementCount, F("epsilon"), s));
                break;
            case "transformer.residual-rms-norm":
                Check(si_residual_rms_norm(Ptr("hidden"), Ptr("residual"), Ptr("weight"), Ptr("updated"), Ptr("output"),
                    (long)T("hidden").ElementCount, F("epsilon"), s));
                break;
            case "transformer.swiglu":
                Check(si_swiglu(Ptr("gate_up"), Ptr("output"), (long)T("output").ElementCount, s));
                break;
            case "transformer.scaled-add":
                Check(si_scaled_add(Ptr("input"), Ptr("update"), Ptr("output"), (long)T("output").ElementCount, F("scale"), s));
                break;
            case "transformer.rope-kv-write":
            {
                var kc = T("key_cache"); // [context, kv_heads, head_size]
                Check(si_rope_kv_write(Ptr("qkv"), Ptr("position"), Ptr("frequencies"), Ptr("query"), Ptr("key_cache"),
                    Ptr("value_cache"), (long)T("query").ElementCount, kc.Dimensions[1], I("head_size"), I("rotary_size"),
                    kc.Dimensions[0], F("rope_scale"), s));
                break;
            }
            case "transformer.grouped-query-attention":
            {
                var q = T("query");     // [query_heads, head_size]
                var kc = T("key_cache"); // [context, kv_heads, head_size]
                Check(si_grouped_query_attention(Ptr("query"), Ptr("key_cache"), Ptr("value_cache"), Ptr("position"),
                    Ptr("output"), q.Dimensions[0], kc.Dimensions[1], q.Dimensions[1], kc.Dimensions[0], s));
                break;
            }
            case "transformer.argmax":
                Check(si_argmax(Ptr("input"), (long)T("input").ElementCount, Ptr("output"), s));
                break;
            default:
                throw new NotSupportedException($"No CUDA dispatch for '{op.InstructionCollectionId:D}/{op.InstructionName}'.");
        }
    }

    private static TensorType ToNative(VmElementType type) => type switch
    {
        VmElementType.Float32 => TensorType.F32,
        VmElementType.Float16 => TensorType.F16,
        VmElementType.Int32 => TensorType.I32,
        VmElementType.Q8_0 => TensorType.Q8_0,
        VmElementType.Q4_K => TensorType.Q4_K,
        VmElementType.Q6_K => TensorType.Q6_K,
        _ => throw new NotSupportedException($"VM element type {type} has no CUDA tensor type."),
    };
}
