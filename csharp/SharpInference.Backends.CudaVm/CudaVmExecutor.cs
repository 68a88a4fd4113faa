// CUDA counterpart of D3D12VmExecutor (D3D12VmExecutor.cs:17-900): one
// native context (device + stream) per executor, one device buffer per VM
// slot, and every entry recorded once into a CUDA graph and replayed. Calls
// are serialised under one lock, as the D3D12 executor's are
// (D3D12VmExecutor.cs:285,307,457); concurrency comes from several executors
// in VmEngine queues, each with its own context.
//
// Source only here: built as SharpInference.Backends.CudaVm against the
// reference's SharpInference.Vm. The program walk dispatches each VmOperator
// to the native entry point of its instruction; Phi-4 sessions that want the
// fused decode step use the native si_decoder_* session instead (see
// INTEGRATION.md).
using System.Runtime.InteropServices;
using SharpInference.Instructions;
using SharpInference.Vm;
using static SharpInference.Backends.CudaVm.SharpInferCuda;

namespace SharpInference.Backends.CudaVm;

public sealed unsafe class CudaVmExecutor : IVmTaskExecutable
{
    private readonly object gate = new();
    private readonly nint context;
    private readonly nint stream;
    private readonly nint[] buffers;
    private readonly Dictionary<string, int> slotIndex;
    private readonly Dictionary<string, nint> graphs = new(StringComparer.Ordinal);
    private readonly Dictionary<string, nint> transferGraphs = new(StringComparer.Ordinal);
    private readonly List<(nint Pointer, ulong Bytes)> pinned = [];
    private bool disposed;

    public CudaVmExecutor(VmProgram program, int device = 0)
    {
        ArgumentNullException.ThrowIfNull(program);
        if (program.Target != VmTarget.Cuda)
            throw new ArgumentException($"Program '{program.Name}' targets {program.Target}, not Cuda.", nameof(program));
        if (si_abi_version() != AbiVersion) throw new NotSupportedException("libsharpinfer_cuda ABI version mismatch.");
        Program = program;
        Check(si_context_create(device, out context));
        Check(si_context_stream(context, out stream));
        buffers = new nint[program.Slots.Count];
        slotIndex = new(StringComparer.Ordinal);
        for (var i = 0; i < buffers.Length; i++)
        {
            // VmTensor.ByteLength is block-aware for the quantised element types
            Check(si_buffer_create(context, program.Slots[i].Tensor.ByteLength, out buffers[i]));
            slotIndex[program.Slots[i].Id] = i;
        }
    }

    public VmProgram Program { get; }

    public ulong SubmissionCount
    {
        get { lock (gate) { Check(si_context_submission_count(context, out var n)); return n; } }
    }

    public int SlotIndex(string slot) =>
        slotIndex.TryGetValue(slot, out var index) ? index : throw new ArgumentException($"Unknown VM slot '{slot}'.", nameof(slot));

    public void Upload(string slot, ReadOnlySpan<byte> bytes) => Upload(SlotIndex(slot), bytes);
    public void Upload(int slot, ReadOnlySpan<byte> bytes)
    {
        lock (gate)
        {
            ThrowIfDisposed();
            ValidateLength(slot, (ulong)bytes.Length);
            fixed (byte* p = bytes) Check(si_buffer_upload(context, buffers[slot], 0, p, (ulong)bytes.Length));
        }
    }

    public byte[] Readback(string slot) => Readback(SlotIndex(slot));
    public byte[] Readback(int slot)
    {
        var bytes = new byte[checked((int)Program.Slots[slot].Tensor.ByteLength)];
        Readback(slot, bytes);
        return bytes;
    }
    public void Readback(string slot, byte[] destination) => Readback(SlotIndex(slot), destination);
    public void Readback(int slot, byte[] destination)
    {
        ArgumentNullException.ThrowIfNull(destination);
        lock (gate)
        {
            ThrowIfDisposed();
            ValidateLength(slot, (ulong)destination.Length);
            fixed (byte* p = destination) Check(si_buffer_readback(context, buffers[slot], 0, p, (ulong)destination.Length));
        }
    }

    /// <summary>Replays the entry's recorded graph (recording it on first use) and waits for it.</summary>
    public void Execute(string entry)
    {
        lock (gate)
        {
            ThrowIfDisposed();
            Check(si_graph_launch(context, EntryGraph(entry)));
            Check(si_context_synchronize(context));
        }
    }

    /// <summary>
    /// One control upload, the entry and one result readback as one recorded submission and one wait
    /// (D3D12VmExecutor.cs:298-361): the copies go through pinned staging recorded into the graph.
    /// </summary>
    public void ExecuteWithTransfers(string entry, string uploadSlot, byte[] uploadBytes, string readbackSlot,
        byte[] readbackBytes)
    {
        ArgumentNullException.ThrowIfNull(uploadBytes);
        ArgumentNullException.ThrowIfNull(readbackBytes);
        lock (gate)
        {
            ThrowIfDisposed();
            int up = SlotIndex(uploadSlot), down = SlotIndex(readbackSlot);
            ValidateLength(up, (ulong)uploadBytes.Length);
            ValidateLength(down, (ulong)readbackBytes.Length);
            var key = $"{entry}\0{up}\0{down}\0{uploadBytes.Length}\0{readbackBytes.Length}";
            var (src, dst) = Staging(key, (ulong)uploadBytes.Length, (ulong)readbackBytes.Length);
            if (!transferGraphs.TryGetValue(key, out var graph))
            {
                Check(si_graph_begin(context));
                Check(si_buffer_upload_async(context, buffers[up], 0, (void*)src, (ulong)uploadBytes.Length));
                Record(entry);
                Check(si_buffer_readback_async(context, buffers[down], 0, (void*)dst, (ulong)readbackBytes.Length));
                Check(si_graph_end(context, out graph));
                transferGraphs[key] = graph;
            }
            Marshal.Copy(uploadBytes, 0, src, uploadBytes.Length);
            Check(si_graph_launch(context, graph));
            Check(si_context_synchronize(context));
            Marshal.Copy(dst, readbackBytes, 0, readbackBytes.Length);
        }
    }

    /// <summary>Mean GPU microseconds of the entry over `repetitions` back-to-back replays.</summary>
    public double MeasureGpuMicroseconds(string entry, int repetitions = 8)
    {
        if (repetitions is < 1 or > 1024) throw new ArgumentOutOfRangeException(nameof(repetitions));
        lock (gate)
        {
            ThrowIfDisposed();
            var graph = EntryGraph(entry);
            Check(si_graph_launch(context, graph));
            Check(si_context_synchronize(context));
            var start = System.Diagnostics.Stopwatch.GetTimestamp();
            for (var i = 0; i < repetitions; i++) Check(si_graph_launch(context, graph));
            Check(si_context_synchronize(context));
            var elapsed = System.Diagnostics.Stopwatch.GetElapsedTime(start);
            return elapsed.TotalMicroseconds / repetitions;
        }
    }

    /// <summary>Slot-ordered byte[][] bridge (D3D12VmExecutor.cs:514-545): upload all, execute, read back writable slots.</summary>
    public void Execute(string entryName, byte[][] slots)
    {
        ArgumentNullException.ThrowIfNull(slots);
        if (slots.Length != buffers.Length) throw new ArgumentException("Context must match Program.Slots order.", nameof(slots));
        lock (gate)
        {
            for (var i = 0; i < slots.Length; i++) Upload(i, slots[i]);
            Execute(entryName);
            for (var i = 0; i < slots.Length; i++)
                if (Program.Slots[i].Access == VmAccess.ReadWrite) Readback(i, slots[i]);
        }
    }

    public void ExecuteTask(string entryName, VmExecutionLease lease, CancellationToken cancellation)
    {
        ArgumentNullException.ThrowIfNull(lease);
        cancellation.ThrowIfCancellationRequested();
        Execute(entryName, lease.GetBuffers());
    }

    // ---- recording -----------------------------------------------------------

    private nint EntryGraph(string entry)
    {
        if (graphs.TryGetValue(entry, out var graph)) return graph;
        Check(si_graph_begin(context));
        try { Record(entry); }
        finally { Check(si_graph_end(context, out graph)); }
        graphs[entry] = graph;
        return graph;
    }

    private void Record(string entryName)
    {
        var entry = Program.Entries.SingleOrDefault(e => e.Name == entryName)
            ?? throw new ArgumentException($"Unknown VM entry '{entryName}'.", nameof(entryName));
        var binding = entry.Arguments.ToDictionary(a => a.Parameter, a => (Slot: SlotIndex(a.Source), a.ByteOffset),
            StringComparer.Ordinal);
        RecordDefinition(entry.Definition, binding);
    }

    private void RecordDefinition(string definitionId, IReadOnlyDictionary<string, (int Slot, ulong Offset)> binding)
    {
        var definition = Program.Definitions.Single(d => d.Id == definitionId);
        foreach (var node in definition.Nodes)
        {
            switch (node.Instruction)
            {
                case VmOperator op:
                    CudaVmDispatch.Launch(this, op, Resolve(op.Arguments, binding));
                    break;
                case VmCall call:
                    RecordDefinition(call.Definition, Resolve(call.Arguments, binding));
                    break;
                case VmDispatch dispatch:
                    // kernel definitions hold instruction nodes; each runs as its own native launch
                    RecordDefinition(dispatch.Definition, Resolve(dispatch.Arguments, binding));
                    break;
                case VmBarrier:
                    break; // launches on one stream are ordered already
                default:
                    throw new NotSupportedException($"VM instruction {node.Instruction.GetType().Name} is not supported on CUDA.");
            }
        }
    }

    private Dictionary<string, (int Slot, ulong Offset)> Resolve(IEnumerable<VmArgument> arguments,
        IReadOnlyDictionary<string, (int Slot, ulong Offset)> outer)
    {
        var result = new Dictionary<string, (int, ulong)>(StringComparer.Ordinal);
        foreach (var a in arguments)
        {
            if (outer.TryGetValue(a.Source, out var bound)) result[a.Parameter] = (bound.Slot, bound.Offset + a.ByteOffset);
            else result[a.Parameter] = (SlotIndex(a.Source), a.ByteOffset);
        }
        return result;
    }

    internal nint Context => context;
    internal nint Stream => stream;
    internal nint Buffer(int slot) => buffers[slot];
    internal VmTensor Tensor(int slot) => Program.Slots[slot].Tensor;

    internal nint DevicePointer(int slot, ulong offset)
    {
        Check(si_buffer_device_pointer(buffers[slot], out var p, out var bytes));
        if (offset > bytes) throw new ArgumentException($"Offset {offset} beyond slot '{Program.Slots[slot].Id}'.");
        return p + (nint)offset;
    }

    private (nint Src, nint Dst) Staging(string key, ulong up, ulong down)
    {
        Check(si_host_alloc_pinned(Math.Max(up, 1), out var src));
        Check(si_host_alloc_pinned(Math.Max(down, 1), out var dst));
        pinned.Add((src, up));
        pinned.Add((dst, down));
        return (src, dst);
    }

    private void ValidateLength(int slot, ulong bytes)
    {
        if ((uint)slot >= (uint)buffers.Length) throw new ArgumentOutOfRangeException(nameof(slot));
        if (bytes != Program.Slots[slot].Tensor.ByteLength)
            throw new ArgumentException($"Slot '{Program.Slots[slot].Id}' holds {Program.Slots[slot].Tensor.ByteLength} bytes, got {bytes}.");
    }

    private void ThrowIfDisposed() => ObjectDisposedException.ThrowIf(disposed, this);

    public void Dispose()
    {
        lock (gate)
        {
            if (disposed) return;
            disposed = true;
            foreach (var g in graphs.Values.Concat(transferGraphs.Values)) si_graph_destroy(g);
            foreach (var (p, _) in pinned) si_host_free_pinned(p);
            foreach (var b in buffers) si_buffer_destroy(context, b);
            si_context_destroy(context);
        }
    }
}
