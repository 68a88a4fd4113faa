"""ctypes binding of libsharpinfer_cuda (the C ABI in include/sharpinfer_cuda.h).

Status codes become the exception types the reference raises for the same
condition (SharpInference.Instructions/InstructionCollection.cs:152-156 for
InstructionAdaptationException; ArgumentException / NotSupportedException /
InvalidDataException elsewhere). The library is required: importing this
module without the built shared object raises, there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libsharpinfer_cuda.so"

# GGUF tensor type ids (GgufModelFile.cs:24-46)
F32, F16, Q8_0, Q4_K, Q6_K, I32 = 0, 1, 8, 12, 14, 26
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", I32: "I32"}

MATVEC_DEFAULT, MATVEC_COOPERATIVE, MATVEC_QUANT_STAGED = 0, 1, 2

(SI_OK, SI_ERR_INVALID_ARGUMENT, SI_ERR_UNSUPPORTED, SI_ERR_ADAPTATION, SI_ERR_INVALID_DATA, SI_ERR_CUDA,
 SI_ERR_OUT_OF_MEMORY, SI_ERR_NCCL, SI_ERR_TIMEOUT, SI_ERR_NO_DEVICE) = range(10)


class SiError(RuntimeError):
    status = -1


class ArgumentError(SiError, ValueError):          # ArgumentException
    status = SI_ERR_INVALID_ARGUMENT


class NotSupportedError(SiError):                  # NotSupportedException
    status = SI_ERR_UNSUPPORTED


class InstructionAdaptationError(SiError):         # InstructionAdaptationException
    status = SI_ERR_ADAPTATION


class InvalidDataError(SiError):                   # InvalidDataException
    status = SI_ERR_INVALID_DATA


class CudaError(SiError):
    status = SI_ERR_CUDA


class OutOfMemoryError(SiError, MemoryError):
    status = SI_ERR_OUT_OF_MEMORY


class NcclError(SiError):
    status = SI_ERR_NCCL


class DeviceTimeoutError(SiError, TimeoutError):
    status = SI_ERR_TIMEOUT


class NoDeviceError(SiError):
    status = SI_ERR_NO_DEVICE


_ERRORS = {c.status: c for c in (ArgumentError, NotSupportedError, InstructionAdaptationError, InvalidDataError,
                                 CudaError, OutOfMemoryError, NcclError, DeviceTimeoutError, NoDeviceError)}

_vp, _u64, _i64, _u32, _i32 = C.c_void_p, C.c_uint64, C.c_int64, C.c_uint32, C.c_int
_pu64, _pu32 = C.POINTER(C.c_uint64), C.POINTER(C.c_uint32)

# name -> argtypes (restype is si_status unless listed in _RESTYPE)
SIGNATURES = {
    "si_abi_version": [],
    "si_last_error": [C.c_char_p, C.c_size_t],
    "si_device_count": [C.POINTER(C.c_int)],
    "si_tensor_byte_length": [_u32, _pu64, _i32, _pu64],
    "si_row_bytes": [_u32, _i64, _pu64],
    "si_quantize": [_u32, _vp, _i64, _vp],
    "si_dequantize": [_u32, _vp, _i64, _vp],
    "si_synth_normal": [_u64, _u64, _i64, C.c_float, _vp, _i32],
    "si_synth_weights": [_u32, _u64, _i64, _i64, C.c_float, _vp, _i32],
    "si_synth_weight_rows": [_u32, _u64, _i64, _i64, _i64, C.c_float, _vp, _i32],
    "si_synth_weight_rows_device": [_u32, _u64, _i64, _i64, _i64, C.c_float, _vp, _vp],
    "si_synth_weight_block_device": [_u32, _u64, _i64, _i64, _i64, _i64, _i64, C.c_float, _vp, _vp],
    "si_matvec": [_u32, _vp, _u32, _vp, _u32, _vp, _i64, _i64, _u32, _vp],
    "si_batch_shared_matvec": [_u32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "si_gemv_default_plan": [_u32, _i64, _i64, _vp],
    "si_matvec_quant_planned": [_u32, _vp, _vp, _vp, _i64, _i64, _vp, _vp],
    "si_matrix_multiply_workspace_bytes": [_u32, _i64, _i64, _i64, _pu64],
    "si_matrix_multiply": [_u32, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _u64, _vp],
    "si_matrix_multiply_static_workspace": [_u32, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "si_device_error_take": [_i32, _pu32],
    "si_context_create": [_i32, C.POINTER(_vp)],
    "si_context_destroy": [_vp],
    "si_context_stream": [_vp, C.POINTER(_vp)],
    "si_context_synchronize": [_vp],
    "si_context_submission_count": [_vp, _pu64],
    "si_buffer_create": [_vp, _u64, C.POINTER(_vp)],
    "si_buffer_destroy": [_vp, _vp],
    "si_buffer_device_pointer": [_vp, C.POINTER(_vp), _pu64],
    "si_buffer_upload": [_vp, _vp, _u64, _vp, _u64],
    "si_buffer_readback": [_vp, _vp, _u64, _vp, _u64],
    "si_buffer_upload_async": [_vp, _vp, _u64, _vp, _u64],
    "si_buffer_readback_async": [_vp, _vp, _u64, _vp, _u64],
    "si_host_alloc_pinned": [_u64, C.POINTER(_vp)],
    "si_host_free_pinned": [_vp],
    "si_ctx_matvec": [_vp, _u32, _vp, _u64, _u32, _vp, _u64, _u32, _vp, _u64, _i64, _i64, _u32],
    "si_ctx_batch_shared_matvec": [_vp, _u32, _vp, _u64, _vp, _u64, _vp, _u64, _vp, _u64, _i64, _i64, _i64],
    "si_ctx_matrix_multiply": [_vp, _u32, _vp, _u64, _vp, _u64, _vp, _u64, _i64, _i64, _i64],
    "si_rowshard_plan": [_i64, _i32, _i32, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)],
    "si_comm_unique_id": [_vp, C.c_size_t],
    "si_comm_create": [_i32, _i32, _i32, _vp, _i32, C.POINTER(_vp)],
    "si_comm_destroy": [_vp],
    "si_rowshard_matvec_allgather": [_vp, _u32, _vp, _vp, _vp, _i64, _i64, _vp],
    "si_ipc_export": [_vp, _vp, C.c_size_t],
    "si_ipc_open": [_i32, _vp, C.POINTER(_vp)],
    "si_ipc_close": [_i32, _vp],
    "si_peer_group_create": [_i32, _i32, _i32, C.POINTER(C.c_uint64), C.c_uint64, C.POINTER(_vp)],
    "si_peer_group_destroy": [_vp],
    "si_rowshard_matvec_peer": [_vp, _u32, _vp, _vp, C.c_uint64, _i64, _i64, _vp],
    "si_graph_begin": [_vp],
    "si_graph_end": [_vp, C.POINTER(_vp)],
    "si_graph_launch": [_vp, _vp],
    "si_graph_destroy": [_vp],
    "si_instruction_resolve": [C.c_char_p, C.c_char_p, C.POINTER(C.c_int)],
    "si_instruction_validate": [_i32, _pu32, _i32, C.c_char_p],
    # transformer instructions (device pointers, stream last)
    "si_gather_row": [_u32, _vp, _i64, _i64, _vp, _vp, _vp],
    "si_rms_norm": [_vp, _vp, _vp, _i64, C.c_float, _vp],
    "si_residual_rms_norm": [_vp, _vp, _vp, _vp, _vp, _i64, C.c_float, _vp],
    "si_swiglu": [_vp, _vp, _i64, _vp],
    "si_scaled_add": [_vp, _vp, _vp, _i64, C.c_float, _vp],
    "si_rope_kv_write": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, C.c_float, _vp],
    "si_grouped_query_attention": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64, _vp],
    "si_rope_grouped_query_attention": [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i64, C.c_float, _vp],
    "si_gqa_scores": [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64, _vp],
    "si_causal_softmax": [_vp, _vp, _vp, _i32, _i64, _vp],
    "si_gqa_values": [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64, _vp],
    "si_argmax": [_vp, _i64, _vp, _vp],
    "si_embedding_gather_batch": [_vp, _i64, _vp, _vp, _i64, _i64, _vp],
    "si_copy_embedding_rows": [_vp, _vp, _i64, _i64, _i64, _i64, _vp],
    "si_batch_rms_norm": [_vp, _vp, _vp, _vp, _i64, _i64, C.c_float, _vp],
    "si_batch_residual_rms_norm": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, C.c_float, _vp],
    "si_batch_swiglu": [_vp, _vp, _vp, _i64, _i64, _vp],
    "si_batch_rope_kv_write": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i64, C.c_float, _vp],
    "si_batch_gqa_scores": [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _vp],
    "si_batch_causal_softmax": [_vp, _vp, _vp, _i64, _i32, _i64, _vp],
    "si_batch_gqa_values": [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _vp],
    "si_batch_grouped_query_attention": [_vp, _vp, _vp, _i32, _i32, _vp, _i32, _i32, _i32, _i64, _vp],
    "si_batch_select_last": [_vp, _vp, _vp, _i64, _i64, _vp],
    "si_batch_gather_rows": [_vp, _i64, _vp, _vp, _i64, _i64, _vp],
    # decoder session
    "si_decoder_create": [_i32, _vp, C.POINTER(_vp)],
    "si_decoder_create_typed": [_i32, _vp, _vp, _i32, C.POINTER(_vp)],
    "si_decoder_arena_bytes": [_vp, _pu64],
    "si_decoder_create_streams": [_i32, _vp, _i32, C.POINTER(_vp)],
    "si_decoder_step_streams": [_vp, _vp, _vp, _vp],
    "si_decoder_generate_streams": [_vp, _vp, _vp, _i32, _vp],
    "si_decoder_prefill_stream": [_vp, _i32, _vp, _i32, _i32, _vp],
    "si_decoder_create_sharded": [_i32, _vp, _vp, _u64, C.POINTER(_vp)],
    "si_tp_partition_plan": [_vp, _i32, _i32, _vp],
    "si_decoder_tp_arena_bytes": [_vp, _i32, _pu64],
    "si_decoder_create_tensor_parallel": [_i32, _vp, _vp, C.POINTER(_vp)],
    "si_decoder_destroy": [_vp],
    "si_decoder_slot": [_vp, C.c_char_p, C.POINTER(_vp), _pu64],
    "si_decoder_upload": [_vp, C.c_char_p, _u64, _vp, _u64],
    "si_decoder_read": [_vp, C.c_char_p, _u64, _vp, _u64],
    "si_decoder_stream": [_vp, C.POINTER(_vp)],
    "si_decoder_forward_token": [_vp, C.c_int32, C.POINTER(C.c_int32)],
    "si_decoder_generate": [_vp, _vp, C.c_int32, C.c_int32, _vp],
    "si_decoder_prefill": [_vp, _vp, C.c_int32, _vp],
    "si_decoder_prefill_embeddings": [_vp, _vp, C.c_int32, _vp],
    "si_decoder_reset": [_vp],
    "si_decoder_position": [_vp, C.POINTER(C.c_int32)],
    # GGUF files
    "si_gguf_open": [C.c_char_p, C.POINTER(_vp)],
    "si_gguf_close": [_vp],
    "si_gguf_tensor_count": [_vp, C.POINTER(_i64)],
    "si_gguf_find_tensor": [_vp, C.c_char_p, C.POINTER(_i64)],
    "si_gguf_tensor_info": [_vp, _i64, C.c_char_p, C.c_size_t, _pu32, C.POINTER(C.c_int32), _pu64, _pu64,
                            C.POINTER(_vp)],
    "si_gguf_metadata_count": [_vp, C.POINTER(_i64)],
    "si_gguf_metadata_key": [_vp, _i64, C.c_char_p, C.c_size_t, _pu32, _pu32, _pu64],
    "si_gguf_metadata_number": [_vp, C.c_char_p, C.POINTER(C.c_double)],
    "si_gguf_metadata_string": [_vp, C.c_char_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)],
    "si_gguf_metadata_array": [_vp, C.c_char_p, _pu32, _pu64, C.POINTER(_vp)],
}
_RESTYPE = {"si_abi_version": C.c_int}


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m sharpinference_b200.build` "
                          "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, C.c_int)
    return lib


lib = _load()


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    lib.si_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != SI_OK:
        raise _ERRORS.get(status, SiError)(last_error() or f"status {status}")


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args))


def device_count() -> int:
    n = C.c_int(0)
    call("si_device_count", C.byref(n))
    return n.value


def row_bytes(wtype: int, cols: int) -> int:
    b = C.c_uint64()
    call("si_row_bytes", wtype, cols, C.byref(b))
    return b.value


def tensor_byte_length(wtype: int, dims) -> int:
    arr = (C.c_uint64 * len(dims))(*dims)
    b = C.c_uint64()
    call("si_tensor_byte_length", wtype, arr, len(dims), C.byref(b))
    return b.value


def rowshard_plan(rows: int, nranks: int, rank: int) -> tuple[int, int, int]:
    """(row_begin, row_count, rows_per_rank) of `rank` for a row-sharded weight."""
    b, c, p = C.c_int64(), C.c_int64(), C.c_int64()
    call("si_rowshard_plan", rows, nranks, rank, C.byref(b), C.byref(c), C.byref(p))
    return b.value, c.value, p.value


def comm_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    call("si_comm_unique_id", buf, 128)
    return bytes(buf)


class Comm:
    """NCCL communicator for row-sharded mat-vec (one rank per GPU)."""

    def __init__(self, device: int, nranks: int, rank: int, uid: bytes, timeout_ms: int = 60000):
        arr = (C.c_uint8 * 128).from_buffer_copy(uid)
        h = C.c_void_p()
        call("si_comm_create", device, nranks, rank, arr, timeout_ms, C.byref(h))
        self.handle, self.nranks, self.rank = h, nranks, rank

    def rowshard_matvec_allgather(self, wtype, weight_shard_ptr, x_ptr, y_full_ptr, rows, cols, stream):
        call("si_rowshard_matvec_allgather", self.handle, wtype, weight_shard_ptr, x_ptr, y_full_ptr, rows, cols,
             C.c_void_p(stream))

    def close(self):
        if self.handle:
            call("si_comm_destroy", self.handle)
            self.handle = None


def ipc_export(device_ptr: int) -> bytes:
    """64-byte CUDA IPC handle of a device allocation (e.g. Buffer.device_pointer)."""
    buf = (C.c_uint8 * 64)()
    call("si_ipc_export", C.c_void_p(device_ptr), buf, 64)
    return bytes(buf)


def ipc_open(device: int, handle: bytes) -> int:
    arr = (C.c_uint8 * 64).from_buffer_copy(handle)
    p = C.c_void_p()
    call("si_ipc_open", device, arr, C.byref(p))
    return p.value


def ipc_close(device: int, ptr: int) -> None:
    call("si_ipc_close", device, C.c_void_p(ptr))


class PeerGroup:
    """Row-sharded GEMV whose kernel writes every rank's output arena over
    NVLink (si_rowshard_matvec_peer). arena_addrs[q] is rank q's arena as
    mapped in this process."""

    def __init__(self, device: int, nranks: int, rank: int, arena_addrs, arena_bytes: int):
        addrs = (C.c_uint64 * nranks)(*arena_addrs)
        h = C.c_void_p()
        call("si_peer_group_create", device, nranks, rank, addrs, arena_bytes, C.byref(h))
        self.handle, self.nranks, self.rank = h, nranks, rank

    def rowshard_matvec(self, wtype, weight_shard_ptr, x_ptr, output_offset, rows, cols, stream):
        call("si_rowshard_matvec_peer", self.handle, wtype, C.c_void_p(weight_shard_ptr), C.c_void_p(x_ptr),
             output_offset, rows, cols, C.c_void_p(stream))

    def close(self):
        if self.handle:
            call("si_peer_group_destroy", self.handle)
            self.handle = None


def device_error_take(device: int = 0) -> int:
    v = C.c_uint32()
    call("si_device_error_take", device, C.byref(v))
    return v.value


# ---- numpy helpers (host codecs) -------------------------------------------------
def _np():
    import numpy as np
    return np


def synth_normal(seed: int, count: int, sigma: float = 1.0, offset: int = 0, threads: int = 0):
    np = _np()
    out = np.empty(count, dtype=np.float32)
    call("si_synth_normal", seed, offset, count, sigma, out.ctypes.data, threads)
    return out


def synth_weights(wtype: int, seed: int, rows: int, cols: int, sigma: float = 0.02, threads: int = 0):
    np = _np()
    out = np.empty(row_bytes(wtype, cols) * rows, dtype=np.uint8)
    call("si_synth_weights", wtype, seed, rows, cols, sigma, out.ctypes.data, threads)
    return out


def synth_weight_rows(wtype: int, seed: int, row_begin: int, rows: int, cols: int, sigma: float = 0.02,
                      threads: int = 0):
    np = _np()
    out = np.empty(row_bytes(wtype, cols) * rows, dtype=np.uint8)
    call("si_synth_weight_rows", wtype, seed, row_begin, rows, cols, sigma, out.ctypes.data, threads)
    return out


def synth_weight_rows_device(wtype: int, seed: int, row_begin: int, rows: int, cols: int, sigma: float, dst: int,
                             stream=None) -> None:
    """si_synth_weight_rows_device: the seeded rows generated in device memory."""
    call("si_synth_weight_rows_device", wtype, seed, row_begin, rows, cols, sigma, dst, stream)


def synth_weight_block_device(wtype: int, seed: int, row_begin: int, rows: int, col_begin: int, col_count: int,
                              cols: int, sigma: float, dst: int, stream) -> None:
    call("si_synth_weight_block_device", wtype, seed, row_begin, rows, col_begin, col_count, cols, sigma, dst, stream)


def quantize(wtype: int, values):
    np = _np()
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.empty(tensor_byte_length(wtype, [values.size]), dtype=np.uint8)
    call("si_quantize", wtype, values.ctypes.data, values.size, out.ctypes.data)
    return out


def dequantize(wtype: int, blob, count: int):
    np = _np()
    blob = np.ascontiguousarray(blob).view(np.uint8)
    out = np.empty(count, dtype=np.float32)
    call("si_dequantize", wtype, blob.ctypes.data, count, out.ctypes.data)
    return out


# ---- executor ----------------------------------------------------------------------
class GemvPlan(C.Structure):
    """si_gemv_plan: launch shape of the tensor-core Q8_0 / Q4_K GEMV."""
    _fields_ = [(n, C.c_int32) for n in ("cluster", "rows_per_tile", "smem_kb", "mma_path", "warps_per_column",
                                         "superblocks_per_warp", "ctas_per_sm", "max_groups")]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


def gemv_default_plan(wtype: int, rows: int, cols: int) -> GemvPlan:
    plan = GemvPlan()
    call("si_gemv_default_plan", wtype, rows, cols, C.byref(plan))
    return plan


def gemv_plan(**fields) -> GemvPlan:
    """A plan with the default's fields for a K = 3072 matrix, overridden by `fields`."""
    base = {"cluster": 1, "rows_per_tile": 32, "smem_kb": 226, "mma_path": 1, "warps_per_column": 1,
            "superblocks_per_warp": 0, "ctas_per_sm": 1, "max_groups": 0}
    base.update(fields)
    return GemvPlan(**base)


class Buffer:
    """A device slot owned by a Context (D3D12VmResourcePool-style ownership)."""

    def __init__(self, ctx: "Context", nbytes: int):
        self.ctx = ctx
        self.nbytes = nbytes
        h = C.c_void_p()
        call("si_buffer_create", ctx.handle, nbytes, C.byref(h))
        self.handle = h
        p, n = C.c_void_p(), C.c_uint64()
        call("si_buffer_device_pointer", h, C.byref(p), C.byref(n))
        self.device_pointer = p.value

    def upload(self, data, offset: int = 0) -> None:
        np = _np()
        arr = np.ascontiguousarray(data)
        call("si_buffer_upload", self.ctx.handle, self.handle, offset, arr.ctypes.data, arr.nbytes)

    def readback(self, nbytes: int | None = None, offset: int = 0):
        np = _np()
        n = self.nbytes - offset if nbytes is None else nbytes
        out = np.empty(n, dtype=np.uint8)
        call("si_buffer_readback", self.ctx.handle, self.handle, offset, out.ctypes.data, n)
        return out

    def free(self) -> None:
        if self.handle:
            call("si_buffer_destroy", self.ctx.handle, self.handle)
            self.handle = None


class Graph:
    """A recorded submission replayed with one launch."""

    def __init__(self, ctx: "Context", handle):
        self.ctx, self.handle = ctx, handle

    def launch(self) -> None:
        call("si_graph_launch", self.ctx.handle, self.handle)

    def close(self) -> None:
        if self.handle:
            call("si_graph_destroy", self.handle)
            self.handle = None


class Context:
    """Executor context: one device, one stream, serialised calls
    (the native counterpart of D3D12VmExecutor)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        call("si_context_create", device, C.byref(h))
        self.handle = h
        self.device = device
        s = C.c_void_p()
        call("si_context_stream", h, C.byref(s))
        self.stream = s.value

    def buffer(self, nbytes: int) -> Buffer:
        return Buffer(self, nbytes)

    def synchronize(self) -> None:
        call("si_context_synchronize", self.handle)

    def record(self, fn) -> "Graph":
        """Captures everything `fn` issues on the context stream into a graph."""
        call("si_graph_begin", self.handle)
        try:
            fn()
        finally:
            h = C.c_void_p()
            st = lib.si_graph_end(self.handle, C.byref(h))
        check(st)
        return Graph(self, h)

    @property
    def submission_count(self) -> int:
        v = C.c_uint64()
        call("si_context_submission_count", self.handle, C.byref(v))
        return v.value

    def matvec(self, wtype, weight: Buffer, input: Buffer, output: Buffer, rows, cols, *, weight_offset=0,
               input_offset=0, output_offset=0, input_type=F32, output_type=F32, config=MATVEC_DEFAULT):
        call("si_ctx_matvec", self.handle, wtype, weight.handle, weight_offset, input_type, input.handle,
             input_offset, output_type, output.handle, output_offset, rows, cols, config)

    def matvec_planned(self, wtype, weight: Buffer, input: Buffer, output: Buffer, rows, cols, plan: "GemvPlan"):
        """core.mat-vec on Q8_0 / Q4_K weights with an explicit launch shape, on this context's stream."""
        call("si_matvec_quant_planned", wtype, weight.device_pointer, input.device_pointer, output.device_pointer,
             rows, cols, C.byref(plan), self.stream)

    def batch_shared_matvec(self, wtype, weight: Buffer, input: Buffer, control: Buffer, output: Buffer, batch,
                            out_features, in_features, *, weight_offset=0, input_offset=0, control_offset=0,
                            output_offset=0):
        call("si_ctx_batch_shared_matvec", self.handle, wtype, weight.handle, weight_offset, input.handle,
             input_offset, control.handle, control_offset, output.handle, output_offset, batch, out_features,
             in_features)

    def matrix_multiply(self, wtype, x: Buffer, weight: Buffer, y: Buffer, m, n, k, *, x_offset=0,
                        weight_offset=0, y_offset=0):
        call("si_ctx_matrix_multiply", self.handle, wtype, x.handle, x_offset, weight.handle, weight_offset,
             y.handle, y_offset, m, n, k)

    def close(self) -> None:
        if self.handle:
            call("si_context_destroy", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---- instruction registry ----------------------------------------------------------
TIER_ZERO_FLOAT32 = "00000000-0000-0000-0000-000000000000"
TIER_ZERO_FLOAT16 = "00000000-0000-0000-0000-000000000001"
TRANSFORMER_FLOAT32 = "824d0f9c-16c7-46d8-b49d-0f91d6a4ec83"


def resolve(collection_id: str, name: str) -> int:
    v = C.c_int()
    call("si_instruction_resolve", collection_id.encode(), name.encode(), C.byref(v))
    return v.value


def validate(instruction_id: int, port_types, configuration: str = "") -> None:
    arr = (C.c_uint32 * len(port_types))(*port_types)
    call("si_instruction_validate", instruction_id, arr, len(port_types), configuration.encode())


def header_functions(header: Path | None = None) -> list[str]:
    """Function names declared in include/sharpinfer_cuda.h."""
    import re
    header = header or _HERE.parent / "include" / "sharpinfer_cuda.h"
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(si_[a-z0-9_]+)\s*\(", text)))



# ---- Phi-4 decoder session -----------------------------------------------------------
class DecoderConfig(C.Structure):
    """si_decoder_config."""
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("query_heads", C.c_int32), ("kv_heads", C.c_int32),
                ("head_size", C.c_int32), ("rotary_size", C.c_int32), ("intermediate", C.c_int32),
                ("vocab", C.c_int32), ("context", C.c_int64), ("epsilon", C.c_float), ("rope_base", C.c_float),
                ("rope_scale", C.c_float), ("weight_type", C.c_uint32), ("embedding_type", C.c_uint32)]


def decoder_slot_names(layers: int) -> list[str]:
    """Weight slots of the decode program (Phi4D3D12TextSession.cs:391-410)."""
    names = ["token_embedding", "output_norm"]
    for layer in range(layers):
        names += [f"attn_norm_{layer}", f"ffn_norm_{layer}", f"qkv_weight_{layer}", f"attn_output_weight_{layer}",
                  f"ffn_up_weight_{layer}", f"ffn_down_weight_{layer}"]
    return names


class TpPartition(C.Structure):
    """si_tp_partition: one rank's slices of a tensor-parallel session."""
    _fields_ = [("kv_head_begin", C.c_int32), ("kv_heads", C.c_int32), ("query_head_begin", C.c_int32),
                ("query_heads", C.c_int32), ("ffn_begin", C.c_int64), ("ffn_rows", C.c_int64),
                ("vocab_begin", C.c_int64), ("vocab_rows", C.c_int64)]


def tp_partition(cfg: dict, nranks: int, rank: int) -> TpPartition:
    part = TpPartition()
    call("si_tp_partition_plan", C.byref(DecoderConfig(**cfg)), nranks, rank, C.byref(part))
    return part


def tp_arena_bytes(cfg: dict, nranks: int) -> int:
    v = C.c_uint64()
    call("si_decoder_tp_arena_bytes", C.byref(DecoderConfig(**cfg)), nranks, C.byref(v))
    return v.value


def decoder_arena_bytes(cfg: dict) -> int:
    """Arena bytes a row-sharded session needs (si_decoder_arena_bytes)."""
    c, v = DecoderConfig(**cfg), C.c_uint64()
    call("si_decoder_arena_bytes", C.byref(c), C.byref(v))
    return v.value


class Decoder:
    """Phi4D3D12TextSession on CUDA: ForwardToken, Reset, Position, plus a
    device-resident greedy loop (generate). With a PeerGroup, the row-sharded
    session of that rank (si_decoder_create_sharded)."""

    def __init__(self, cfg: dict, device: int = 0, group: "PeerGroup | None" = None, streams: int = 1,
                 shard_min_bytes: int = 0, slot_types: "list[int] | None" = None, tensor_parallel: bool = False):
        self.cfg = DecoderConfig(**cfg)
        self.streams = streams
        h = C.c_void_p()
        if tensor_parallel:  # si_decoder_create_tensor_parallel on the group's rank
            call("si_decoder_create_tensor_parallel", device, C.byref(self.cfg), group.handle, C.byref(h))
        elif slot_types is not None:  # one GGUF type per slot (decoder_slot_names order)
            t = (C.c_uint32 * len(slot_types))(*slot_types)
            call("si_decoder_create_typed", device, C.byref(self.cfg), t, len(slot_types), C.byref(h))
        elif group is not None:
            call("si_decoder_create_sharded", device, C.byref(self.cfg), group.handle, shard_min_bytes, C.byref(h))
        elif streams != 1:
            call("si_decoder_create_streams", device, C.byref(self.cfg), streams, C.byref(h))
        else:
            call("si_decoder_create", device, C.byref(self.cfg), C.byref(h))
        self.handle = h
        s = C.c_void_p()
        call("si_decoder_stream", h, C.byref(s))
        self.stream = s.value

    def slot(self, name: str) -> tuple[int, int]:
        p, n = C.c_void_p(), C.c_uint64()
        call("si_decoder_slot", self.handle, name.encode(), C.byref(p), C.byref(n))
        return p.value, n.value

    def upload(self, name: str, data, offset: int = 0) -> None:
        np = _np()
        arr = np.ascontiguousarray(data)
        call("si_decoder_upload", self.handle, name.encode(), offset, arr.ctypes.data, arr.nbytes)

    def read(self, name: str, dtype=None, count: int | None = None, offset: int = 0):
        np = _np()
        dtype = np.dtype(dtype or np.float32)
        if count is None:
            count = (self.slot(name)[1] - offset) // dtype.itemsize
        out = np.empty(count, dtype=dtype)
        call("si_decoder_read", self.handle, name.encode(), offset, out.ctypes.data, out.nbytes)
        return out

    def forward_token(self, token: int) -> int:
        v = C.c_int32()
        call("si_decoder_forward_token", self.handle, token, C.byref(v))
        return v.value

    def generate(self, prompt, steps: int):
        np = _np()
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(p.size + steps, dtype=np.int32)
        call("si_decoder_generate", self.handle, p.ctypes.data, p.size, steps, out.ctypes.data)
        return out

    def prefill(self, prompt) -> int:
        """Batched prompt prefill; returns the prediction after the last token."""
        np = _np()
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        v = C.c_int32()
        call("si_decoder_prefill", self.handle, p.ctypes.data, p.size, C.byref(v))
        return v.value

    def prefill_embeddings(self, rows) -> int:
        """Prefill from ready FP32 embedding rows [n, hidden]."""
        np = _np()
        r = np.ascontiguousarray(rows, dtype=np.float32)
        if r.ndim != 2 or r.shape[1] != self.cfg.hidden:
            raise ArgumentError(f"embedding rows must be [n, {self.cfg.hidden}], got {r.shape}")
        v = C.c_int32()
        call("si_decoder_prefill_embeddings", self.handle, r.ctypes.data, r.shape[0], C.byref(v))
        return v.value

    def _stream_args(self, tokens, positions):
        np = _np()
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        if t.size != self.streams or p.size != self.streams:
            raise ArgumentError(f"need {self.streams} tokens and positions")
        return t, p

    def step_streams(self, tokens, positions):
        """One step of every stream; returns each stream's argmax."""
        np = _np()
        t, p = self._stream_args(tokens, positions)
        out = np.empty(self.streams, dtype=np.int32)
        call("si_decoder_step_streams", self.handle, t.ctypes.data, p.ctypes.data, out.ctypes.data)
        return out

    def generate_streams(self, tokens, positions, steps: int):
        """`steps` greedy steps of every stream: [steps, streams] argmax ids."""
        np = _np()
        t, p = self._stream_args(tokens, positions)
        out = np.empty((max(steps, 0), self.streams), dtype=np.int32)
        call("si_decoder_generate_streams", self.handle, t.ctypes.data, p.ctypes.data, steps, out.ctypes.data)
        return out

    def prefill_stream(self, stream: int, prompt, start: int = 0) -> int:
        """Batched prefill of one stream's prompt from position `start`."""
        np = _np()
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        v = C.c_int32()
        call("si_decoder_prefill_stream", self.handle, stream, pr.ctypes.data, pr.size, start, C.byref(v))
        return v.value

    def reset(self) -> None:
        call("si_decoder_reset", self.handle)

    @property
    def position(self) -> int:
        v = C.c_int32()
        call("si_decoder_position", self.handle, C.byref(v))
        return v.value

    def close(self) -> None:
        if self.handle:
            call("si_decoder_destroy", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---- GGUF model files ----------------------------------------------------------------
GGUF_SCALARS = {0: "u1", 1: "i1", 2: "<u2", 3: "<i2", 4: "<u4", 5: "<i4", 6: "<f4", 7: "u1", 10: "<u8", 11: "<i8",
                12: "<f8"}


class GgufTensor:
    def __init__(self, name, type_, dims, nbytes, address, owner):
        self.name, self.type, self.dims, self.nbytes, self._address, self._owner = name, type_, dims, nbytes, address, owner

    @property
    def data(self):
        """The tensor's bytes in the mapping (read-only view, no copy)."""
        np = _np()
        buf = (C.c_uint8 * self.nbytes).from_address(self._address)
        arr = np.frombuffer(buf, dtype=np.uint8)
        arr.flags.writeable = False
        return arr


class GgufFile:
    """GgufModelFile: metadata and tensors of a GGUF v3 file (si_gguf_*)."""

    def __init__(self, path):
        h = C.c_void_p()
        call("si_gguf_open", str(path).encode(), C.byref(h))
        self.handle = h
        n = C.c_int64()
        call("si_gguf_tensor_count", h, C.byref(n))
        self.tensors = {}
        name = C.create_string_buffer(4096)
        t, rank, nbytes, data = C.c_uint32(), C.c_int32(), C.c_uint64(), C.c_void_p()
        dims = (C.c_uint64 * 8)()
        for i in range(n.value):
            call("si_gguf_tensor_info", h, i, name, 4096, C.byref(t), C.byref(rank), dims, C.byref(nbytes),
                 C.byref(data))
            nm = name.value.decode()
            self.tensors[nm] = GgufTensor(nm, t.value, [dims[d] for d in range(rank.value)], nbytes.value,
                                          data.value, self)
        call("si_gguf_metadata_count", h, C.byref(n))
        self.metadata = {}
        et, cnt = C.c_uint32(), C.c_uint64()
        for i in range(n.value):
            call("si_gguf_metadata_key", h, i, name, 4096, C.byref(t), C.byref(et), C.byref(cnt))
            key = name.value.decode()
            self.metadata[key] = self._value(key, t.value, et.value, cnt.value)

    def _value(self, key, type_, elem, count):
        np = _np()
        k = key.encode()
        if type_ == 8:
            n = C.c_size_t()
            call("si_gguf_metadata_string", self.handle, k, None, 0, C.byref(n))
            buf = C.create_string_buffer(n.value + 1)
            call("si_gguf_metadata_string", self.handle, k, buf, n.value + 1, None)
            return buf.raw[:n.value].decode("utf-8")
        if type_ == 9:
            if elem not in GGUF_SCALARS:
                return ("array", elem, count)
            p = C.c_void_p()
            call("si_gguf_metadata_array", self.handle, k, None, None, C.byref(p))
            dt = np.dtype(GGUF_SCALARS[elem])
            arr = np.frombuffer((C.c_uint8 * (count * dt.itemsize)).from_address(p.value), dtype=dt).copy()
            return arr.astype(bool) if elem == 7 else arr
        v = C.c_double()
        call("si_gguf_metadata_number", self.handle, k, C.byref(v))
        if type_ == 7:
            return bool(v.value)
        return v.value if type_ in (6, 12) else int(v.value)

    def close(self):
        if self.handle:
            call("si_gguf_close", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
