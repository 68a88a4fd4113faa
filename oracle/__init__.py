"""CPU oracle (test infrastructure only): ctypes binding of oracle/liboracle.so,
a plain-C restatement of SharpInference's mat-vec numerics. Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / reference legs use it;
the shipped library never does. See oracle/oracle.h for the parity status.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

F32, F16, Q8_0, Q4_K = 0, 1, 8, 12


def build(force: bool = False) -> Path:
    src = HERE / "oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(src.stat().st_mtime,
                                                                          (HERE / "oracle.h").stat().st_mtime):
        subprocess.run(["make", "-s", "-C", str(HERE), "-B" if force else "liboracle.so"], check=True)
    return LIB_PATH


def _load() -> C.CDLL:
    build()
    lib = C.CDLL(str(LIB_PATH))
    vp, i64, u64, u32, i32 = C.c_void_p, C.c_int64, C.c_uint64, C.c_uint32, C.c_int
    sig = {
        "or_splitmix64": ([u64, u64], u64),
        "or_normal_fill": ([u64, u64, i64, C.c_float, vp], None),
        "or_f16_to_f32": ([C.c_uint16], C.c_float),
        "or_f32_to_f16": ([C.c_float], C.c_uint16),
        "or_byte_length": ([u32, u64, C.POINTER(u64)], i32),
        "or_quantize_q8_0": ([vp, i64, vp], None),
        "or_dequantize_q8_0": ([vp, i64, vp], None),
        "or_quantize_q4_k": ([vp, i64, vp], None),
        "or_dequantize_q4_k": ([vp, i64, vp], None),
        "or_dequantize_row": ([u32, vp, i64, vp], i32),
        "or_matvec": ([u32, vp, vp, vp, i64, i64, i32], i32),
        "or_matvec_f64": ([u32, vp, vp, vp, i64, i64, i32], i32),
        "or_matvec_cooperative": ([u32, u32, u32, vp, vp, vp, i64, i64, i32], i32),
        "or_batch_shared_matvec": ([u32, vp, vp, vp, vp, i64, i64, i64], i32),
        "or_matrix_multiply_tr": ([u32, vp, vp, vp, i64, i64, i64, i32], i32),
        "or_online_cores": ([], i32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise ValueError(f"oracle {what} failed with code {rc}")


def byte_length(wtype: int, elements: int) -> int:
    b = C.c_uint64()
    _check(lib.or_byte_length(wtype, elements, C.byref(b)), "byte_length")
    return b.value


def normal(seed: int, count: int, sigma: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib.or_normal_fill(seed, offset, count, sigma, _ptr(out))
    return out


def quantize(wtype: int, values: np.ndarray) -> np.ndarray:
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.empty(byte_length(wtype, values.size), dtype=np.uint8)
    if wtype == Q8_0:
        lib.or_quantize_q8_0(_ptr(values), values.size, _ptr(out))
    elif wtype == Q4_K:
        lib.or_quantize_q4_k(_ptr(values), values.size, _ptr(out))
    elif wtype == F16:
        out = np.array([lib.or_f32_to_f16(float(v)) for v in values], dtype=np.uint16).view(np.uint8)
    else:
        out = values.view(np.uint8).copy()
    return out


def dequantize(wtype: int, blob: np.ndarray, count: int) -> np.ndarray:
    blob = np.ascontiguousarray(blob).view(np.uint8)
    out = np.empty(count, dtype=np.float32)
    _check(lib.or_dequantize_row(wtype, _ptr(blob), count, _ptr(out)), "dequantize")
    return out


def matvec(wtype: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    y = np.empty(rows, dtype=np.float32)
    _check(lib.or_matvec(wtype, _ptr(w), _ptr(x), _ptr(y), rows, cols, threads), "matvec")
    return y


def matvec_f64(wtype: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    y = np.empty(rows, dtype=np.float64)
    _check(lib.or_matvec_f64(wtype, _ptr(w), _ptr(x), _ptr(y), rows, cols, threads), "matvec_f64")
    return y


def matvec_cooperative(wtype: int, xtype: int, ytype: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int,
                       lanes: int = 64) -> np.ndarray:
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x)
    y = np.empty(rows, dtype=np.float16 if ytype == F16 else np.float32)
    _check(lib.or_matvec_cooperative(wtype, xtype, ytype, _ptr(w), _ptr(x), _ptr(y), rows, cols, lanes),
           "matvec_cooperative")
    return y


def batch_shared_matvec(wtype: int, w: np.ndarray, inp: np.ndarray, control, out: np.ndarray, batch: int,
                        out_features: int, in_features: int) -> np.ndarray:
    w = np.ascontiguousarray(w)
    inp = np.ascontiguousarray(inp, dtype=np.float32)
    ctl = np.ascontiguousarray(control, dtype=np.int32)
    out = np.ascontiguousarray(out, dtype=np.float32).copy()
    _check(lib.or_batch_shared_matvec(wtype, _ptr(w), _ptr(inp), _ptr(ctl), _ptr(out), batch, out_features,
                                      in_features), "batch_shared_matvec")
    return out


def matrix_multiply_tr(wtype: int, x: np.ndarray, w: np.ndarray, m: int, n: int, k: int,
                       threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    y = np.empty(m * n, dtype=np.float32)
    _check(lib.or_matrix_multiply_tr(wtype, _ptr(x), _ptr(w), _ptr(y), m, n, k, threads), "matrix_multiply_tr")
    return y


def online_cores() -> int:
    return lib.or_online_cores()
