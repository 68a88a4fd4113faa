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

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14


def build(force: bool = False) -> Path:
    newest = max((HERE / n).stat().st_mtime for n in ("oracle.c", "transformer.c", "oracle.h", "Makefile"))
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest:
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
        "or_quantize_q6_k": ([vp, i64, vp], None),
        "or_dequantize_q6_k": ([vp, i64, vp], None),
        "or_dequantize_row": ([u32, vp, i64, vp], i32),
        "or_matvec": ([u32, vp, vp, vp, i64, i64, i32], i32),
        "or_matvec_f64": ([u32, vp, vp, vp, i64, i64, i32], i32),
        "or_matvec_cooperative": ([u32, u32, u32, vp, vp, vp, i64, i64, i32], i32),
        "or_batch_shared_matvec": ([u32, vp, vp, vp, vp, i64, i64, i64], i32),
        "or_matrix_multiply_tr": ([u32, vp, vp, vp, i64, i64, i64, i32], i32),
        "or_online_cores": ([], i32),
        # transformer instructions (transformer.c)
        "or_rms_norm": ([vp, vp, vp, i64, C.c_float], None),
        "or_residual_rms_norm": ([vp, vp, vp, vp, vp, i64, C.c_float], None),
        "or_swiglu": ([vp, vp, i64], None),
        "or_scaled_add": ([vp, vp, vp, i64, C.c_float], None),
        "or_gather_row": ([u32, vp, i64, i64, C.c_int32, vp], i32),
        "or_rope_kv_write": ([vp, C.c_int32, vp, vp, vp, vp, i64, i64, i32, i32, i64, C.c_float], None),
        "or_grouped_query_attention": ([vp, vp, vp, C.c_int32, vp, i32, i32, i32, i64], None),
        "or_gqa_scores": ([vp, vp, C.c_int32, vp, i32, i32, i32, i64], None),
        "or_causal_softmax": ([vp, C.c_int32, vp, i32, i64], None),
        "or_gqa_values": ([vp, vp, C.c_int32, vp, i32, i32, i32, i64], None),
        "or_argmax": ([vp, i64], C.c_int32),
        "or_batch_rms_norm": ([vp, vp, vp, vp, i64, i64, C.c_float], None),
        "or_batch_residual_rms_norm": ([vp, vp, vp, vp, vp, vp, i64, i64, C.c_float], None),
        "or_batch_swiglu": ([vp, vp, vp, i64, i64], None),
        "or_batch_rope_kv_write": ([vp, vp, vp, vp, vp, vp, i64, i64, i64, i32, i32, i64, C.c_float], None),
        "or_batch_gqa_scores": ([vp, vp, vp, vp, i64, i32, i32, i32, i64], None),
        "or_batch_causal_softmax": ([vp, vp, vp, i64, i32, i64], None),
        "or_batch_gqa_values": ([vp, vp, vp, vp, i64, i32, i32, i32, i64], None),
        "or_batch_select_last": ([vp, vp, vp, i64, i64], None),
        "or_batch_gather_rows": ([vp, i64, vp, vp, i64, i64], None),
        "or_embedding_gather_batch": ([vp, i64, vp, vp, i64, i64], None),
        "or_copy_embedding_rows": ([vp, vp, i64, i64, i64], None),
        "or_rope_frequencies": ([C.c_float, i32, vp], None),
        "or_decoder_step": ([vp, vp, vp, vp, vp, C.c_int32, C.c_int32, vp, C.POINTER(C.c_int32), i32], i32),
        "or_decoder_step_typed": ([vp, vp, vp, vp, vp, vp, C.c_int32, C.c_int32, vp, C.POINTER(C.c_int32), i32], i32),
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


_PAR_MIN = 1 << 22  # elements: below this one call, above it chunks over host threads


def _chunks(count: int, align: int):
    """[begin, end) ranges covering count elements in multiples of align, one per host thread."""
    threads = max(1, int(lib.or_online_cores()))
    step = max(align, -(-count // threads) // align * align)
    return [(b, min(count, b + step)) for b in range(0, count, step)]


def _parallel(fn, ranges) -> None:
    # ctypes releases the GIL inside the C calls, so the chunks run in parallel
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(len(ranges)) as ex:
        list(ex.map(lambda r: fn(*r), ranges))


def normal(seed: int, count: int, sigma: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    if count < _PAR_MIN:
        lib.or_normal_fill(seed, offset, count, sigma, _ptr(out))
    else:  # element i depends on (seed, offset + i) only: chunks give the same values
        _parallel(lambda b, e: lib.or_normal_fill(seed, offset + b, e - b, sigma, _ptr(out) + 4 * b),
                  _chunks(count, 2))
    return out


def quantize(wtype: int, values: np.ndarray) -> np.ndarray:
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.empty(byte_length(wtype, values.size), dtype=np.uint8)
    if wtype in (Q8_0, Q4_K, Q6_K):
        fn, per, nb = {Q8_0: (lib.or_quantize_q8_0, 32, 34), Q4_K: (lib.or_quantize_q4_k, 256, 144),
                       Q6_K: (lib.or_quantize_q6_k, 256, 210)}[wtype]
        if values.size < _PAR_MIN or values.size % per:
            fn(_ptr(values), values.size, _ptr(out))
        else:  # blocks are independent
            _parallel(lambda b, e: fn(_ptr(values) + 4 * b, e - b, _ptr(out) + b // per * nb),
                      _chunks(values.size, per))
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


# ---- transformer instructions (transformer.c) ---------------------------------------
def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def rms_norm(x, weight, eps: float) -> np.ndarray:
    x, weight = _f32(x), _f32(weight)
    out = np.empty_like(x)
    lib.or_rms_norm(_ptr(x), _ptr(weight), _ptr(out), x.size, eps)
    return out


def residual_rms_norm(hidden, residual, weight, eps: float):
    hidden, residual, weight = _f32(hidden), _f32(residual), _f32(weight)
    updated, out = np.empty_like(hidden), np.empty_like(hidden)
    lib.or_residual_rms_norm(_ptr(hidden), _ptr(residual), _ptr(weight), _ptr(updated), _ptr(out), hidden.size, eps)
    return updated, out


def swiglu(gate_up) -> np.ndarray:
    gate_up = _f32(gate_up)
    out = np.empty(gate_up.size // 2, dtype=np.float32)
    lib.or_swiglu(_ptr(gate_up), _ptr(out), out.size)
    return out


def scaled_add(x, update, scale: float) -> np.ndarray:
    x, update = _f32(x), _f32(update)
    out = np.empty_like(x)
    lib.or_scaled_add(_ptr(x), _ptr(update), _ptr(out), x.size, scale)
    return out


def gather_row(ttype: int, table, rows: int, cols: int, index: int) -> np.ndarray:
    table = np.ascontiguousarray(table)
    out = np.empty(cols, dtype=np.float32)
    _check(lib.or_gather_row(ttype, _ptr(table), rows, cols, index, _ptr(out)), "gather_row")
    return out


def rope_kv_write(qkv, position: int, freq, key_cache, value_cache, query_size: int, kv_heads: int, head_size: int,
                  rotary_size: int, context: int, rope_scale: float):
    """Returns (query, key_cache, value_cache); the caches are updated copies."""
    qkv, freq = _f32(qkv), _f32(freq)
    kc, vc = _f32(key_cache).copy(), _f32(value_cache).copy()
    query = np.zeros(query_size, dtype=np.float32)
    lib.or_rope_kv_write(_ptr(qkv), position, _ptr(freq), _ptr(query), _ptr(kc), _ptr(vc), query_size,
                         kv_heads * head_size, head_size, rotary_size, context, rope_scale)
    return query, kc, vc


def grouped_query_attention(query, key_cache, value_cache, position: int, query_heads: int, kv_heads: int,
                            head_size: int, context: int) -> np.ndarray:
    query, kc, vc = _f32(query), _f32(key_cache), _f32(value_cache)
    out = np.empty(query_heads * head_size, dtype=np.float32)
    lib.or_grouped_query_attention(_ptr(query), _ptr(kc), _ptr(vc), position, _ptr(out), query_heads, kv_heads,
                                   head_size, context)
    return out


def gqa_scores(query, key_cache, position: int, query_heads: int, kv_heads: int, head_size: int, context: int):
    query, kc = _f32(query), _f32(key_cache)
    out = np.empty(query_heads * context, dtype=np.float32)
    lib.or_gqa_scores(_ptr(query), _ptr(kc), position, _ptr(out), query_heads, kv_heads, head_size, context)
    return out


def causal_softmax(scores, position: int, heads: int, context: int):
    scores = _f32(scores)
    out = np.empty_like(scores)
    lib.or_causal_softmax(_ptr(scores), position, _ptr(out), heads, context)
    return out


def gqa_values(probs, value_cache, position: int, query_heads: int, kv_heads: int, head_size: int, context: int):
    probs, vc = _f32(probs), _f32(value_cache)
    out = np.empty(query_heads * head_size, dtype=np.float32)
    lib.or_gqa_values(_ptr(probs), _ptr(vc), position, _ptr(out), query_heads, kv_heads, head_size, context)
    return out


def argmax(x) -> int:
    x = _f32(x)
    return int(lib.or_argmax(_ptr(x), x.size))


def batch_rms_norm(x, weight, control, out, eps: float):
    x, weight, ctl, out = _f32(x), _f32(weight), _i32(control), _f32(out).copy()
    batch, width = x.shape
    lib.or_batch_rms_norm(_ptr(x), _ptr(weight), _ptr(ctl), _ptr(out), batch, width, eps)
    return out


def batch_residual_rms_norm(hidden, residual, weight, control, updated, out, eps: float):
    hidden, residual, weight, ctl = _f32(hidden), _f32(residual), _f32(weight), _i32(control)
    updated, out = _f32(updated).copy(), _f32(out).copy()
    batch, width = hidden.shape
    lib.or_batch_residual_rms_norm(_ptr(hidden), _ptr(residual), _ptr(weight), _ptr(ctl), _ptr(updated), _ptr(out),
                                   batch, width, eps)
    return updated, out


def batch_swiglu(gate_up, control, out):
    gate_up, ctl, out = _f32(gate_up), _i32(control), _f32(out).copy()
    batch, width = out.shape
    lib.or_batch_swiglu(_ptr(gate_up), _ptr(ctl), _ptr(out), batch, width)
    return out


def batch_rope_kv_write(qkv, control, freq, query, key_cache, value_cache, query_size: int, kv_heads: int,
                        head_size: int, rotary_size: int, context: int, rope_scale: float):
    qkv, ctl, freq = _f32(qkv), _i32(control), _f32(freq)
    query, kc, vc = _f32(query).copy(), _f32(key_cache).copy(), _f32(value_cache).copy()
    batch = qkv.shape[0]
    lib.or_batch_rope_kv_write(_ptr(qkv), _ptr(ctl), _ptr(freq), _ptr(query), _ptr(kc), _ptr(vc), batch, query_size,
                               kv_heads * head_size, head_size, rotary_size, context, rope_scale)
    return query, kc, vc


def batch_gqa_scores(query, key_cache, control, scores, query_heads: int, kv_heads: int, head_size: int,
                     context: int):
    query, kc, ctl, scores = _f32(query), _f32(key_cache), _i32(control), _f32(scores).copy()
    batch = query.shape[0]
    lib.or_batch_gqa_scores(_ptr(query), _ptr(kc), _ptr(ctl), _ptr(scores), batch, query_heads, kv_heads, head_size,
                            context)
    return scores


def batch_causal_softmax(scores, control, probs, heads: int, context: int):
    scores, ctl, probs = _f32(scores), _i32(control), _f32(probs).copy()
    batch = scores.shape[0]
    lib.or_batch_causal_softmax(_ptr(scores), _ptr(ctl), _ptr(probs), batch, heads, context)
    return probs


def batch_gqa_values(probs, value_cache, control, out, query_heads: int, kv_heads: int, head_size: int,
                     context: int):
    probs, vc, ctl, out = _f32(probs), _f32(value_cache), _i32(control), _f32(out).copy()
    batch = probs.shape[0]
    lib.or_batch_gqa_values(_ptr(probs), _ptr(vc), _ptr(ctl), _ptr(out), batch, query_heads, kv_heads, head_size,
                            context)
    return out


def batch_select_last(x, control, out):
    x, ctl, out = _f32(x), _i32(control), _f32(out).copy()
    batch, width = x.shape
    lib.or_batch_select_last(_ptr(x), _ptr(ctl), _ptr(out), batch, width)
    return out


def batch_gather_rows(table, control, out):
    table, ctl, out = _f32(table), _i32(control), _f32(out).copy()
    rows, width = table.shape
    lib.or_batch_gather_rows(_ptr(table), rows, _ptr(ctl), _ptr(out), out.shape[0], width)
    return out


def embedding_gather_batch(table_f16, rows: int, indices, width: int) -> np.ndarray:
    table = np.ascontiguousarray(table_f16).view(np.uint16)
    idx = _i32(indices)
    out = np.empty(idx.size * width, dtype=np.float32)
    lib.or_embedding_gather_batch(_ptr(table), rows, _ptr(idx), _ptr(out), idx.size, width)
    return out


def copy_embedding_rows(x, out, rows: int, width: int, output_start: int):
    x, out = _f32(x), _f32(out).copy()
    lib.or_copy_embedding_rows(_ptr(x), _ptr(out), rows, width, output_start)
    return out


def rope_frequencies(base: float, rotary_size: int) -> np.ndarray:
    out = np.empty(rotary_size // 2, dtype=np.float32)
    lib.or_rope_frequencies(base, rotary_size, _ptr(out))
    return out


class DecoderConfig(C.Structure):
    """or_decoder_config (oracle.h); the same fields as si_decoder_config."""
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("query_heads", C.c_int32), ("kv_heads", C.c_int32),
                ("head_size", C.c_int32), ("rotary_size", C.c_int32), ("intermediate", C.c_int32),
                ("vocab", C.c_int32), ("context", C.c_int64), ("epsilon", C.c_float), ("rope_base", C.c_float),
                ("rope_scale", C.c_float), ("weight_type", C.c_uint32), ("embedding_type", C.c_uint32)]


class Decoder:
    """The Phi-4 decode program on the CPU (or_decoder_step). `weights` maps
    the reference's slot names to numpy arrays (raw GGUF bytes or FP32)."""

    def __init__(self, cfg: dict, weights: dict, threads: int = 0, slot_types=None):
        self.cfg = DecoderConfig(**cfg)
        self._types = None if slot_types is None else (C.c_uint32 * len(slot_types))(*slot_types)
        c = self.cfg
        names = ["token_embedding", "output_norm"]
        for layer in range(c.layers):
            names += [f"attn_norm_{layer}", f"ffn_norm_{layer}", f"qkv_weight_{layer}",
                      f"attn_output_weight_{layer}", f"ffn_up_weight_{layer}", f"ffn_down_weight_{layer}"]
        self._keep = [np.ascontiguousarray(weights[n]) for n in names]
        self._ptrs = (C.c_void_p * len(names))(*[a.ctypes.data for a in self._keep])
        self.freq = rope_frequencies(c.rope_base, c.rotary_size)
        kv = c.layers * c.context * c.kv_heads * c.head_size
        self.key_cache = np.zeros(kv, dtype=np.float32)
        self.value_cache = np.zeros(kv, dtype=np.float32)
        self.logits = np.zeros(c.vocab, dtype=np.float32)
        self.position = 0
        self.threads = threads

    def forward_token(self, token: int) -> int:
        nxt = C.c_int32()
        _check(lib.or_decoder_step_typed(C.byref(self.cfg), self._ptrs, self._types, _ptr(self.freq),
                                         _ptr(self.key_cache), _ptr(self.value_cache), token, self.position,
                                         _ptr(self.logits), C.byref(nxt), self.threads), "decoder_step")
        self.position += 1
        return int(nxt.value)

    def generate(self, prompt, steps: int) -> list[int]:
        out, tok = [], None
        for i in range(len(prompt) + steps):
            tok = self.forward_token(int(prompt[i]) if i < len(prompt) else tok)
            out.append(tok)
        return out
