"""Phi-4 text decoder shapes and seeded random-init weights for the CUDA
decoder session (native.Decoder, the counterpart of Phi4D3D12TextSession).

The dimensions follow Phi4D3D12TextSession.cs:14-25 (Phi-4-mini); the 14B
shape is the Phi-4 (14B) text model. Weights are synthetic: every linear
slot is N(0, sigma) quantised to the configured GGUF type with its own seed
(slot ordinal i of native.decoder_slot_names -> seed * 1_000_003 + i), norm
weights are ones. Weights are generated and uploaded one slot at a time so
host memory stays at one slot.
"""
from __future__ import annotations

import re

import numpy as np

from . import native

# Phi4D3D12TextSession.cs:14-25; epsilon / rope metadata of the Phi-4-mini GGUF
# (phi3.attention.layer_norm_rms_epsilon, phi3.rope.freq_base,
# phi3.rope.scaling.attn_factor = sqrt(1 + ln(32) / ln(4096))).
PHI4_MINI = dict(layers=32, hidden=3072, query_heads=24, kv_heads=8, head_size=128, rotary_size=96,
                 intermediate=8192, vocab=200064, context=4096, epsilon=1e-5, rope_base=10000.0,
                 rope_scale=1.1902381, weight_type=native.Q4_K, embedding_type=native.Q4_K)
PHI4_14B = dict(layers=40, hidden=5120, query_heads=40, kv_heads=10, head_size=128, rotary_size=128,
                intermediate=17920, vocab=100352, context=4096, epsilon=1e-5, rope_base=250000.0, rope_scale=1.0,
                weight_type=native.Q8_0, embedding_type=native.Q8_0)
TINY = dict(layers=2, hidden=256, query_heads=2, kv_heads=1, head_size=128, rotary_size=96, intermediate=512,
            vocab=640, context=128, epsilon=1e-5, rope_base=10000.0, rope_scale=1.1902381, weight_type=native.Q4_K,
            embedding_type=native.Q4_K)


def linear_shapes(cfg: dict) -> dict[str, tuple[int, int]]:
    """(rows, cols) of every quantised slot (Phi4D3D12TextSession.cs:391-410)."""
    h, f = cfg["hidden"], cfg["intermediate"]
    kv = cfg["kv_heads"] * cfg["head_size"]
    shapes = {"token_embedding": (cfg["vocab"], h)}
    for layer in range(cfg["layers"]):
        shapes[f"qkv_weight_{layer}"] = (h + 2 * kv, h)
        shapes[f"attn_output_weight_{layer}"] = (h, h)
        shapes[f"ffn_up_weight_{layer}"] = (2 * f, h)
        shapes[f"ffn_down_weight_{layer}"] = (h, f)
    return shapes


def weight_bytes(cfg: dict) -> int:
    """Bytes of weights one decode step reads: every linear slot once (the
    tied token_embedding as the vocabulary projection) plus the norms."""
    total = 0
    for name, (rows, cols) in linear_shapes(cfg).items():
        wt = cfg["embedding_type"] if name == "token_embedding" else cfg["weight_type"]
        total += rows * native.row_bytes(wt, cols)
    return total + (2 * cfg["layers"] + 1) * cfg["hidden"] * 4


def synthetic_weights(cfg: dict, seed: int, sigma: float = 0.02, threads: int = 0):
    """Yields (slot name, bytes) for every linear slot, one at a time."""
    shapes = linear_shapes(cfg)
    for i, name in enumerate(native.decoder_slot_names(cfg["layers"])):
        if name not in shapes:
            continue
        rows, cols = shapes[name]
        wt = cfg["embedding_type"] if name == "token_embedding" else cfg["weight_type"]
        yield name, native.synth_weights(wt, seed * 1_000_003 + i, rows, cols, sigma, threads)


def load_synthetic(decoder: "native.Decoder", cfg: dict, seed: int, sigma: float = 0.02, threads: int = 0) -> None:
    for name, blob in synthetic_weights(cfg, seed, sigma, threads):
        decoder.upload(name, blob)


def random_prompt(seed: int, tokens: int, vocab: int) -> np.ndarray:
    """Uniform random token ids (splitmix64 of the index, modulo vocab)."""
    idx = np.arange(tokens, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = idx * np.uint64(0x9E3779B97F4A7C15) + np.uint64(seed * 0x632BE59BD9B4E019 & 0xFFFFFFFFFFFFFFFF)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return (z % np.uint64(vocab)).astype(np.int32)


# ---- GGUF files: the session's weights by the reference's tensor names ------------
# Phi4D3D12TextSession.cs:391-410: slot <- GGUF tensor.
def gguf_tensor_name(slot: str) -> str:
    if slot == "token_embedding":
        return "token_embd.weight"
    if slot == "output_norm":
        return "output_norm.weight"
    name, layer = slot.rsplit("_", 1)
    return {"attn_norm": f"blk.{layer}.attn_norm.weight", "ffn_norm": f"blk.{layer}.ffn_norm.weight",
            "qkv_weight": f"blk.{layer}.attn_qkv.weight", "attn_output_weight": f"blk.{layer}.attn_output.weight",
            "ffn_up_weight": f"blk.{layer}.ffn_up.weight", "ffn_down_weight": f"blk.{layer}.ffn_down.weight"}[name]


def config_from_gguf(f: "native.GgufFile", context: int = 4096) -> dict:
    """The decoder configuration of a phi3-architecture GGUF file: the
    metadata the reference session reads (phi3.rope.freq_base,
    phi3.attention.layer_norm_rms_epsilon, phi3.rope.scaling.attn_factor),
    the shape keys, and the weight types of the tensors themselves."""
    m = f.metadata
    emb = f.tensors["token_embd.weight"]
    heads = int(m.get("phi3.attention.head_count", PHI4_MINI["query_heads"]))
    hidden = int(m.get("phi3.embedding_length", emb.dims[0]))
    cfg = dict(layers=int(m.get("phi3.block_count", PHI4_MINI["layers"])), hidden=hidden, query_heads=heads,
               kv_heads=int(m.get("phi3.attention.head_count_kv", heads)), head_size=hidden // heads,
               rotary_size=int(m.get("phi3.rope.dimension_count", hidden // heads)),
               intermediate=int(m.get("phi3.feed_forward_length", PHI4_MINI["intermediate"])), vocab=int(emb.dims[1]),
               context=context, epsilon=float(m["phi3.attention.layer_norm_rms_epsilon"]),
               rope_base=float(m["phi3.rope.freq_base"]),
               rope_scale=float(m.get("phi3.rope.scaling.attn_factor", 1.0)),
               weight_type=f.tensors["blk.0.attn_qkv.weight"].type, embedding_type=emb.type)
    return cfg


def slot_types_from_gguf(f: "native.GgufFile", layers: int) -> list[int]:
    """The GGUF type of every session slot's tensor (decoder_slot_names
    order), for si_decoder_create_typed: mixed-type files such as Q4_K_M keep
    some projections and the embedding in Q6_K."""
    return [f.tensors[gguf_tensor_name(slot)].type for slot in native.decoder_slot_names(layers)]


def open_session_gguf(f: "native.GgufFile", context: int = 4096, device: int = 0) -> "native.Decoder":
    """A decoder session for a phi3 GGUF file: per-slot types when the file
    mixes weight types, every tensor uploaded unchanged."""
    cfg = config_from_gguf(f, context)
    types = slot_types_from_gguf(f, cfg["layers"])
    names = native.decoder_slot_names(cfg["layers"])
    mixed = any(t != cfg["weight_type"] for t, slot in zip(types, names) if "_weight_" in slot)
    dec = native.Decoder(cfg, device, slot_types=types if mixed else None)
    load_gguf(dec, f)
    return dec


def load_gguf(decoder: "native.Decoder", f: "native.GgufFile") -> None:
    """Uploads every slot's GGUF tensor unchanged (Phi4D3D12TextSession.cs:56-57)."""
    for slot in native.decoder_slot_names(decoder.cfg.layers):
        t = f.tensors[gguf_tensor_name(slot)]
        size = decoder.slot(slot)[1]
        if t.nbytes != size:
            raise native.InvalidDataError(f"GGUF tensor '{t.name}' has {t.nbytes} bytes, slot '{slot}' {size}")
        decoder.upload(slot, t.data)


def save_gguf(path, cfg: dict, weights: dict) -> None:
    """Writes a model (the session's slots -> arrays) as a phi3 GGUF file."""
    from . import gguf
    h, f_ = cfg["hidden"], cfg["intermediate"]
    shapes = linear_shapes(cfg)
    meta = {"general.architecture": "phi3", "general.alignment": (gguf.U32, 32),
            "phi3.block_count": (gguf.U32, cfg["layers"]), "phi3.embedding_length": (gguf.U32, h),
            "phi3.feed_forward_length": (gguf.U32, f_), "phi3.attention.head_count": (gguf.U32, cfg["query_heads"]),
            "phi3.attention.head_count_kv": (gguf.U32, cfg["kv_heads"]),
            "phi3.rope.dimension_count": (gguf.U32, cfg["rotary_size"]),
            "phi3.attention.layer_norm_rms_epsilon": (gguf.F32, cfg["epsilon"]),
            "phi3.rope.freq_base": (gguf.F32, cfg["rope_base"]),
            "phi3.rope.scaling.attn_factor": (gguf.F32, cfg["rope_scale"])}
    tensors = []
    for slot in native.decoder_slot_names(cfg["layers"]):
        if slot in shapes:
            rows, cols = shapes[slot]
            t = cfg["embedding_type"] if slot == "token_embedding" else cfg["weight_type"]
            tensors.append((gguf_tensor_name(slot), t, [cols, rows], weights[slot]))
        else:
            tensors.append((gguf_tensor_name(slot), 0, [h], np.asarray(weights[slot], dtype=np.float32)))
    gguf.write(path, meta, tensors)


def _col_slice(blob: np.ndarray, wtype: int, rows: int, cols: int, c0: int, c1: int) -> np.ndarray:
    """Columns [c0, c1) of a [rows, cols] matrix in GGUF bytes (c0, c1 on block boundaries)."""
    rb = native.row_bytes(wtype, cols)
    b0 = native.row_bytes(wtype, c0) if c0 else 0
    b1 = native.row_bytes(wtype, c1)
    return np.ascontiguousarray(np.asarray(blob).view(np.uint8).reshape(rows, rb)[:, b0:b1]).reshape(-1)


def _row_slice(blob: np.ndarray, wtype: int, cols: int, ranges) -> np.ndarray:
    rb = native.row_bytes(wtype, cols)
    m = np.asarray(blob).view(np.uint8).reshape(-1, rb)
    return np.ascontiguousarray(np.concatenate([m[a:b] for a, b in ranges])).reshape(-1)


def tp_slot_layout(cfg: dict, part, name: str):
    """How one rank's slot of a tensor-parallel session (si_tp_partition_plan)
    is cut from the whole tensor: ("rows", [(r0, r1), ...]) for the qkv rows
    of the rank's heads (query, then key, then value rows) and its gate / up
    rows of the intermediate; ("cols", c0, c1) for the out projection's
    columns of its query heads and down's columns of its intermediate slice;
    ("whole",) for token_embedding (gather-row reads every row; the
    vocabulary projection uses the rank's rows of it in place) and the norms."""
    base = re.sub(r"_\d+$", "", name)  # slot name without its layer index
    h, f, hs = cfg["hidden"], cfg["intermediate"], cfg["head_size"]
    kv = cfg["kv_heads"] * hs
    q0, q1 = part.query_head_begin * hs, (part.query_head_begin + part.query_heads) * hs
    k0, k1 = part.kv_head_begin * hs, (part.kv_head_begin + part.kv_heads) * hs
    f0, f1 = part.ffn_begin, part.ffn_begin + part.ffn_rows
    if base == "qkv_weight":
        return ("rows", [(q0, q1), (h + k0, h + k1), (h + kv + k0, h + kv + k1)])
    if base == "ffn_up_weight":
        return ("rows", [(f0, f1), (f + f0, f + f1)])
    if base == "attn_output_weight":
        return ("cols", q0, q1)
    if base == "ffn_down_weight":
        return ("cols", f0, f1)
    return ("whole",)


def tp_slice_weights(cfg: dict, weights: dict, part) -> dict:
    """One rank's slots of a tensor-parallel session (si_tp_partition_plan),
    cut from the whole model's GGUF bytes as tp_slot_layout says."""
    shapes = linear_shapes(cfg)
    wt = cfg["weight_type"]
    out = {}
    for name, arr in weights.items():
        lay = tp_slot_layout(cfg, part, name)
        if lay[0] == "rows":
            out[name] = _row_slice(arr, wt, shapes[name][1], lay[1])
        elif lay[0] == "cols":
            rows, cols = shapes[name]
            out[name] = _col_slice(arr, wt, rows, cols, lay[1], lay[2])
        else:
            out[name] = arr
    return out

