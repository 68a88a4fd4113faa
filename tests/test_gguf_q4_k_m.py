"""A Q4_K_M-layout model file written by an independent GGUF writer
(gguf-py 0.19.0's GGUFWriter, llama.cpp's Python package) read by the
library's GGUF reader (si_gguf_*) and decoded by a session whose slots take
each tensor's own type byte-for-byte (Phi4D3D12TextSession.cs:56-57 uploads
GgufModelTensor.Bytes). Q4_K_M files keep most projections in Q4_K and the
embedding plus some ffn_down tensors in Q6_K; the reference's reader sizes
neither (GgufModelFile.cs:314-320 throws for the K-quants)."""
import numpy as np
import pytest

import oracle
from sharpinference_b200 import native, phi4

gguf = pytest.importorskip("gguf")
QT = gguf.GGMLQuantizationType

CFG = dict(layers=2, hidden=256, query_heads=2, kv_heads=1, head_size=128, rotary_size=96, intermediate=512,
           vocab=640, context=64, epsilon=1e-5, rope_base=10000.0, rope_scale=1.1902381, weight_type=native.Q4_K,
           embedding_type=native.Q6_K)
# per slot (decoder_slot_names order): Q6_K embedding, Q4_K attention and ffn_up,
# ffn_down Q6_K in layer 0 and Q4_K in layer 1, F32 norms
TYPES = {"token_embedding": native.Q6_K, "ffn_down_weight_0": native.Q6_K}


def _model(seed=41):
    names = native.decoder_slot_names(CFG["layers"])
    shapes = phi4.linear_shapes(CFG)
    types, weights = [], {}
    for i, name in enumerate(names):
        if name in shapes:
            rows, cols = shapes[name]
            t = TYPES.get(name, native.Q4_K)
            weights[name] = oracle.quantize(t, oracle.normal(seed * 1000 + i, rows * cols, 0.02))
        else:
            t = native.F32
            weights[name] = (1.0 + oracle.normal(seed * 1000 + i, CFG["hidden"], 0.1)).astype(np.float32)
        types.append(t)
    return names, types, weights


def _write(path, names, types, weights):
    w = gguf.GGUFWriter(str(path), "phi3")
    w.add_uint32("phi3.block_count", CFG["layers"])
    w.add_uint32("phi3.embedding_length", CFG["hidden"])
    w.add_uint32("phi3.feed_forward_length", CFG["intermediate"])
    w.add_uint32("phi3.attention.head_count", CFG["query_heads"])
    w.add_uint32("phi3.attention.head_count_kv", CFG["kv_heads"])
    w.add_uint32("phi3.rope.dimension_count", CFG["rotary_size"])
    w.add_float32("phi3.attention.layer_norm_rms_epsilon", CFG["epsilon"])
    w.add_float32("phi3.rope.freq_base", CFG["rope_base"])
    w.add_float32("phi3.rope.scaling.attn_factor", CFG["rope_scale"])
    shapes = phi4.linear_shapes(CFG)
    qt = {native.Q4_K: QT.Q4_K, native.Q6_K: QT.Q6_K}
    for name, t in zip(names, types):
        if t == native.F32:
            w.add_tensor(phi4.gguf_tensor_name(name), weights[name])
        else:  # raw blocks, shape [rows, bytes per row]
            rows = shapes[name][0]
            w.add_tensor(phi4.gguf_tensor_name(name), weights[name].reshape(rows, -1), raw_dtype=qt[t])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_gguf_writer_file_reads_back(tmp_path):
    names, types, weights = _model()
    path = tmp_path / "q4_k_m.gguf"
    _write(path, names, types, weights)
    with native.GgufFile(path) as f:
        cfg = phi4.config_from_gguf(f, context=CFG["context"])
        for k, v in CFG.items():
            assert cfg[k] == pytest.approx(v), k
        assert phi4.slot_types_from_gguf(f, CFG["layers"]) == types
        for name in names:
            t = f.tensors[phi4.gguf_tensor_name(name)]
            assert np.array_equal(t.data, np.ascontiguousarray(weights[name]).view(np.uint8).reshape(-1)), name


@pytest.mark.gpu
def test_q4_k_m_file_decodes_the_oracle_tokens(tmp_path):
    names, types, weights = _model()
    path = tmp_path / "q4_k_m.gguf"
    _write(path, names, types, weights)
    prompt = np.random.default_rng(41).integers(0, CFG["vocab"], 10)
    want = oracle.Decoder(CFG, weights, slot_types=types).generate(prompt, 12)
    with native.GgufFile(path) as f:
        with phi4.open_session_gguf(f, context=CFG["context"]) as dec:
            assert list(dec.generate(prompt, 12)) == want
            # the batched prompt path over the same mixed-type slots
            dec.reset()
            assert dec.prefill(prompt) == want[len(prompt) - 1]
    assert native.device_error_take(0) == 0
