"""GGUF v3 files: the library's reader (si_gguf_*) against files written by
sharpinference_b200.gguf, with the checks GgufModelFile.Open performs
(GgufModelFile.cs:57-160) and its byte-length table (:301-331, plus the
K-quant superblocks). No GPU needed."""
import struct

import numpy as np
import pytest

from sharpinference_b200 import gguf, native, phi4
from test_transformer_oracle import tiny_decoder_config, tiny_decoder_weights

N = native


def _write(path, meta, tensors, alignment=32):
    gguf.write(path, meta, tensors, alignment)
    return path


def test_round_trip_metadata_and_tensors(tmp_path):
    data = np.arange(256 * 4, dtype=np.uint8)
    floats = np.linspace(-1, 1, 7, dtype=np.float32)
    meta = {"general.name": "tiny", "n": 7, "big": 1 << 40, "f": 1.5, "flag": True,
            "u16": (gguf.U16, 65535), "f64": (gguf.F64, 0.25), "ids": [1, 2, 3], "names": ["a", "bc"],
            "vals": [0.5, 1.5]}
    p = _write(tmp_path / "m.gguf", meta, [("w", 8, [32, 4], np.arange(4 * 34, dtype=np.uint8)),
                                            ("v", 0, [7], floats), ("raw", 24, [1024], data)])
    with N.GgufFile(p) as f:
        m = f.metadata
        assert m["general.name"] == "tiny" and m["n"] == 7 and m["big"] == 1 << 40
        assert m["f"] == 1.5 and m["flag"] is True and m["u16"] == 65535 and m["f64"] == 0.25
        assert list(m["ids"]) == [1, 2, 3] and m["names"] == ("array", gguf.STRING, 2)
        assert np.allclose(m["vals"], [0.5, 1.5])
        assert list(f.tensors) == ["w", "v", "raw"]
        w = f.tensors["w"]
        assert w.type == 8 and w.dims == [32, 4] and w.nbytes == 4 * 34
        assert np.array_equal(w.data, np.arange(4 * 34, dtype=np.uint8))
        assert np.array_equal(f.tensors["v"].data.view(np.float32), floats)
        assert np.array_equal(f.tensors["raw"].data, data)


def test_byte_length_table():
    # GetByteLength (GgufModelFile.cs:301-331) and the K-quant superblocks
    cases = {0: 4 * 256, 1: 2 * 256, 30: 2 * 256, 24: 256, 25: 512, 26: 1024, 27: 2048, 28: 2048,
             2: 8 * 18, 3: 8 * 20, 6: 8 * 22, 7: 8 * 24, 8: 8 * 34, 9: 8 * 36,
             10: 84, 11: 110, 12: 144, 13: 176, 14: 210, 15: 292}
    for t, want in cases.items():
        assert N.tensor_byte_length(t, [256]) == want, t
    with pytest.raises(N.InvalidDataError):
        N.tensor_byte_length(14, [100])  # Q6_K needs whole superblocks
    with pytest.raises(N.NotSupportedError):
        N.tensor_byte_length(4, [32])    # type id 4 does not exist


def _raw_header(tensors=0, meta=0, magic=0x46554747, version=3):
    return struct.pack("<IIQQ", magic, version, tensors, meta)


def _s(x):
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


@pytest.mark.parametrize("blob,err", [
    (_raw_header(magic=0x12345678), N.InvalidDataError),
    (_raw_header(version=2), N.InvalidDataError),
    (_raw_header(meta=2) + _s("k") + struct.pack("<Ii", 5, 1) + _s("k") + struct.pack("<Ii", 5, 2), N.InvalidDataError),
    (_raw_header(meta=1) + _s("  ") + struct.pack("<Ii", 5, 1), N.InvalidDataError),
    (_raw_header(meta=1) + _s("k") + struct.pack("<IB", 7, 2), N.InvalidDataError),      # Bool 2
    (_raw_header(meta=1) + _s("k") + struct.pack("<II", 9, 9), N.InvalidDataError),      # nested array
    (_raw_header(meta=1) + _s("k") + struct.pack("<I", 77), N.InvalidDataError),         # unknown type
    (_raw_header(meta=1) + _s("general.alignment") + struct.pack("<II", 4, 24), N.InvalidDataError),
    (_raw_header(tensors=1) + _s("t") + struct.pack("<I", 9) + b"\0" * 72, N.InvalidDataError),   # rank 9
    (_raw_header(tensors=1) + _s("t") + struct.pack("<IQIQ", 1, 0, 0, 0), N.InvalidDataError),     # empty dim
    (_raw_header(tensors=1) + _s("t") + struct.pack("<IQIQ", 1, 1 << 20, 0, 0), N.InvalidDataError),  # past EOF
    (_raw_header(tensors=1) + _s("t") + struct.pack("<IQIQ", 1, 32, 99, 0), N.NotSupportedError),
    (_raw_header(tensors=2) + (_s("t") + struct.pack("<IQIQ", 1, 4, 0, 0)) * 2, N.InvalidDataError),
])
def test_malformed_files_are_rejected(tmp_path, blob, err):
    p = tmp_path / "bad.gguf"
    p.write_bytes(blob + b"\0" * 64)
    with pytest.raises(err):
        N.GgufFile(p)


def test_truncated_files_are_rejected(tmp_path):
    whole = _raw_header(meta=1, tensors=1) + _s("key") + struct.pack("<Ii", 5, 1) + _s("t") + struct.pack(
        "<IQIQ", 1, 4, 0, 0)
    for cut in (3, 10, 30, len(whole) - 1):
        p = tmp_path / f"cut{cut}.gguf"
        p.write_bytes(whole[:cut])
        with pytest.raises(N.InvalidDataError):
            N.GgufFile(p)


def test_legacy_32bit_array_count(tmp_path):
    # GgufModelFile.ReadArrayCount: an older converter's 32-bit count is read
    # as such when the 64-bit value is out of range.
    body = _s("arr") + struct.pack("<III", 9, 5, 3) + struct.pack("<iii", 7, 8, 9)
    p = tmp_path / "legacy.gguf"
    p.write_bytes(_raw_header(meta=1) + body + b"\0" * 64)
    with N.GgufFile(p) as f:
        assert list(f.metadata["arr"]) == [7, 8, 9]


def test_missing_file_is_an_argument_error(tmp_path):
    with pytest.raises(N.ArgumentError):
        N.GgufFile(tmp_path / "none.gguf")


def test_phi4_model_round_trip(tmp_path):
    cfg = tiny_decoder_config()
    w = tiny_decoder_weights(cfg, seed=9)
    p = tmp_path / "phi4_tiny.gguf"
    phi4.save_gguf(p, cfg, w)
    with N.GgufFile(p) as f:
        got = phi4.config_from_gguf(f, context=cfg["context"])
        for k in ("layers", "hidden", "query_heads", "kv_heads", "head_size", "rotary_size", "intermediate", "vocab",
                  "weight_type", "embedding_type", "context"):
            assert got[k] == cfg[k], k
        assert np.float32(got["epsilon"]) == np.float32(cfg["epsilon"])
        assert np.float32(got["rope_scale"]) == np.float32(cfg["rope_scale"])
        for slot, arr in w.items():
            t = f.tensors[phi4.gguf_tensor_name(slot)]
            assert np.array_equal(t.data, np.ascontiguousarray(arr).view(np.uint8).reshape(-1)), slot
