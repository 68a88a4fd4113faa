"""Host-side GGUF helpers of the library against the oracle (bit-exact), and
the block codecs' own invariants (round trips, error bounds, layout)."""
import numpy as np
import pytest

import oracle
from sharpinference_b200 import native
from helpers import known_answers, TYPES


def test_byte_length_table_matches_reference_cases():
    c = known_answers()["byte_lengths"]
    for case in c["cases"]:
        assert native.tensor_byte_length(TYPES[case["type"]], case["dims"]) == case["bytes"]
    for case in c["invalid_data"]:
        with pytest.raises(native.InvalidDataError):
            native.tensor_byte_length(TYPES[case["type"]], case["dims"])
    with pytest.raises(native.NotSupportedError):
        native.tensor_byte_length(c["unsupported_type"], [32])


@pytest.mark.parametrize("seed", [0, 1, 7, 11])
def test_normal_generator_matches_oracle(seed):
    a = native.synth_normal(seed, 4099, 0.02, offset=5)
    b = oracle.normal(seed, 4099, 0.02, offset=5)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    big = native.synth_normal(seed, 1 << 16, 1.0)
    assert abs(float(big.mean())) < 0.02 and abs(float(big.std()) - 1.0) < 0.02


@pytest.mark.parametrize("wtype", [native.Q8_0, native.Q4_K, native.Q6_K])
@pytest.mark.parametrize("sigma", [0.02, 1.0, 300.0])
def test_quantizer_bit_exact_with_oracle(wtype, sigma):
    x = oracle.normal(3, 256 * 37, sigma)
    x[:256] = 0.0                    # all-zero block
    x[256:512] = np.abs(x[256:512])  # non-negative block (min term 0)
    x[512:768] = -np.abs(x[512:768])
    assert np.array_equal(native.quantize(wtype, x), oracle.quantize(wtype, x))


@pytest.mark.parametrize("wtype", [native.Q8_0, native.Q4_K, native.Q6_K])
def test_dequantize_bit_exact_with_oracle(wtype):
    x = oracle.normal(5, 256 * 19, 0.02)
    blob = oracle.quantize(wtype, x)
    a = native.dequantize(wtype, blob, x.size)
    b = oracle.dequantize(wtype, blob, x.size)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_synth_weights_equals_generate_then_quantize():
    rows, cols = 33, 512
    for wtype in (native.Q8_0, native.Q4_K, native.Q6_K, native.F16, native.F32):
        blob = native.synth_weights(wtype, 9, rows, cols, 0.02)
        ref = native.quantize(wtype, oracle.normal(9, rows * cols, 0.02)) if wtype != native.F16 else \
            oracle.normal(9, rows * cols, 0.02).astype(np.float16).view(np.uint8)
        assert np.array_equal(blob, ref), wtype


def test_q8_0_block_layout_and_error_bound():
    x = oracle.normal(1, 32 * 64, 1.0)
    blob = native.quantize(native.Q8_0, x).reshape(-1, 34)
    d = blob[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    amax = np.abs(x.reshape(-1, 32)).max(axis=1)
    assert np.allclose(d, (amax / 127).astype(np.float16).astype(np.float32))
    q = blob[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    w = native.dequantize(native.Q8_0, blob, x.size).reshape(-1, 32)
    # round-to-nearest: |w - x| <= d/2 (+ fp16 rounding of d, 2^-11 relative)
    assert np.all(np.abs(w - x.reshape(-1, 32)) <= (amax / 127)[:, None] * (0.5 + 127 * 2.0 ** -11) + 1e-7)


def test_q4_k_layout_and_error_bound():
    x = oracle.normal(2, 256 * 64, 0.02)
    blob = native.quantize(native.Q4_K, x).reshape(-1, 144)
    w = native.dequantize(native.Q4_K, blob, x.size).reshape(-1, 8, 32)
    xs = x.reshape(-1, 8, 32)
    rng = xs.max(axis=2) - np.minimum(xs.min(axis=2), 0)
    # 15 steps per sub-block plus 6-bit scale / min quantisation error
    err = np.abs(w - xs).max(axis=2)
    assert np.all(err <= rng / 15 * 0.5 + rng / 15 / 63 * 15 + rng / 63 * 0.6 + 1e-7)
    # nibble layout: byte l of chunk j holds elements 64j+l (low) and 64j+32+l (high)
    qs = blob[:, 16:].reshape(-1, 4, 32)
    assert qs.dtype == np.uint8


def test_round_trip_is_idempotent():
    """quantize(dequantize(q)) == q for Q8_0 blocks whose absmax value is
    exactly representable (round trip through the format)."""
    x = (np.arange(-64, 64, dtype=np.float32) / 8.0)
    blob = native.quantize(native.Q8_0, x)
    w = native.dequantize(native.Q8_0, blob, x.size)
    assert np.array_equal(native.quantize(native.Q8_0, w), blob)


def test_q6_k_block_layout_and_error_bound():
    """Q6_K round trip: |w - x| <= half a step of each 16-element group
    (d * scale / 2, plus the binary16 rounding of d), codes inside [0, 63]."""
    x = oracle.normal(4, 256 * 32, 0.02)
    blob = native.quantize(native.Q6_K, x)
    assert blob.size == 32 * 210
    w = native.dequantize(native.Q6_K, blob, x.size)
    blocks = blob.reshape(32, 210)
    d = blocks[:, 208:210].copy().view(np.float16).astype(np.float32).reshape(32, 1)
    sc = blocks[:, 192:208].view(np.int8).astype(np.float32)
    step = np.repeat(d * sc, 16, axis=1).reshape(-1)
    assert np.all(np.abs(w - x) <= 0.5 * step * 1.001 + 1e-12)
