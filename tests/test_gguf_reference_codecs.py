"""Pins the GGUF block codecs to an independent published implementation:
gguf-py 0.19.0 (llama.cpp's `gguf.quants`, installed in this image). The
reference itself has no quantized arithmetic (GgufModelFile.cs:301-331 only
sizes the blocks), so the oracle's dequantisers are checked bit for bit
against gguf-py on the BASELINE workloads' blocks (config 1 Q8_0 seed 0, the
five config-2 Q4_K shapes with seeds 0-4, sampled rows including the last),
on odd shapes, and on random valid blocks that reach every code, scale and
minimum the formats can hold. Q8_0 quantisation is also pinned (gguf-py
quantises Q8_0; it has no K-quant quantiser)."""
import numpy as np
import pytest

import oracle

gguf = pytest.importorskip("gguf")
quants = pytest.importorskip("gguf.quants")
QT = gguf.GGMLQuantizationType
KIND = {oracle.Q8_0: QT.Q8_0, oracle.Q4_K: QT.Q4_K}
BLOCK = {oracle.Q8_0: (32, 34), oracle.Q4_K: (256, 144)}
if hasattr(oracle, "Q6_K"):
    KIND[oracle.Q6_K] = QT.Q6_K
    BLOCK[oracle.Q6_K] = (256, 210)

CONFIG2 = [("qkv", 5120, 3072, 0), ("o", 3072, 3072, 1), ("gate_up", 16384, 3072, 2), ("down", 3072, 8192, 3),
           ("lm_head", 200064, 3072, 4)]


def _same_bits(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    assert a.shape == b.shape
    diff = np.flatnonzero(a.view(np.uint32) != b.view(np.uint32))
    assert diff.size == 0, f"{diff.size} elements differ, first at {diff[0]}: {a[diff[0]]} vs {b[diff[0]]}"


def _rows(wtype, seed, rows, cols, sigma=0.02):
    """Rows `rows` of the seeded [*, cols] matrix, quantised by the oracle (the
    generator is a counter, so row r is the values at offset r * cols)."""
    vals = np.concatenate([oracle.normal(seed, cols, sigma, offset=r * cols) for r in rows])
    return oracle.quantize(wtype, vals), vals.size


def _check(wtype, blob, count):
    per, nbytes = BLOCK[wtype]
    ref = quants.dequantize(np.ascontiguousarray(blob).reshape(-1, nbytes), KIND[wtype])
    _same_bits(oracle.dequantize(wtype, blob, count), ref)


def test_q8_0_config1_full_matrix():
    """Config 1: Q8_0 8192 x 3072, seed 0, every row."""
    blob = oracle.quantize(oracle.Q8_0, oracle.normal(0, 8192 * 3072, 0.02))
    _check(oracle.Q8_0, blob, 8192 * 3072)


@pytest.mark.parametrize("name,n,k,seed", CONFIG2, ids=[c[0] for c in CONFIG2])
def test_q4_k_config2_sampled_rows(name, n, k, seed):
    rows = sorted({0, 1, 2, 127, 128, n // 2, n - 2, n - 1})
    blob, count = _rows(oracle.Q4_K, seed, rows, k)
    _check(oracle.Q4_K, blob, count)


@pytest.mark.parametrize("wtype", [oracle.Q8_0, oracle.Q4_K])
@pytest.mark.parametrize("sigma", [1e-4, 0.02, 1.0, 300.0])
def test_odd_shapes_and_scales(wtype, sigma):
    per, _ = BLOCK[wtype]
    x = oracle.normal(17, per * 37, sigma)
    x[:per] = 0.0                        # all-zero block
    x[per:2 * per] = np.abs(x[per:2 * per])  # non-negative block (Q4_K min term 0)
    x[2 * per:3 * per] = -np.abs(x[2 * per:3 * per])
    x[3 * per + 5] = 40 * sigma          # one outlier
    _check(wtype, oracle.quantize(wtype, x), x.size)


def _random_blocks(wtype, nblocks, seed):
    """Random valid blocks: random code bytes, finite FP16 scales of both
    signs and a wide range of magnitudes."""
    rng = np.random.default_rng(seed)
    per, nbytes = BLOCK[wtype]
    raw = rng.integers(0, 256, size=(nblocks, nbytes), dtype=np.uint8)

    def f16(n):
        return (rng.standard_normal(n) * 10.0 ** rng.integers(-4, 2, n)).astype(np.float16).view(np.uint8).reshape(n, 2)

    if wtype == oracle.Q8_0:
        raw[:, 0:2] = f16(nblocks)
    elif wtype == oracle.Q4_K:
        raw[:, 0:2] = f16(nblocks)
        raw[:, 2:4] = f16(nblocks)
    else:  # Q6_K: d is the last two bytes
        raw[:, nbytes - 2:nbytes] = f16(nblocks)
    return raw.reshape(-1), nblocks * per


@pytest.mark.parametrize("wtype", sorted(KIND))
def test_random_valid_blocks(wtype):
    blob, count = _random_blocks(wtype, 4096, 5 + wtype)
    _check(wtype, blob, count)


def test_q8_0_quantiser_equals_gguf():
    """The oracle's (and the library's, checked bit-exact elsewhere) Q8_0
    quantiser writes the bytes gguf-py's Q8_0 quantiser writes."""
    for seed, sigma in ((0, 0.02), (3, 1.0), (9, 250.0)):
        x = oracle.normal(seed, 32 * 4096, sigma)
        x[:32] = 0.0
        ref = quants.quantize(x.reshape(-1, 1024), QT.Q8_0)
        assert np.array_equal(oracle.quantize(oracle.Q8_0, x), np.asarray(ref).reshape(-1))
