"""The few-row GEMM with the dequantised weights in tensor memory
(gemm_fewrow.cu), behind transformer.batch-shared-matvec for 2..32 input
rows of Q4_K / Q8_0 weights (GpuBatchTransformerInstructions.cs:224-279),
against the oracle's double-precision mat-vec under the north-star gate:
single stage and single tile, row tails, 16- and 32-row passes, K split over
clusters of 2..8 CTAs, persistent CTAs over more tiles than SMs, validCount,
rows scaled into the FP16 operand range, every code and scale of the block
formats, determinism, and the range flag of an oversized Q8_0 scale."""
import numpy as np
import pytest

import oracle
from helpers import north_star_gate, row_norm_max
from sharpinference_b200 import native

pytestmark = pytest.mark.gpu
N = native


def _run(ctx, wtype, blob, x, m, n, k, valid):
    W, X, C, Y = ctx.buffer(blob.nbytes), ctx.buffer(x.nbytes), ctx.buffer(8), ctx.buffer(m * n * 4)
    try:
        W.upload(blob), X.upload(x), C.upload(np.array([0, valid], np.int32))
        Y.upload(np.full(m * n, -31.0, np.float32))
        ctx.batch_shared_matvec(wtype, W, X, C, Y, m, n, k)
        return Y.readback().view(np.float32).reshape(m, n).copy()
    finally:
        for b in (W, X, C, Y):
            b.free()


def _check(wtype, blob, x, y, m, n, k, valid):
    assert np.all(y[valid:] == -31.0), "rows at or beyond validCount were written"
    rn = row_norm_max(wtype, blob, n, k)
    xs = x.reshape(m, k)
    for b in range(valid):
        north_star_gate(y[b], oracle.matvec_f64(wtype, blob, xs[b], n, k), xs[b], rn, k)


@pytest.mark.parametrize("wtype", [N.Q4_K, N.Q8_0])
@pytest.mark.parametrize("m,valid,n,k", [
    (2, 2, 128, 256),        # one stage, one tile
    (5, 4, 129, 2560),       # row tail of one, 16-row pass
    (16, 16, 5120, 3072),    # Phi-4-mini qkv at the reference's 16 rows
    (17, 17, 1000, 768),     # 32-row pass, tail tile
    (32, 29, 300, 17920),    # narrow and long: K split over a cluster
    (32, 32, 3072, 8192),    # Phi-4-mini down at 32 streams
    (24, 24, 24000, 3072),   # 188 tiles: persistent CTAs take two
])
def test_fewrow_shapes_match_oracle(ctx, wtype, m, valid, n, k):
    blob = native.synth_weights(wtype, m + n, n, k, 0.02)
    x = native.synth_normal(900 + m, m * k, 1.0)
    y = _run(ctx, wtype, blob, x, m, n, k, valid)
    y2 = _run(ctx, wtype, blob, x, m, n, k, valid)
    np.testing.assert_array_equal(y, y2)  # deterministic (split-K partials added in rank order)
    _check(wtype, blob, x, y, m, n, k, valid)
    assert native.device_error_take(0) == 0


@pytest.mark.parametrize("wtype", [N.Q4_K, N.Q8_0])
def test_fewrow_rows_scaled_into_fp16_range(ctx, wtype):
    """Rows whose largest magnitude is above 2^10 or below 2^-6 are scaled by a
    power of two before the FP16 split (32-element sums of 1e4-sized values
    would overflow FP16); the result is unscaled exactly."""
    m, n, k = 6, 700, 1536
    blob = native.synth_weights(wtype, 3, n, k, 0.02)
    x = native.synth_normal(31, m * k, 1.0).reshape(m, k)
    x[1] *= 3.0e4        # above 2^10
    x[2] *= 1.0e-5       # below 2^-6
    x[3, 17] = 5.0e3     # one outlier
    x[4] = 0.0           # all zero
    x = np.ascontiguousarray(x.reshape(-1), dtype=np.float32)
    y = _run(ctx, wtype, blob, x, m, n, k, m)
    assert np.all(y[4] == 0.0)
    _check(wtype, blob, x, y, m, n, k, m)
    assert native.device_error_take(0) == 0


def _random_blocks(wtype, rng, rows, k):
    """Valid blocks with every code and scale value reachable: random code and
    scale bytes, small random FP16 block scales."""
    rb = oracle.byte_length(wtype, k)
    blob = rng.integers(0, 256, size=rows * rb, dtype=np.uint8)
    if wtype == N.Q4_K:
        blocks = blob.reshape(-1, 144)
        d = rng.uniform(1e-4, 2e-3, blocks.shape[0]).astype(np.float16)
        dmin = rng.uniform(1e-4, 2e-3, blocks.shape[0]).astype(np.float16)
        blocks[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
        blocks[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    else:
        blocks = blob.reshape(-1, 34)
        d = rng.uniform(-3e-3, 3e-3, blocks.shape[0]).astype(np.float16)
        blocks[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    return blob


@pytest.mark.parametrize("wtype", [N.Q4_K, N.Q8_0])
def test_fewrow_every_code_and_scale(ctx, wtype):
    rng = np.random.default_rng(5)
    m, n, k = 12, 384, 2048
    blob = _random_blocks(wtype, rng, n, k)
    x = rng.standard_normal(m * k).astype(np.float32)
    y = _run(ctx, wtype, blob, x, m, n, k, m)
    _check(wtype, blob, x, y, m, n, k, m)
    assert native.device_error_take(0) == 0


def test_fewrow_flags_q8_0_scale_outside_fp16_range(ctx):
    """A Q8_0 block scale above 512 (weights beyond +-65,000) cannot be split
    into FP16 operands: the kernel sets bit 32 of the device error word."""
    m, n, k = 4, 128, 512
    blob = native.synth_weights(N.Q8_0, 9, n, k, 0.02)
    blocks = blob.reshape(-1, 34)
    blocks[5, 0:2] = np.array([1000.0], np.float16).view(np.uint8)
    x = native.synth_normal(10, m * k, 1.0)
    _run(ctx, N.Q8_0, blob, x, m, n, k, m)
    assert native.device_error_take(0) & 32
