"""transformer.batch-shared-matvec and core.matrix-multiply (transpose_right)
on the GPU through the C ABI, against the oracle and the reference's known
answers (GpuTransformerInstructionTests.cs:280-324, CpuVmMixedWeightsTests.cs)."""
import numpy as np
import pytest

import oracle
from helpers import known_answers, north_star_gate, row_norm_max, to_f16_bytes
from sharpinference_b200 import native

pytestmark = pytest.mark.gpu
N = native


def test_batch_shared_known_answer(ctx):
    c = known_answers()["batch_shared_matvec"]
    W = ctx.buffer(16); X = ctx.buffer(48); C = ctx.buffer(8); Y = ctx.buffer(24)
    try:
        W.upload(to_f16_bytes(c["weight"]))
        X.upload(np.array(c["input"], np.float32))
        C.upload(np.array(c["control"], np.int32))
        Y.upload(np.full(6, c["fill"], np.float32))
        ctx.batch_shared_matvec(N.F16, W, X, C, Y, c["batch"], c["out_features"], c["in_features"])
        assert Y.readback().view(np.float32).tolist() == c["expected"]
    finally:
        for b in (W, X, C, Y):
            b.free()


def test_mixed_weights_batched_known_answer(ctx):
    c = known_answers()["mixed_weights_batched"]
    W = ctx.buffer(32); X = ctx.buffer(64); Y = ctx.buffer(16)
    try:
        W.upload(to_f16_bytes(c["matrix"]))
        X.upload(np.array(c["input"], np.float32))
        ctx.matrix_multiply(N.F16, X, W, Y, 2, 2, 8)
        assert Y.readback().view(np.float32).tolist() == c["expected"]
    finally:
        for b in (W, X, Y):
            b.free()


def _shared_case(ctx, wtype, batch, n, k, valid, seed):
    blob = native.synth_weights(wtype, seed, n, k, 0.02)
    x = native.synth_normal(500 + seed, batch * k, 1.0)
    W, X, C, Y = ctx.buffer(blob.nbytes), ctx.buffer(x.nbytes), ctx.buffer(8), ctx.buffer(batch * n * 4)
    try:
        W.upload(blob), X.upload(x), C.upload(np.array([0, valid], np.int32))
        Y.upload(np.full(batch * n, -31.0, np.float32))
        ctx.batch_shared_matvec(wtype, W, X, C, Y, batch, n, k)
        y = Y.readback().view(np.float32).reshape(batch, n).copy()
    finally:
        for b in (W, X, C, Y):
            b.free()
    return blob, x.reshape(batch, k), y


@pytest.mark.parametrize("wtype", [N.F16, N.Q8_0, N.Q4_K, N.Q6_K])
@pytest.mark.parametrize("batch,valid", [(16, 16), (16, 11), (32, 32), (5, 0), (3, 7)])
def test_batch_shared_quant_parity_and_valid_mask(ctx, wtype, batch, valid):
    n, k = 300, 512
    blob, x, y = _shared_case(ctx, wtype, batch, n, k, valid, seed=batch + valid)
    valid_rows = min(batch, max(valid, 0))
    assert np.all(y[valid_rows:] == -31.0), "rows at or beyond validCount were written"
    rn = row_norm_max(wtype, blob, n, k)
    for b in range(valid_rows):
        ref = oracle.matvec_f64(wtype, blob, x[b], n, k)
        north_star_gate(y[b], ref, x[b], rn, k)


@pytest.mark.parametrize("wtype", [N.Q4_K, N.Q8_0])
@pytest.mark.parametrize("batch,valid,n,k", [(13, 13, 5120, 3072), (9, 7, 3072, 8192), (32, 30, 2000, 1024),
                                             (8, 8, 4099, 768)])
def test_batch_shared_tensor_core_shapes(ctx, wtype, batch, valid, n, k):
    """Q4_K runs the batched tensor-core GEMV (eight input rows per weight
    pass, K split over clusters for K = 8192), Q8_0 one GEMV per row."""
    blob, x, y = _shared_case(ctx, wtype, batch, n, k, valid, seed=batch * 7 + n)
    assert np.all(y[valid:] == -31.0), "rows at or beyond validCount were written"
    rn = row_norm_max(wtype, blob, n, k)
    for b in range(valid):
        ref = oracle.matvec_f64(wtype, blob, x[b], n, k)
        north_star_gate(y[b], ref, x[b], rn, k)
    assert native.device_error_take(0) == 0


@pytest.mark.parametrize("wtype", [N.F32, N.F16, N.Q8_0, N.Q4_K, N.Q6_K])
@pytest.mark.parametrize("m,n,k", [(1, 64, 256), (33, 129, 512), (64, 1000, 768), (300, 200, 256), (257, 128, 1024),
                                   (64, 7, 256)])
def test_matrix_multiply_parity(ctx, wtype, m, n, k):
    """m >= 64 with k % 64 == 0 runs the tcgen05 kernel (tails in m, n and a
    single K stage included); smaller m runs the SIMT kernel."""
    blob = native.synth_weights(wtype, m + n, n, k, 0.02)
    x = native.synth_normal(77, m * k, 1.0)
    X, W, Y = ctx.buffer(x.nbytes), ctx.buffer(blob.nbytes), ctx.buffer(m * n * 4)
    try:
        X.upload(x), W.upload(blob)
        ctx.matrix_multiply(wtype, X, W, Y, m, n, k)
        y = Y.readback().view(np.float32).reshape(m, n).copy()
    finally:
        for b in (X, W, Y):
            b.free()
    ref = oracle.matrix_multiply_tr(wtype, x, blob, m, n, k).reshape(m, n)
    rn = row_norm_max(wtype, blob, n, k)
    for r in range(m):
        north_star_gate(y[r], ref[r], x[r * k:(r + 1) * k], rn, k)


@pytest.mark.parametrize("m", [512])
def test_prefill_gemm_q4_k_config3_shape(ctx, m):
    """BASELINE config 3 shape (X 512x3072 over the qkv Q4_K weight)."""
    n, k = 5120, 3072
    blob = native.synth_weights(N.Q4_K, 0, n, k, 0.02)
    x = native.synth_normal(3000, m * k, 1.0)
    X, W, Y = ctx.buffer(x.nbytes), ctx.buffer(blob.nbytes), ctx.buffer(m * n * 4)
    try:
        X.upload(x), W.upload(blob)
        ctx.matrix_multiply(N.Q4_K, X, W, Y, m, n, k)
        y = Y.readback().view(np.float32).reshape(m, n).copy()
    finally:
        for b in (X, W, Y):
            b.free()
    rows = [0, 1, 255, 511]
    rn = row_norm_max(N.Q4_K, blob, n, k)
    for r in rows:
        ref = oracle.matvec_f64(N.Q4_K, blob, x[r * k:(r + 1) * k], n, k)
        north_star_gate(y[r], ref, x[r * k:(r + 1) * k], rn, k)
    assert native.device_error_take(0) == 0


@pytest.mark.parametrize("wtype", [N.Q4_K, N.Q8_0, N.F16])
@pytest.mark.parametrize("batch,valid,n,k", [(2, 2, 256, 8192), (16, 15, 130, 4096), (24, 24, 640, 17920),
                                             (64, 60, 384, 2048), (100, 100, 200, 1024)])
def test_few_row_gemm_split_k_row_tiles_deterministic(ctx, wtype, batch, valid, n, k):
    """The few-row tcgen05 GEMM behind batch-shared-matvec: narrow weights
    with long rows split K over a cluster (2 or 4 CTAs, partials summed
    through distributed shared memory), 16/32/64-row tiles, more than one
    row tile (100 rows); two runs give identical bits."""
    blob, x, y = _shared_case(ctx, wtype, batch, n, k, valid, seed=batch * 3 + k)
    _, _, y2 = _shared_case(ctx, wtype, batch, n, k, valid, seed=batch * 3 + k)
    np.testing.assert_array_equal(y, y2)
    assert np.all(y[valid:] == -31.0), "rows at or beyond validCount were written"
    rn = row_norm_max(wtype, blob, n, k)
    for b in range(valid):
        north_star_gate(y[b], oracle.matvec_f64(wtype, blob, x[b], n, k), x[b], rn, k)
    assert native.device_error_take(0) == 0
