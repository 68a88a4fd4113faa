"""core.mat-vec on the GPU through the C ABI, against the oracle and the
reference's known answers (GpuMatVecTests.cs, CpuVmMixedWeightsTests.cs)."""
import math

import numpy as np
import pytest

import oracle
from helpers import (cooperative_fixture, known_answers, north_star_gate, reference_gate, row_norm_max, TYPES)
from sharpinference_b200 import native

pytestmark = pytest.mark.gpu
N = native
SENTINEL = 13.0
PAD = 3


def _bytes(values, t):
    v = np.asarray(values, dtype=np.float32)
    return (v.astype(np.float16) if t == N.F16 else v).view(np.uint8)


def _values(raw, t):
    return (raw.view(np.float16).astype(np.float32) if t == N.F16 else raw.view(np.float32)).copy()


def run_padded(ctx, rows, cols, matrix, vector, wt, xt, yt, repeats=3, config=0):
    """GpuMatVecTests.Execute (GpuMatVecTests.cs:288-315): every buffer is
    padded by 3 sentinel elements (13) on both sides, the kernel sees views at
    that offset, runs 3 times; padding and inputs must be untouched."""
    es = {N.F16: 2, N.F32: 4}
    wbuf = np.concatenate([np.full(PAD, SENTINEL), matrix, np.full(PAD, SENTINEL)])
    xbuf = np.concatenate([np.full(PAD, SENTINEL), vector, np.full(PAD, SENTINEL)])
    ybuf = np.full(rows + 2 * PAD, SENTINEL)
    wb, xb, yb = _bytes(wbuf, wt), _bytes(xbuf, xt), _bytes(ybuf, yt)
    W, X, Y = ctx.buffer(wb.nbytes), ctx.buffer(xb.nbytes), ctx.buffer(yb.nbytes)
    try:
        W.upload(wb), X.upload(xb), Y.upload(yb)
        outs = []
        for _ in range(repeats):
            ctx.matvec(wt, W, X, Y, rows, cols, weight_offset=PAD * es[wt], input_offset=PAD * es[xt],
                       output_offset=PAD * es[yt], input_type=xt, output_type=yt, config=config)
            y = _values(Y.readback(), yt)
            assert np.all(y[:PAD] == SENTINEL) and np.all(y[-PAD:] == SENTINEL), "padding overwritten"
            outs.append(y[PAD:-PAD])
        assert np.array_equal(W.readback(), wb), "weight modified"
        assert np.array_equal(X.readback(), xb), "input modified"
        assert native.device_error_take(0) == 0
        return outs
    finally:
        W.free(), X.free(), Y.free()


@pytest.mark.parametrize("sig", [("F32", "F32", "F32"), ("F16", "F32", "F32"), ("F16", "F16", "F16")])
def test_cooperative_signatures_tails_views_and_repeats(ctx, sig):
    fx = cooperative_fixture()
    wt, xt, yt = (TYPES[s] for s in sig)
    for rows, cols in fx["shapes"]:
        rows, cols = int(rows), int(cols)
        m = ((np.arange(rows * cols) % 9 - 4) * 0.125).astype(np.float32)
        v = ((np.arange(cols) % 7 - 3) * 0.25).astype(np.float32)
        expected = fx[f"expected_{rows}x{cols}_{'f16' if yt == N.F16 else 'f32'}"]
        for y in run_padded(ctx, rows, cols, m, v, wt, xt, yt, config=N.MATVEC_COOPERATIVE):
            reference_gate(y, expected)


@pytest.mark.parametrize("final", [4095, 4032])
def test_cooperative_cancellation_exact(ctx, final):
    c = known_answers()["cooperative_cancellation"]
    x = np.ones(4096, np.float32)
    x[0], x[final] = c["big"], -c["big"]
    for y in run_padded(ctx, 3, 4096, np.ones(3 * 4096, np.float32), x, N.F32, N.F32, N.F32):
        assert y.tolist() == c["expected"]


def test_cooperative_nonfinite_classes(ctx):
    c = known_answers()["cooperative_nonfinite"]
    for inp, exp in zip(c["inputs"], c["expected"]):
        x = np.array([float(v) for v in inp], np.float32)
        for y in run_padded(ctx, 3, 2, np.ones(6, np.float32), x, N.F32, N.F32, N.F32):
            for v in y:
                assert math.isnan(v) if exp == "nan" else v == float(exp)


def test_mixed_weights_known_answer(ctx):
    c = known_answers()["mixed_weights_matvec"]
    for y in run_padded(ctx, 2, 8, np.array(c["matrix"], np.float32), np.ones(8, np.float32), N.F16, N.F32, N.F32):
        assert y.tolist() == c["expected"]


@pytest.mark.parametrize("shape", [(3, 2051), (64, 1024)])
def test_bounded_conversion_blocks(ctx, shape):
    rows, cols = shape
    for y in run_padded(ctx, rows, cols, np.ones(rows * cols, np.float32), np.full(cols, 0.25, np.float32),
                        N.F16, N.F32, N.F32):
        assert np.all(y == cols * 0.25)


def test_grid_limit_rows(ctx):
    c = known_answers()["matvec_grid"]
    for y in run_padded(ctx, c["rows"], 3, np.ones(c["rows"] * 3, np.float32), np.array(c["input"], np.float32),
                        N.F32, N.F32, N.F32, repeats=1):
        assert np.all(y == c["expected_value"])


# ---------------------------------------------------------------- quantized
def quant_case(ctx, wtype, rows, cols, seed, *, offset=0, x_seed=None, check_sentinels=True, repeats=2):
    blob = native.synth_weights(wtype, seed, rows, cols, 0.02)
    x = native.synth_normal(1000 + seed if x_seed is None else x_seed, cols, 1.0)
    W = ctx.buffer(blob.nbytes + offset + 64)
    X = ctx.buffer(x.nbytes + 64)
    Y = ctx.buffer(rows * 4 + 2 * 64)
    try:
        W.upload(blob, offset=offset)
        X.upload(x)
        Y.upload(np.full(rows + 32, SENTINEL, np.float32))
        outs = []
        for _ in range(repeats):
            ctx.matvec(wtype, W, X, Y, rows, cols, weight_offset=offset, output_offset=64)
            raw = Y.readback().view(np.float32)
            if check_sentinels:
                assert np.all(raw[:16] == SENTINEL) and np.all(raw[16 + rows:] == SENTINEL)
            outs.append(raw[16:16 + rows].copy())
        assert native.device_error_take(0) == 0
        assert np.array_equal(W.readback(blob.nbytes, offset), blob)
        return blob, x, outs
    finally:
        W.free(), X.free(), Y.free()


def check_quant(wtype, blob, x, outs, rows, cols):
    ref = oracle.matvec(wtype, blob, x, rows, cols)
    exact = oracle.matvec_f64(wtype, blob, x, rows, cols)
    rn = row_norm_max(wtype, blob, rows, cols)
    for y in outs:
        north_star_gate(y, exact, x, rn, cols)
        north_star_gate(y, ref, x, rn, cols)
    assert np.array_equal(outs[0], outs[-1]), "repeated execution is not deterministic"


@pytest.mark.parametrize("rows,cols", [(1, 256), (7, 256), (65, 512), (1000, 768), (333, 3072), (29, 8192),
                                       (17, 17920), (5, 30720)])
def test_q4_k_shapes_and_tails(ctx, rows, cols):
    blob, x, outs = quant_case(ctx, N.Q4_K, rows, cols, seed=rows + cols)
    check_quant(N.Q4_K, blob, x, outs, rows, cols)


@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (65, 288), (1000, 256), (333, 3072), (29, 5120),
                                       (17, 17920), (3, 32 * 1001)])
def test_q8_0_shapes_and_tails(ctx, rows, cols):
    blob, x, outs = quant_case(ctx, N.Q8_0, rows, cols, seed=rows + cols)
    check_quant(N.Q8_0, blob, x, outs, rows, cols)


@pytest.mark.parametrize("rows,cols", [(1, 256), (7, 512), (300, 3072), (29, 5120), (3, 8192), (5, 17920),
                                       (40, 1024)])
def test_q6_k_shapes(ctx, rows, cols):
    """Q6_K (210-byte superblocks: 16-bit aligned, 16-element int8-scaled
    groups) against the oracle, odd superblock counts included."""
    blob, x, outs = quant_case(ctx, N.Q6_K, rows, cols, seed=rows + cols)
    check_quant(N.Q6_K, blob, x, outs, rows, cols)


@pytest.mark.parametrize("wtype", [N.Q8_0, N.Q4_K, N.Q6_K])
def test_quant_unaligned_weight_view_uses_row_warp_path(ctx, wtype):
    rows, cols = 77, 1024
    blob, x, outs = quant_case(ctx, wtype, rows, cols, seed=5, offset=2)
    check_quant(wtype, blob, x, outs, rows, cols)


def test_config1_q8_0_8192x3072(ctx):
    """W 8192x3072 ~ N(0,0.02) seed 0, Q8_0; x ~ N(0,1)."""
    blob, x, outs = quant_case(ctx, N.Q8_0, 8192, 3072, seed=0)
    check_quant(N.Q8_0, blob, x, outs, 8192, 3072)


PHI4_MINI = [("qkv", 5120, 3072, 0), ("o", 3072, 3072, 1), ("gate_up", 16384, 3072, 2), ("down", 3072, 8192, 3),
             ("lm_head", 200064, 3072, 4)]


@pytest.mark.parametrize("name,rows,cols,seed", PHI4_MINI)
def test_config2_q4_k_phi4_mini_shapes(ctx, name, rows, cols, seed):
    """Q4_K GEMV sweep over the Phi-4-mini projections,
    seeds 0-4, compared in full with the oracle."""
    blob, x, outs = quant_case(ctx, N.Q4_K, rows, cols, seed=seed)
    check_quant(N.Q4_K, blob, x, outs, rows, cols)


@pytest.mark.parametrize("wtype", [N.Q8_0, N.Q4_K])
def test_full_size_linearity_and_zero(ctx, wtype):
    """Size-independent properties on the largest shape: W(a x1 + b x2) =
    a W x1 + b W x2 within the gate, and W 0 = 0 exactly."""
    rows, cols = 200064, 3072
    blob = native.synth_weights(wtype, 4, rows, cols, 0.02)
    x1 = native.synth_normal(71, cols, 1.0)
    x2 = native.synth_normal(72, cols, 1.0)
    xs = [x1, x2, (2.0 * x1 - 0.5 * x2).astype(np.float32), np.zeros(cols, np.float32)]
    W, X, Y = ctx.buffer(blob.nbytes), ctx.buffer(cols * 4), ctx.buffer(rows * 4)
    try:
        W.upload(blob)
        ys = []
        for x in xs:
            X.upload(x)
            ctx.matvec(wtype, W, X, Y, rows, cols)
            ys.append(Y.readback().view(np.float32).copy())
    finally:
        W.free(), X.free(), Y.free()
    assert np.all(ys[3] == 0.0)
    combo = 2.0 * ys[0].astype(np.float64) - 0.5 * ys[1]
    d = ys[2] - combo
    assert np.linalg.norm(d) / np.linalg.norm(combo) <= 1e-4


def test_chained_gemvs_and_async_uploads_keep_stream_order(ctx):
    """Launch ordering of the decode GEMV (launched with programmatic
    dependent launch): (1) an asynchronous upload of x followed by the GEMV
    must see the new x; (2) a GEMV whose input is the previous GEMV's output
    must see that output; (3) a GEMV that overwrites the previous GEMV's
    input must not race with it."""
    import ctypes as C
    k, n1, n2 = 3072, 3072, 3072
    w1 = native.synth_weights(N.Q4_K, 41, n1, k, 0.02)
    w2 = native.synth_weights(N.Q4_K, 42, n2, n1, 0.02)
    W1, W2 = ctx.buffer(w1.nbytes), ctx.buffer(w2.nbytes)
    X, H, Y = ctx.buffer(k * 4), ctx.buffer(n1 * 4), ctx.buffer(n2 * 4)
    px = C.c_void_p()
    native.call("si_host_alloc_pinned", k * 4, C.byref(px))
    try:
        W1.upload(w1), W2.upload(w2)
        host = np.ctypeslib.as_array(C.cast(px, C.POINTER(C.c_float)), shape=(k,))
        for step in range(4):
            x = native.synth_normal(900 + step, k, 1.0)
            host[:] = x
            native.call("si_buffer_upload_async", ctx.handle, X.handle, 0, px, k * 4)
            ctx.matvec(N.Q4_K, W1, X, H, n1, k)     # H = W1 x
            ctx.matvec(N.Q4_K, W2, H, Y, n2, n1)    # Y = W2 H   (reads the previous output)
            ctx.matvec(N.Q4_K, W1, X, H, n1, k)     # rewrites H while nothing may still read it
            y = Y.readback().view(np.float32)
            h = H.readback().view(np.float32)
            h_ref = oracle.matvec_f64(N.Q4_K, w1, x, n1, k)
            y_ref = oracle.matvec_f64(N.Q4_K, w2, h.astype(np.float32), n2, n1)
            assert np.linalg.norm(h - h_ref) / np.linalg.norm(h_ref) <= 1e-4, step
            assert np.linalg.norm(y - y_ref) / np.linalg.norm(y_ref) <= 1e-4, step
    finally:
        native.call("si_host_free_pinned", px)
        for b in (W1, W2, X, H, Y):
            b.free()


def test_recorded_submission_replays_with_new_pinned_inputs(ctx):
    """si_graph_*: upload (async, pinned) -> GEMV -> readback recorded once,
    replayed with new host inputs (ExecuteWithTransfers analog)."""
    import ctypes as C
    rows, cols = 3072, 3072
    blob = native.synth_weights(N.Q4_K, 51, rows, cols, 0.02)
    W, X, Y = ctx.buffer(blob.nbytes), ctx.buffer(cols * 4), ctx.buffer(rows * 4)
    px, py = C.c_void_p(), C.c_void_p()
    native.call("si_host_alloc_pinned", cols * 4, C.byref(px))
    native.call("si_host_alloc_pinned", rows * 4, C.byref(py))
    try:
        W.upload(blob)
        hx = np.ctypeslib.as_array(C.cast(px, C.POINTER(C.c_float)), shape=(cols,))
        hy = np.ctypeslib.as_array(C.cast(py, C.POINTER(C.c_float)), shape=(rows,))

        def issue():
            native.call("si_buffer_upload_async", ctx.handle, X.handle, 0, px, cols * 4)
            ctx.matvec(N.Q4_K, W, X, Y, rows, cols)
            native.call("si_buffer_readback_async", ctx.handle, Y.handle, 0, py, rows * 4)

        before = ctx.submission_count
        g = ctx.record(issue)
        try:
            for step in range(3):
                x = native.synth_normal(700 + step, cols, 1.0)
                hx[:] = x
                g.launch()
                ctx.synchronize()
                ref = oracle.matvec_f64(N.Q4_K, blob, x, rows, cols)
                assert np.linalg.norm(hy - ref) / np.linalg.norm(ref) <= 1e-4
            assert ctx.submission_count == before + 1 + 3  # the recorded dispatch + 3 replays
        finally:
            g.close()
    finally:
        native.call("si_host_free_pinned", px)
        native.call("si_host_free_pinned", py)
        for b in (W, X, Y):
            b.free()
