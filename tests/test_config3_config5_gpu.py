"""BASELINE config 3 and config 5 at full width, against the oracle.

Config 3: the prefill GEMM Y = X W^T (core.matrix-multiply, transpose_right;
CpuInstructionNumerics.cs:61-82 restated as one mat-vec per row) over all
five Phi-4-mini Q4_K shapes at M = 512 and M = 2048, X ~ N(0,1). Sampled rows
of Y (the first, both sides of the 128- and 256-row tile edges, the middle
and the last) are checked over all N columns, which covers the last weight
row tile of lm_head (200064 = 1563 * 128) and the split-K reduction of down
(K = 8192).

Config 5: one Phi-4-14B-shaped layer (hidden 5120, 40 / 10 heads of 128, FFN
17920, Q8_0 weights) through the decode session, greedy ids and logits
against the oracle's restatement of the program (cut vocabulary, so the CPU
oracle stays quick)."""
import numpy as np
import pytest

import oracle
from helpers import north_star_gate, row_norm_max
from sharpinference_b200 import native
from test_transformer_oracle import tiny_decoder_weights

pytestmark = pytest.mark.gpu
N = native

CONFIG2 = [("qkv", 5120, 3072, 0), ("o", 3072, 3072, 1), ("gate_up", 16384, 3072, 2), ("down", 3072, 8192, 3),
           ("lm_head", 200064, 3072, 4)]


@pytest.mark.parametrize("m", [512, 2048])
@pytest.mark.parametrize("name,n,k,seed", CONFIG2, ids=[c[0] for c in CONFIG2])
def test_prefill_gemm_config3(ctx, m, name, n, k, seed):
    blob = native.synth_weights(N.Q4_K, seed, n, k, 0.02)
    x = native.synth_normal(3000 + seed, m * k, 1.0)
    X, W, Y = ctx.buffer(x.nbytes), ctx.buffer(blob.nbytes), ctx.buffer(m * n * 4)
    try:
        X.upload(x), W.upload(blob)
        Y.upload(np.full(m * n, np.nan, np.float32))
        ctx.matrix_multiply(N.Q4_K, X, W, Y, m, n, k)
        y = Y.readback().view(np.float32).reshape(m, n)
    finally:
        for b in (X, W, Y):
            b.free()
    assert native.device_error_take(0) == 0
    rows = sorted({0, 1, 127, 128, 255, 256, m // 2 + 3, m - 1})
    rn = row_norm_max(N.Q4_K, blob, n, k)
    for r in rows:
        xr = x[r * k:(r + 1) * k]
        north_star_gate(y[r], oracle.matvec_f64(N.Q4_K, blob, xr, n, k), xr, rn, k)
    # every element was written (no NaN fill left) and is finite
    assert np.all(np.isfinite(y))


def test_phi4_14b_full_width_layer_q8_0():
    cfg = dict(layers=1, hidden=5120, query_heads=40, kv_heads=10, head_size=128, rotary_size=128,
               intermediate=17920, vocab=2048, context=64, epsilon=1e-5, rope_base=250000.0, rope_scale=1.0,
               weight_type=native.Q8_0, embedding_type=native.Q8_0)
    weights = tiny_decoder_weights(cfg, seed=11)
    ref = oracle.Decoder(cfg, weights)
    prompt = np.random.default_rng(11).integers(0, cfg["vocab"], 6)
    with native.Decoder(cfg) as dec:
        for name, arr in weights.items():
            dec.upload(name, arr)
        tok = None
        for i in range(10):
            t_in = int(prompt[i]) if i < len(prompt) else tok
            tok = dec.forward_token(t_in)
            assert tok == ref.forward_token(t_in), f"step {i}"
            got, want = np.asarray(dec.read("logits"), np.float64), np.asarray(ref.logits, np.float64)
            assert np.all(np.isfinite(got))
            assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-4
    assert native.device_error_take(0) == 0
