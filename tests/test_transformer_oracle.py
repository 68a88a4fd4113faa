"""The CPU oracle of the transformer instructions, pinned to the known answers
of the reference's GpuTransformerInstructionTests (fixtures in
tests/golden/transformer_known_answers.json) and checked against float64
restatements of the same formulas. No GPU needed."""
import json

import numpy as np
import pytest

import oracle
from helpers import GOLDEN


def _cases():
    return json.loads((GOLDEN / "transformer_known_answers.json").read_text())


def _close(actual, expected, tol):
    actual, expected = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    assert actual.shape == expected.shape
    assert np.max(np.abs(actual - expected)) <= tol, (actual, expected)


def test_residual_rms_norm_known_answer():
    c = _cases()["residual_rms_norm"]
    updated, out = oracle.residual_rms_norm(c["hidden"], c["residual"], c["weight"], c["epsilon"])
    _close(updated, c["expected_updated"], c["tolerance"])
    _close(out, c["expected_output"], c["tolerance"])


def test_swiglu_and_scaled_add_known_answers():
    c = _cases()
    _close(oracle.swiglu(c["swiglu"]["gate_up"]), c["swiglu"]["expected"], c["swiglu"]["tolerance"])
    s = c["scaled_add"]
    _close(oracle.scaled_add(s["input"], s["update"], s["scale"]), s["expected"], s["tolerance"])


def test_batch_rms_norm_known_answer_skips_padding():
    c = _cases()["batch_rms_norm"]
    x = np.float32(c["input"]).reshape(c["batch"], c["width"])
    out = oracle.batch_rms_norm(x, c["weight"], c["control"], np.full_like(x, c["fill"]), c["epsilon"])
    _close(out.reshape(-1), c["expected"], c["tolerance"])


def test_batch_gather_rows_known_answer():
    c = _cases()["batch_gather_rows"]
    table = np.float32(c["table"]).reshape(c["rows"], c["width"])
    out = oracle.batch_gather_rows(table, c["control"], np.full((c["batch"], c["width"]), c["fill"], np.float32))
    _close(out.reshape(-1), c["expected"], c["tolerance"])


def test_batch_attention_known_answer():
    c = _cases()["batch_attention"]
    qh, kvh, hs, ctx = c["query_heads"], c["kv_heads"], c["head_size"], c["context"]
    qkv = np.float32(c["qkv"]).reshape(c["batch"], -1)
    query = np.zeros((c["batch"], qh * hs), np.float32)
    query, kc, vc = oracle.batch_rope_kv_write(qkv, c["control"], c["frequencies"], query, c["key_cache"],
                                               c["value_cache"], qh * hs, kvh, hs, c["rotary_size"], ctx,
                                               c["rope_scale"])
    _close(kc, c["expected_key_cache"], c["cache_tolerance"])
    _close(vc, c["expected_value_cache"], c["cache_tolerance"])
    scores = oracle.batch_gqa_scores(query, kc, c["control"], np.zeros((c["batch"], qh, ctx), np.float32), qh, kvh,
                                     hs, ctx)
    probs = oracle.batch_causal_softmax(scores, c["control"], np.zeros_like(scores), qh, ctx)
    out = oracle.batch_gqa_values(probs, vc, c["control"], np.zeros((c["batch"], qh * hs), np.float32), qh, kvh, hs,
                                  ctx)
    _close(out.reshape(-1), c["expected_output"], c["output_tolerance"])


def _attention_f64(query, kc, vc, active, qh, kvh, hs):
    out = np.zeros(qh * hs)
    for h in range(qh):
        kv = h // (qh // kvh)
        k = kc.reshape(-1, kvh, hs)[: active + 1, kv].astype(np.float64)
        v = vc.reshape(-1, kvh, hs)[: active + 1, kv].astype(np.float64)
        s = k @ query[h * hs:(h + 1) * hs].astype(np.float64) / np.sqrt(hs)
        p = np.exp(s - s.max())
        out[h * hs:(h + 1) * hs] = p @ v / p.sum()
    return out


@pytest.mark.parametrize("position", [0, 5, 63, 200, -3])
def test_grouped_query_attention_matches_float64(position):
    qh, kvh, hs, ctx = 6, 2, 32, 64
    rng = np.random.default_rng(position + 10)
    q = rng.standard_normal(qh * hs).astype(np.float32)
    kc = rng.standard_normal(ctx * kvh * hs).astype(np.float32)
    vc = rng.standard_normal(ctx * kvh * hs).astype(np.float32)
    out = oracle.grouped_query_attention(q, kc, vc, position, qh, kvh, hs, ctx)
    active = min(max(0, position), ctx - 1)  # GpuTransformerInstructionCollection.cs:90-93
    np.testing.assert_allclose(out, _attention_f64(q, kc, vc, active, qh, kvh, hs), rtol=1e-5, atol=1e-5)
    # the unfused scores -> softmax -> values chain agrees for positions inside the cache
    if 0 <= position < ctx:
        s = oracle.gqa_scores(q, kc, position, qh, kvh, hs, ctx)
        p = oracle.causal_softmax(s, position, qh, ctx)
        np.testing.assert_allclose(oracle.gqa_values(p, vc, position, qh, kvh, hs, ctx), out, rtol=1e-5, atol=1e-5)


def test_gqa_scores_unsigned_position_scores_every_token():
    # token <= uint(active): a negative position wraps to a large unsigned value
    qh, kvh, hs, ctx = 2, 1, 4, 5
    q = np.ones(qh * hs, np.float32)
    kc = np.arange(ctx * hs, dtype=np.float32)
    s = oracle.gqa_scores(q, kc, -1, qh, kvh, hs, ctx).reshape(qh, ctx)
    assert np.all(s > -3e38)
    s = oracle.gqa_scores(q, kc, 1, qh, kvh, hs, ctx).reshape(qh, ctx)
    assert np.all(s[:, 2:] == np.float32(-3.402823466e38)) and np.all(s[:, :2] > -3e38)


def test_rope_kv_write_matches_rotation_formula():
    qh, kvh, hs, rot, ctx, pos, scale = 2, 1, 8, 6, 4, 3, 1.25
    rng = np.random.default_rng(3)
    qkv = rng.standard_normal(qh * hs + 2 * kvh * hs).astype(np.float32)
    freq = oracle.rope_frequencies(10000.0, rot)
    np.testing.assert_allclose(freq, 1.0 / 10000.0 ** (2 * np.arange(rot // 2) / rot), rtol=1e-6)
    kc0 = np.full(ctx * kvh * hs, -5, np.float32)
    query, kc, vc = oracle.rope_kv_write(qkv, pos, freq, kc0, kc0, qh * hs, kvh, hs, rot, ctx, scale)

    def rotate(head):
        out = head.astype(np.float64).copy()
        half = rot // 2
        for d in range(rot):
            ang = pos * float(freq[d % half])
            c, s = np.cos(ang) * scale, np.sin(ang) * scale
            out[d] = head[d] * c - head[d + half] * s if d < half else head[d] * c + head[d - half] * s
        return out

    for h in range(qh):
        np.testing.assert_allclose(query[h * hs:(h + 1) * hs], rotate(qkv[h * hs:(h + 1) * hs]), rtol=1e-5, atol=1e-6)
    k = qkv[qh * hs:qh * hs + kvh * hs]
    np.testing.assert_allclose(kc[pos * kvh * hs:(pos + 1) * kvh * hs], rotate(k), rtol=1e-5, atol=1e-6)
    assert np.all(vc[pos * kvh * hs:(pos + 1) * kvh * hs] == qkv[-kvh * hs:])
    assert np.all(np.delete(kc, np.s_[pos * kvh * hs:(pos + 1) * kvh * hs]) == -5)
    # outside [0, context): nothing is written
    _, kc2, _ = oracle.rope_kv_write(qkv, ctx, freq, kc0, kc0, qh * hs, kvh, hs, rot, ctx, scale)
    assert np.all(kc2 == -5)


def test_argmax_ties_nan_and_sentinel():
    assert oracle.argmax([1, 3, 3, 2]) == 1
    assert oracle.argmax([np.nan, 2, np.nan, 2]) == 1
    assert oracle.argmax([-np.inf, -np.inf]) == 0
    assert oracle.argmax([-1, -0.0, 0.0]) == 1  # -0 == +0: the smaller index wins
    x = np.zeros(1000, np.float32)
    x[[300, 700]] = 5
    assert oracle.argmax(x) == 300


def test_gather_row_dequantises_and_flags_invalid_index():
    rng = np.random.default_rng(4)
    table = rng.standard_normal((6, 256)).astype(np.float32) * 0.02
    blob = oracle.quantize(oracle.Q4_K, table)
    row = oracle.gather_row(oracle.Q4_K, blob, 6, 256, 4)
    np.testing.assert_array_equal(row, oracle.dequantize(oracle.Q4_K, blob[4 * 144:5 * 144], 256))
    assert np.all(np.isnan(oracle.gather_row(oracle.Q4_K, blob, 6, 256, 6)))
    assert np.all(np.isnan(oracle.gather_row(oracle.Q4_K, blob, 6, 256, -1)))


def test_embedding_gather_batch_and_copy_rows():
    table = np.arange(12, dtype=np.float32).reshape(4, 3).astype(np.float16)
    out = oracle.embedding_gather_batch(table, 4, [2, 0, 9], 3)
    np.testing.assert_array_equal(out, [6, 7, 8, 0, 1, 2, 0, 0, 0])
    out = oracle.copy_embedding_rows(np.float32([1, 2, 3, 4]), np.zeros(8, np.float32), 2, 2, 1)
    np.testing.assert_array_equal(out, [0, 0, 1, 2, 3, 4, 0, 0])


def test_batch_forms_leave_rows_past_valid_count():
    rng = np.random.default_rng(5)
    gate_up = rng.standard_normal((3, 8)).astype(np.float32)
    out = oracle.batch_swiglu(gate_up, [0, 2], np.full((3, 4), 7, np.float32))
    np.testing.assert_allclose(out[:2].reshape(-1), np.concatenate([oracle.swiglu(g) for g in gate_up[:2]]))
    assert np.all(out[2] == 7)
    sel = oracle.batch_select_last(np.arange(6, dtype=np.float32).reshape(3, 2), [0, 2], np.zeros(2, np.float32))
    np.testing.assert_array_equal(sel, [2, 3])
    sel = oracle.batch_select_last(np.arange(6, dtype=np.float32).reshape(3, 2), [0, 4], np.full(2, 9, np.float32))
    np.testing.assert_array_equal(sel, [9, 9])


def tiny_decoder_config(wtype=oracle.Q4_K):
    return dict(layers=2, hidden=256, query_heads=2, kv_heads=1, head_size=128, rotary_size=96, intermediate=512,
                vocab=640, context=64, epsilon=1e-5, rope_base=10000.0, rope_scale=1.1902381, weight_type=wtype,
                embedding_type=wtype)


def tiny_decoder_weights(cfg, seed=7):
    """Seeded random-init weights: linears N(0, 0.02) quantised, norms 1 + N(0, 0.1)."""
    from sharpinference_b200 import native
    h, f, kv = cfg["hidden"], cfg["intermediate"], cfg["kv_heads"] * cfg["head_size"]
    shapes = {"token_embedding": (cfg["vocab"], h)}
    for layer in range(cfg["layers"]):
        shapes[f"qkv_weight_{layer}"] = (h + 2 * kv, h)
        shapes[f"attn_output_weight_{layer}"] = (h, h)
        shapes[f"ffn_up_weight_{layer}"] = (2 * f, h)
        shapes[f"ffn_down_weight_{layer}"] = (h, f)
    weights = {}
    for i, name in enumerate(native.decoder_slot_names(cfg["layers"])):
        if name in shapes:
            rows, cols = shapes[name]
            wt = cfg["embedding_type"] if name == "token_embedding" else cfg["weight_type"]
            values = oracle.normal(seed * 1000 + i, rows * cols, 0.02)
            weights[name] = (values.astype(np.float16).view(np.uint8) if wt == oracle.F16
                             else oracle.quantize(wt, values))
        else:
            weights[name] = (1.0 + oracle.normal(seed * 1000 + i, h, 0.1)).astype(np.float32)
    return weights


def test_oracle_decoder_is_deterministic_and_finite():
    cfg = tiny_decoder_config()
    w = tiny_decoder_weights(cfg)
    a = oracle.Decoder(cfg, w).generate([1, 2, 3, 4], 4)
    b = oracle.Decoder(cfg, w).generate([1, 2, 3, 4], 4)
    assert a == b
    assert all(0 <= t < cfg["vocab"] for t in a)
    d = oracle.Decoder(cfg, w)
    d.forward_token(5)
    assert np.all(np.isfinite(d.logits))
