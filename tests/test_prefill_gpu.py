"""Batched prompt prefill (si_decoder_prefill / si_decoder_prefill_embeddings,
the reference's prefill_fused_16 program) and its fused chunk attention
(si_batch_grouped_query_attention) against the oracle: the attention equals
batch-gqa-scores -> batch-causal-softmax -> batch-gqa-values to a relative
2e-5; a prefilled session predicts the oracle's token after the prompt,
holds the oracle's KV cache rows, and decodes on to the oracle's greedy ids."""
import numpy as np
import pytest

import oracle
from sharpinference_b200 import native
from test_decoder_gpu import _load, _logit_gate
from test_transformer_gpu import S, dev, p  # noqa: F401  (dev is a fixture)
from test_transformer_oracle import tiny_decoder_config, tiny_decoder_weights

pytestmark = pytest.mark.gpu
N = native


@pytest.mark.parametrize("hs,qh,kvh,start,count,ctx_len", [
    (128, 6, 2, 0, 77, 77),      # context not a multiple of the key tile
    (128, 24, 8, 40, 100, 300),  # Phi-4-mini heads, rows after a cached prefix
    (64, 8, 1, 3, 64, 80),       # eight query heads per key/value head
    (256, 2, 2, 10, 33, 64),
    (192, 3, 3, 0, 1, 16),       # one row
])
def test_fused_batch_attention_matches_oracle(ctx, dev, hs, qh, kvh, start, count, ctx_len):
    rng = np.random.default_rng(hs + start + count)
    T = ctx_len
    q = rng.standard_normal((count, qh * hs)).astype(np.float32)
    kc = rng.standard_normal(T * kvh * hs).astype(np.float32)
    vc = rng.standard_normal(T * kvh * hs).astype(np.float32)
    out = dev.zeros(count * qh * hs, fill=-4)
    N.call("si_batch_grouped_query_attention", p(dev.put(q)), p(dev.put(kc)), p(dev.put(vc)), start, count, p(out),
           qh, kvh, hs, T, S(ctx))
    ctl = [start, count]
    s_ref = oracle.batch_gqa_scores(q, kc, ctl, np.zeros((count, qh, T), np.float32), qh, kvh, hs, T)
    p_ref = oracle.batch_causal_softmax(s_ref, ctl, np.zeros((count, qh, T), np.float32), qh, T)
    o_ref = oracle.batch_gqa_values(p_ref, vc, ctl, np.zeros((count, qh * hs), np.float32), qh, kvh, hs, T)
    np.testing.assert_allclose(dev.get(out), o_ref.reshape(-1), rtol=2e-5, atol=2e-6)


def test_fused_batch_attention_argument_errors(ctx, dev):
    q, kc = dev.zeros(4 * 128), dev.zeros(8 * 128)
    with pytest.raises(N.ArgumentError):
        N.call("si_batch_grouped_query_attention", p(q), p(kc), p(kc), 6, 4, p(q), 1, 1, 128, 8, S(ctx))
    with pytest.raises(N.NotSupportedError):
        N.call("si_batch_grouped_query_attention", p(q), p(kc), p(kc), 0, 4, p(q), 2, 1, 32, 8, S(ctx))


def _prefill_cfg(wtype=native.Q4_K, context=640):
    cfg = tiny_decoder_config(wtype)
    cfg["context"] = context
    return cfg


@pytest.mark.parametrize("wtype,tokens", [(native.Q4_K, 600), (native.Q4_K, 40), (native.Q8_0, 257),
                                          (native.F16, 96), (native.Q8_0, 513)])
def test_prefill_matches_oracle(wtype, tokens):
    """Chunks of 512 rows (600 = 512 + 88, 513 = 512 + 1), GEMMs on the
    tensor cores from 64 rows and the few-row paths below, then greedy
    decode from there."""
    cfg = _prefill_cfg(wtype)
    weights = tiny_decoder_weights(cfg, seed=50 + wtype)
    prompt = np.random.default_rng(tokens).integers(0, cfg["vocab"], tokens)
    ref = oracle.Decoder(cfg, weights)
    want = ref.generate(prompt, 12)
    with native.Decoder(cfg) as dec:
        _load(dec, weights)
        nxt = dec.prefill(prompt)
        assert dec.position == tokens
        assert nxt == want[tokens - 1]
        kc = dec.read("key_cache_1").reshape(cfg["context"], -1)
        kc_ref = ref.key_cache.reshape(cfg["layers"], cfg["context"], -1)[1]
        np.testing.assert_allclose(kc[:tokens], kc_ref[:tokens], rtol=1e-3, atol=2e-4)
        assert list(dec.generate([nxt], 11)) == want[tokens:]


def test_prefill_logits_and_resume_after_decode():
    """Prefill from a position already advanced by ForwardToken (start > 0)
    and a second prefill after the first: logits of the last prompt row
    within the north-star gate of the oracle's."""
    cfg = _prefill_cfg()
    weights = tiny_decoder_weights(cfg, seed=77)
    prompt = np.random.default_rng(77).integers(0, cfg["vocab"], 150)
    ref = oracle.Decoder(cfg, weights)
    with native.Decoder(cfg) as dec:
        _load(dec, weights)
        for t in prompt[:5]:
            assert dec.forward_token(int(t)) == ref.forward_token(int(t))
        for t in prompt[5:100]:
            tok_ref = ref.forward_token(int(t))
        assert dec.prefill(prompt[5:100]) == tok_ref
        _logit_gate(dec.read("logits"), ref.logits)
        for t in prompt[100:]:
            tok_ref = ref.forward_token(int(t))
        assert dec.prefill(prompt[100:]) == tok_ref
        _logit_gate(dec.read("logits"), ref.logits)
        assert dec.position == 150


def test_prefill_embeddings_equals_token_prefill():
    """PrefillFusedEmbeddings on the prompt's dequantised embedding rows
    gives the token prefill's prediction and caches."""
    cfg = _prefill_cfg()
    weights = tiny_decoder_weights(cfg, seed=91)
    prompt = np.random.default_rng(91).integers(0, cfg["vocab"], 70)
    rows = np.stack([oracle.gather_row(cfg["embedding_type"], weights["token_embedding"], cfg["vocab"],
                                       cfg["hidden"], int(t)) for t in prompt])
    with native.Decoder(cfg) as a, native.Decoder(cfg) as b:
        _load(a, weights)
        _load(b, weights)
        assert a.prefill(prompt) == b.prefill_embeddings(rows)
        np.testing.assert_array_equal(a.read("value_cache_0"), b.read("value_cache_0"))
        np.testing.assert_array_equal(a.read("logits"), b.read("logits"))


def test_prefill_argument_errors():
    cfg = _prefill_cfg(context=64)
    with native.Decoder(cfg) as dec:
        with pytest.raises(native.ArgumentError):
            dec.prefill([1, cfg["vocab"]])
        with pytest.raises(native.ArgumentError):
            dec.prefill([])
        with pytest.raises(native.ArgumentError, match="capacity"):
            dec.prefill(np.ones(65, np.int32))
        with pytest.raises(native.ArgumentError):
            dec.prefill_embeddings(np.zeros((3, cfg["hidden"] + 1), np.float32))
        assert dec.position == 0
        dec.prefill(np.ones(64, np.int32))
        with pytest.raises(native.ArgumentError, match="capacity"):
            dec.prefill([1])
    assert native.device_error_take(0) == 0
