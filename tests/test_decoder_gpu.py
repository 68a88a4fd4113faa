"""The Phi-4 decode program on CUDA (si_decoder_*) against the oracle's
restatement of the same program (or_decoder_step): identical greedy token
ids on seeded random-init models, logits within the north-star gate, the
device-resident greedy loop equal to ForwardToken, and the session's
argument errors."""
import numpy as np
import pytest

import oracle
from sharpinference_b200 import native
from test_transformer_oracle import tiny_decoder_config, tiny_decoder_weights

pytestmark = pytest.mark.gpu


def _load(dec, weights):
    for name, arr in weights.items():
        dec.upload(name, arr)


def _logit_gate(gpu, ref):
    gpu, ref = np.asarray(gpu, np.float64), np.asarray(ref, np.float64)
    assert np.all(np.isfinite(gpu))
    rel_l2 = np.linalg.norm(gpu - ref) / np.linalg.norm(ref)
    assert rel_l2 <= 1e-4, rel_l2


@pytest.mark.parametrize("wtype", [native.Q4_K, native.Q8_0, native.F16, native.Q6_K])
def test_forward_token_matches_oracle(wtype):
    cfg = tiny_decoder_config(wtype)
    weights = tiny_decoder_weights(cfg, seed=7 + wtype)
    ref = oracle.Decoder(cfg, weights)
    rng = np.random.default_rng(wtype)
    prompt = rng.integers(0, cfg["vocab"], 20)
    with native.Decoder(cfg) as dec:
        _load(dec, weights)
        tok_gpu = tok_ref = None
        for i in range(32):
            t_in = int(prompt[i]) if i < len(prompt) else tok_gpu
            tok_gpu = dec.forward_token(t_in)
            tok_ref = ref.forward_token(t_in)
            _logit_gate(dec.read("logits"), ref.logits)
            assert tok_gpu == tok_ref, f"step {i}: {tok_gpu} != {tok_ref}"
        assert dec.position == 32
        # the caches hold exactly the rows written so far
        kc = dec.read("key_cache_1").reshape(cfg["context"], -1)
        kc_ref = ref.key_cache.reshape(cfg["layers"], cfg["context"], -1)[1]
        np.testing.assert_allclose(kc[:32], kc_ref[:32], rtol=1e-3, atol=1e-4)
        assert np.all(kc[32:] == 0)


def test_generate_equals_forward_token_loop_and_oracle():
    cfg = tiny_decoder_config()
    weights = tiny_decoder_weights(cfg, seed=3)
    prompt = np.random.default_rng(11).integers(0, cfg["vocab"], 16)
    ref = oracle.Decoder(cfg, weights).generate(prompt, 24)
    with native.Decoder(cfg) as dec:
        _load(dec, weights)
        fused = dec.generate(prompt, 24)
        assert dec.position == 40
        assert list(fused) == ref
        dec.reset()
        assert dec.position == 0
        loop, tok = [], None
        for i in range(40):
            tok = dec.forward_token(int(prompt[i]) if i < 16 else tok)
            loop.append(tok)
        assert loop == ref
        # continuing from the current position: prompt = the last prediction
        dec.reset()
        first = dec.generate(prompt, 0)
        rest = dec.generate([first[-1]], 23)
        assert list(first) + list(rest) == ref


def test_full_width_layer_matches_oracle():
    """Phi-4-mini layer widths (hidden 3072, 24/8 heads of 128, FFN 8192) with
    a cut vocabulary and one layer, so the CPU oracle stays quick."""
    cfg = dict(layers=1, hidden=3072, query_heads=24, kv_heads=8, head_size=128, rotary_size=96,
               intermediate=8192, vocab=4096, context=256, epsilon=1e-5, rope_base=10000.0, rope_scale=1.1902381,
               weight_type=native.Q4_K, embedding_type=native.Q4_K)
    weights = tiny_decoder_weights(cfg, seed=5)
    ref = oracle.Decoder(cfg, weights)
    prompt = np.random.default_rng(5).integers(0, cfg["vocab"], 12)
    with native.Decoder(cfg) as dec:
        _load(dec, weights)
        for i, t in enumerate(prompt):
            assert dec.forward_token(int(t)) == ref.forward_token(int(t)), i
            _logit_gate(dec.read("logits"), ref.logits)


def test_session_argument_errors():
    cfg = tiny_decoder_config()
    cfg["context"] = 4
    with native.Decoder(cfg) as dec:
        with pytest.raises(native.ArgumentError):
            dec.forward_token(cfg["vocab"])
        with pytest.raises(native.ArgumentError):
            dec.forward_token(-1)
        with pytest.raises(native.ArgumentError):
            dec.generate([1, 2, 3], 2)  # five positions, context of four
        for _ in range(4):
            dec.forward_token(1)
        with pytest.raises(native.ArgumentError, match="capacity"):
            dec.forward_token(1)
        with pytest.raises(native.ArgumentError):
            dec.upload("no_such_slot", np.zeros(4, np.float32))
        with pytest.raises(native.ArgumentError):
            dec.upload("output_norm", np.zeros(cfg["hidden"] + 1, np.float32))
    bad = tiny_decoder_config()
    bad["query_heads"] = 3
    with pytest.raises(native.InstructionAdaptationError):
        native.Decoder(bad)
    assert native.device_error_take(0) == 0


def test_session_from_gguf_file(tmp_path):
    """A model saved as a phi3 GGUF file, opened by the library's reader and
    uploaded byte-for-byte into the session, decodes the oracle's tokens."""
    from sharpinference_b200 import phi4
    cfg = tiny_decoder_config()
    weights = tiny_decoder_weights(cfg, seed=33)
    path = tmp_path / "tiny.gguf"
    phi4.save_gguf(path, cfg, weights)
    prompt = np.random.default_rng(33).integers(0, cfg["vocab"], 10)
    want = oracle.Decoder(cfg, weights).generate(prompt, 10)
    with native.GgufFile(path) as f:
        gcfg = phi4.config_from_gguf(f, context=cfg["context"])
        with native.Decoder(gcfg) as dec:
            phi4.load_gguf(dec, f)
            assert list(dec.generate(prompt, 10)) == want
