"""Multi-stream decoder session (si_decoder_create_streams): several
independent sequences share the weights, each with its own KV cache and
position; one step runs the decode program over all of them (projections
as the few-row tensor-core GEMM). Every stream must decode the oracle's
greedy ids of its own prompt, whatever the other streams hold."""
import numpy as np
import pytest

import oracle
from sharpinference_b200 import native
from test_decoder_gpu import _load
from test_transformer_oracle import tiny_decoder_config, tiny_decoder_weights

pytestmark = pytest.mark.gpu


def _prompts(cfg, lengths, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, cfg["vocab"], n) for n in lengths]


@pytest.mark.parametrize("wtype", [native.Q4_K, native.Q8_0, native.F16])
def test_streams_decode_each_prompt_like_the_oracle(wtype):
    cfg = tiny_decoder_config(wtype)
    weights = tiny_decoder_weights(cfg, seed=40 + wtype)
    lengths, steps = [5, 9, 3, 12], 10
    prompts = _prompts(cfg, lengths, 40 + wtype)
    want = [oracle.Decoder(cfg, weights).generate(p, steps) for p in prompts]
    with native.Decoder(cfg, streams=len(prompts)) as dec:
        _load(dec, weights)
        first = [dec.prefill_stream(b, p) for b, p in enumerate(prompts)]
        assert first == [w[n - 1] for w, n in zip(want, lengths)]
        out = dec.generate_streams(first, lengths, steps)
        assert out.shape == (steps, len(prompts))
        for b, (w, n) in enumerate(zip(want, lengths)):
            assert list(out[:, b]) == w[n:n + steps], f"stream {b}"
        # one host-driven step from the same state equals the loop's first step
        again = dec.step_streams(first, lengths)
        assert list(again) == list(out[0])
    assert native.device_error_take(0) == 0


def test_streams_long_prompts_take_several_staging_passes():
    """Prompts long enough that the decode attention's CTAs (8 per stream and
    key/value head, each a contiguous range of the stream's tokens) stage
    their cache rows in more than one pass: in the multi-stream form a CTA
    holds at most 113 KB of shared memory (two per SM), 96 rows of this
    model, and the ranges here reach 150 rows. Streams of different lengths
    take one or two passes side by side."""
    cfg = dict(tiny_decoder_config(native.Q8_0), context=1280)
    weights = tiny_decoder_weights(cfg, seed=51)
    lengths, steps = [1100, 700, 1200], 4
    prompts = _prompts(cfg, lengths, 51)
    want = [oracle.Decoder(cfg, weights).generate(p, steps) for p in prompts]
    with native.Decoder(cfg, streams=len(prompts)) as dec:
        _load(dec, weights)
        first = [dec.prefill_stream(b, p) for b, p in enumerate(prompts)]
        assert first == [w[n - 1] for w, n in zip(want, lengths)]
        out = dec.generate_streams(first, lengths, steps)
        for b, (w, n) in enumerate(zip(want, lengths)):
            assert list(out[:, b]) == w[n:n + steps], f"stream {b}"
    assert native.device_error_take(0) == 0


def test_streams_stepwise_prompt_equals_prefill():
    """Feeding the prompts through step_streams (all streams advancing
    together, shorter prompts padded by repeating their last token at the
    same position) leaves the caches the prefill leaves."""
    cfg = tiny_decoder_config()
    weights = tiny_decoder_weights(cfg, seed=47)
    prompts = _prompts(cfg, [6, 6], 47)
    want = [oracle.Decoder(cfg, weights).generate(p, 4) for p in prompts]
    with native.Decoder(cfg, streams=2) as dec:
        _load(dec, weights)
        nxt = None
        for i in range(6):
            nxt = dec.step_streams([prompts[0][i], prompts[1][i]], [i, i])
        assert list(nxt) == [want[0][5], want[1][5]]
        out = dec.generate_streams(nxt, [6, 6], 4)
        assert [list(out[:, b]) for b in range(2)] == [want[0][6:10], want[1][6:10]]


def test_streams_argument_errors():
    cfg = tiny_decoder_config()
    with native.Decoder(cfg, streams=3) as dec:
        with pytest.raises(native.ArgumentError):
            dec.step_streams([1, 2], [0, 0])
        with pytest.raises(native.ArgumentError, match="capacity"):
            dec.generate_streams([1, 2, 3], [0, cfg["context"] - 2, 0], 4)
        with pytest.raises(native.ArgumentError):
            dec.step_streams([1, cfg["vocab"], 3], [0, 0, 0])
        with pytest.raises(native.ArgumentError):
            dec.prefill_stream(3, [1, 2])
    with pytest.raises(native.ArgumentError):
        native.Decoder(cfg, streams=0)
    single = tiny_decoder_config()
    with native.Decoder(single) as dec:
        with pytest.raises(native.ArgumentError, match="multi-stream"):
            native.call("si_decoder_step_streams", dec.handle, np.zeros(1, np.int32).ctypes.data,
                        np.zeros(1, np.int32).ctypes.data, np.zeros(1, np.int32).ctypes.data)
