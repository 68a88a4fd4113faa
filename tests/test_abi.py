"""The C ABI: the shared library loads, exports every function the header
declares, and rejects invalid launches on the host with the status that maps
to the reference's exception (no GPU needed: validation runs before any
device call)."""
import ctypes as C
import subprocess

import numpy as np
import pytest

from sharpinference_b200 import native

N = native


def test_library_exports_every_header_symbol():
    declared = native.header_functions()
    assert len(declared) >= 30
    missing = [name for name in declared if not hasattr(native.lib, name)]
    assert not missing, missing
    # and the binding covers all of them
    assert sorted(native.SIGNATURES) == declared


def test_exported_dynamic_symbols_are_the_header():
    out = subprocess.run(["nm", "-D", "--defined-only", str(native.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line and line.split()[-1].startswith("si_")}
    assert exported == set(native.header_functions())


def test_abi_version():
    assert native.lib.si_abi_version() == 1


FAKE = 0x1000  # never dereferenced: every case below fails validation first


def _mv(wtype=N.Q8_0, xt=N.F32, yt=N.F32, rows=8, cols=256, cfg=0, w=FAKE, x=FAKE * 1000, y=FAKE * 2000):
    return native.lib.si_matvec(wtype, w, xt, x, yt, y, rows, cols, cfg, None)


def test_matvec_rejects_nonpositive_shapes():
    assert _mv(rows=0) == N.SI_ERR_INVALID_ARGUMENT
    assert "Mixed matvec requires" in native.last_error()
    assert _mv(cols=-1) == N.SI_ERR_INVALID_ARGUMENT


def test_matvec_rejects_rows_beyond_thread_indexing():
    # GpuMatVecExecution.Groups(uint.MaxValue) throws (GpuMatVecTests.cs:113)
    assert _mv(rows=0xFFFFFFFF) == N.SI_ERR_INVALID_ARGUMENT
    assert "32-bit thread indexing" in native.last_error()


def test_matvec_rejects_unknown_type_and_partial_blocks():
    assert _mv(wtype=99) == N.SI_ERR_UNSUPPORTED
    assert _mv(wtype=N.Q8_0, cols=33) == N.SI_ERR_INVALID_DATA
    assert _mv(wtype=N.Q4_K, cols=300) == N.SI_ERR_INVALID_DATA


def test_matvec_rejects_wrong_configuration_and_signature():
    assert _mv(wtype=N.Q4_K, cfg=N.MATVEC_COOPERATIVE) == N.SI_ERR_ADAPTATION
    assert _mv(wtype=N.F32, cfg=N.MATVEC_QUANT_STAGED) == N.SI_ERR_ADAPTATION
    assert _mv(wtype=N.F32, cfg=7) == N.SI_ERR_ADAPTATION
    assert _mv(wtype=N.Q8_0, xt=N.F16) == N.SI_ERR_ADAPTATION
    assert _mv(wtype=N.F32, xt=N.Q8_0) == N.SI_ERR_ADAPTATION


def test_matvec_rejects_aliasing_and_null():
    # output overlapping the weight (D3D12 compiler refuses aliasing, GpuMatVecTests.cs:104-112)
    assert _mv(w=FAKE, y=FAKE + 16) == N.SI_ERR_UNSUPPORTED
    assert _mv(w=None) == N.SI_ERR_INVALID_ARGUMENT


def test_matvec_rejects_host_pointers_without_touching_a_device():
    w = np.zeros(N.row_bytes(N.Q8_0, 256) * 8, np.uint8)
    x = np.zeros(256, np.float32)
    y = np.zeros(8, np.float32)
    st = _mv(w=w.ctypes.data, x=x.ctypes.data, y=y.ctypes.data)
    assert st == N.SI_ERR_INVALID_ARGUMENT
    assert "not" in native.last_error()


def test_batch_shared_and_matmul_validation():
    lib = native.lib
    assert lib.si_batch_shared_matvec(N.Q4_K, FAKE, FAKE * 1000, None, FAKE * 3000, 2, 8, 256, None) == \
        N.SI_ERR_INVALID_ARGUMENT
    assert lib.si_batch_shared_matvec(N.F32, FAKE, FAKE * 1000, FAKE * 500, FAKE * 3000, 2, 8, 256, None) == \
        N.SI_ERR_ADAPTATION
    assert lib.si_batch_shared_matvec(N.Q4_K, FAKE, FAKE * 1000, FAKE * 500, FAKE * 3000, 0, 8, 256, None) == \
        N.SI_ERR_ADAPTATION
    assert lib.si_matrix_multiply(N.Q4_K, FAKE * 1000, FAKE, FAKE * 3000, 4, 8, 100, None, 0, None) == \
        N.SI_ERR_INVALID_DATA
    b = C.c_uint64()
    assert lib.si_matrix_multiply_workspace_bytes(N.Q4_K, 0, 8, 256, C.byref(b)) == N.SI_ERR_INVALID_ARGUMENT


def test_context_without_device_reports_no_device():
    if native.device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(native.NoDeviceError):
        native.Context(0)


def test_registry_resolves_cuda_instructions():
    mv = native.resolve(native.TIER_ZERO_FLOAT32, "core.mat-vec")
    mv16 = native.resolve(native.TIER_ZERO_FLOAT16, "core.mat-vec")
    mm = native.resolve(native.TIER_ZERO_FLOAT32, "core.matrix-multiply")
    bs = native.resolve(native.TRANSFORMER_FLOAT32, "transformer.batch-shared-matvec")
    assert len({mv, mv16, mm, bs}) == 4
    # collection not installed / no CUDA implementation -> NotSupportedException
    with pytest.raises(native.NotSupportedError):
        native.resolve("11111111-2222-3333-4444-555555555555", "core.mat-vec")
    with pytest.raises(native.NotSupportedError):
        native.resolve(native.TIER_ZERO_FLOAT32, "core.copy")
    with pytest.raises(native.NotSupportedError):
        native.resolve(native.TRANSFORMER_FLOAT32, "core.gather-row")  # a tier-zero instruction


# The 22 names of GpuTransformerInstructionCollection.cs:8-33 with their port types.
TRANSFORMER_PORTS = {
    "transformer.rms-norm": "fff", "transformer.residual-rms-norm": "fffff", "transformer.swiglu": "ff",
    "transformer.rope-kv-write": "fiffff", "transformer.gqa-scores": "ffif", "transformer.causal-softmax": "fif",
    "transformer.gqa-values": "ffif", "transformer.grouped-query-attention": "fffif", "transformer.argmax": "fi",
    "transformer.scaled-add": "fff", "transformer.embedding-gather-batch": "hif",
    "transformer.copy-embedding-rows": "ff", "transformer.batch-rms-norm": "ffif",
    "transformer.batch-residual-rms-norm": "fffiff", "transformer.batch-shared-matvec": "hfif",
    "transformer.batch-swiglu": "fif", "transformer.batch-rope-kv-write": "fiffff",
    "transformer.batch-gqa-scores": "ffif", "transformer.batch-causal-softmax": "fif",
    "transformer.batch-gqa-values": "ffif", "transformer.batch-select-last": "fif",
    "transformer.batch-gather-rows": "fif",
}


def test_registry_covers_every_transformer_instruction():
    code = {"f": N.F32, "i": N.I32, "h": N.F16}
    ids = set()
    for name, ports in TRANSFORMER_PORTS.items():
        iid = native.resolve(native.TRANSFORMER_FLOAT32, name)
        ids.add(iid)
        types = [code[c] for c in ports]
        native.validate(iid, types)
        wrong = list(types)
        wrong[-1] = N.F16 if wrong[-1] != N.F16 else N.F32
        with pytest.raises(native.InstructionAdaptationError):
            native.validate(iid, wrong)
        with pytest.raises(native.InstructionAdaptationError):
            native.validate(iid, types[:-1])
        with pytest.raises(native.InstructionAdaptationError):
            native.validate(iid, types, "some-config")
    assert len(ids) == len(TRANSFORMER_PORTS) == 22
    gr = native.resolve(native.TIER_ZERO_FLOAT32, "core.gather-row")
    for t in (N.F32, N.F16, N.Q8_0, N.Q4_K):
        native.validate(gr, [t, N.I32, N.F32])
    with pytest.raises(native.InstructionAdaptationError):
        native.validate(gr, [N.F32, N.F32, N.F32])


def test_transformer_entry_points_reject_bad_shapes_on_the_host():
    lib = native.lib
    f = FAKE
    # rope: odd rotary size, rotary above head size, query not whole heads (rope-kv-write Generate)
    assert lib.si_rope_kv_write(f, f, f, f, f, f, 256, 1, 128, 95, 16, 1.0, None) == N.SI_ERR_ADAPTATION
    assert lib.si_rope_kv_write(f, f, f, f, f, f, 256, 1, 128, 130, 16, 1.0, None) == N.SI_ERR_ADAPTATION
    assert lib.si_rope_kv_write(f, f, f, f, f, f, 200, 1, 128, 96, 16, 1.0, None) == N.SI_ERR_ADAPTATION
    assert lib.si_rope_kv_write(f, f, f, f, f, f, 256, 1, 128, 96, 16, 0.0, None) == N.SI_ERR_ADAPTATION
    # attention: heads not divisible
    assert lib.si_grouped_query_attention(f, f, f, f, f, 24, 7, 128, 64, None) == N.SI_ERR_ADAPTATION
    assert "divisible" in native.last_error()
    assert lib.si_gqa_scores(f, f, f, f, 6, 4, 32, 16, None) == N.SI_ERR_ADAPTATION
    # norms: epsilon must be finite and positive
    assert lib.si_rms_norm(f, f, f, 16, 0.0, None) == N.SI_ERR_ADAPTATION
    assert lib.si_residual_rms_norm(f, f, f, f, f, 16, float("nan"), None) == N.SI_ERR_ADAPTATION
    assert lib.si_scaled_add(f, f, f, 16, -2.0, None) == N.SI_ERR_ADAPTATION
    assert lib.si_copy_embedding_rows(f, f, 4, 0, 8, 0, None) == N.SI_ERR_ADAPTATION
    assert lib.si_copy_embedding_rows(f, f, 4, 2, 8, 3, None) == N.SI_ERR_ADAPTATION
    assert lib.si_argmax(f, 0, f, None) == N.SI_ERR_ADAPTATION
    assert lib.si_gather_row(N.Q4_K, f, 4, 300, f, f, None) == N.SI_ERR_INVALID_DATA
    assert lib.si_gather_row(99, f, 4, 256, f, f, None) == N.SI_ERR_UNSUPPORTED


def test_decoder_config_is_validated_before_any_device_call():
    base = dict(layers=2, hidden=256, query_heads=2, kv_heads=1, head_size=128, rotary_size=96, intermediate=512,
                vocab=640, context=64, epsilon=1e-5, rope_base=10000.0, rope_scale=1.0, weight_type=N.Q4_K,
                embedding_type=N.Q4_K)
    for change, err in [({"query_heads": 3}, native.InstructionAdaptationError),
                        ({"kv_heads": 3, "query_heads": 2}, native.InstructionAdaptationError),
                        ({"rotary_size": 97}, native.InstructionAdaptationError),
                        ({"intermediate": 500}, native.InvalidDataError),
                        ({"layers": 0}, native.ArgumentError),
                        ({"weight_type": 99}, native.NotSupportedError)]:
        cfg = dict(base, **change)
        with pytest.raises(err):
            native.Decoder(cfg)


def test_session_variants_and_fused_attention_validate_on_the_host():
    """The multi-stream and row-sharded sessions and the fused batch
    attention check their arguments before touching a device."""
    lib = native.lib
    base = dict(layers=2, hidden=256, query_heads=2, kv_heads=1, head_size=128, rotary_size=96, intermediate=512,
                vocab=640, context=64, epsilon=1e-5, rope_base=10000.0, rope_scale=1.0, weight_type=N.Q4_K,
                embedding_type=N.Q4_K)
    with pytest.raises(native.ArgumentError):
        native.Decoder(base, streams=0)
    with pytest.raises(native.InstructionAdaptationError):
        native.Decoder(dict(base, query_heads=3), streams=4)
    # arena bytes: the four per-layer projection outputs twice (even / odd
    # layers) and the logits, each 256-byte aligned, + 4 KB of state
    qkv = 256 + 2 * 128
    al = lambda n: (n * 4 + 255) // 256 * 256  # noqa: E731
    want = 2 * sum(al(n) for n in (qkv, 256, 2 * 512, 256)) + al(640) + 4096
    assert native.decoder_arena_bytes(base) == want
    with pytest.raises(native.InstructionAdaptationError):
        native.decoder_arena_bytes(dict(base, rotary_size=97))
    h = C.c_void_p()
    cfg = native.DecoderConfig(**base)
    assert lib.si_decoder_create_sharded(0, C.byref(cfg), None, 0, C.byref(h)) == N.SI_ERR_INVALID_ARGUMENT
    f = FAKE
    assert lib.si_batch_grouped_query_attention(f, f, f, 0, 0, f, 2, 1, 128, 64, None) == N.SI_ERR_ADAPTATION
    assert lib.si_batch_grouped_query_attention(f, f, f, 0, 4, f, 3, 2, 128, 64, None) == N.SI_ERR_ADAPTATION
    assert lib.si_batch_grouped_query_attention(f, f, f, 0, 4, f, 2, 1, 96, 64, None) == N.SI_ERR_UNSUPPORTED
    assert lib.si_synth_weight_rows_device(N.Q4_K, 1, 0, 1, 256, 0.02, f, None) == N.SI_ERR_UNSUPPORTED
    assert lib.si_synth_weight_rows_device(N.Q8_0, 1, 0, 1, 48, 0.02, f, None) == N.SI_ERR_INVALID_ARGUMENT


def test_registry_signatures_and_configurations():
    mv = native.resolve(native.TIER_ZERO_FLOAT32, "core.mat-vec")
    for wt in (N.F32, N.F16, N.Q8_0, N.Q4_K):
        native.validate(mv, [wt, N.F32, N.F32])
    native.validate(mv, [N.F16, N.F32, N.F32], "cooperative-matvec")
    native.validate(mv, [N.Q4_K, N.F32, N.F32], "cuda-gemv-staged")
    with pytest.raises(native.InstructionAdaptationError):
        native.validate(mv, [N.Q4_K, N.F32, N.F32], "cooperative-matvec")
    with pytest.raises(native.InstructionAdaptationError):
        native.validate(mv, [N.F32, N.F32, N.F32], "missing")  # unknown configuration
    with pytest.raises(native.InstructionAdaptationError):
        native.validate(mv, [N.F16, N.F16, N.F16])
    mv16 = native.resolve(native.TIER_ZERO_FLOAT16, "core.mat-vec")
    native.validate(mv16, [N.F16, N.F16, N.F16])
    bs = native.resolve(native.TRANSFORMER_FLOAT32, "transformer.batch-shared-matvec")
    native.validate(bs, [N.Q4_K, N.F32, N.I32, N.F32])
    with pytest.raises(native.InstructionAdaptationError):
        native.validate(bs, [N.F32, N.F32, N.I32, N.F32])
    mm = native.resolve(native.TIER_ZERO_FLOAT32, "core.matrix-multiply")
    native.validate(mm, [N.F32, N.Q8_0, N.F32])
    with pytest.raises(native.InstructionAdaptationError):
        native.validate(mm, [N.Q8_0, N.F32, N.F32])


def test_last_error_is_thread_local():
    import threading
    _mv(rows=0)
    msg = native.last_error()
    seen = []

    def other():
        _mv(wtype=99)
        seen.append(native.last_error())

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert native.last_error() == msg
    assert seen and seen[0] != msg
