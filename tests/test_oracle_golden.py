"""Pins the CPU oracle to the reference's own known-answer tests
(fixtures in tests/golden/, restated from the cited C# tests)."""
import math

import numpy as np
import pytest

import oracle
from helpers import cooperative_fixture, known_answers, TYPES

KA = known_answers()


def _f16(values):
    return np.asarray(values, dtype=np.float32).astype(np.float16).view(np.uint8)


def test_mixed_weights_cpu_matvec_exact():
    c = KA["mixed_weights_matvec"]
    y = oracle.matvec(oracle.F16, _f16(c["matrix"]), np.array(c["input"], np.float32), c["rows"], c["cols"])
    assert y.tolist() == c["expected"]


def test_mixed_weights_batched_exact():
    c = KA["mixed_weights_batched"]
    w = _f16(c["matrix"])
    x = np.array(c["input"], np.float32).reshape(c["batch"], c["cols"])
    y = oracle.matrix_multiply_tr(oracle.F16, x, w, c["batch"], c["rows"], c["cols"])
    assert y.tolist() == c["expected"]
    out = oracle.batch_shared_matvec(oracle.F16, w, x, [0, c["batch"]], np.zeros(c["batch"] * c["rows"]),
                                     c["batch"], c["rows"], c["cols"])
    assert out.tolist() == c["expected"]


@pytest.mark.parametrize("shape", KA["bounded_conversion_blocks"]["shapes"])
def test_bounded_conversion_blocks(shape):
    rows, cols = shape
    w = _f16(np.ones(rows * cols))
    y = oracle.matvec(oracle.F16, w, np.full(cols, 0.25, np.float32), rows, cols)
    assert np.all(y == np.float32(cols * 0.25))


@pytest.mark.parametrize("final", KA["cooperative_cancellation"]["final_indices"])
@pytest.mark.parametrize("lanes", [64, 32])
def test_cooperative_cancellation(final, lanes):
    c = KA["cooperative_cancellation"]
    x = np.ones(c["cols"], np.float32)
    x[0] = c["big"]
    x[final] = -c["big"]
    w = np.ones(c["rows"] * c["cols"], np.float32)
    y = oracle.matvec_cooperative(oracle.F32, oracle.F32, oracle.F32, w, x, c["rows"], c["cols"], lanes)
    assert y.tolist() == c["expected"]


@pytest.mark.parametrize("case", range(4))
@pytest.mark.parametrize("lanes", [64, 32])
def test_cooperative_nonfinite(case, lanes):
    c = KA["cooperative_nonfinite"]
    x = np.array([float(v) for v in c["inputs"][case]], np.float32)
    expected = float(c["expected"][case])
    y = oracle.matvec_cooperative(oracle.F32, oracle.F32, oracle.F32, np.ones(6, np.float32), x, 3, 2, lanes)
    for v in y:
        if math.isnan(expected):
            assert math.isnan(v)
        else:
            assert v == expected


@pytest.mark.parametrize("sig", [("F32", "F32", "F32"), ("F16", "F32", "F32"), ("F16", "F16", "F16")])
@pytest.mark.parametrize("lanes", [64, 32])
def test_cooperative_signatures_match_reference_expectations(sig, lanes):
    fx = cooperative_fixture()
    wt, xt, yt = (TYPES[s] for s in sig)
    for rows, cols in fx["shapes"]:
        rows, cols = int(rows), int(cols)
        m = ((np.arange(rows * cols) % 9 - 4) * 0.125).astype(np.float32)
        v = ((np.arange(cols) % 7 - 3) * 0.25).astype(np.float32)
        w = m.astype(np.float16) if wt == oracle.F16 else m
        x = v.astype(np.float16) if xt == oracle.F16 else v
        y = oracle.matvec_cooperative(wt, xt, yt, w, x, rows, cols, lanes).astype(np.float32)
        expected = fx[f"expected_{rows}x{cols}_{'f16' if yt == oracle.F16 else 'f32'}"]
        err = np.abs(y - expected)
        assert np.all(err <= 3e-5 + 3e-5 * np.abs(expected)), (rows, cols, sig)


def test_batch_shared_known_answer():
    c = KA["batch_shared_matvec"]
    out = oracle.batch_shared_matvec(oracle.F16, _f16(c["weight"]), np.array(c["input"], np.float32), c["control"],
                                     np.full(c["batch"] * c["out_features"], c["fill"], np.float32), c["batch"],
                                     c["out_features"], c["in_features"])
    assert out.tolist() == c["expected"]


def test_byte_lengths():
    c = KA["byte_lengths"]
    for case in c["cases"]:
        assert oracle.byte_length(TYPES[case["type"]], int(np.prod(case["dims"]))) == case["bytes"]
    for case in c["invalid_data"]:
        with pytest.raises(ValueError):
            oracle.byte_length(TYPES[case["type"]], int(np.prod(case["dims"])))
    with pytest.raises(ValueError):
        oracle.byte_length(c["unsupported_type"], 32)


def test_grid_fixture_values():
    c = KA["matvec_grid"]
    rows = c["rows"]
    # GpuMatVecExecution.Groups restated: y = ceil(rows/65535), x = ceil(rows/y)
    y = (rows + 65534) // 65535
    x = (rows + y - 1) // y
    assert [x, y] == c["groups"]
    w = np.ones(rows * c["cols"], np.float32)
    out = oracle.matvec(oracle.F32, w, np.array(c["input"], np.float32), rows, c["cols"])
    assert np.all(out == c["expected_value"])
