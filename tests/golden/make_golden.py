"""Writes the golden fixtures that pin the CPU oracle and the CUDA kernels to
the reference's own known-answer tests.

The reference is C#/.NET + Direct3D 12 and cannot run here, so each fixture
is restated from the test source that holds it (inputs and expected values
exactly as that test constructs them; cited per case):

  reference_known_answers.json  small known-answer cases
  cooperative_matvec.npz        GpuMatVecTests shapes x signatures, with the
                                double-precision expected values that test
                                computes
  transformer_known_answers.json  GpuTransformerInstructionTests cases, with
                                the expected values computed the way each
                                test computes them

Run:  python tests/golden/make_golden.py   (deterministic; no inputs needed)
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def known_answers() -> dict:
    cases = {}
    # CpuVmMixedWeightsTests.cs:95-104 -- FP16 weights, FP32 accumulation:
    # half accumulation would lose the unit terms next to 2048.
    matrix = [2048, 1, -2048, 1, 0, 0, 0, 0, 2, 0.5, 4, -1, 0, 0, 0, 0]
    cases["mixed_weights_matvec"] = {
        "source": "src/SharpInference.Tests/CpuVmMixedWeightsTests.cs:95-104",
        "weight_type": "F16", "rows": 2, "cols": 8,
        "matrix": matrix, "input": [1.0] * 8, "expected": [2.0, 5.5],
    }
    # Same matrix, batched form: the second input row is all 2s
    # (CpuVmMixedWeightsTests.cs:98-103, expected [2, 5.5, 4, 11]).
    cases["mixed_weights_batched"] = {
        "source": "src/SharpInference.Tests/CpuVmMixedWeightsTests.cs:98-103",
        "weight_type": "F16", "batch": 2, "rows": 2, "cols": 8,
        "matrix": matrix, "input": [1.0] * 8 + [2.0] * 8, "expected": [2.0, 5.5, 4.0, 11.0],
    }
    # CpuVmMixedWeightsTests.cs:62-72 -- bounded conversion blocks and parallel
    # rows: all-ones FP16 matrix times 0.25 gives columns * 0.25 exactly.
    cases["bounded_conversion_blocks"] = {
        "source": "src/SharpInference.Tests/CpuVmMixedWeightsTests.cs:62-72",
        "shapes": [[3, 2051], [64, 1024]], "matrix_value": 1.0, "input_value": 0.25,
        "expected_per_row": "columns * 0.25",
    }
    # GpuMatVecTests.cs:41-52 -- cancellation across and within lanes.
    cases["cooperative_cancellation"] = {
        "source": "src/SharpInference.Tests/GpuMatVecTests.cs:41-52",
        "rows": 3, "cols": 4096, "matrix_value": 1.0, "input_value": 1.0,
        "big": 100000000.0, "final_indices": [4095, 4032], "expected": [4094.0, 4094.0, 4094.0],
    }
    # GpuMatVecTests.cs:54-67 -- non-finite sums keep their class.
    cases["cooperative_nonfinite"] = {
        "source": "src/SharpInference.Tests/GpuMatVecTests.cs:54-67",
        "rows": 3, "cols": 2, "matrix_value": 1.0,
        "inputs": [["inf", 1.0], ["-inf", 1.0], ["inf", "-inf"], ["nan", 1.0]],
        "expected": ["inf", "-inf", "nan", "nan"],
    }
    # GpuMatVecTests.cs:69-85,87-114 and GpuMatVecExecution.cs:15-24 -- launch
    # geometry: Groups(65536) = (32768, 2); rows > uint.MaxValue / 64 rejected.
    cases["matvec_grid"] = {
        "source": "src/SharpInference.Tests/GpuMatVecTests.cs:69-85,113; "
                  "src/SharpInference.Instructions/GpuMatVecExecution.cs:15-24",
        "rows": 65536, "cols": 3, "groups": [32768, 2], "input": [1.0, 2.0, 3.0], "expected_value": 6.0,
        "max_rows": 0xFFFFFFFF // 64, "rejected_rows": 0xFFFFFFFF,
    }
    # GpuTransformerInstructionTests.cs:280-324 -- batch-shared-matvec with
    # validCount = 2 of 3 rows; the third output row keeps its -31 fill.
    cases["batch_shared_matvec"] = {
        "source": "src/SharpInference.Tests/GpuTransformerInstructionTests.cs:280-324",
        "weight_type": "F16", "batch": 3, "in_features": 4, "out_features": 2,
        "weight": [1, -0.5, 2, 0.25, -1, 3, 0.5, -2],
        "input": [2, 4, -1, 8, -3, 1, 2, -2, 9, 9, 9, 9],
        "control": [0, 2], "fill": -31.0, "expected": [0, -6.5, 0, 11, -31, -31],
    }
    # GgufModelFile.cs:301-331 -- byte lengths; Q4_K is new (the reference
    # throws NotSupportedException for it at :320).
    cases["byte_lengths"] = {
        "source": "src/SharpInference.Gguf/GgufModelFile.cs:301-331",
        "cases": [
            {"type": "F32", "dims": [7, 3], "bytes": 84},
            {"type": "F16", "dims": [7, 3], "bytes": 42},
            {"type": "Q8_0", "dims": [8192, 3072], "bytes": 26738688},
            {"type": "Q8_0", "dims": [32], "bytes": 34},
            {"type": "Q4_K", "dims": [256], "bytes": 144},
            {"type": "Q4_K", "dims": [5120, 3072], "bytes": 8847360},
            {"type": "Q4_K", "dims": [200064, 3072], "bytes": 345710592},
        ],
        "invalid_data": [{"type": "Q8_0", "dims": [33]}, {"type": "Q4_K", "dims": [3, 100]}],
        "unsupported_type": 99,
    }
    return cases


def _avg_f32(values) -> np.float32:
    """Enumerable.Average over floats: double accumulation, float result."""
    return np.float32(np.sum(np.asarray(values, dtype=np.float64)) / len(values))


def _rms_expected(row, weight, eps=np.float32(1e-5)):
    row = np.asarray(row, dtype=np.float32)
    scale = np.float32(1.0) / np.sqrt(_avg_f32(row * row) + eps, dtype=np.float32)
    return (row * scale * np.asarray(weight, dtype=np.float32)).astype(np.float32)


def _attention_reference(qkv, key_cache, value_cache, batch, qh, kvh, hs, start):
    """AttentionReference of GpuTransformerInstructionTests.cs:514-559."""
    qsize, kvsize = qh * hs, kvh * hs
    width = qsize + 2 * kvsize
    out = np.zeros(batch * qsize, dtype=np.float64)
    for row in range(batch):
        active = start + row
        for head in range(qh):
            kv = head // (qh // kvh)
            scores = np.array([sum(qkv[row * width + head * hs + d] * key_cache[(t * kvh + kv) * hs + d]
                                   for d in range(hs)) for t in range(active + 1)]) / np.sqrt(hs)
            e = np.exp(scores - scores.max())
            for d in range(hs):
                out[row * qsize + head * hs + d] = sum(e[t] / e.sum() * value_cache[(t * kvh + kv) * hs + d]
                                                       for t in range(active + 1))
    return out


def transformer_known_answers() -> dict:
    src = "src/SharpInference.Tests/GpuTransformerInstructionTests.cs"
    cases = {}
    hidden = [1, -2, 3, -4, 5, -6, 7, -8]
    residual = [0.5, 1, -1.5, 2, -2.5, 3, -3.5, 4]
    weight = [1, 0.5, 1.5, 2, 0.75, 1.25, 0.25, 1.75]
    updated = (np.float32(hidden) + np.float32(residual)).astype(np.float32)
    cases["residual_rms_norm"] = {
        "source": f"{src}:12-78", "epsilon": 1e-5, "hidden": hidden, "residual": residual, "weight": weight,
        "expected_updated": updated.tolist(), "expected_output": _rms_expected(updated, weight).tolist(),
        "tolerance": 1e-5,
    }
    gate_up = np.float32([-2, -1, 1, 2, 0.5, 1.5, -2, 3])
    g, u = gate_up[:4], gate_up[4:]
    cases["swiglu"] = {
        "source": f"{src}:80-137", "gate_up": gate_up.tolist(),
        "expected": (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32).tolist(), "tolerance": 1e-5,
    }
    cases["scaled_add"] = {
        "source": f"{src}:139-185", "input": [1, -2, 3, -4], "update": [0.5, 1, -1.5, 2], "scale": 2.0,
        "expected": [2, 0, 0, 0], "tolerance": 1e-5,
    }
    rms_in = np.float32([1, -2, 3, -4, 5, 2, 4, -1, -3, 0.5, 9, 9, 9, 9, 9]).reshape(3, 5)
    rms_w = [1, 0.5, 1.5, 2, 0.25]
    expected = np.full((3, 5), -77.0, dtype=np.float32)
    for row in range(2):
        expected[row] = _rms_expected(rms_in[row], rms_w)
    cases["batch_rms_norm"] = {
        "source": f"{src}:187-235", "epsilon": 1e-5, "batch": 3, "width": 5, "input": rms_in.reshape(-1).tolist(),
        "weight": rms_w, "control": [7, 2], "fill": -77.0, "expected": expected.reshape(-1).tolist(),
        "tolerance": 1e-5,
    }
    cases["batch_gather_rows"] = {
        "source": f"{src}:237-277", "rows": 5, "batch": 4, "width": 3,
        "table": [0, 1, 2, 10, 11, 12, 20, 21, 22, 30, 31, 32, 40, 41, 42], "control": [2, 2], "fill": -17.0,
        "expected": [20, 21, 22, 30, 31, 32, -17, -17, -17, -17, -17, -17], "tolerance": 1e-5,
    }
    qkv = [1, 0, 0, 1, 1, 1, 10, 20, 1, 1, 2, 0, 0, 2, 30, 40]
    exp_k = [1, 0, 1, 1, 0, 2, -9, -9]
    exp_v = [2, 4, 10, 20, 30, 40, -8, -8]
    cases["batch_attention"] = {
        "source": f"{src}:327-441,514-559", "batch": 2, "query_heads": 2, "kv_heads": 1, "head_size": 2,
        "context": 4, "rotary_size": 2, "rope_scale": 1.0, "frequencies": [0.0], "qkv": qkv, "control": [1, 2],
        "key_cache": [1, 0, -9, -9, -9, -9, -9, -9], "value_cache": [2, 4, -8, -8, -8, -8, -8, -8],
        "expected_key_cache": exp_k, "expected_value_cache": exp_v,
        "expected_output": _attention_reference(qkv, exp_k, exp_v, 2, 2, 1, 2, 1).tolist(),
        "cache_tolerance": 1e-5, "output_tolerance": 2e-5,
    }
    return cases


# GpuMatVecTests.cs:13-39: shapes x signatures, values (i%9-4)*0.125 and
# (i%7-3)*0.25, expected = (float) double-precision row sum, rounded through
# Half for an FP16 output; padding sentinel 13 around every buffer.
SHAPES = [(1, 1), (7, 17), (7, 63), (7, 64), (7, 65), (3, 4096), (65536, 3), (65537, 3)]
SIGNATURES = [("F32", "F32", "F32"), ("F16", "F32", "F32"), ("F16", "F16", "F16")]


def cooperative_fixture() -> dict:
    out = {}
    for rows, cols in SHAPES:
        matrix = ((np.arange(rows * cols) % 9 - 4) * 0.125).astype(np.float32)
        vector = ((np.arange(cols) % 7 - 3) * 0.25).astype(np.float32)
        exact = (matrix.reshape(rows, cols).astype(np.float64) @ vector.astype(np.float64)).astype(np.float32)
        out[f"expected_{rows}x{cols}_f32"] = exact
        out[f"expected_{rows}x{cols}_f16"] = exact.astype(np.float16).astype(np.float32)
    out["shapes"] = np.array(SHAPES, dtype=np.int64)
    return out


def main() -> None:
    (HERE / "reference_known_answers.json").write_text(json.dumps(known_answers(), indent=1) + "\n")
    np.savez_compressed(HERE / "cooperative_matvec.npz", **cooperative_fixture())
    (HERE / "transformer_known_answers.json").write_text(json.dumps(transformer_known_answers(), indent=1) + "\n")
    print("wrote", HERE / "reference_known_answers.json", HERE / "cooperative_matvec.npz",
          HERE / "transformer_known_answers.json")


if __name__ == "__main__":
    main()
