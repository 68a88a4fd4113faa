"""Shared test helpers: golden fixtures, the parity gates and device I/O."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
TYPES = {"F32": 0, "F16": 1, "Q8_0": 8, "Q4_K": 12}


def known_answers() -> dict:
    return json.loads((GOLDEN / "reference_known_answers.json").read_text())


def cooperative_fixture():
    return np.load(GOLDEN / "cooperative_matvec.npz")


def fnum(v):
    return float(v) if not isinstance(v, str) else float(v.replace("inf", "inf"))


def reference_gate(actual, expected, rel=3e-5, abs_=3e-5):
    """Operator gate of the reference (GpuMatVecTests.cs:307-311):
    NaN stays NaN, +/-Inf equal, otherwise |d| <= 3e-5 + 3e-5 |ref|."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape
    nan = np.isnan(expected)
    assert np.all(np.isnan(actual[nan])), "NaN class lost"
    inf = np.isinf(expected)
    assert np.array_equal(actual[inf], expected[inf]), "Inf class lost"
    fin = ~(nan | inf)
    err = np.abs(actual[fin] - expected[fin])
    bound = abs_ + rel * np.abs(expected[fin])
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, f"{bad.size} elements outside 3e-5+3e-5|ref|; first {bad[:5]}, err {err[bad[:5]]}"


def north_star_gate(actual, reference, x, row_norm_max, k):
    """Parity gate for quantized mat-vec / GEMM outputs:
    max|d| <= 1e-3 * ||x||_2 * max_row ||W||_2 / sqrt(K) and relative L2 <= 1e-4."""
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    r = np.asarray(reference, dtype=np.float64).reshape(-1)
    assert np.all(np.isfinite(a)), "non-finite output"
    d = a - r
    bound = 1e-3 * float(np.linalg.norm(np.asarray(x, dtype=np.float64))) * row_norm_max / np.sqrt(k)
    max_abs = float(np.max(np.abs(d))) if d.size else 0.0
    rel_l2 = float(np.linalg.norm(d) / max(np.linalg.norm(r), 1e-300))
    assert max_abs <= bound, f"max|d| {max_abs:.3e} > bound {bound:.3e}"
    assert rel_l2 <= 1e-4, f"relative L2 {rel_l2:.3e} > 1e-4"
    return max_abs, rel_l2


def row_norm_max(wtype: int, blob: np.ndarray, rows: int, cols: int) -> float:
    import oracle
    rb = oracle.byte_length(wtype, cols)
    best = 0.0
    step = max(1, rows // 2048)  # bound the cost on the largest shapes
    for r in range(0, rows, step):
        w = oracle.dequantize(wtype, blob[r * rb:(r + 1) * rb], cols)
        best = max(best, float(np.linalg.norm(w.astype(np.float64))))
    return best


def to_f16_bytes(values) -> np.ndarray:
    return np.asarray(values, dtype=np.float32).astype(np.float16).view(np.uint8)
