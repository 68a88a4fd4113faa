"""Child process of test_gemv_plans_gpu.py: runs the Q4_K and Q8_0 GEMV on
lists of shapes under the launch shape given in SI_Q4K_GEMV_PLAN (read once per
process by the library) and prints one JSON line of per-shape parity results."""
import json
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import oracle  # noqa: E402
from helpers import north_star_gate, row_norm_max  # noqa: E402
from sharpinference_b200 import native  # noqa: E402

SHAPES = [(1, 256), (37, 512), (77, 1024), (300, 3072), (1000, 2048), (4099, 768), (513, 8192), (3072, 4096),
          (40, 12288)]
Q8_SHAPES = [(1, 256), (37, 512), (300, 3072), (1000, 5120), (4099, 768), (50, 17920), (20, 12288), (129, 8192)]


def main() -> None:
    out = []
    cases = [(native.Q4_K, r, c) for r, c in SHAPES] + [(native.Q8_0, r, c) for r, c in Q8_SHAPES]
    with native.Context(0) as ctx:
        for i, (wt, rows, cols) in enumerate(cases):
            blob = native.synth_weights(wt, 700 + i, rows, cols, 0.02)
            x = native.synth_normal(1700 + i, cols, 1.0)
            W, X, Y = ctx.buffer(blob.nbytes), ctx.buffer(4 * cols), ctx.buffer(4 * rows)
            W.upload(blob), X.upload(x)
            ctx.matvec(wt, W, X, Y, rows, cols)
            y = Y.readback().view(np.float32).copy()
            ref = oracle.matvec(wt, blob, x, rows, cols)
            entry = {"type": wt, "rows": rows, "cols": cols}
            try:
                entry["max_abs"], entry["rel_l2"] = north_star_gate(y, ref, x, row_norm_max(wt, blob, rows, cols),
                                                                    cols)
                entry["ok"] = True
            except AssertionError as e:
                entry["ok"], entry["why"] = False, str(e)
            out.append(entry)
            W.free(), X.free(), Y.free()
        err = native.device_error_take(0)
    print(json.dumps({"shapes": out, "device_error_word": err}), flush=True)


if __name__ == "__main__":
    main()
