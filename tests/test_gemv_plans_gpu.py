"""Every launch shape of the tensor-core Q4_K and Q8_0 GEMV (K split over
1..8-CTA clusters, 16/32-row tiles, full or half shared-memory ring, one or
two CTAs per SM, one or two superblocks per warp, FP16 or INT8 MMA path, one
or two warps per superblock column) against the oracle on ragged shapes.
Each shape is passed explicitly through si_matvec_quant_planned."""
import numpy as np
import pytest

import oracle
from helpers import north_star_gate, row_norm_max
from sharpinference_b200 import native

pytestmark = pytest.mark.gpu

SHAPES = [(1, 256), (37, 512), (77, 1024), (300, 3072), (1000, 2048), (4099, 768), (513, 8192), (3072, 4096),
          (40, 12288)]
Q8_SHAPES = [(1, 256), (37, 512), (300, 3072), (1000, 5120), (4099, 768), (50, 17920), (20, 12288), (129, 8192)]

# (cluster, rows_per_tile, smem_kb, mma_path, warps_per_column, superblocks_per_warp, ctas_per_sm, max_groups)
PLANS = [(1, 16, 100, 0, 1, 0, 1, 0), (1, 32, 220, 0, 1, 0, 1, 0), (2, 16, 100, 0, 1, 0, 1, 0),
         (2, 32, 220, 0, 1, 0, 1, 0), (4, 16, 100, 0, 1, 0, 1, 0), (4, 32, 64, 0, 1, 0, 1, 0),
         (1, 16, 100, 1, 1, 0, 1, 0), (1, 32, 220, 1, 1, 0, 1, 0), (2, 16, 100, 1, 1, 0, 1, 0),
         (2, 32, 220, 1, 1, 0, 1, 0), (4, 32, 64, 1, 1, 0, 1, 0), (1, 32, 226, 1, 2, 0, 1, 0),
         (2, 32, 226, 1, 2, 0, 1, 0), (4, 32, 120, 1, 2, 0, 1, 0), (3, 16, 226, 1, 1, 0, 1, 0),
         (5, 32, 226, 1, 1, 0, 1, 0), (8, 16, 160, 1, 1, 0, 1, 0),
         # two CTAs per SM (half the shared memory each), two superblocks per warp
         (1, 16, 112, 1, 1, 2, 2, 0), (1, 32, 112, 1, 1, 2, 2, 0), (2, 16, 112, 1, 1, 2, 2, 0),
         (2, 16, 112, 1, 1, 0, 2, 0), (4, 16, 112, 1, 1, 0, 2, 0), (1, 16, 112, 0, 1, 2, 2, 0),
         (1, 16, 112, 1, 1, 1, 2, 7), (4, 32, 112, 1, 1, 2, 2, 0)]


def _cases():
    return [(native.Q4_K, r, c) for r, c in SHAPES] + [(native.Q8_0, r, c) for r, c in Q8_SHAPES]


@pytest.fixture(scope="module")
def data():
    out = []
    for i, (wt, rows, cols) in enumerate(_cases()):
        blob = native.synth_weights(wt, 700 + i, rows, cols, 0.02)
        x = native.synth_normal(1700 + i, cols, 1.0)
        out.append((wt, rows, cols, blob, x, oracle.matvec(wt, blob, x, rows, cols)))
    return out


def test_default_plan_is_reported():
    p = native.gemv_default_plan(native.Q4_K, 200064, 3072)
    assert p.rows_per_tile in (16, 32) and p.ctas_per_sm in (1, 2) and 1 <= p.cluster <= 8
    with pytest.raises(native.NotSupportedError):
        native.gemv_default_plan(native.F32, 8, 256)


def test_plan_fields_are_validated(ctx):
    W, X, Y = ctx.buffer(144 * 4), ctx.buffer(4 * 256), ctx.buffer(16)
    for bad in (dict(cluster=9), dict(rows_per_tile=8), dict(smem_kb=16), dict(ctas_per_sm=3),
                dict(ctas_per_sm=2, smem_kb=200), dict(superblocks_per_warp=3), dict(mma_path=2)):
        with pytest.raises(native.ArgumentError):
            ctx.matvec_planned(native.Q4_K, W, X, Y, 4, 256, native.gemv_plan(**bad))
    for b in (W, X, Y):
        b.free()


@pytest.mark.parametrize("plan", PLANS, ids=lambda p: ",".join(map(str, p)))
def test_launch_shape_parity(ctx, data, plan):
    fields = dict(zip(("cluster", "rows_per_tile", "smem_kb", "mma_path", "warps_per_column",
                       "superblocks_per_warp", "ctas_per_sm", "max_groups"), plan))
    ran = 0
    for wt, rows, cols, blob, x, ref in data:
        W, X, Y = ctx.buffer(blob.nbytes), ctx.buffer(4 * cols), ctx.buffer(4 * rows)
        W.upload(blob), X.upload(x)
        try:
            ctx.matvec_planned(wt, W, X, Y, rows, cols, native.gemv_plan(**fields))
        except native.NotSupportedError:
            W.free(), X.free(), Y.free()
            continue  # this shape cannot cover the matrix (e.g. K slice too long for one superblock per warp)
        ctx.synchronize()
        y = Y.readback().view(np.float32).copy()
        north_star_gate(y, ref, x, row_norm_max(wt, blob, rows, cols), cols)
        ran += 1
        W.free(), X.free(), Y.free()
    assert ran >= len(data) // 2
    assert native.device_error_take(0) == 0
