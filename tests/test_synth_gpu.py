"""Device-side synthetic weights (si_synth_weight_rows_device) against the
host generator: the same seeded matrix rows, byte-identical except where the
device library's double log/sin/cos moved a rounding boundary."""
import numpy as np
import pytest

from sharpinference_b200 import native as N

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wt,rows,cols,begin", [(N.F32, 33, 256, 5), (N.F16, 64, 4096, 7),
                                                (N.Q8_0, 300, 5120, 0), (N.Q8_0, 257, 3072, 1000)])
def test_device_rows_match_host_rows(ctx, wt, rows, cols, begin):
    host = N.synth_weight_rows(wt, 11, begin, rows, cols, 0.02)
    buf = ctx.buffer(host.nbytes)
    try:
        N.synth_weight_rows_device(wt, 11, begin, rows, cols, 0.02, buf.device_pointer, ctx.stream)
        ctx.synchronize()
        dev = buf.readback().view(np.uint8)
    finally:
        buf.free()
    same = float(np.mean(dev == host))
    diag = ""
    if same < 0.9999:
        if wt == N.F32:
            a, b = dev.view(np.float32), host.view(np.float32)
            bad = np.nonzero(a != b)[0]
            diag = f"f32 mismatches {bad.size}: first {bad[:8].tolist()} dev {a[bad[:4]].tolist()} host {b[bad[:4]].tolist()}"
        elif wt == N.Q8_0:
            pos = (np.nonzero(dev != host)[0] % 34)
            diag = f"scale-byte mismatches {int(np.sum(pos < 2))}, quant-byte mismatches {int(np.sum(pos >= 2))}"
    assert same >= 0.9999, (same, diag)
    if wt == N.F32:
        np.testing.assert_allclose(dev.view(np.float32), host.view(np.float32), rtol=1e-6, atol=0)


def test_device_synthesis_argument_errors(ctx):
    buf = ctx.buffer(1 << 16)
    try:
        with pytest.raises(N.NotSupportedError):
            N.synth_weight_rows_device(N.Q4_K, 1, 0, 1, 256, 0.02, buf.device_pointer, ctx.stream)
        with pytest.raises(N.ArgumentError):
            N.synth_weight_rows_device(N.Q8_0, 1, 0, 1, 48, 0.02, buf.device_pointer, ctx.stream)
        with pytest.raises(N.ArgumentError):  # 2000 rows of 34 bytes overflow the 64 KB buffer
            N.synth_weight_rows_device(N.Q8_0, 1, 0, 2000, 32, 0.02, buf.device_pointer, ctx.stream)
    finally:
        buf.free()
