"""si_matrix_multiply_static_workspace: the GEMM for callers that cannot
allocate device memory (a host pool that owns every device byte, or a loop
that must not reach cudaMalloc/cudaFree, which can synchronise the device).
Its scratch is a fixed 64 MiB device array inside the library. Checked
through the C ABI against si_ctx_matrix_multiply (context-owned workspace)
on two calls in a row. Collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from helpers import north_star_gate, row_norm_max
from sharpinference_b200 import native

pytestmark = pytest.mark.gpu
N = native


def _static_call(ctx, wtype, X, W, Y, m, n, k):
    st = native.lib.si_matrix_multiply_static_workspace(wtype, X.device_pointer, W.device_pointer, Y.device_pointer,
                                                        m, n, k, C.c_void_p(ctx.stream))
    native.check(st)
    ctx.synchronize()


@pytest.mark.parametrize("wtype,m,n,k", [(N.Q4_K, 512, 640, 3072), (N.Q8_0, 300, 200, 1024)])
def test_static_workspace_matches_allocating_entry_point(ctx, wtype, m, n, k):
    blob = native.synth_weights(wtype, 21, n, k, 0.02)
    W, X, Y, R = ctx.buffer(blob.nbytes), ctx.buffer(m * k * 4), ctx.buffer(m * n * 4), ctx.buffer(m * n * 4)
    try:
        W.upload(blob)
        rn = row_norm_max(wtype, blob, n, k)
        for call, seed in enumerate((31, 32)):  # two calls in a row, different inputs
            x = native.synth_normal(seed, m * k, 1.0)
            X.upload(x)
            Y.upload(np.full(m * n, np.nan, np.float32))
            _static_call(ctx, wtype, X, W, Y, m, n, k)
            ctx.matrix_multiply(wtype, X, W, R, m, n, k)
            y = Y.readback().view(np.float32).reshape(m, n)
            ref = R.readback().view(np.float32).reshape(m, n)
            assert np.all(np.isfinite(y)), f"call {call}: output not fully written"
            for r in (0, m // 2, m - 1):
                north_star_gate(y[r], ref[r], x[r * k:(r + 1) * k], rn, k)
            assert np.array_equal(y, ref), f"call {call}: differs from the allocating entry point"
        assert native.device_error_take(0) == 0
    finally:
        for b in (W, X, Y, R):
            b.free()


def _align256(v):
    return (v + 255) // 256 * 256


def test_static_workspace_call_allocates_nothing(ctx):
    """The entry point's claim: after the first call on a device (which looks
    up the array's address), a call takes no device memory. The shape splits
    K, so the partial sums live in the shared array too."""
    import torch
    wtype, m, n, k = N.Q4_K, 512, 640, 3072
    need = C.c_uint64()
    native.check(native.lib.si_matrix_multiply_workspace_bytes(wtype, m, n, k, C.byref(need)))
    assert need.value > 2 * _align256(m * k * 2), "shape must split K (partial sums in the workspace)"
    blob = native.synth_weights(wtype, 23, n, k, 0.02)
    W, X, Y = ctx.buffer(blob.nbytes), ctx.buffer(m * k * 4), ctx.buffer(m * n * 4)
    try:
        W.upload(blob)
        X.upload(native.synth_normal(41, m * k, 1.0))
        for _ in range(2):  # first calls: address lookup and kernel module loading
            _static_call(ctx, wtype, X, W, Y, m, n, k)
        free_before, _ = torch.cuda.mem_get_info(0)
        for _ in range(3):
            _static_call(ctx, wtype, X, W, Y, m, n, k)
        free_after, _ = torch.cuda.mem_get_info(0)
        assert free_after == free_before, f"device memory changed by {free_before - free_after} bytes"
    finally:
        for b in (W, X, Y):
            b.free()


def test_static_workspace_rejects_oversized_request(ctx):
    m, n, k = 4096, 128, 8192  # needs 4*m*k = 128 MiB of scratch
    W, X, Y = ctx.buffer(native.row_bytes(N.Q4_K, k) * n), ctx.buffer(m * k * 4), ctx.buffer(m * n * 4)
    try:
        st = native.lib.si_matrix_multiply_static_workspace(N.Q4_K, X.device_pointer, W.device_pointer,
                                                            Y.device_pointer, m, n, k, C.c_void_p(ctx.stream))
        assert st == N.SI_ERR_INVALID_ARGUMENT
        assert "static workspace" in native.last_error()
    finally:
        for b in (W, X, Y):
            b.free()
