"""Launch state is per device and thread-safe: two host threads, each with
its own context (one executor each, as the reference's engine pools
executors), run the tcgen05 GEMM and the tensor-core GEMV concurrently on
one GPU in a fresh process (the shared-memory opt-ins and SM counts are
looked up on first use by both threads at once) and match the oracle."""
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

CHILD = r'''
import sys, threading
sys.path.insert(0, ROOT); sys.path.insert(0, ROOT + "/tests")
import numpy as np
import oracle
from helpers import north_star_gate, row_norm_max
from sharpinference_b200 import native
errors = []
def work(seed):
    try:
        with native.Context(0) as ctx:
            for wt in (native.Q4_K, native.Q8_0):
                n, k, m = 640, 3072, 96
                blob = native.synth_weights(wt, seed, n, k, 0.02)
                x = native.synth_normal(seed + 1, m * k, 1.0)
                W, X, Y, V = ctx.buffer(blob.nbytes), ctx.buffer(x.nbytes), ctx.buffer(m * n * 4), ctx.buffer(n * 4)
                W.upload(blob), X.upload(x)
                for _ in range(3):
                    ctx.matrix_multiply(wt, X, W, Y, m, n, k)
                    ctx.matvec(wt, W, X, V, n, k)
                y = Y.readback().view(np.float32).reshape(m, n)
                v = V.readback().view(np.float32)
                rn = row_norm_max(wt, blob, n, k)
                for r in (0, m - 1):
                    north_star_gate(y[r], oracle.matvec_f64(wt, blob, x[r * k:(r + 1) * k], n, k),
                                    x[r * k:(r + 1) * k], rn, k)
                north_star_gate(v, oracle.matvec_f64(wt, blob, x[:k], n, k), x[:k], rn, k)
                for b in (W, X, Y, V):
                    b.free()
    except Exception as e:  # reported by the parent
        errors.append(repr(e))
ts = [threading.Thread(target=work, args=(s,)) for s in (3, 9)]
for t in ts: t.start()
for t in ts: t.join()
assert native.device_error_take(0) == 0
print("ERRORS" if errors else "OK", errors)
'''


def test_two_host_threads_two_contexts_one_gpu():
    root = str(Path(__file__).resolve().parents[1])
    r = subprocess.run([sys.executable, "-c", f"ROOT = {root!r}\n" + CHILD], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().startswith("OK"), r.stdout[-2000:]
