"""Every launch shape of the tensor-core Q4_K and Q8_0 GEMV (K split over
1/2/4-CTA clusters, 16/32-row tiles, full or half shared-memory ring, FP16 or INT8
MMA path, one or two warps per superblock column) against the
oracle on ragged shapes. The shape is forced through SI_Q4K_GEMV_PLAN, which
the library reads once per process, so each plan runs in a child process."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
CHILD = Path(__file__).resolve().parent / "gemv_plan_child.py"
PLANS = ["default", "1,16,100", "1,32,220", "2,16,100", "2,32,220", "4,16,100", "4,32,64",
         "1,16,100,1", "1,32,220,1", "2,16,100,1", "2,32,220,1", "4,32,64,1", "1,32,226,1,2", "2,32,226,1,2",
         "4,32,120,1,2", "3,16,226", "5,32,226", "8,16,160"]


@pytest.mark.parametrize("plan", PLANS)
def test_launch_shape_parity(plan):
    env = dict(os.environ)
    env.pop("SI_Q4K_GEMV_PLAN", None)
    if plan != "default":
        env["SI_Q4K_GEMV_PLAN"] = plan
    r = subprocess.run([sys.executable, str(CHILD)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["device_error_word"] == 0
    bad = [s for s in res["shapes"] if not s["ok"]]
    assert not bad, bad
