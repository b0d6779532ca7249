"""GPU parity of q8 GEMM plans the planner does not pick for these shapes by
itself: the SMEM x SMEM kernel (REELS_Q8_TS=0, the plan for reduction scales
that are not 16-byte aligned), each token tile of the weight-in-TMEM kernel
(REELS_Q8_TS=256/192/128, and 1282 for 128-token tiles with 128-wide
pipeline stages), the single-CTA forms of the plans the planner runs on
CTA pairs (REELS_Q8_PAIR=0), and the 128-token tiles with one MMA issuer
instead of two (REELS_Q8_ISS2=0).  The overrides are read once
per process, so each plan runs its cases in a child process."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys
sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
import torch
import lora_case as lc
from reels_b200 import lora_forward, lora_backward, saved_buffer, check_device_status
out = []
for (M, K, N, r, layout, dt) in {cases!r}:
    c = lc.make_case(M, K, N, r, dtype=dt, layout=layout, seed=M + N)
    tdt = lc.torch_dtype(torch, dt)
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(tdt); dy = torch.from_numpy(c.dY).cuda().to(tdt)
    saved = saved_buffer(layer, x)
    y = lora_forward(layer, x, saved=saved)
    g = lora_backward(layer, x, dy, saved=saved)
    check_device_status()
    ref = lc.oracle_outputs(c)
    got = (y.float().cpu().numpy(), g.dx.float().cpu().numpy(), g.A.t().contiguous().cpu().numpy(),
           g.B.t().contiguous().cpu().numpy())
    out.append([lc.rel_l2(a, b) for a, b in zip(got, ref)])
print(json.dumps(out))
"""

CASES = [(512, 512, 768, 16, 0, "bf16"), (300, 256, 512, 65, 1, "bf16"), (256, 1024, 512, 8, 0, "f16"),
         (1000, 640, 1152, 32, 1, "f16"), (2048, 1536, 640, 32, 0, "bf16")]


@pytest.mark.parametrize("overrides", [{"REELS_Q8_TS": "0"}, {"REELS_Q8_TS": "256"}, {"REELS_Q8_TS": "192"},
                                       {"REELS_Q8_TS": "128"}, {"REELS_Q8_TS": "1282"}, {"REELS_Q8_PAIR": "0"},
                                       {"REELS_Q8_TS": "1282", "REELS_Q8_ISS2": "0"},
                                       {"REELS_Q8_TS": "1282", "REELS_Q8_PAIR": "1", "REELS_Q8_ISS2": "0"}],
                         ids=lambda o: ",".join(f"{k[9:]}={v}" for k, v in o.items()))
def test_forced_plan_parity(overrides):
    from reels_b200 import build
    build.build()
    env = dict(os.environ)
    for k in ("REELS_Q8_TILE", "REELS_Q8_TS", "REELS_Q8_PAIR", "REELS_Q8_ISS2"):
        env.pop(k, None)
    env.update(overrides)
    code = CHILD.format(root=ROOT, tests=os.path.join(ROOT, "tests"), cases=CASES)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    errs = json.loads(res.stdout.strip().splitlines()[-1])
    for case, e in zip(CASES, errs):
        assert max(e) <= 3e-3, (case, e)
