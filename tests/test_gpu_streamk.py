"""GPU parity of the stream-K schedule of the weight-in-TMEM q8 GEMM.

With stream-K every CTA takes an equal run of (tile, pipeline stage) units;
a tile cut across runs is finished by the CTA holding its first stages, which
adds the other pieces' fp32 accumulators (left in the workspace, announced
by per-warp flags) in its epilogue.  REELS_Q8_STREAMK=1 keeps only stream-K
plans and REELS_Q8_TS picks the tile, so each forced plan runs in a child
process.  The shapes make cut tiles in both passes, LoRA blocks that land in
a different piece than the reduction stages (rank 65 over 64-wide stages),
ragged token and feature tails, and the hybrid schedule (whole tiles first,
stream-K for the last rounds).  Reference: fp32 torch on the same
dequantised weight (relative L2 <= 3e-3, the north star's bound); the
result must also be identical from run to run.
"""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import ctypes, json, sys
sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
import torch
import lora_case as lc
from reels_b200 import (lora_forward, lora_forward_gelu, lora_backward, materialize_weight, saved_buffer,
                        check_device_status, weight_mul, weight_transpose_mul)
from reels_b200 import _native as nat
torch.manual_seed(0)
L = nat.lib()

def plan(M, Nout, Kred):
    info = (ctypes.c_int64 * 7)()
    nat.check("plan", L.reels_q8_plan(M, Nout, Kred, 0, 0, info))
    return int(info[0])

def rel(a, b):
    return float((a.float() - b).norm() / b.norm())

out = []
for (M, K, N, r, layout, dt, gelu) in {cases!r}:
    c = lc.make_case(16, K, N, max(r, 1), dtype=dt, layout=layout, seed=K + N + r)   # weights and adapter
    tdt = lc.torch_dtype(torch, dt)
    layer = lc.device_layer(torch, c)
    x = torch.randn(M, K, device="cuda").to(tdt)
    dy = torch.randn(M, N, device="cuda").to(tdt)
    W = materialize_weight(layer.weight, torch.float32)          # (N, K)
    xf, dyf = x.float(), dy.float()
    res = dict(plans=[plan(M, N, K), plan(M, K, N)])
    if r == 0:
        # the frozen linear alone: _weight_mul and _weight_transpose_mul
        y, y2 = weight_mul(layer.weight, x), weight_mul(layer.weight, x)
        dx, dx2 = weight_transpose_mul(layer.weight, dy), weight_transpose_mul(layer.weight, dy)
        check_device_status()
        res.update(y=rel(y, xf @ W.t()), dx=rel(dx, dyf @ W), dA=0.0, dB=0.0,
                   same=bool(torch.equal(y, y2) and torch.equal(dx, dx2)))
        out.append(res)
        continue
    A, B, s = layer.A.float(), layer.B.float(), layer.alpha / r
    saved = saved_buffer(layer, x)
    if gelu:
        y, pre = lora_forward_gelu(layer, x, saved=saved)
        y2, _ = lora_forward_gelu(layer, x, saved=saved)
        h = xf @ W.t() + s * (xf @ A.t()) @ B.t()
        res["pre"] = rel(pre, h)
        res["y"] = rel(y, torch.nn.functional.gelu(pre.float(), approximate="tanh"))
        xa = torch.nn.functional.gelu(xf, approximate="tanh").to(tdt)   # the next linear's input
        g = lora_backward(layer, xa, dy, x_pre=x)
        g2 = lora_backward(layer, xa, dy, x_pre=x)
        gp = torch.ops.aten.gelu_backward(torch.ones_like(xf), xf, approximate="tanh")
        xaf = xa.float()
        res["dx"] = rel(g.dx, (dyf @ W + s * (dyf @ B) @ A) * gp)
        res["dA"] = rel(g.A, s * (dyf @ B).t() @ xaf)
        res["dB"] = rel(g.B, s * dyf.t() @ (xaf @ A.t()))
    else:
        y = lora_forward(layer, x, saved=saved)
        y2 = lora_forward(layer, x, saved=saved)
        g = lora_backward(layer, x, dy, saved=saved)
        g2 = lora_backward(layer, x, dy, saved=saved)
        res["y"] = rel(y, xf @ W.t() + s * (xf @ A.t()) @ B.t())
        res["dx"] = rel(g.dx, dyf @ W + s * (dyf @ B) @ A)
        res["dA"] = rel(g.A, s * (dyf @ B).t() @ xf)
        res["dB"] = rel(g.B, s * dyf.t() @ (xf @ A.t()))
    check_device_status()
    res["same"] = bool(torch.equal(y, y2) and torch.equal(g.dx, g2.dx) and torch.equal(g.A, g2.A)
                       and torch.equal(g.B, g2.B))
    out.append(res)
print(json.dumps(out))
"""

# (M, K, N, r, layout, dtype, gelu): every case cuts tiles in the forward
# (Nout = N) and in dX (Nout = K) for each forced tile shape.
CASES = [(700, 1024, 1536, 32, 0, "bf16", False),
         (300, 2048, 1024, 65, 1, "f16", False),
         (136, 2560, 6912, 8, 0, "f16", False),
         (520, 1536, 2048, 0, 0, "bf16", False),
         (700, 1024, 1536, 16, 1, "bf16", True)]
# 320 output tiles of 256 tokens in the forward: one round of whole tiles,
# then stream-K over the rest
HYBRID = [(4096, 512, 2560, 16, 0, "bf16", False)]


def _run(env_extra, cases):
    from reels_b200 import build
    build.build()
    env = dict(os.environ)
    for k in ("REELS_Q8_TILE", "REELS_Q8_TS", "REELS_Q8_STREAMK"):
        env.pop(k, None)
    env.update(env_extra)
    code = CHILD.format(root=ROOT, tests=os.path.join(ROOT, "tests"), cases=cases)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stderr[-3000:]
    return json.loads(res.stdout.strip().splitlines()[-1])


def _check(cases, results, want_sk=True):
    for case, e in zip(cases, results):
        if want_sk:
            assert e["plans"] == [2, 2], (case, e)
        for k in ("y", "dx", "dA", "dB") + (("pre",) if case[6] else ()):
            assert e[k] <= 3e-3, (case, k, e)
        assert e["same"], (case, e)


@pytest.mark.parametrize("ts", ["256", "192", "128", "1282", "2562"])
def test_stream_k_plans(ts):
    _check(CASES, _run({"REELS_Q8_STREAMK": "1", "REELS_Q8_TS": ts}, CASES))


def test_stream_k_after_whole_tile_rounds():
    _check(HYBRID, _run({"REELS_Q8_STREAMK": "1", "REELS_Q8_TS": "256"}, HYBRID))


def test_default_plans_on_the_same_cases():
    """The planner's own choice (stream-K or not) on the same shapes."""
    _check(CASES, _run({}, CASES), want_sk=False)
