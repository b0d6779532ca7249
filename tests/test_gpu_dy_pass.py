"""GPU parity of the backward's one pass over dy (sk_dual_kernel), which
computes G = s*B'*dy and dB = s*T*dy (lora.jl:112-114) from a single read of
dy.

Each case is pinned to one way the pass writes its outputs (checked through
the planner query first, so a planner change cannot silently drop a case):
  - both final (one token range, one feature range);
  - G split over feature ranges, dB final;
  - dB split over token ranges, G final (rank 128: the widest rank the pass
    takes, TMEM full);
  - both split, summed by one reduce launch.
Every case runs plain and with fp32 accumulators (grad_scale 0.5), and is
checked against the CPU oracle within the north star's bound, and against
the separate G and dB passes (REELS_SK_DUAL=0, read at each call): dB is the
same fp32 sum of the same bf16 products in another order, so it agrees to
1e-5; dX and dA see G rounded to bf16 from a differently ordered fp32 sum,
so a few roundings may land on the other side."""
import ctypes
import os

import pytest

import lora_case as lc

pytestmark = pytest.mark.gpu

# (M, K, N, r, layout, dtype, expected (splits_m > 1, splits_n > 1))
CASES = [
    (7, 64, 48, 3, 0, "bf16", (False, False)),
    (96, 256, 512, 65, 1, "bf16", (False, True)),
    (8000, 128, 256, 128, 0, "bf16", (True, False)),
    (1000, 640, 1152, 32, 1, "f16", (True, True)),
    (2048, 384, 640, 64, 0, "bf16", (True, True)),
]


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("needs a GPU")
    from reels_b200 import build
    build.build()
    return t


def plan(M, N, r):
    from reels_b200 import _native as nat
    info = (ctypes.c_int64 * 6)()
    assert nat.lib().reels_sk_dual_plan(M, N, r, 148, info) == 0
    return list(info)


def run(torch, c, accumulate, separate):
    from reels_b200 import check_device_status, lora_backward, lora_forward, saved_buffer
    tdt = lc.torch_dtype(torch, c.dtype)
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(tdt)
    dy = torch.from_numpy(c.dY).cuda().to(tdt)
    saved = saved_buffer(layer, x)
    lora_forward(layer, x, saved=saved)
    if separate:
        os.environ["REELS_SK_DUAL"] = "0"
    try:
        if accumulate:
            accA = torch.full((c.K, c.r), 0.5, device="cuda").t()
            accB = torch.full((c.r, c.N), -0.25, device="cuda").t()
            g = lora_backward(layer, x, dy, saved=saved, dA_acc=accA, dB_acc=accB, grad_scale=0.5)
            dA, dB = (accA - 0.5) / 0.5, (accB + 0.25) / 0.5
        else:
            g = lora_backward(layer, x, dy, saved=saved)
            dA, dB = g.A, g.B
        torch.cuda.synchronize()
    finally:
        os.environ.pop("REELS_SK_DUAL", None)
    check_device_status()
    return (g.dx.float().cpu().numpy(), dA.t().contiguous().cpu().numpy(), dB.t().contiguous().cpu().numpy())


@pytest.mark.parametrize("M,K,N,r,layout,dt,split", CASES)
@pytest.mark.parametrize("accumulate", [False, True])
def test_dy_pass_matches_oracle_and_separate_passes(torch, M, K, N, r, layout, dt, split, accumulate):
    p = plan(M, N, r)
    assert p[0] == 1 and (p[1] > 1, p[2] > 1) == split, p
    os.environ["REELS_SK_DUAL"] = "0"
    try:
        assert plan(M, N, r)[0] == 0
    finally:
        os.environ.pop("REELS_SK_DUAL", None)
    c = lc.make_case(M, K, N, r, dtype=dt, layout=layout, seed=M + N + r)
    fused = run(torch, c, accumulate, separate=False)
    sep = run(torch, c, accumulate, separate=True)
    _, dX, dA, dB = lc.oracle_outputs(c)
    for name, got, ref in zip(("dX", "dA", "dB"), fused, (dX, dA, dB)):
        assert lc.rel_l2(got, ref) <= lc.TOL, (name, lc.rel_l2(got, ref))
    assert lc.rel_l2(fused[2], sep[2]) <= 1e-5, lc.rel_l2(fused[2], sep[2])
    assert lc.rel_l2(fused[0], sep[0]) <= 1e-3
    assert lc.rel_l2(fused[1], sep[1]) <= 1e-3


def test_rank_above_128_keeps_separate_passes():
    # the dB accumulators of a 129..256-rank pass do not fit next to G's in TMEM
    assert plan(4096, 1536, 256)[0] == 0
    assert plan(4096, 1536, 129)[0] == 0
