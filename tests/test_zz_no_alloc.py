"""GPU test of reels_q8lora_forward_static_ws, the forward entry point that
allocates nothing.

It serves callers that cannot allocate device memory themselves (a binding
handed only raw device pointers, or a loop held to a fixed memory budget):
its scratch is a 32 MiB device array inside the library.  The test calls it
through the C ABI twice in a row and checks both results against the
ordinary entry point (caller workspace) within the parity tolerance used
elsewhere (relative L2 <= 3e-3), that the device's free memory does not
change across a call, and that oversized shapes are refused.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import pytest

import lora_case as lc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    from reels_b200 import _native as nat
    from reels_b200 import build
    build.build()
    return torch, nat, nat.lib()


def _call_both(torch, nat, L, c, dt_torch, dt_code):
    """y, saved from the ordinary forward (caller workspace), then twice from
    the static-scratch forward."""
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(c.X).to(dev).to(dt_torch)
    q = torch.from_numpy(c.q).to(dev)
    s = torch.from_numpy(c.s).to(dev)
    A = torch.from_numpy(c.A).to(dev).to(dt_torch)     # [K][r]
    B = torch.from_numpy(c.B).to(dev).to(dt_torch)     # [r][N]
    nsaved = max(L.reels_q8lora_saved_bytes(c.M, c.r, dt_code), 16)
    wsn = L.reels_q8lora_workspace_bytes(c.M, c.K, c.N, c.r, dt_code, nat.PASS_FORWARD)
    ws = torch.empty((max(wsn, 256),), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream

    # Outputs are allocated up front so that the free-memory check below sees
    # only what the library itself might allocate.
    outs = [(torch.empty((c.M, c.N), dtype=dt_torch, device=dev), torch.zeros((nsaved,), dtype=torch.uint8, device=dev))
            for _ in range(3)]

    def run(static, k):
        y, saved = outs[k]
        if static:
            rc = L.reels_q8lora_forward_static_ws(x.data_ptr(), q.data_ptr(), s.data_ptr(), c.layout, A.data_ptr(),
                                                  B.data_ptr(), None, c.M, c.K, c.N, c.r, c.alpha, dt_code,
                                                  y.data_ptr(), saved.data_ptr(), st)
        else:
            rc = L.reels_q8lora_forward(x.data_ptr(), q.data_ptr(), s.data_ptr(), c.layout, A.data_ptr(),
                                        B.data_ptr(), None, c.M, c.K, c.N, c.r, c.alpha, dt_code, y.data_ptr(),
                                        saved.data_ptr(), ws.data_ptr(), wsn, st)
        nat.check("forward", rc)
        return y, saved

    ref = run(False, 0)
    first = run(True, 1)          # the first call on the device also looks up the scratch address
    torch.cuda.synchronize(dev)
    free_before = torch.cuda.mem_get_info(dev)[0]
    second = run(True, 2)
    torch.cuda.synchronize(dev)
    free_after = torch.cuda.mem_get_info(dev)[0]
    nat.check("device status", L.reels_lowvram_check_device_status(st))
    return ref, first, second, free_before, free_after


@pytest.mark.parametrize("M,K,N,r,layout", [
    (8192, 1536, 1536, 32, 0),   # many tiles: scratch holds A^T, A*x and the LoRA operand
    (64, 1536, 512, 16, 1),      # few tiles: split reduction, fp32 partials in the scratch
])
def test_static_scratch_forward_matches_workspace_forward(env, M, K, N, r, layout):
    torch, nat, L = env
    c = lc.make_case(M, K, N, r, dtype="bf16", layout=layout, seed=M + r)
    assert L.reels_q8lora_workspace_bytes(M, K, N, r, nat.BF16, nat.PASS_FORWARD) <= (32 << 20)
    (y0, s0), (y1, s1), (y2, s2), free_before, free_after = _call_both(torch, nat, L, c, torch.bfloat16, nat.BF16)
    ref = y0.float().cpu().numpy()
    for y in (y1, y2):
        assert lc.rel_l2(y.float().cpu().numpy(), ref) <= lc.TOL
    assert torch.equal(s1, s0) and torch.equal(s2, s0)
    # the oracle agrees too
    assert lc.rel_l2(y2.float().cpu().numpy(), lc.oracle_outputs(c)[0]) <= lc.TOL
    assert free_after == free_before


def test_static_scratch_rejects_oversized_shapes(env):
    torch, nat, L = env
    M, K, N, r = 256, 16384, 8192, 16
    assert L.reels_q8lora_workspace_bytes(M, K, N, r, nat.BF16, nat.PASS_FORWARD) > (32 << 20)
    dev = torch.device("cuda", 0)
    x = torch.empty((16,), dtype=torch.bfloat16, device=dev)
    p = x.data_ptr()
    rc = L.reels_q8lora_forward_static_ws(p, p, p, 0, p, p, None, M, K, N, r, 16.0, nat.BF16, p, None,
                                          torch.cuda.current_stream(dev).cuda_stream)
    assert rc == nat.EINVAL
    assert b"static array" in L.reels_lowvram_last_error()
