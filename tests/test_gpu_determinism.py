"""Run-to-run determinism of the q8 LoRA linear (forward Y, backward dX, dA,
dB) on the plans the planner picks for these shapes.  No reduction in the
library uses atomics: split partials are summed in index order, and the two
MMA issuers of the 128-token tiles accumulate into two accumulators that the
epilogue adds as acc0 + acc1.  Repeating a call must therefore give the same
bits; a race in a pipeline shows up here as a difference between repeats.

Plans (reels_q8_plan on 148 SMs, forward / dX):
  96 x 4096 -> 8192    128-token tiles, two issuers, 2 / 4 reduction splits,
                       a ragged token tile
  128 x 3072 -> 12288  128-token tiles, two issuers, no split / 4 splits (fp16, r = 64)
  512 x 1536 -> 1536   four 128-token tiles per column tile, two issuers
  2048 x 1536 -> 8960  256-token tiles on CTA pairs / 192-token tiles, several per CTA
"""
import pytest

pytestmark = pytest.mark.gpu

# the last field: also compare the first run with the oracle (the 2048-token
# plans have their parity cases elsewhere; the oracle takes ~30 s there)
CASES = [(96, 4096, 8192, 8, "bf16", True), (128, 3072, 12288, 64, "f16", True), (512, 1536, 1536, 32, "bf16", True),
         (2048, 1536, 8960, 32, "bf16", False)]


@pytest.mark.parametrize("M,K,N,r,dt,check_oracle", CASES)
def test_repeat_is_bit_identical(M, K, N, r, dt, check_oracle):
    import torch

    import lora_case as lc
    from reels_b200 import check_device_status, lora_backward, lora_forward, saved_buffer

    c = lc.make_case(M, K, N, r, dtype=dt, layout=0, seed=M + r)
    tdt = lc.torch_dtype(torch, dt)
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(tdt)
    dy = torch.from_numpy(c.dY).cuda().to(tdt)
    runs = []
    for _ in range(3):
        saved = saved_buffer(layer, x)
        y = lora_forward(layer, x, saved=saved)
        g = lora_backward(layer, x, dy, saved=saved)
        runs.append([t.clone() for t in (y, g.dx, g.A, g.B)])
    torch.cuda.synchronize()
    check_device_status()
    for rep in runs[1:]:
        for name, a, b in zip(("Y", "dX", "dA", "dB"), runs[0], rep):
            assert torch.equal(a, b), (name, (a.float() - b.float()).abs().max().item())
    if not check_oracle:
        return
    # and the first run is the right product
    ref = lc.oracle_outputs(c)
    got = (runs[0][0].float().cpu().numpy(), runs[0][1].float().cpu().numpy(),
           runs[0][2].t().contiguous().cpu().numpy(), runs[0][3].t().contiguous().cpu().numpy())
    for name, a, b in zip(("Y", "dX", "dA", "dB"), got, ref):
        assert lc.rel_l2(a, b) <= lc.TOL, (name, lc.rel_l2(a, b))
