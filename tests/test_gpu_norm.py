"""GPU parity of the fused LayerNorm + modulation and its pullback against
the oracle (src/layers/linear.jl:26-36,49-59; modulation.jl:13-22).

Forward: the kernel's fp32 sums run in a different order from the oracle's
fp64 ones, so the rounded outputs may differ where a value lies at a
rounding boundary; the bar is relative L2 <= 3e-3 with at most 1% of
elements one rounding step apart (fp32: 1e-5).  Backward: dx, dscale and
dshift against the oracle fed the kernel's own rounded LayerNorm output."""
import numpy as np
import pytest

import lora_case as lc
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as _t
    from reels_b200 import build
    build.build()
    return _t


CASES = [  # (M, K, tokens_per_sample, dtype, modulate, ln affine)
    (1024, 1536, 512, "bf16", True, False),
    (300, 5120, 300, "bf16", True, True),
    (257, 1000, 100, "f16", True, False),
    (64, 4096, 64, "f32", False, True),
    (128, 24, 32, "bf16", True, True),
    (512, 5120, 256, "bf16", False, False),  # one row per warp, no modulation
]


@pytest.mark.parametrize("M,K,tps,dtype,mod,aff", CASES)
def test_layernorm_modulate_parity(torch, M, K, tps, dtype, mod, aff):
    from reels_b200 import check_device_status, layernorm_modulate, layernorm_modulate_backward
    rng = np.random.default_rng(M + K)
    batch = (M + tps - 1) // tps
    x = lc.round_to(rng.standard_normal((M, K)) * 2 + 0.5, dtype)
    scale = lc.round_to(0.1 * rng.standard_normal((batch, K)), dtype) if mod else None
    shift = lc.round_to(0.1 * rng.standard_normal((batch, K)), dtype) if mod else None
    w = lc.round_to(rng.uniform(0.5, 1.5, K), dtype) if aff else None
    b = lc.round_to(0.1 * rng.standard_normal(K), dtype) if aff else None
    dout = lc.round_to(rng.standard_normal((M, K)), dtype)
    tdt = lc.torch_dtype(torch, dtype)
    T = lambda a: None if a is None else torch.from_numpy(a).cuda().to(tdt)
    eps = 1e-6
    out = layernorm_modulate(T(x), T(scale), T(shift), eps, T(w), T(b), tps)
    dx, dscale, dshift = layernorm_modulate_backward(T(x), T(dout), T(scale), eps, T(w), T(b), tps, param_grads=True)
    dx2, _, _ = layernorm_modulate_backward(T(x), T(dout), T(scale), eps, T(w), T(b), tps, param_grads=True)
    check_device_status()
    ln = lc.round_to(oracle.layernorm(x, eps, w, b), dtype)
    ref = lc.round_to(oracle.modulate(ln, tps, scale, shift), dtype)
    got = out.float().cpu().numpy()
    tol = lc.TOL_F32 if dtype == "f32" else lc.TOL
    assert lc.rel_l2(got, ref) <= tol
    if dtype != "f32":
        assert np.mean(got != ref) <= 0.01
    # backward: g = round(dout * (1 + scale)), then the LayerNorm's pullback
    g = dout if scale is None else lc.round_to(dout * (np.float32(1) + np.repeat(scale, tps, 0)[:M]), dtype)
    dx_ref = oracle.layernorm_backward(x, g, eps, w)
    assert lc.rel_l2(dx.float().cpu().numpy(), dx_ref) <= tol
    assert torch.equal(dx, dx2)
    sample = np.arange(M) // tps
    ds_ref = np.stack([(dout * ln)[sample == i].sum(0, dtype=np.float64) for i in range(batch)])
    dh_ref = np.stack([dout[sample == i].sum(0, dtype=np.float64) for i in range(batch)])
    assert lc.rel_l2(dscale.cpu().numpy(), ds_ref) <= 1e-4
    assert lc.rel_l2(dshift.cpu().numpy(), dh_ref) <= 1e-5


def test_autograd(torch):
    from reels_b200 import LayerNormModulateFunction, layernorm_modulate_backward
    rng = np.random.default_rng(3)
    M, K = 256, 1536
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda().to(torch.bfloat16)
    sc = torch.from_numpy((0.1 * rng.standard_normal((1, K))).astype(np.float32)).cuda().to(torch.bfloat16)
    sh = torch.from_numpy((0.1 * rng.standard_normal((1, K))).astype(np.float32)).cuda().to(torch.bfloat16)
    x.requires_grad_(True)
    sc.requires_grad_(True)
    sh.requires_grad_(True)
    y = LayerNormModulateFunction.apply(x, sc, sh, 1e-6)
    dy = torch.ones_like(y)
    y.backward(dy)
    dx, ds, dh = layernorm_modulate_backward(x.detach(), dy, sc.detach(), 1e-6, param_grads=True)
    assert torch.equal(x.grad, dx)
    assert torch.equal(sc.grad, ds.to(torch.bfloat16)) and torch.equal(sh.grad, dh.to(torch.bfloat16))


@pytest.mark.parametrize("M,N,tps,dtype", [(1024, 1536, 512, "bf16"), (300, 1000, 100, "f16"), (64, 96, 64, "f32")])
def test_gated_residual(torch, M, N, tps, dtype):
    """mixed_add(x, mixed_mul(y, gate)) (transformer.jl:272,293) and its
    pullback: the forward bit for bit (elementwise fp32 operations, each
    rounded), dy bit for bit, dgate within fp32 summation order."""
    from reels_b200 import check_device_status, gated_residual, gated_residual_backward
    rng = np.random.default_rng(M + N)
    batch = (M + tps - 1) // tps
    x = lc.round_to(rng.standard_normal((M, N)), dtype)
    y = lc.round_to(rng.standard_normal((M, N)), dtype)
    gate = lc.round_to(rng.standard_normal((batch, N)), dtype)
    dout = lc.round_to(rng.standard_normal((M, N)), dtype)
    tdt = lc.torch_dtype(torch, dtype)
    T = lambda a: torch.from_numpy(a).cuda().to(tdt)
    out = gated_residual(T(x), T(y), T(gate), tps)
    xin = T(x)
    gated_residual(xin, T(y), T(gate), tps, out=xin)  # in place
    dy, dgate = gated_residual_backward(T(dout), T(y), T(gate), tps)
    check_device_status()
    g_rows = np.repeat(gate, tps, 0)[:M]
    ref = lc.round_to(x + lc.round_to(y * g_rows, dtype), dtype)
    assert np.array_equal(out.float().cpu().numpy(), ref)
    assert torch.equal(xin, out)
    assert np.array_equal(dy.float().cpu().numpy(), lc.round_to(dout * g_rows, dtype))
    sample = np.arange(M) // tps
    dg_ref = np.stack([(dout * y)[sample == i].sum(0, dtype=np.float64) for i in range(batch)])
    assert lc.rel_l2(dgate.cpu().numpy(), dg_ref) <= 1e-5


def test_modulation_finite_differences(torch):
    """The reference's modulation test (test/unit/layers.jl:43-54) on the
    fused LayerNorm + modulation in fp32: 3 features, 4 tokens per sample, 2
    samples; dx, dscale and dshift against central differences of
    sum(out .* dy) with step 1e-3, rtol 3e-3."""
    from reels_b200 import layernorm_modulate, layernorm_modulate_backward
    rng = np.random.default_rng(22)
    x = torch.from_numpy(rng.standard_normal((8, 3)).astype(np.float32)).cuda()
    scale = torch.from_numpy(rng.standard_normal((2, 3)).astype(np.float32)).cuda()
    shift = torch.from_numpy(rng.standard_normal((2, 3)).astype(np.float32)).cuda()
    dy = torch.from_numpy(rng.standard_normal((8, 3)).astype(np.float32)).cuda()
    eps = 1e-6

    def objective():
        return float((layernorm_modulate(x, scale, shift, eps, tokens_per_sample=4).double() * dy.double()).sum())

    def fd(t, idx, h=1e-3):
        old = t[idx].item()
        t[idx] = old + h
        plus = objective()
        t[idx] = old - h
        minus = objective()
        t[idx] = old
        return (plus - minus) / (2 * h)

    dx, dscale, dshift = layernorm_modulate_backward(x, dy, scale, eps, tokens_per_sample=4, param_grads=True)
    for idx in ((1, 2), (5, 0), (6, 1)):
        assert dx[idx].item() == pytest.approx(fd(x, idx), rel=3e-3, abs=1e-4)
    assert dscale[0, 1].item() == pytest.approx(fd(scale, (0, 1)), rel=3e-3, abs=1e-4)
    assert dshift[1, 2].item() == pytest.approx(fd(shift, (1, 2)), rel=3e-3, abs=1e-4)
