"""GPU parity of the LoRA linear over Int8 weights against the CPU oracle.

Bar (north star): relative L2 error <= 3e-3 for Y, dX, dA and dB against the
reference arithmetic in fp32 on the same dequantised weights
(src/layers/lora.jl:56-95, 106-118); fp32 activations (CUDA-core path)
<= 1e-5.  Calls go through the Python mirror, which calls the C ABI.
"""
import glob
import os

import numpy as np
import pytest

import lora_case as lc

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch():
    import torch as _t
    from reels_b200 import build
    build.build()
    return _t


def run_gpu(torch, c: lc.Case, use_saved=True, grad_scale=1.0):
    from reels_b200 import lora_backward, lora_forward, saved_buffer
    from reels_b200 import _native as nat
    dt = lc.torch_dtype(torch, c.dtype)
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(dt)
    dy = torch.from_numpy(c.dY).cuda().to(dt)
    saved = saved_buffer(layer, x) if use_saved else None
    y = lora_forward(layer, x, saved=saved)
    path_f = nat.last_path()
    g = lora_backward(layer, x, dy, saved=saved, grad_scale=grad_scale)
    path_b = nat.last_path()
    from reels_b200 import check_device_status
    check_device_status()
    return (y.float().cpu().numpy(), g.dx.float().cpu().numpy(), g.A.t().contiguous().cpu().numpy(),
            g.B.t().contiguous().cpu().numpy(), path_f, path_b)


def check(c, got, ref, tol=None, scale=(1.0, 1.0, 1.0, 1.0)):
    tol = tol if tol is not None else (lc.TOL_F32 if c.dtype == "f32" else lc.TOL)
    names = ["Y", "dX", "dA", "dB"]
    errs = {}
    for name, a, b, sc in zip(names, got[:4], ref, scale):
        errs[name] = lc.rel_l2(a, np.asarray(b) * sc)
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"rel L2 over {tol}: {errs}"
    return errs


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "linear_*.npz"))))
def test_committed_fixtures(torch, path):
    f = np.load(path)
    c = lc.case_from_fixture(f)
    got = run_gpu(torch, c)
    check(c, got, (f["Y"], f["dX"], f["dA"], f["dB"]))


@pytest.fixture(scope="module")
def cfg1(torch):
    # Wan-2.1-1.3B FFN up-proj, M=1280, K=1536, N=8960,
    # r=16, alpha=16, bf16, seed 0.
    c = lc.make_case(1280, 1536, 8960, 16, alpha=16.0, dtype="bf16", layout=0, seed=0, a_std=1.0 / 16)
    return c, lc.oracle_outputs(c)


@pytest.mark.parametrize("layout", [0, 1])
def test_config1_parity(torch, cfg1, layout):
    from reels_b200 import _native as nat
    c, ref = cfg1
    if layout == 1:
        c = lc.Case(**{**c.__dict__, "layout": 1, "Wmem": np.ascontiguousarray(c.Wmem.T),
                       "q": np.ascontiguousarray(c.q.T)})
    got = run_gpu(torch, c)
    assert got[4] == nat.PATH_TENSORCORE and got[5] == nat.PATH_TENSORCORE
    check(c, got, ref)


def test_config1_recompute_matches_saved(torch, cfg1):
    c, ref = cfg1
    a = run_gpu(torch, c, use_saved=True)
    b = run_gpu(torch, c, use_saved=False)
    for x, y in zip(a[:4], b[:4]):
        assert np.array_equal(x, y)


@pytest.mark.parametrize("M,K,N,r,layout", [
    (1, 64, 256, 16, 0),        # one token
    (7, 80, 48, 3, 1),          # ragged everything (K, N multiples of 16 only)
    (129, 128, 272, 8, 0),      # one row past a tile
    (300, 1536, 1536, 32, 1),   # Wan attention shape, few tokens (split-K)
    (64, 512, 512, 1, 0),       # rank 1
    (96, 256, 512, 65, 1),      # rank just over one 64-wide extension block
    (200, 256, 256, 128, 0),    # two extension blocks
    (128, 256, 256, 256, 1),    # maximum rank
    (520, 320, 640, 32, 0),     # MT=2 tiles with a ragged tail
    (2048, 1536, 1536, 32, 0),  # many tiles, no split
])
def test_shapes_bf16(torch, M, K, N, r, layout):
    from reels_b200 import _native as nat
    c = lc.make_case(M, K, N, r, dtype="bf16", layout=layout, seed=M + K + N + r)
    got = run_gpu(torch, c)
    assert got[4] == nat.PATH_TENSORCORE
    check(c, got, lc.oracle_outputs(c))


@pytest.mark.parametrize("r", [8, 64])
@pytest.mark.parametrize("layout", [0, 1])
def test_fp16_with_loss_scale(torch, r, layout):
    # config 5 style: fp16 activations, dY multiplied by the static loss scale
    # 1024, adapter gradients unscaled by 1/1024 (src/training/precision.jl:8-12).
    from reels_b200 import _native as nat
    c = lc.make_case(256, 1024, 1536, r, dtype="f16", layout=layout, seed=r, dy_scale=1024.0)
    got = run_gpu(torch, c, grad_scale=1.0 / 1024)
    assert got[4] == nat.PATH_TENSORCORE
    Y, dX, dA, dB = lc.oracle_outputs(c)
    check(c, got, (Y, dX, dA / 1024, dB / 1024))


@pytest.mark.parametrize("M,K,N,r,layout", [(4, 5, 7, 2, 0), (33, 24, 40, 3, 1), (5, 64, 48, 8, 0)])
def test_fp32_cuda_core_path(torch, M, K, N, r, layout):
    from reels_b200 import _native as nat
    c = lc.make_case(M, K, N, r, dtype="f32", layout=layout, seed=3)
    got = run_gpu(torch, c)
    assert got[4] == nat.PATH_CUDACORE
    check(c, got, lc.oracle_outputs(c))


def test_ragged_bf16_cuda_core_path(torch):
    from reels_b200 import _native as nat
    c = lc.make_case(11, 24, 40, 2, dtype="bf16", layout=1, seed=9)
    got = run_gpu(torch, c)
    assert got[4] == nat.PATH_CUDACORE
    check(c, got, lc.oracle_outputs(c))


def test_bias_and_disabled_adapter(torch):
    from reels_b200 import lora_forward, set_adapter_enabled
    c = lc.make_case(64, 256, 512, 8, dtype="bf16", layout=0, seed=2, bias=True)
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(torch.bfloat16)
    y = lora_forward(layer, x).float().cpu().numpy()
    assert lc.rel_l2(y, lc.oracle_outputs(c)[0]) <= lc.TOL
    set_adapter_enabled(layer, False)
    y0 = lora_forward(layer, x).float().cpu().numpy()
    import oracle
    base = oracle.lora_forward(c.X, c.q, c.s, c.layout, c.A[:, :0].copy(), c.B[:0].copy(), 1.0, bias=c.bias)
    assert lc.rel_l2(y0, base) <= lc.TOL


def test_zero_B_equals_weight_mul(torch):
    # test/unit/lora.jl:6 on the device: B = 0 gives the plain quantised linear.
    from reels_b200 import lora_forward, weight_mul
    c = lc.make_case(256, 512, 768, 16, dtype="bf16", layout=0, seed=4)
    c.B[:] = 0
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(torch.bfloat16)
    y = lora_forward(layer, x)
    y0 = weight_mul(layer.weight, x)
    assert torch.equal(y, y0)


def test_empty_token_batch(torch):
    """No tokens (the reference's (in, 0) activations): empty outputs, zero
    adapter gradients, accumulators left as they are, and the same for the
    block neighbours and the dropout path."""
    from reels_b200 import (check_device_status, gated_residual, gated_residual_backward, layernorm_modulate,
                            layernorm_modulate_backward, lora_backward, lora_forward, saved_buffer,
                            weight_transpose_mul)
    c = lc.make_case(16, 256, 384, 8, dtype="bf16", layout=0, seed=9)
    layer = lc.device_layer(torch, c)
    x = torch.empty((0, 256), dtype=torch.bfloat16, device="cuda")
    dy = torch.empty((0, 384), dtype=torch.bfloat16, device="cuda")
    saved = saved_buffer(layer, x)
    y = lora_forward(layer, x, saved=saved)
    assert tuple(y.shape) == (0, 384)
    g = lora_backward(layer, x, dy, saved=saved)
    assert tuple(g.dx.shape) == (0, 256)
    assert not g.A.any() and not g.B.any()
    accA = torch.full((256, 8), 0.5, device="cuda").t()
    accB = torch.full((8, 384), -1.0, device="cuda").t()
    lora_backward(layer, x, dy, dA_acc=accA, dB_acc=accB, need_dx=False)
    assert bool((accA == 0.5).all()) and bool((accB == -1.0).all())
    assert tuple(weight_transpose_mul(layer.weight, dy).shape) == (0, 256)
    layer.dropout = 0.25
    assert tuple(lora_forward(layer, x, training=True, dropout_seed=3).shape) == (0, 384)
    scale = torch.zeros((1, 256), dtype=torch.bfloat16, device="cuda")
    assert tuple(layernorm_modulate(x, scale, scale).shape) == (0, 256)
    dxn, ds, dh = layernorm_modulate_backward(x, x, scale, param_grads=True)
    assert tuple(dxn.shape) == (0, 256) and not ds.any() and not dh.any()
    gate = torch.ones((1, 256), dtype=torch.bfloat16, device="cuda")
    assert tuple(gated_residual(x, x, gate).shape) == (0, 256)
    dyr, dg = gated_residual_backward(x, x, gate)
    assert tuple(dyr.shape) == (0, 256) and not dg.any()
    check_device_status()


def test_accumulate_into_fp32_buffers(torch):
    from reels_b200 import lora_backward
    c = lc.make_case(512, 256, 384, 16, dtype="bf16", layout=1, seed=6)
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(torch.bfloat16)
    dy = torch.from_numpy(c.dY).cuda().to(torch.bfloat16)
    g1 = lora_backward(layer, x, dy)
    accA = torch.full((c.K, c.r), 0.5, device="cuda").t()
    accB = torch.full((c.r, c.N), -0.25, device="cuda").t()
    lora_backward(layer, x, dy, dA_acc=accA, dB_acc=accB, grad_scale=0.5, need_dx=False)
    assert torch.allclose(accA, 0.5 + 0.5 * g1.A, rtol=1e-6, atol=1e-6)
    assert torch.allclose(accB, -0.25 + 0.5 * g1.B, rtol=1e-6, atol=1e-6)


def test_weight_transpose_mul_is_the_frozen_pullback(torch):
    # ad_rules.jl:70-80: the frozen weight's pullback is dequant(W)' * dy.
    from reels_b200 import weight_transpose_mul
    import oracle
    c = lc.make_case(300, 512, 1024, 0, dtype="bf16", layout=1, seed=8)
    layer = lc.device_layer(torch, c)
    dy = torch.from_numpy(c.dY).cuda().to(torch.bfloat16)
    dx = weight_transpose_mul(layer.weight, dy).float().cpu().numpy()
    Wd = oracle.dequantize_f32(c.q, c.s, 1)
    assert lc.rel_l2(dx, c.dY.astype(np.float64) @ Wd.astype(np.float64)) <= lc.TOL


def test_frozen_linear_autograd_is_the_transpose_mul(torch):
    """rrule(linear) (ad_rules.jl:55-68): the frozen dense layer's pullback
    is exactly dequant(W)' * dy, with no tangent for the weight or bias."""
    from reels_b200 import DenseLayer, FrozenLinearFunction, linear, weight_transpose_mul
    c = lc.make_case(300, 512, 640, 8, dtype="bf16", layout=1, seed=12, bias=True)
    layer = lc.device_layer(torch, c)
    dense = DenseLayer(layer.weight, layer.bias)
    x = torch.from_numpy(c.X).cuda().to(torch.bfloat16).requires_grad_(True)
    dy = torch.from_numpy(c.dY).cuda().to(torch.bfloat16)
    y = FrozenLinearFunction.apply(x, dense)
    assert torch.equal(y, linear(dense, x.detach()))
    y.backward(dy)
    assert torch.equal(x.grad, weight_transpose_mul(dense.weight, dy))


def test_autograd_function_matches_explicit_backward(torch):
    from reels_b200 import LoRALinearFunction, lora_backward
    c = lc.make_case(256, 512, 512, 16, dtype="bf16", layout=0, seed=10)
    layer = lc.device_layer(torch, c)
    x = torch.from_numpy(c.X).cuda().to(torch.bfloat16).requires_grad_(True)
    A = layer.A.detach().clone().requires_grad_(True)
    B = layer.B.detach().clone().requires_grad_(True)
    y = LoRALinearFunction.apply(x, A, B, layer)
    dy = torch.from_numpy(c.dY).cuda().to(torch.bfloat16)
    y.backward(dy)
    g = lora_backward(layer, x.detach(), dy)
    assert torch.equal(x.grad, g.dx)
    assert torch.allclose(A.grad.float(), g.A.to(torch.bfloat16).float())


@pytest.mark.parametrize("M,K,N", [(8192, 1536, 8960), (32760, 1536, 1536)])
def test_full_size_against_torch_fp32(torch, M, K, N):
    """At the benchmark's full sizes the CPU oracle is too slow; compare with an fp32
    torch computation on the same dequantised weight (this is a floating-
    point kernel) -- Y and dX, r = 32."""
    from reels_b200 import lora_backward, lora_forward, materialize_weight
    torch.manual_seed(0)
    r = 32
    c = lc.make_case(16, K, N, r, dtype="bf16", layout=0, seed=1)   # weights only; tokens below
    layer = lc.device_layer(torch, c)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    dy = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    y = lora_forward(layer, x)
    g = lora_backward(layer, x, dy)
    W = materialize_weight(layer.weight, torch.float32)          # (N, K)
    A = layer.A.float()
    B = layer.B.float()
    s = layer.alpha / r
    xf, dyf = x.float(), dy.float()
    y_ref = xf @ W.t() + s * (xf @ A.t()) @ B.t()
    dx_ref = dyf @ W + s * (dyf @ B) @ A
    dA_ref = s * (dyf @ B).t() @ xf
    dB_ref = s * dyf.t() @ (xf @ A.t())

    def rel(a, b):
        return float((a.float() - b).norm() / b.norm())

    assert rel(y, y_ref) <= lc.TOL
    assert rel(g.dx, dx_ref) <= lc.TOL
    assert rel(g.A, dA_ref) <= lc.TOL
    assert rel(g.B, dB_ref) <= lc.TOL
