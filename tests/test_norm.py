"""CPU checks of the LayerNorm + modulation oracle (src/layers/linear.jl:
26-36,49-59; modulation.jl:13-22) and of the argument checks of its C ABI."""
import ctypes

import numpy as np
import pytest

import oracle
from reels_b200 import _native as nat
from reels_b200 import build as native_build


def test_layernorm_moments():
    x = np.random.default_rng(0).standard_normal((16, 300)).astype(np.float32) * 3 + 1
    y = oracle.layernorm(x, 1e-6)
    assert np.abs(y.mean(1)).max() < 1e-6
    assert np.abs(y.std(1) - 1).max() < 1e-5
    w = np.linspace(0.5, 2, 300).astype(np.float32)
    b = np.linspace(-1, 1, 300).astype(np.float32)
    assert np.allclose(oracle.layernorm(x, 1e-6, w, b), y * w + b, atol=1e-6)


def test_modulate_per_sample():
    ln = np.ones((6, 4), np.float32)
    scale = np.array([[1, 2, 3, 4], [0, 0, 0, 0]], np.float32)
    shift = np.array([[0, 0, 0, 0], [5, 5, 5, 5]], np.float32)
    out = oracle.modulate(ln, 3, scale, shift)
    assert np.array_equal(out[:3], np.tile([2, 3, 4, 5], (3, 1)))
    assert np.array_equal(out[3:], np.full((3, 4), 6, np.float32))


def test_layernorm_backward_finite_differences():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 40)).astype(np.float64)
    g = rng.standard_normal((3, 40))
    w = rng.uniform(0.5, 1.5, 40)
    eps = 1e-5

    def f(xx):
        mu = xx.mean(1, keepdims=True)
        v = ((xx - mu) ** 2).mean(1, keepdims=True)
        return ((xx - mu) / np.sqrt(v + eps) * w * g).sum()

    h = 1e-6
    num = np.zeros_like(x)
    for i in range(x.shape[0]):
        for j in range(x.shape[1]):
            e = np.zeros_like(x)
            e[i, j] = h
            num[i, j] = (f(x + e) - f(x - e)) / (2 * h)
    got = oracle.layernorm_backward(x.astype(np.float32), g.astype(np.float32), eps, w.astype(np.float32))
    assert np.abs(got - num).max() < 2e-4 * np.abs(num).max()


@pytest.fixture(scope="module")
def lib():
    native_build.build()
    return nat.lib()


def test_layernorm_rejects_bad_arguments(lib):
    p = ctypes.c_void_p(0x1000)
    f = lib.reels_layernorm_modulate
    assert f(None, 4, 16, 4, None, None, None, None, 1e-6, nat.BF16, p, None) == nat.EINVAL
    assert f(p, 4, 0, 4, None, None, None, None, 1e-6, nat.BF16, p, None) == nat.EINVAL
    assert f(p, 4, 20000, 4, None, None, None, None, 1e-6, nat.BF16, p, None) == nat.EINVAL
    assert f(p, 4, 16, 0, None, None, None, None, 1e-6, nat.BF16, p, None) == nat.EINVAL
    assert f(p, 4, 16, 4, None, None, None, None, float("nan"), nat.BF16, p, None) == nat.EINVAL
    assert f(p, 4, 16, 4, None, None, None, None, 1e-6, 9, p, None) == nat.EINVAL
    assert f(p, 4, 16, 4, None, None, None, None, 1e-6, nat.BF16, None, None) == nat.EINVAL
    b = lib.reels_layernorm_modulate_backward
    assert b(p, None, 4, 16, 4, None, None, None, 1e-6, nat.BF16, p, None, None, 0, None, 0, None) == nat.EINVAL
    assert b(p, p, 4, 16, 4, None, None, None, 1e-6, nat.BF16, None, None, None, 0, None, 0, None) == nat.EINVAL
    # parameter gradients need a workspace
    assert b(p, p, 4, 16, 4, None, None, None, 1e-6, nat.BF16, p, p, p, 0, None, 0, None) == nat.EINVAL
    assert lib.reels_layernorm_modulate_workspace_bytes(4, 16, 4) > 0


def test_gated_residual_rejects_bad_arguments(lib):
    p = ctypes.c_void_p(0x1000)
    f = lib.reels_gated_residual
    assert f(None, p, p, 4, 16, 4, nat.BF16, p, None) == nat.EINVAL
    assert f(p, p, p, 4, 0, 4, nat.BF16, p, None) == nat.EINVAL
    assert f(p, p, p, 4, 16, 0, nat.BF16, p, None) == nat.EINVAL
    b = lib.reels_gated_residual_backward
    assert b(p, None, p, 4, 16, 4, nat.BF16, p, p, 0, p, 1 << 20, None) == nat.EINVAL  # dgate needs y
    assert b(p, p, p, 4, 16, 4, nat.BF16, p, p, 0, None, 0, None) == nat.EINVAL       # and a workspace
