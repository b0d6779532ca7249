"""CPU checks of the optimizer step's host logic and of its oracle.

The schedule, the weight-decay mask and the bias corrections follow
src/training/optimizer.jl:26-60; the oracle's AdamW step follows
optimizer.jl:63-71 with the clip of wan_runner.jl:213-221.  The GPU kernels
are compared with this oracle bit for bit in test_gpu_optim.py.
"""
import ctypes
import math

import numpy as np
import pytest

import oracle
from reels_b200 import _native as nat
from reels_b200 import build as native_build
from reels_b200 import optim

f32 = np.float32


def test_weight_decay_mask_is_occursin():
    names = ["blocks.0.attn.q.lora_A", "blocks.0.norm.bias", "blocks.1.ffn.lora_B"]
    assert optim.weight_decay_mask(names, [r"\.bias$", "norm"]) == [True, False, True]
    assert optim.weight_decay_mask(names, []) == [True, True, True]
    assert optim.weight_decay_mask(names, ["lora_[AB]"]) == [False, True, False]


def test_learning_rate_schedule():
    # warmup: base * step / warm
    assert optim.learning_rate(1e-3, "cosine", 10, 5, 100) == float(f32(5e-4))
    assert optim.learning_rate(1e-3, "linear", 10, 10, 100) == float(f32(1e-3))
    # after warmup, progress = (step - warm) / (total - warm), clamped
    assert optim.learning_rate(1e-3, "constant", 10, 50, 100) == float(f32(1e-3))
    lin = optim.learning_rate(1e-3, "linear", 10, 55, 100)
    assert lin == float(f32(1e-3) * (f32(1) - f32(0.5)))
    cos = optim.learning_rate(2e-3, "cosine", 0, 30, 120)
    assert cos == pytest.approx(2e-3 * (1 + math.cos(math.pi * 0.25)) / 2, rel=1e-6)
    assert optim.learning_rate(1e-3, "linear", 0, 500, 100) == 0.0  # progress clamps at 1
    # warm-up in Float32 arithmetic (base::Float32 * step / warm, each op
    # rounded): at the last warm-up step 1f-4 * 5 / 5 is 9.999999f-5, not 1f-4
    assert optim.learning_rate(1e-4, "constant", 5, 5, 100) == float(f32(9.999999e-05))
    assert optim.learning_rate(3e-4, "cosine", 7, 5, 100) == float(f32(0.00021428571))
    with pytest.raises(ValueError):
        optim.learning_rate(1e-3, "step", 0, 1, 10)


def test_bias_corrections_follow_float32_power():
    # beta^1 = beta; beta^3 = beta*beta*beta in fp32; others rounded from fp64
    assert optim.f32_pow(0.9, 1) == f32(0.9)
    b = f32(0.999)
    assert optim.f32_pow(0.999, 3) == f32(f32(b * b) * b)
    for step in (2, 5, 10, 1000, 12345):
        assert optim.f32_pow(0.999, step) == f32(float(b) ** step)
    c1, c2 = optim.bias_corrections(optim.AdamW(), 1)
    assert c1 == float(f32(1) - f32(0.9)) and c2 == float(f32(1) - f32(0.999))


def test_oracle_adamw_known_answer():
    # g = 1, zero moments, w = 1, step 1: m/c1 = v/c2 = 1, so the step is
    # 1/(1 + 1e-8) = 1 in fp32, plus decay 0.01 * w.
    c1, c2 = optim.bias_corrections(optim.AdamW(), 1)
    m, v, w = oracle.adamw_update(np.ones(2, f32), np.zeros(2), np.zeros(2), np.ones(2), 1e-4, 0.9, 0.999, 1e-8,
                                  0.01, c1, c2)
    assert m[0] == f32(1) - f32(0.9)  # (1f0 - beta1) g: 0.100000024, not 0.1
    assert w[0] == f32(1) - f32(f32(1e-4) * f32(f32(1) + f32(0.01)))
    # no decay: w moves by exactly lr
    _, _, w0 = oracle.adamw_update(np.ones(1, f32), np.zeros(1), np.zeros(1), np.ones(1), 1e-4, 0.9, 0.999, 1e-8,
                                   0.0, c1, c2)
    assert w0[0] == f32(1) - f32(1e-4)


def test_oracle_adamw_matches_numpy_restatement():
    rng = np.random.default_rng(3)
    n = 1000
    g = rng.standard_normal(n).astype(f32)
    m = (0.1 * rng.standard_normal(n)).astype(f32)
    v = (0.01 * rng.random(n)).astype(f32)
    w = rng.standard_normal(n).astype(f32)
    lr, b1, b2, eps, decay, c1, c2, gs, cs = (f32(3e-4), f32(0.9), f32(0.999), f32(1e-8), f32(0.01), f32(0.19),
                                              f32(0.002), f32(0.5), f32(0.25))
    gg = (g * gs) * cs
    mm = b1 * m + (f32(1) - b1) * gg
    vv = b2 * v + (f32(1) - b2) * (gg * gg)
    ww = w - lr * ((mm / c1) / (np.sqrt(vv / c2) + eps) + decay * w)
    om, ov, ow = oracle.adamw_update(g, m, v, w, lr, b1, b2, eps, decay, c1, c2, gs, cs)
    assert np.array_equal(om, mm) and np.array_equal(ov, vv) and np.array_equal(ow, ww)


def test_oracle_sumsq():
    assert oracle.sumsq([np.array([3, 4], f32)]) == 25.0
    assert oracle.sumsq([np.ones(4, f32), np.ones(5, f32)], 0.5) == 9 * 0.25


@pytest.fixture(scope="module")
def lib():
    native_build.build()
    return nat.lib()


def test_prepare_rejects_bad_tables(lib):
    p = 0x1000
    ws = ctypes.c_void_p(0x10000)  # never dereferenced: the checks come first
    good = nat.OptTensor(p, p, p, p, p, 10, nat.BF16, 1)
    n = lib.reels_opt_workspace_bytes(1)
    assert n >= 256 and lib.reels_opt_workspace_bytes(3) > n
    bad_dtype = (nat.OptTensor * 1)(nat.OptTensor(p, p, p, p, p, 10, 7, 1))
    assert lib.reels_opt_prepare(bad_dtype, 1, ws, n, None) == nat.EINVAL
    assert "param_dtype" in lib.reels_lowvram_last_error().decode()
    null_ptr = (nat.OptTensor * 1)(nat.OptTensor(p, None, p, p, p, 10, nat.BF16, 1))
    assert lib.reels_opt_prepare(null_ptr, 1, ws, n, None) == nat.EINVAL
    neg = (nat.OptTensor * 1)(nat.OptTensor(p, p, p, p, p, -1, nat.BF16, 1))
    assert lib.reels_opt_prepare(neg, 1, ws, n, None) == nat.EINVAL
    one = (nat.OptTensor * 1)(good)
    assert lib.reels_opt_prepare(one, 1, ws, n - 8, None) == nat.EINVAL  # too small
    assert lib.reels_opt_prepare(one, 1, ctypes.c_void_p(0x10008), n, None) == nat.EINVAL  # misaligned
    assert lib.reels_opt_prepare(one, -1, ws, n, None) == nat.EINVAL
    assert lib.reels_grad_norm_sq(None, 1.0, ws, None) == nat.EINVAL
    assert lib.reels_adamw_update(ws, 1e-4, 0.9, 0.999, 1e-8, 0.01, 0.0, 0.001, 1.0, None, 0.0, None) == nat.EINVAL
    assert "corrections" in lib.reels_lowvram_last_error().decode()
    assert lib.reels_adamw_update(ws, float("nan"), 0.9, 0.999, 1e-8, 0.01, 0.1, 0.001, 1.0, None, 0.0,
                                  None) == nat.EINVAL
    assert lib.reels_adamw_update(ws, 1e-4, 0.9, 0.999, 1e-8, 0.01, 0.1, 0.001, 1.0, ws, 0.0, None) == nat.EINVAL


def test_reference_known_answers_on_the_oracle():
    """The reference's own AdamW cases (test/unit/training.jl:87-127):
    named weight-decay exclusions give exactly 0.95 and 1 after one step of
    lr 0.1, weight decay 0.5 on zero gradients."""
    assert optim.weight_decay_mask(["blocks.0.attn.lora_A.weight", "blocks.0.attn.bias"], [r"bias$"]) == [True, False]
    c1, c2 = optim.bias_corrections(optim.AdamW(), 1)
    for decay, expect in ((0.5, 0.95), (0.0, 1.0)):
        _, _, w = oracle.adamw_update(np.zeros(2, f32), np.zeros(2), np.zeros(2), np.ones(2), 0.1, 0.9, 0.999, 1e-8,
                                      decay, c1, c2)
        assert np.array_equal(w, np.full(2, f32(expect)))
