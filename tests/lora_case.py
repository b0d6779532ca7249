"""Shared helpers for the GPU parity tests: seeded inputs in the reference's
memory layouts, the device layer built from them, and the comparison metric.

Inputs follow the measurement plan: numpy Generator(PCG64(seed)), X and dY
~ N(0, 1), W ~ N(0, 0.02) quantised per output row, A ~ N(0, a_std),
B ~ N(0, 0.01); 16-bit inputs are rounded to the activation type first so
the oracle sees exactly the values the GPU sees.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import oracle

TOL = 3e-3          # relative L2 bound of the north star, Y / dX / dA / dB
TOL_F32 = 1e-5      # fp32 activations (CUDA-core path) vs the fp64 oracle


def round_to(x, dtype):
    x = np.asarray(x, np.float32)
    if dtype == "bf16":
        return oracle.bf16_round(x)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


@dataclass
class Case:
    M: int
    K: int
    N: int
    r: int
    alpha: float
    dtype: str
    layout: int
    X: np.ndarray
    Wmem: np.ndarray
    q: np.ndarray
    s: np.ndarray
    A: np.ndarray     # [K][r]
    B: np.ndarray     # [r][N]
    dY: np.ndarray
    bias: np.ndarray | None = None


def make_case(M, K, N, r, alpha=None, dtype="bf16", layout=0, seed=0, a_std=None, dy_scale=1.0, bias=False):
    g = np.random.Generator(np.random.PCG64(seed))
    X = round_to(g.standard_normal((M, K)), dtype)
    W = (0.02 * g.standard_normal((N, K))).astype(np.float32)
    Wmem = np.ascontiguousarray(W.T) if layout == 0 else W
    a_std = (1.0 / np.sqrt(K)) if a_std is None else a_std
    A = round_to(a_std * g.standard_normal((K, max(r, 0))), dtype)
    B = round_to(0.01 * g.standard_normal((max(r, 0), N)), dtype)
    dY = round_to(dy_scale * g.standard_normal((M, N)), dtype)
    q, s = oracle.quantize(Wmem, layout)
    b = round_to(0.1 * g.standard_normal(N), dtype) if bias else None
    return Case(M, K, N, r, float(alpha if alpha is not None else max(r, 1)), dtype, layout, X, Wmem, q, s, A, B, dY,
                b)


def case_from_fixture(f):
    import json
    meta = json.loads(str(f["meta"]))
    return Case(meta["M"], meta["K"], meta["N"], meta["r"], meta["alpha"], meta["dtype"], meta["layout"], f["X"],
                f["W"], f["q"], f["s"], f["A"], f["B"], f["dY"])


def torch_dtype(torch, name):
    return {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[name]


def device_layer(torch, c: Case):
    """The LoRALinear on the GPU with the reference's column-major storage."""
    from reels_b200 import LoRALinear, QuantizedMatrix
    dt = torch_dtype(torch, c.dtype)
    q = torch.from_numpy(c.q).cuda()
    values = q.t() if c.layout == 0 else q          # logical (out, in)
    qm = QuantizedMatrix(values, torch.from_numpy(c.s).cuda(), dt)
    A = torch.from_numpy(c.A).cuda().to(dt).t()      # logical (rank, in), column-major
    B = torch.from_numpy(c.B).cuda().to(dt).t()      # logical (out, rank), column-major
    bias = torch.from_numpy(c.bias).cuda().to(dt) if c.bias is not None else None
    return LoRALinear(qm, bias, A, B, c.alpha)


def oracle_outputs(c: Case):
    Y = oracle.lora_forward(c.X, c.q, c.s, c.layout, c.A, c.B, c.alpha, bias=c.bias)
    dX, dA, dB = oracle.lora_backward(c.X, c.dY, c.q, c.s, c.layout, c.A, c.B, c.alpha)
    return Y, dX, dA, dB


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    den = np.sqrt((b * b).sum())
    num = np.sqrt(((a - b) ** 2).sum())
    return float(num / den) if den > 0 else float(num)
