"""The optimizer step after the gradient all-reduce, on the GPU.

Mirrors src/training/optimizer.jl and the step of src/training/wan_runner.jl:

==============================  =============================================
reference                       here
==============================  =============================================
AdamW                           :class:`AdamW` (optimizer.jl:1-7)
AdamWState                      :class:`AdamWState` (optimizer.jl:9-24)
weight_decay_mask               :func:`weight_decay_mask` (optimizer.jl:26-37)
learning_rate                   :func:`learning_rate` (optimizer.jl:39-47)
update!                         :func:`update_` (optimizer.jl:48-73)
norm + clip (wan_runner.jl)     :func:`grad_norm_sq`, ``max_gradient_norm`` of
                                :func:`update_` (wan_runner.jl:213-221)
==============================  =============================================

The reference loops over the parameter list with several broadcasts per
tensor and reads the gradient norm back to the host before clipping.  Here
the norm is one launch over every tensor and the clip, moments, master
update and the rewrite of the model's copy are one more, reading the norm on
the device: no host round trip inside the step.  Per element the arithmetic
is the reference's, rounded once per operation in fp32 (no fused
multiply-adds), so the master weights, moments and parameters equal a
restatement of update! bit for bit given the same gradients and clip factor.

Bias corrections ``1 - beta^step`` are formed on the host as Julia forms
``beta1^state.step`` for a Float32 ``beta1`` and an integer step: for step 3
the product ``beta*beta*beta`` in fp32, otherwise the power by squaring in
fp64, rounded to fp32 (Julia 1.11 Base, ``^(::Float32, ::Integer)`` and
``Base.power_by_squaring``).
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _native as nat

_DT = {torch.float32: nat.F32, torch.float16: nat.F16, torch.bfloat16: nat.BF16}


@dataclass(frozen=True)
class AdamW:
    """AdamW hyperparameters (optimizer.jl:1-7)."""
    learning_rate: float = 1e-4
    beta1: float = 0.9
    beta2: float = 0.999
    epsilon: float = 1e-8
    weight_decay: float = 0.01


def weight_decay_mask(names: Sequence[str], exclusions: Sequence[str]) -> List[bool]:
    """One flag per parameter name; False where any exclusion pattern occurs
    in the name (optimizer.jl:26-37, ``occursin(Regex, name)``)."""
    patterns = [re.compile(e) for e in exclusions]
    return [not any(p.search(n) for p in patterns) for n in names]


def learning_rate(base: float, kind: str, warmup_steps: int, step: int, total: int) -> float:
    """Scheduled learning rate of optimizer.jl:39-47 (kind: constant, linear
    or cosine), as an fp32 value."""
    f32 = np.float32
    if warmup_steps > 0 and step <= warmup_steps:
        # base is the Float32 training.learning_rate (config/schema.jl:40):
        # Float32 * Int and Float32 / Int each round to Float32
        return float(f32(f32(base) * f32(step)) / f32(warmup_steps))
    progress = f32(min(max((step - warmup_steps) / max(total - warmup_steps, 1), 0.0), 1.0))
    if kind == "constant":
        return float(f32(base))
    if kind == "linear":
        return float(f32(base) * (f32(1.0) - progress))
    if kind == "cosine":
        return float(f32(base) * (f32(1.0) + f32(math.cos(math.pi * float(progress)))) / f32(2.0))
    raise ValueError(f"unknown scheduler {kind}")


def _power_by_squaring(x: float, p: int) -> float:
    """Julia Base.power_by_squaring for p >= 0, in fp64 (Python floats)."""
    if p == 1:
        return x
    if p == 0:
        return 1.0
    if p == 2:
        return x * x
    t = ((p & -p).bit_length() - 1) + 1  # trailing_zeros(p) + 1
    p >>= t
    t -= 1
    while t > 0:
        x = x * x
        t -= 1
    y = x
    while p > 0:
        t = ((p & -p).bit_length() - 1) + 1
        p >>= t
        t -= 1
        while t >= 0:
            x = x * x
            t -= 1
        y = y * x
    return y


def f32_pow(beta: float, step: int) -> np.float32:
    """``Float32(beta)^step`` as Julia 1.11 evaluates it."""
    b = np.float32(beta)
    if step == 3:
        return np.float32(np.float32(b * b) * b)
    if step < 0:
        raise ValueError("negative step")
    return np.float32(_power_by_squaring(float(b), step))


def bias_corrections(opt: AdamW, step: int):
    """(1 - beta1^step, 1 - beta2^step) in fp32 (optimizer.jl:59-60)."""
    one = np.float32(1.0)
    return float(one - f32_pow(opt.beta1, step)), float(one - f32_pow(opt.beta2, step))


class AdamWState:
    """Moments and fp32 masters of every parameter (optimizer.jl:9-24), plus
    the prepared device table of the last (params, grads) set."""

    def __init__(self, params: Sequence[torch.Tensor]):
        for p in params:
            if p.dtype not in _DT or not p.is_cuda or not p.is_contiguous():
                raise ValueError("parameters must be contiguous CUDA fp32/fp16/bf16 tensors")
        self.step = 0
        self.m = [torch.zeros(p.numel(), dtype=torch.float32, device=p.device) for p in params]
        self.v = [torch.zeros(p.numel(), dtype=torch.float32, device=p.device) for p in params]
        self.master = [p.detach().reshape(-1).to(torch.float32).clone() for p in params]
        self._ws: Optional[torch.Tensor] = None
        self._key = None

    def _prepare(self, params, grads, mask) -> torch.Tensor:
        if not (len(params) == len(grads) == len(self.m) == len(self.v) == len(self.master)):
            raise ValueError("parameter, gradient, and optimizer state lengths differ")
        if mask is not None and len(mask) != len(params):
            raise ValueError("weight-decay mask and parameter lengths differ")
        for p, g, w in zip(params, grads, self.master):
            if p.dtype not in _DT or not p.is_contiguous() or p.numel() != w.numel() or p.device != w.device:
                raise ValueError("parameters must be the contiguous fp32/fp16/bf16 tensors the state was made for")
            if g.dtype != torch.float32 or not g.is_contiguous() or g.numel() != w.numel() or g.device != w.device:
                raise ValueError("gradients must be contiguous fp32 tensors of the parameters' sizes")
        # the table holds pointers, element types and the decay flags
        key = (tuple((p.data_ptr(), p.dtype) for p in params), tuple(g.data_ptr() for g in grads),
               tuple(bool(x) for x in mask) if mask is not None else None)
        if key == self._key and self._ws is not None:
            return self._ws
        n = len(params)
        table = (nat.OptTensor * max(n, 1))()
        for i, (p, g, m, v, w) in enumerate(zip(params, grads, self.m, self.v, self.master)):
            table[i] = nat.OptTensor(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), w.data_ptr(), p.numel(),
                                     _DT[p.dtype], 1 if (mask is None or mask[i]) else 0)
        L = nat.lib()
        nbytes = L.reels_opt_workspace_bytes(n)
        dev = params[0].device if n else torch.device("cuda", torch.cuda.current_device())
        ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
        off = (-ws.data_ptr()) % 256
        ws = ws[off: off + nbytes]
        stream = torch.cuda.current_stream(dev).cuda_stream
        nat.check("reels_opt_prepare", L.reels_opt_prepare(table, n, ws.data_ptr(), nbytes, stream))
        self._ws, self._key = ws, key
        return ws


def grad_norm_sq(state: AdamWState, params, grads, grad_scale: float = 1.0,
                 weight_decay_mask: Optional[Sequence[bool]] = None) -> torch.Tensor:
    """Sum of squared gradients over every tensor, as a device fp32 scalar
    (the ``norm_squared`` of wan_runner.jl:215; no host synchronisation)."""
    ws = state._prepare(params, grads, weight_decay_mask)
    out = torch.empty((), dtype=torch.float32, device=ws.device)
    stream = torch.cuda.current_stream(ws.device).cuda_stream
    nat.check("reels_grad_norm_sq", nat.lib().reels_grad_norm_sq(ws.data_ptr(), float(grad_scale), out.data_ptr(),
                                                                 stream))
    return out


def update_(opt: AdamW, state: AdamWState, params, grads, learning_rate: Optional[float] = None,
            weight_decay_mask: Optional[Sequence[bool]] = None, max_gradient_norm: Optional[float] = None,
            grad_scale: float = 1.0) -> Optional[torch.Tensor]:
    """One AdamW step ``update!`` (optimizer.jl:48-73) over every parameter:
    moments, fp32 master and the parameter itself rewritten in place.

    ``max_gradient_norm``: clip first as wan_runner.jl:215-221 does (scale
    every gradient by max/norm when the global norm exceeds it); the norm is
    computed and applied on the device and returned as its square (a device
    scalar, for metrics).  ``grad_scale`` multiplies the gradients first (e.g.
    1/gradient_accumulation)."""
    ws = state._prepare(params, grads, weight_decay_mask)
    stream = torch.cuda.current_stream(ws.device).cuda_stream
    L = nat.lib()
    sumsq = None
    if max_gradient_norm is not None:
        sumsq = torch.empty((), dtype=torch.float32, device=ws.device)
        nat.check("reels_grad_norm_sq", L.reels_grad_norm_sq(ws.data_ptr(), float(grad_scale), sumsq.data_ptr(),
                                                             stream))
    state.step += 1
    c1, c2 = bias_corrections(opt, state.step)
    lr = opt.learning_rate if learning_rate is None else learning_rate
    nat.check("reels_adamw_update", L.reels_adamw_update(
        ws.data_ptr(), float(np.float32(lr)), float(np.float32(opt.beta1)), float(np.float32(opt.beta2)),
        float(np.float32(opt.epsilon)), float(np.float32(opt.weight_decay)), c1, c2, float(grad_scale),
        sumsq.data_ptr() if sumsq is not None else None,
        float(max_gradient_norm) if max_gradient_norm is not None else 0.0, stream))
    return sumsq
