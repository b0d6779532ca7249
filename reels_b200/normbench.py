"""Time the fused LayerNorm + modulation (forward, and the pullback with the
modulation's parameter gradients) on one GPU against PyTorch evaluating the
same expression as separate kernels, the way the reference's broadcasts do.

    python -m reels_b200.normbench [--M 32760] [--K 5120] [--dtype bf16]

One JSON line: microseconds per pass (CUDA events on the launching stream,
best of three rounds after warm-up) and the HBM bandwidth of the fused
kernels, counted as one read of x and one write of the output for the
forward, and reads of x and dout plus the write of dx for dx (the
parameter-gradient pass re-reads x and dout).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from . import build as native_build


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=32760)
    ap.add_argument("--K", type=int, default=5120)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16"])
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    native_build.build()
    from .lowvram import layernorm_modulate, layernorm_modulate_backward
    dev = torch.device("cuda", 0)
    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    M, K = a.M, a.K
    x = torch.randn(M, K, device=dev).to(dt)
    dout = torch.randn(M, K, device=dev).to(dt)
    scale = (0.1 * torch.randn(1, K, device=dev)).to(dt)
    shift = (0.1 * torch.randn(1, K, device=dev)).to(dt)

    def fused():
        layernorm_modulate(x, scale, shift, 1e-6)

    def fused_bwd():
        layernorm_modulate_backward(x, dout, scale, 1e-6, param_grads=True)

    def torch_fwd():  # linear.jl:49-59 then 26-36, as separate kernels
        x32 = x.float()
        mu = x32.mean(-1, keepdim=True)
        c = x32 - mu
        var = (c * c).mean(-1, keepdim=True)
        ln = (c / torch.sqrt(var + 1e-6)).to(dt)
        (ln.float() * (1 + scale.float()) + shift.float()).to(dt)

    passes = [("fused_fwd", fused), ("torch_fwd", torch_fwd), ("fused_bwd_with_param_grads", fused_bwd)]
    for _, fn in passes:
        for _ in range(3):
            fn()
    torch.cuda.synchronize(dev)
    best = {}
    for _ in range(3):
        for name, fn in passes:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.reps):
                fn()
            e1.record()
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) / a.reps * 1e3
            best[name] = min(best.get(name, us), us)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as fh:
            hbm = float(json.load(fh)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        hbm = 6650.0
    e = 2
    out = {"M": M, "K": K, "dtype": a.dtype}
    for name, us in best.items():
        out[name] = {"us": round(us, 1)}
    gb = 2 * M * K * e / (best["fused_fwd"] * 1e-6) / 1e9
    out["fused_fwd"]["gbs"] = round(gb, 1)
    out["fused_fwd"]["hbm_frac"] = round(gb / hbm, 3)
    gbb = 5 * M * K * e / (best["fused_bwd_with_param_grads"] * 1e-6) / 1e9
    out["fused_bwd_with_param_grads"]["gbs"] = round(gbb, 1)
    out["fused_bwd_with_param_grads"]["hbm_frac"] = round(gbb / hbm, 3)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
