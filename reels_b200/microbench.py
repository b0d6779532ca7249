"""Time the q8 GEMM of the forward (_weight_mul) and of dX
(_weight_transpose_mul) for one shape through the C ABI.

    python -m reels_b200.microbench M K N [layout] [--reps R] [--once]

Prints one JSON line: microseconds and TFLOP/s (2*M*N*K / time) per pass,
CUDA-event timed on the launching stream after warm-up.  The kernel and tile
shape follow the library's planner; REELS_Q8_TS (256, 192, 128, or 0 for the
SMEM x SMEM kernel) and REELS_Q8_TILE ("2x256", "2x128", "1x256", "1x128",
"pair") force one.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _native as nat
from . import build as native_build


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("M", type=int)
    ap.add_argument("K", type=int)
    ap.add_argument("N", type=int)
    ap.add_argument("layout", type=int, nargs="?", default=0)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16"])
    ap.add_argument("--once", action="store_true",
                    help="one forward and one dX launch, no timing (for a profiler capture)")
    a = ap.parse_args()
    native_build.build()
    L = nat.lib()
    M, K, N, layout = a.M, a.K, a.N, a.layout
    tdt, dt = (torch.bfloat16, nat.BF16) if a.dtype == "bf16" else (torch.float16, nat.F16)
    dev = torch.device("cuda", 0)
    x = torch.randn(M, K, device=dev).to(tdt)
    dy = torch.randn(M, N, device=dev).to(tdt)
    q = torch.randint(-127, 128, (K, N) if layout == 0 else (N, K), device=dev, dtype=torch.int8)
    s = torch.rand(N, device=dev) * 1e-3 + 1e-4
    y = torch.empty(M, N, device=dev, dtype=tdt)
    dx = torch.empty(M, K, device=dev, dtype=tdt)
    wsn = max(L.reels_q8lora_workspace_bytes(M, K, N, 0, dt, p) for p in (0, 1))
    ws = torch.empty(max(wsn, 256), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream

    def fwd():
        nat.check("weight_mul", L.reels_q8_weight_mul(x.data_ptr(), q.data_ptr(), s.data_ptr(), layout, None, M, K,
                                                      N, dt, y.data_ptr(), ws.data_ptr(), wsn, st))

    def bwd():
        nat.check("weight_transpose_mul", L.reels_q8_weight_transpose_mul(
            dy.data_ptr(), q.data_ptr(), s.data_ptr(), layout, M, K, N, dt, dx.data_ptr(), ws.data_ptr(), wsn, st))

    out = {"M": M, "K": K, "N": N, "layout": layout, "dtype": a.dtype}
    if a.once:
        fwd()
        bwd()
        torch.cuda.synchronize(dev)
        nat.check("device status", L.reels_lowvram_check_device_status(st))
        print(json.dumps(out), flush=True)
        return
    for name, fn in (("fwd", fwd), ("dx", bwd)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) / a.reps * 1e3
        out[name] = {"us": round(us, 1), "tflops": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 1)}
    nat.check("device status", L.reels_lowvram_check_device_status(st))
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
