"""Time the q8 GEMM of the forward (_weight_mul) and of dX
(_weight_transpose_mul) for one shape through the C ABI.

    python -m reels_b200.microbench M K N [layout] [--reps R] [--once] [--gelu]

Prints one JSON line: microseconds and TFLOP/s (2*M*N*K / time) per pass,
CUDA-event timed on the launching stream after warm-up (the best of three
rounds that take the passes in turn).  The kernel and tile
shape follow the library's planner; REELS_Q8_TS (256, 192, 128, or 0 for the
SMEM x SMEM kernel) and REELS_Q8_TILE ("2x256", "2x128", "1x256", "1x128",
"pair") force one.

--gelu adds the passes with gelu_tanh fused into the epilogue
(reels_q8lora_forward_act writing y and the pre-activation; the dX of
reels_q8lora_backward_act through gelu_tanh') beside the same GEMM followed by
PyTorch's own tanh-GELU kernels (F.gelu / aten.gelu_backward), the unfused
way to run the projection and its activation.
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
    ap.add_argument("--gelu", action="store_true", help="also time the fused gelu_tanh epilogues")
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

    pre = torch.empty(M, N, device=dev, dtype=tdt)
    pre_x = torch.randn(M, K, device=dev).to(tdt)

    def fwd_gelu():
        nat.check("forward_act", L.reels_q8lora_forward_act(
            x.data_ptr(), q.data_ptr(), s.data_ptr(), layout, None, None, None, M, K, N, 0, 1.0, dt,
            nat.ACT_GELU_TANH, y.data_ptr(), pre.data_ptr(), None, ws.data_ptr(), wsn, st))

    def bwd_gelu():
        nat.check("backward_act", L.reels_q8lora_backward_act(
            None, dy.data_ptr(), q.data_ptr(), s.data_ptr(), layout, None, None, None, M, K, N, 0, 1.0, 1.0, dt,
            nat.ACT_GELU_TANH, pre_x.data_ptr(), dx.data_ptr(), None, None, 0, ws.data_ptr(), wsn, st))

    def fwd_then_gelu():
        nat.check("weight_mul", L.reels_q8_weight_mul(x.data_ptr(), q.data_ptr(), s.data_ptr(), layout, None, M, K,
                                                      N, dt, pre.data_ptr(), ws.data_ptr(), wsn, st))
        torch.nn.functional.gelu(pre, approximate="tanh", out=y)

    def dx_then_gelu_grad():
        bwd()
        torch.ops.aten.gelu_backward(dx, pre_x, approximate="tanh")

    out = {"M": M, "K": K, "N": N, "layout": layout, "dtype": a.dtype}
    if a.once:
        fwd()
        bwd()
        torch.cuda.synchronize(dev)
        nat.check("device status", L.reels_lowvram_check_device_status(st))
        print(json.dumps(out), flush=True)
        return
    passes = [("fwd", fwd), ("dx", bwd)]
    if a.gelu:
        passes += [("fwd_gelu_fused", fwd_gelu), ("fwd_then_torch_gelu", fwd_then_gelu),
                   ("dx_gelu_fused", bwd_gelu), ("dx_then_torch_gelu_grad", dx_then_gelu_grad)]
    # Round-robin over the passes, best of three rounds each: a pass timed
    # late in a long run would otherwise see lower clocks under the power cap.
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
    for name, _ in passes:
        us = best[name]
        out[name] = {"us": round(us, 1), "tflops": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 1)}
    nat.check("device status", L.reels_lowvram_check_device_status(st))
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
