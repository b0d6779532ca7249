"""Token-count sweep of one int8-weight LoRA linear, fwd+bwd, on one GPU.

    python -m reels_b200.sweep [--N 13824 --K 5120] [--tokens 128,512,...]
                               [--ranks 8,64] [--dtype f16] [--loss-scale 1024]
                               [--dropout P]

Defaults are the bandwidth-bound sweep on the Wan-2.1-14B FFN up-projection
(W 13824 x 5120, int8 per output row; fp16 activations; dY carries a static
loss scale of 1024, removed again through the backward's grad_scale).  For
each (tokens, rank) the forward and the backward run through the C ABI on
seeded synthetic inputs, timed with CUDA events on the launching stream after
warm-up, and one JSON line reports:

  us_fwd, us_bwd, us        device time per pass and for fwd+bwd
  tflops                    algorithmic FLOPs / time (below)
  hbm_gbs                   algorithmic bytes / time, and its fraction of the
                            measured copy bandwidth (MEASURED_PEAKS.json)
  tensor_frac               tflops / the measured bf16 burst peak

Algorithmic FLOPs (fwd+bwd): the two GEMMs over the frozen weight (Y and dX;
dW is not computed, the weight is frozen), 4*M*N*K, and the six rank-r
products (T, the adapter term of Y, G, that of dX, dA, dB), 2*M*r*(3K + 3N).  Algorithmic bytes:
what must cross HBM at least once per pass -- forward: x, W (int8 + scales),
y; backward: dy, W, x (for dA), dx; the rank-r tensors are counted too.

--dropout P runs the training forward and backward with LoRA dropout
(reels_q8lora_forward_dropout / _backward_dropout): the same algorithmic
FLOPs and bytes, plus the dropped-out input's pass and the masked adapter
part of dx, which the figures then include as overhead.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from . import _native as nat
from . import build as native_build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--N", type=int, default=13824)
    ap.add_argument("--K", type=int, default=5120)
    ap.add_argument("--tokens", default="128,512,2048,8192,32760")
    ap.add_argument("--ranks", default="8,64")
    ap.add_argument("--dtype", default="f16", choices=["f16", "bf16"])
    ap.add_argument("--loss-scale", type=float, default=1024.0)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--dropout", type=float, default=0.0)
    a = ap.parse_args()
    native_build.build()
    L = nat.lib()
    hbm, tf_peak, src = peaks()
    dev = torch.device("cuda", 0)
    tdt, dt = (torch.float16, nat.F16) if a.dtype == "f16" else (torch.bfloat16, nat.BF16)
    N, K = a.N, a.K
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    from . import quantize_frozen_matrix
    w = torch.empty((K, N), device=dev).normal_(0.0, 0.02, generator=g).t()  # (out, in), column-major
    qm = quantize_frozen_matrix(w)
    del w
    q, s = qm.values, qm.scales
    st = torch.cuda.current_stream(dev).cuda_stream
    for r in [int(v) for v in a.ranks.split(",")]:
        alpha = float(r)
        A = (torch.randn((K, r), device=dev, generator=g) / K ** 0.5).to(tdt)
        B = (0.01 * torch.randn((r, N), device=dev, generator=g)).to(tdt)
        for M in [int(v) for v in a.tokens.split(",")]:
            x = torch.randn((M, K), device=dev, generator=g).to(tdt)
            dy = (torch.randn((M, N), device=dev, generator=g) * a.loss_scale).to(tdt)
            y = torch.empty((M, N), device=dev, dtype=tdt)
            dx = torch.empty((M, K), device=dev, dtype=tdt)
            saved = torch.empty((max(L.reels_q8lora_saved_bytes(M, r, dt), 16),), dtype=torch.uint8, device=dev)
            grad = torch.zeros((r * (K + N),), dtype=torch.float32, device=dev)
            flag = nat.PASS_DROPOUT if a.dropout > 0 else 0
            wsn = max(L.reels_q8lora_workspace_bytes(M, K, N, r, dt, p | flag) for p in (0, 1))
            ws = torch.empty((max(wsn, 256),), dtype=torch.uint8, device=dev)

            def fwd():
                if a.dropout > 0:
                    nat.check("forward", L.reels_q8lora_forward_dropout(
                        x.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(), None, M, K, N, r,
                        alpha, dt, a.dropout, 1, 0, y.data_ptr(), saved.data_ptr(), ws.data_ptr(), wsn, st))
                    return
                nat.check("forward", L.reels_q8lora_forward(
                    x.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(), None, M, K, N, r, alpha,
                    dt, y.data_ptr(), saved.data_ptr(), ws.data_ptr(), wsn, st))

            def bwd():
                if a.dropout > 0:
                    nat.check("backward", L.reels_q8lora_backward_dropout(
                        x.data_ptr(), dy.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(),
                        saved.data_ptr(), M, K, N, r, alpha, 1.0 / a.loss_scale, dt, a.dropout, 1, 0, dx.data_ptr(),
                        grad.data_ptr(), grad.data_ptr() + 4 * K * r, 0, ws.data_ptr(), wsn, st))
                    return
                nat.check("backward", L.reels_q8lora_backward(
                    x.data_ptr(), dy.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(),
                    saved.data_ptr(), M, K, N, r, alpha, 1.0 / a.loss_scale, dt, dx.data_ptr(), grad.data_ptr(),
                    grad.data_ptr() + 4 * K * r, 0, ws.data_ptr(), wsn, st))

            res = {}
            for name, fn in (("fwd", fwd), ("bwd", bwd)):
                for _ in range(3):
                    fn()
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(a.reps):
                    fn()
                e1.record()
                torch.cuda.synchronize(dev)
                res[name] = e0.elapsed_time(e1) / a.reps * 1e3
            nat.check("device status", L.reels_lowvram_check_device_status(st))
            us = res["fwd"] + res["bwd"]
            e = 2  # bytes per activation element
            flops = 4.0 * M * N * K + 2.0 * M * r * (3.0 * K + 3.0 * N)
            wbytes = N * K + 4 * N
            rank_bytes = e * r * (K + N) * 2 + e * r * M * 2 + 4 * r * (K + N)
            byts = (e * M * K + wbytes + e * M * N) + (e * M * N + wbytes + e * M * K + e * M * K) + rank_bytes
            gbs = byts / (us * 1e-6) / 1e9
            tfl = flops / (us * 1e-6) / 1e12
            print(json.dumps({
                "shape": f"W {N}x{K}", "tokens": M, "rank": r, "dtype": a.dtype, "loss_scale": a.loss_scale,
                "dropout": a.dropout,
                "us_fwd": round(res["fwd"], 1), "us_bwd": round(res["bwd"], 1), "us": round(us, 1),
                "tflops": round(tfl, 1), "tensor_frac": round(tfl / tf_peak, 3),
                "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 3),
                "algorithmic_bytes": int(byts), "algorithmic_flops": flops,
                "peaks": {"hbm_gbs": hbm, "bf16_tflops": tf_peak, "source": src},
            }), flush=True)


if __name__ == "__main__":
    main()
