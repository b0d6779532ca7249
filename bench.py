"""Benchmark: Int8-weight LoRA linear forward + backward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config block|cfg1|ffn8k|wan14b|wan14b-stack|ltx]
    python bench.py --mode sweep|gemm|norm|adamw [...]     (kernel measurements)

Workload (the default "block"): every linear of one Wan-2.1-1.3B DiT block at
32760 tokens per sample -- self-attention q/k/v/o and cross-attention q/o
(1536x1536 over 32760 tokens), cross-attention k/v (1536x1536 over 512 context
tokens), FFN up 1536->8960 and down 8960->1536 -- int8 per-row weights from
N(0, 0.02), LoRA rank 32 / alpha 32 on every linear, bf16 activations
~N(0,1).  One step = the forward of the ten linears, then their backward in
reverse order (dX, dA, dB), and at N > 1 the fp32 all-reduce of every LoRA
gradient (overlapped with the backward).  Data-parallel weak scaling: each
rank processes its own 32760-token sample.  "wan14b-stack" is the whole
40-block Wan-2.1-14B stack per GPU (153 M adapter parameters, 613 MB of fp32
gradients all-reduced per step in buckets).

Our arm prints one JSON line (rank 0).  ``--impl reference`` times the
reference's CPU code path (oracle/numpy_port.py: dequantise-materialise plus
OpenBLAS sgemm, the op order of src/layers/lora.jl:56-118) on the host cores
instead; the reference itself is Julia and cannot run in this image.

The ``--mode`` measurements print one JSON line per case:
  sweep  token sweep of one linear, fwd+bwd (default: W 13824x5120, fp16,
         static loss scale 1024, M in 128..32760, r in 8, 64)
  gemm   the q8 GEMMs of _weight_mul and _weight_transpose_mul for --shape
         M,K,N (optionally with the fused gelu_tanh epilogues)
  norm   fused LayerNorm + modulation against the same expression as
         separate PyTorch kernels
  adamw  gradient norm + clipped AdamW over the 40-block Wan 14B adapters
  trace  per-role cycle counters of the weight-in-TMEM GEMM (needs a library
         built with -DREELS_TS_TRACE)
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, FFN, CONTEXT = 1536, 8960, 512
L2_BYTES = 126 * 2 ** 20
METRIC = "int8-W LoRA linear fwd+bwd tokens/s (TFLOP/s and % of roofline alongside)"


def l2_note(layers) -> str:
    """How the timed steps stand against the 126 MB L2: the bytes of
    activations, outputs and upstream gradients one step touches."""
    step = sum(2 * (2 * M * K + 2 * M * N) for (_, M, K, N) in layers)
    if step > 2 * L2_BYTES:
        return f"inputs larger than L2 ({step / 2 ** 30:.1f} GB of activations and gradients per step)"
    return (f"inputs fit in L2 ({step / 2 ** 20:.0f} MB of activations and gradients per step); "
            "steps run back to back without a flush (warm L2)")


def block_layers(tokens: int, context: int = CONTEXT, hidden: int = HIDDEN, ffn: int = FFN):
    """(name, M, K, N) of the ten linears of a DiT block (Wan 2.1 1.3B by
    default): self-attention q/k/v/o, cross-attention q/o over the tokens and
    k/v over the context, and the FFN pair."""
    L = []
    for n in ("self_q", "self_k", "self_v", "self_o", "cross_q"):
        L.append((n, tokens, hidden, hidden))
    L.append(("cross_k", context, hidden, hidden))
    L.append(("cross_v", context, hidden, hidden))
    L.append(("cross_o", tokens, hidden, hidden))
    L.append(("ffn_up", tokens, hidden, ffn))
    L.append(("ffn_down", tokens, ffn, hidden))
    return L


def workload(config: str):
    """The linears of one block (``layers``), repeated ``blocks`` times per
    step with distinct weights and adapters."""
    if config == "cfg1":
        return dict(name="wan21-1.3b-ffn-up", layers=[("ffn_up", 1280, 1536, 8960)], tokens=1280, rank=16,
                    alpha=16.0, context=None, blocks=1)
    if config == "ffn8k":
        # One FFN up-projection at 8192 tokens: operands larger than L2 but a
        # few hundred MB in total, the case the ncu captures use.
        return dict(name="wan21-1.3b-ffn-up-8k", layers=[("ffn_up", 8192, 1536, 8960)], tokens=8192, rank=32,
                    alpha=32.0, context=None, blocks=1)
    if config == "wan14b":
        # Wan 2.1 14B, one block of the 40-block stack per GPU (hidden 5120, FFN 13824)
        return dict(name="wan21-14b-block-linears", layers=block_layers(32760, 512, 5120, 13824), tokens=32760,
                    rank=32, alpha=32.0, context=512, blocks=1)
    if config == "wan14b-stack":
        # Wan 2.1 14B in full: the 40-block stack per GPU
        return dict(name="wan21-14b-40-blocks", layers=block_layers(32760, 512, 5120, 13824), tokens=32760,
                    rank=32, alpha=32.0, context=512, blocks=40)
    if config == "ltx":
        # LTX-2.3, per GPU: one block (hidden 4096, FFN 16384), 2 x 6144 tokens, context 2048
        return dict(name="ltx23-block-linears", layers=block_layers(12288, 2048, 4096, 16384), tokens=12288,
                    rank=64, alpha=64.0, context=2048, blocks=1)
    return dict(name="wan21-1.3b-block-linears", layers=block_layers(32760), tokens=32760, rank=32, alpha=32.0,
                context=CONTEXT, blocks=1)


def step_flops(layers, r):
    # 4*M*N*K (forward + dX) + 6*M*r*(K+N) (LoRA forward and backward).
    return float(sum(4.0 * M * N * K + 6.0 * M * r * (K + N) for (_, M, K, N) in layers))


def config_dict(wl, world):
    """The `config` of both arms' JSON lines (the reference arm times the
    same workload on the host)."""
    d = {"workload": wl["name"], "tokens_per_sample": wl["tokens"], "context_tokens": wl["context"],
         "linears": [list(l) for l in wl["layers"]], "rank": wl["rank"], "alpha": wl["alpha"],
         "weight_layout": "out-contiguous (reference)", "global_batch": world, "parallelism": f"dp{world}",
         "l2": l2_note(wl["layers"])}
    if wl["blocks"] > 1:
        d["blocks"] = wl["blocks"]
    return d


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}, "fallback"


def load_traffic_ratio():
    """DRAM traffic / algorithmic bytes of one q8 GEMM launch, from the
    committed ncu summary (a smaller case of the same kernel)."""
    p = os.path.join(ROOT, "profiles", "q8_gemm_traffic.txt")
    if not os.path.exists(p):
        return None, None
    vals = {}
    for line in open(p):
        if "=" in line and not line.startswith("#"):
            k, v = line.split("=", 1)
            vals[k.strip()] = v.strip()
    try:
        return float(vals["traffic_over_algorithmic"]), vals.get("workload")
    except (KeyError, ValueError):
        return None, None


def q8_algorithmic_bytes(layers, r):
    """Minimum DRAM bytes of the step's q8 GEMM launches (forward Y and dX per
    linear, bf16): activations in and out, int8 weight, scales, the rank-r
    operands of the LoRA blocks."""
    rp = ((r + 63) // 64) * 64
    total, n = 0.0, 0
    for (_, M, K, N) in layers:
        total += 2 * M * K + K * N + 4 * N + 2 * M * N + 2 * r * M + 2 * rp * N   # forward
        total += 2 * M * N + K * N + 4 * N + 2 * M * K + 2 * r * M + 2 * rp * K   # dX
        n += 2
    return total, n


def pick_peak(peaks, peak_kind, timed_s, clk):
    """The bf16 denominator that applies to the timed region: the burst figure
    for a region shorter than two seconds that ran at the maximum SM clock
    (the burst figure was measured that way), the sustained figure (seconds
    under the power cap) otherwise."""
    burst = float(peaks.get("bf16_tflops", 1590.0))
    sustained = float(peaks.get("bf16_tflops_sustained", burst))
    at_max = bool(clk) and clk.get("sm_mhz", 0) >= 0.95 * clk.get("sm_max_mhz", 1e9)
    if timed_s < 2.0 and at_max:
        return burst, f"bf16_tflops (burst) of {peak_kind}: timed region {timed_s:.2f} s at the maximum SM clock"
    why = f"{timed_s:.2f} s timed region" if timed_s >= 2.0 else "SM clock below maximum"
    return sustained, f"bf16_tflops_sustained of {peak_kind}: {why}"


# ---------------------------------------------------------------- clocks
def smi_device(local_index: int) -> str:
    """The nvidia-smi id of CUDA device ``local_index``: the matching entry of
    CUDA_VISIBLE_DEVICES (an index or a UUID) when it is set, else the index."""
    cvd = [e.strip() for e in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if e.strip()]
    return cvd[local_index] if local_index < len(cvd) else str(local_index)


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons every INTERVAL_MS.
    Each sample carries nvidia-smi's own timestamp, so only the samples taken
    between :meth:`begin` and :meth:`end` (the timed region) are summarised,
    whatever the pipe's buffering; with none inside, the one nearest the
    region's middle is used and ``window`` says so."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    INTERVAL_MS = 100

    def __init__(self, gpu_index: int, command: str = "nvidia-smi"):
        self.proc = None
        self.gpu = smi_device(gpu_index)
        self.command = command
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                [self.command, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.INTERVAL_MS), "-i", self.gpu],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        # let the sampler come up before the timed region starts
        time.sleep(2 * self.INTERVAL_MS / 1e3)

    def begin(self):
        self.t0 = datetime.datetime.now()

    def end(self):
        self.t1 = datetime.datetime.now()

    @staticmethod
    def _stamp(text: str):
        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.datetime.strptime(text, fmt)
            except ValueError:
                pass
        return None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(2 * self.INTERVAL_MS / 1e3)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        return self.summarise(out)

    def summarise(self, out: str):
        rows = []
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                sm, mx = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            reasons = {nm for nm, v in zip(self.REASONS, parts[6:10]) if v.lower() in ("active", "yes", "1")}
            rows.append((self._stamp(parts[0]), sm, mx, reasons))
        if not rows:
            return None
        window = "timed region"
        if self.t0 is not None and self.t1 is not None and all(r[0] is not None for r in rows):
            inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
            if not inside:
                mid = self.t0 + (self.t1 - self.t0) / 2
                inside = [min(rows, key=lambda r: abs((r[0] - mid).total_seconds()))]
                window = "nearest sample to the timed region"
            rows = inside
        else:
            window = "whole sampler run (timestamps unavailable)"
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": max(r[2] for r in rows),
                "samples": len(rows), "window": window,
                "reasons": sorted(set().union(*(r[3] for r in rows)))}


# ----------------------------------------------------------- CPU baseline
def _blas_threads():
    try:
        from threadpoolctl import threadpool_info
        return max([i.get("num_threads", 1) for i in threadpool_info() if i.get("internal_api") == "openblas"]
                   or [1])
    except Exception:
        return os.cpu_count() or 1


class CpuStep:
    """The reference's CPU code path (numpy + OpenBLAS fp32, oracle/numpy_port.py)
    on a bounded sample of one block: the linears over the sample's tokens run
    at two sample sizes (``small`` and ``large`` tokens), the context linears
    at their own full length.  Per call the reference materialises the
    dequantised weight (a cost that does not grow with the tokens) and runs
    sgemms whose cost grows linearly with them, so the time of the full
    workload is the affine extrapolation of the two samples to ``tokens``,
    plus the context linears once; ``blocks`` repeats that."""

    def __init__(self, wl, small=256, large=512, seed=0):
        import oracle
        self.tokens, self.blocks = wl["tokens"], wl["blocks"]
        self.small, self.large = min(small, self.tokens), min(large, self.tokens)
        r, self.alpha = wl["rank"], wl["alpha"]
        g = np.random.default_rng(seed)
        self.tok, self.ctx = [], []
        for (_, M, K, N) in wl["layers"]:
            m = M if M != self.tokens else self.large
            W = (0.02 * g.standard_normal((K, N), dtype=np.float32))
            q, s = oracle.quantize(W, 0)
            item = (g.standard_normal((m, K), dtype=np.float32), g.standard_normal((m, N), dtype=np.float32), q, s,
                    (g.standard_normal((K, r), dtype=np.float32) / np.sqrt(K)).astype(np.float32),
                    (0.01 * g.standard_normal((r, N), dtype=np.float32)).astype(np.float32))
            (self.tok if M == self.tokens else self.ctx).append(item)
        self.threads = _blas_threads()

    def _run(self, group, m=None):
        from oracle import numpy_port
        t0 = time.perf_counter()
        for (X, dY, q, s, A, B) in group:
            if m is not None:
                X, dY = X[:m], dY[:m]
            numpy_port.lora_step(X, dY, q, s, 0, A, B, self.alpha)
        return time.perf_counter() - t0

    def sample(self):
        """One sample: (estimated seconds of the full workload, measured seconds)."""
        t_small = self._run(self.tok, self.small)
        t_large = self._run(self.tok, self.large)
        t_ctx = self._run(self.ctx) if self.ctx else 0.0
        if self.large > self.small:
            per_tok = max(t_large - t_small, 0.0) / (self.large - self.small)
            t_tok = t_large + per_tok * (self.tokens - self.large)
        else:
            t_tok = t_large
        return self.blocks * (t_tok + t_ctx), t_small + t_large + t_ctx

    def describe(self, n, spent):
        ctx = f" and the context linears at {self.ctx[0][0].shape[0]} tokens" if self.ctx else ""
        return (f"numpy+OpenBLAS fp32 (oracle/numpy_port.py, the op order of lora.jl:56-118): the token linears at "
                f"{self.small} and {self.large} tokens{ctx}, {n} samples in {spent:.1f} s; per-call dequantisation "
                f"plus sgemm time extrapolated affinely to {self.tokens} tokens" +
                (f", times {self.blocks} blocks" if self.blocks > 1 else ""))


def cpu_baseline(wl, seconds):
    cs = CpuStep(wl)
    cs.sample()  # warm-up
    ests, spent, t0 = [], 0.0, time.perf_counter()
    while True:
        est, took = cs.sample()
        ests.append(est)
        spent += took
        if time.perf_counter() - t0 >= seconds:
            break
    est = statistics.median(ests)
    return {"value": wl["tokens"] / est, "unit": "tokens/s", "cores": cs.threads, "kind": "port",
            "sample": cs.describe(len(ests), spent)}


# ------------------------------------------------------ small-token record
def small_m_cases(L, nat, torch, dev, tokens=(128, 512), ranks=(8,), reps=20, N=13824, K=5120, dtype="f16",
                  loss_scale=1024.0, dropout=0.0):
    """fwd+bwd of one linear at small token counts through the C ABI (by default
    the Wan 2.1 14B FFN up-projection: W 13824x5120 int8 per row, fp16, static loss scale
    1024 on dY removed through grad_scale), CUDA-event timed on the launching
    stream after warm-up.  Algorithmic FLOPs: 4*M*N*K (Y and dX) + the six
    rank-r products 2*M*r*(3K + 3N).  Algorithmic bytes: forward x, W (int8 +
    scales), y; backward dy, W, x (for dA), dx; plus the rank-r tensors."""
    from reels_b200 import quantize_frozen_matrix
    peaks, kind = load_peaks()
    hbm, tf_peak = float(peaks["hbm_gbs"]), float(peaks["bf16_tflops"])
    tdt, dt = (torch.float16, nat.F16) if dtype == "f16" else (torch.bfloat16, nat.BF16)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    w = torch.empty((K, N), device=dev).normal_(0.0, 0.02, generator=g).t()  # (out, in), column-major
    qm = quantize_frozen_matrix(w)
    del w
    q, s = qm.values, qm.scales
    st = torch.cuda.current_stream(dev).cuda_stream
    out = []
    for r in ranks:
        alpha = float(r)
        A = (torch.randn((K, r), device=dev, generator=g) / K ** 0.5).to(tdt)
        B = (0.01 * torch.randn((r, N), device=dev, generator=g)).to(tdt)
        for M in tokens:
            x = torch.randn((M, K), device=dev, generator=g).to(tdt)
            dy = (torch.randn((M, N), device=dev, generator=g) * loss_scale).to(tdt)
            y = torch.empty((M, N), device=dev, dtype=tdt)
            dx = torch.empty((M, K), device=dev, dtype=tdt)
            saved = torch.empty((max(L.reels_q8lora_saved_bytes(M, r, dt), 16),), dtype=torch.uint8, device=dev)
            grad = torch.zeros((r * (K + N),), dtype=torch.float32, device=dev)
            flag = nat.PASS_DROPOUT if dropout > 0 else 0
            wsn = max(L.reels_q8lora_workspace_bytes(M, K, N, r, dt, p | flag) for p in (0, 1))
            ws = torch.empty((max(wsn, 256),), dtype=torch.uint8, device=dev)

            def fwd(stream=st):
                if dropout > 0:
                    nat.check("forward", L.reels_q8lora_forward_dropout(
                        x.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(), None, M, K, N, r,
                        alpha, dt, dropout, 1, 0, y.data_ptr(), saved.data_ptr(), ws.data_ptr(), wsn, stream))
                    return
                nat.check("forward", L.reels_q8lora_forward(
                    x.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(), None, M, K, N, r, alpha,
                    dt, y.data_ptr(), saved.data_ptr(), ws.data_ptr(), wsn, stream))

            def bwd(stream=st):
                if dropout > 0:
                    nat.check("backward", L.reels_q8lora_backward_dropout(
                        x.data_ptr(), dy.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(),
                        saved.data_ptr(), M, K, N, r, alpha, 1.0 / loss_scale, dt, dropout, 1, 0, dx.data_ptr(),
                        grad.data_ptr(), grad.data_ptr() + 4 * K * r, 0, ws.data_ptr(), wsn, stream))
                    return
                nat.check("backward", L.reels_q8lora_backward(
                    x.data_ptr(), dy.data_ptr(), q.data_ptr(), s.data_ptr(), 0, A.data_ptr(), B.data_ptr(),
                    saved.data_ptr(), M, K, N, r, alpha, 1.0 / loss_scale, dt, dx.data_ptr(), grad.data_ptr(),
                    grad.data_ptr() + 4 * K * r, 0, ws.data_ptr(), wsn, stream))

            res = {}
            for name, fn in (("fwd", fwd), ("bwd", bwd)):
                for _ in range(3):
                    fn()
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    fn()
                e1.record()
                torch.cuda.synchronize(dev)
                res[name] = e0.elapsed_time(e1) / reps * 1e3
            # The same fwd+bwd captured once in a CUDA graph and replayed: the
            # device time without the host's per-call launch overhead.
            us_graph = None
            try:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    gs = torch.cuda.current_stream(dev).cuda_stream
                    fwd(gs)
                    bwd(gs)
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    graph.replay()
                e1.record()
                torch.cuda.synchronize(dev)
                us_graph = e0.elapsed_time(e1) / reps * 1e3
                del graph
            except Exception as exc:  # reported, not hidden: the eager figures stand
                us_graph = f"graph capture failed: {exc}"
            nat.check("device status", L.reels_lowvram_check_device_status(st))
            us = res["fwd"] + res["bwd"]
            e = 2  # bytes per activation element
            flops = 4.0 * M * N * K + 2.0 * M * r * (3.0 * K + 3.0 * N)
            wbytes = N * K + 4 * N
            rank_bytes = e * r * (K + N) * 2 + e * r * M * 2 + 4 * r * (K + N)
            byts = (e * M * K + wbytes + e * M * N) + (e * M * N + wbytes + e * M * K + e * M * K) + rank_bytes
            gbs = byts / (us * 1e-6) / 1e9
            tfl = flops / (us * 1e-6) / 1e12
            out.append({"shape": f"W {N}x{K}", "tokens": M, "rank": r, "dtype": dtype, "loss_scale": loss_scale,
                        "dropout": dropout, "us_fwd": round(res["fwd"], 1), "us_bwd": round(res["bwd"], 1),
                        "us": round(us, 1),
                        "us_graph": round(us_graph, 1) if isinstance(us_graph, float) else us_graph,
                        "hbm_frac_graph": (round(byts / (us_graph * 1e-6) / 1e9 / hbm, 3)
                                           if isinstance(us_graph, float) else None),
                        "tflops": round(tfl, 1), "tensor_frac": round(tfl / tf_peak, 3),
                        "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 3), "algorithmic_bytes": int(byts),
                        "algorithmic_flops": flops, "peaks": f"hbm_gbs {hbm:.0f}, bf16_tflops {tf_peak:.0f} "
                                                             f"({kind})"})
            del x, dy, y, dx, saved, grad, ws
    return out


# ------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist
    from reels_b200 import build as native_build
    from reels_b200 import _native as nat
    from reels_b200 import distributed as rd
    from reels_b200 import quantize_frozen_matrix

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        rt = rd.init_distributed(backend="nccl", timeout_seconds=120)
    else:
        rt = rd.SingleProcessRuntime()
        torch.cuda.set_device(0)
    dev = torch.device("cuda", local if world > 1 else 0)
    native_build.build()
    L = nat.lib()
    wl = workload(args.config)
    layers, r, alpha, blocks = wl["layers"], wl["rank"], wl["alpha"], wl["blocks"]
    bf = torch.bfloat16
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    class Act:
        """The activations of one linear position of the block, shared by the
        blocks of a stack (synthetic inputs: every block reads the same)."""

    class Lin:
        pass

    acts = []
    for (name, M, K, N) in layers:
        a = Act()
        a.M, a.K, a.N = M, K, N
        a.x = torch.randn((M, K), device=dev, generator=gen).to(bf)
        a.dy = torch.randn((M, N), device=dev, generator=gen).to(bf)
        a.y = torch.empty((M, N), device=dev, dtype=bf)
        a.dx = torch.empty((M, K), device=dev, dtype=bf)
        acts.append(a)
    # fp32 gradients [dA (K*r) | dB (r*N)] of every linear in one buffer, laid
    # out in the order the backward produces them, so that consecutive
    # linears' gradients form contiguous all-reduce buckets
    order = [(b, i) for b in range(blocks) for i in range(len(layers))]
    sizes = {(b, i): r * (layers[i][2] + layers[i][3]) for (b, i) in order}
    total = sum(sizes.values())
    grads = torch.zeros((total,), dtype=torch.float32, device=dev)
    lins, off = {}, 0
    for (b, i) in reversed(order):
        o = Lin()
        name, M, K, N = layers[i]
        o.name, o.M, o.K, o.N, o.act = name, M, K, N, acts[i]
        w = torch.empty((K, N), device=dev).normal_(0.0, 0.02, generator=gen).t()   # (out, in) column-major
        qm = quantize_frozen_matrix(w)
        del w
        o.q, o.s = qm.values, qm.scales
        o.A = (torch.randn((K, r), device=dev, generator=gen) / K ** 0.5).to(bf)     # [K][r] memory
        o.B = (0.01 * torch.randn((r, N), device=dev, generator=gen)).to(bf)         # [r][N] memory
        o.saved = torch.empty((max(L.reels_q8lora_saved_bytes(M, r, nat.BF16), 16),), dtype=torch.uint8,
                              device=dev)
        o.grad = grads[off:off + sizes[(b, i)]]
        off += sizes[(b, i)]
        lins[(b, i)] = o
    lins = [lins[k] for k in order]        # forward order
    wsn = max(max(L.reels_q8lora_workspace_bytes(o.M, o.K, o.N, r, nat.BF16, p) for p in (0, 1)) for o in lins)
    ws = torch.empty((wsn,), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    bucket = int(args.bucket_mb * 2 ** 20) if args.bucket_mb is not None else (64 << 20 if blocks > 1 else 0)
    reducer = rd.OverlappedGradReducer(rt, dev, bucket_bytes=bucket)

    def fwd(o):
        a = o.act
        nat.check("forward", L.reels_q8lora_forward(
            a.x.data_ptr(), o.q.data_ptr(), o.s.data_ptr(), 0, o.A.data_ptr(), o.B.data_ptr(), None, o.M, o.K,
            o.N, r, alpha, nat.BF16, a.y.data_ptr(), o.saved.data_ptr(), ws.data_ptr(), wsn, sp))

    def bwd(o):
        a = o.act
        nat.check("backward", L.reels_q8lora_backward(
            a.x.data_ptr(), a.dy.data_ptr(), o.q.data_ptr(), o.s.data_ptr(), 0, o.A.data_ptr(), o.B.data_ptr(),
            o.saved.data_ptr(), o.M, o.K, o.N, r, alpha, 1.0, nat.BF16, a.dx.data_ptr(), o.grad.data_ptr(),
            o.grad.data_ptr() + 4 * o.K * r, 0, ws.data_ptr(), wsn, sp))

    def step():
        for o in lins:
            fwd(o)
        for o in reversed(lins):
            bwd(o)
            reducer.layer_done(o.grad)
        reducer.finish()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    nat.check("device status", L.reels_lowvram_check_device_status(sp))

    # ---------------- device-timed region ----------------
    clocks = ClockSampler(torch.cuda.current_device() if world == 1 else local)
    clocks.start()
    nat.profile_enable(True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.begin()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks.end()
    clk = clocks.stop()
    q8_ms, q8_n, q8_flops, launches = nat.profile_read()
    nat.profile_enable(False)
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    nat.check("device status", L.reels_lowvram_check_device_status(sp))
    ms_per_step = ms / args.steps
    tokens = wl["tokens"]
    value = world * tokens * args.steps / (ms / 1e3)
    flops = blocks * step_flops(layers, r)

    # ---------------- end to end through the C ABI with host buffers ----------------
    # Every step copies its inputs (each position's activations and upstream
    # gradients, which the blocks of a stack share) from pinned host memory
    # and reads every LoRA gradient back.
    e2e_steps = max(1, min(args.steps, 10 if blocks == 1 else 2))
    hx = [a.x.cpu().pin_memory() for a in acts]
    hdy = [a.dy.cpu().pin_memory() for a in acts]
    hgrad = torch.empty(grads.shape, dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in hx + hdy)
    d2h = hgrad.numel() * hgrad.element_size()

    # The step's inputs cross PCIe on a copy stream in the order the step
    # consumes them (x forward, dy backward), each linear waiting only for its
    # own: the copies overlap the compute.  A step's copies start once the
    # previous step has finished reading the buffers.
    copy_stream = torch.cuda.Stream(dev)
    npos = len(layers)

    def e2e_step():
        ev_x, ev_dy = [], {}
        copy_stream.wait_stream(stream)
        with torch.cuda.stream(copy_stream):
            for a, h in zip(acts, hx):
                a.x.copy_(h, non_blocking=True)
                e = torch.cuda.Event()
                e.record(copy_stream)
                ev_x.append(e)
            for i in reversed(range(npos)):
                acts[i].dy.copy_(hdy[i], non_blocking=True)
                e = torch.cuda.Event()
                e.record(copy_stream)
                ev_dy[i] = e
        for j, o in enumerate(lins):
            if j < npos:
                stream.wait_event(ev_x[j])
            fwd(o)
        for j in reversed(range(len(lins))):
            if j >= len(lins) - npos:
                stream.wait_event(ev_dy[j % npos])
            bwd(lins[j])
            reducer.layer_done(lins[j].grad)
        reducer.finish()
        hgrad.copy_(grads, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(stream)
    torch.cuda.synchronize(dev)
    ems = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([ems], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e_value = world * tokens * e2e_steps / (ems / 1e3)

    peaks, peak_kind = load_peaks()
    q8_tflops = (q8_flops / (q8_ms / 1e3) / 1e12) if q8_ms > 0 else None
    peak, peak_src = pick_peak(peaks, peak_kind, ms / 1e3, clk)
    burst = float(peaks.get("bf16_tflops", peak))
    sustained = float(peaks.get("bf16_tflops_sustained", burst))
    ratio, ratio_src = load_traffic_ratio()
    alg_bytes, alg_n = q8_algorithmic_bytes(layers, r)
    alg_per_launch = alg_bytes / alg_n
    traffic = ratio * alg_per_launch if ratio is not None else None
    step_tflops = flops * world * args.steps / (ms / 1e3) / 1e12

    small = None
    if world == 1 and not args.no_small_m and blocks == 1:
        del ws
        torch.cuda.empty_cache()
        small = small_m_cases(L, nat, torch, dev)

    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(wl, args.cpu_seconds)
        result = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded normal activations, N(0,0.02) weights int8 per row)",
            "config": config_dict(wl, world),
            "tflops": step_tflops,
            "step_frac": {"burst": step_tflops / world / burst, "sustained": step_tflops / world / sustained},
            "roofline": {"bound": "tensor", "kernel": "q8ts_gemm_kernel (forward Y and dX)",
                         "achieved": q8_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": (q8_tflops / peak) if q8_tflops else None,
                         "frac_burst": (q8_tflops / burst) if q8_tflops else None,
                         "frac_sustained": (q8_tflops / sustained) if q8_tflops else None,
                         "peak_source": peak_src,
                         "launches": q8_n, "algorithmic_flops_per_launch": (q8_flops / q8_n) if q8_n else None,
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": alg_per_launch,
                         "traffic_source": (f"ncu DRAM read+write of the same kernel's launches on a smaller case "
                                            f"({ratio_src}) as a fraction of their algorithmic bytes ({ratio:.3f}), "
                                            f"times this workload's algorithmic bytes per launch"
                                            if ratio is not None else None)},
            "small_m": small,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if world > 1:
            result["allreduce"] = {"bytes_per_step": grads.numel() * 4, "bucket_bytes": bucket or "per linear",
                                   "collective": "ncclAllReduce (sum, fp32) on a side stream, then 1/world"}
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        rd.close_distributed(rt)
    return result


# ------------------------------------------------------- reference arm
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    wl = workload(args.config)
    cs = CpuStep(wl)
    for _ in range(args.warmup):
        cs.sample()
    ests, spent = [], 0.0
    for _ in range(args.steps):
        est, took = cs.sample()
        ests.append(est)
        spent += took
    secs = sum(ests)
    value = wl["tokens"] * args.steps / secs
    res = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": secs / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": config_dict(wl, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cs.threads, "kind": "port",
                         "sample": "each step one sample: " + cs.describe(args.steps, spent) +
                                   " (Julia is not installed, so the reference's CPU path runs as its "
                                   "numpy+OpenBLAS restatement)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)
    return res


# ------------------------------------------------------- measurement modes
def _best_of_rounds(torch, dev, passes, reps):
    """Round-robin over the passes, best of three rounds each: a pass timed
    late in a long run would otherwise see lower clocks under the power cap."""
    for _, fn in passes:
        for _ in range(3):
            fn()
    torch.cuda.synchronize(dev)
    best = {}
    for _ in range(3):
        for name, fn in passes:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) / reps * 1e3
            best[name] = min(best.get(name, us), us)
    return best


def mode_sweep(args):
    import torch
    from reels_b200 import _native as nat
    from reels_b200 import build as native_build
    native_build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for rec in small_m_cases(nat.lib(), nat, torch, dev, tokens=[int(v) for v in args.tokens.split(",")],
                             ranks=[int(v) for v in args.ranks.split(",")], reps=args.reps, N=args.N, K=args.K,
                             dtype=args.dtype, loss_scale=args.loss_scale, dropout=args.dropout):
        print(json.dumps(rec), flush=True)


def mode_gemm(args):
    """The q8 GEMMs of the forward (_weight_mul) and of dX
    (_weight_transpose_mul) for one shape, through the C ABI: microseconds and
    TFLOP/s (2*M*N*K / time) per pass.  The planner picks the kernel and tile;
    REELS_Q8_TS (256, 192, 128, or 0 for the SMEM x SMEM kernel) and
    REELS_Q8_TILE force one.  --gelu adds the fused gelu_tanh epilogues beside
    the GEMM followed by PyTorch's own tanh-GELU kernels; --once launches each
    GEMM once without timing (for a profiler capture)."""
    import torch
    from reels_b200 import _native as nat
    from reels_b200 import build as native_build
    native_build.build()
    L = nat.lib()
    M, K, N = (int(v) for v in args.shape.split(","))
    layout = args.layout
    tdt, dt = (torch.bfloat16, nat.BF16) if args.dtype == "bf16" else (torch.float16, nat.F16)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
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
        fwd_into = L.reels_q8_weight_mul(x.data_ptr(), q.data_ptr(), s.data_ptr(), layout, None, M, K, N, dt,
                                         pre.data_ptr(), ws.data_ptr(), wsn, st)
        nat.check("weight_mul", fwd_into)
        torch.nn.functional.gelu(pre, approximate="tanh", out=y)

    def dx_then_gelu_grad():
        bwd()
        torch.ops.aten.gelu_backward(dx, pre_x, approximate="tanh")

    out = {"M": M, "K": K, "N": N, "layout": layout, "dtype": args.dtype}
    if args.once:
        fwd()
        bwd()
        torch.cuda.synchronize(dev)
        nat.check("device status", L.reels_lowvram_check_device_status(st))
        print(json.dumps(out), flush=True)
        return
    passes = [("fwd", fwd), ("dx", bwd)]
    if args.gelu:
        passes += [("fwd_gelu_fused", fwd_gelu), ("fwd_then_torch_gelu", fwd_then_gelu),
                   ("dx_gelu_fused", bwd_gelu), ("dx_then_torch_gelu_grad", dx_then_gelu_grad)]
    best = _best_of_rounds(torch, dev, passes, args.reps)
    for name, _ in passes:
        us = best[name]
        out[name] = {"us": round(us, 1), "tflops": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 1)}
    nat.check("device status", L.reels_lowvram_check_device_status(st))
    print(json.dumps(out), flush=True)


def mode_norm(args):
    """The fused LayerNorm + modulation (forward, and the pullback with the
    modulation's parameter gradients) against PyTorch evaluating the same
    expression as separate kernels, the way the reference's broadcasts do;
    and the gated residual with its pullback.  Bandwidth counts the arrays
    each pass moves (see below)."""
    import torch
    from reels_b200 import build as native_build
    native_build.build()
    from reels_b200.lowvram import layernorm_modulate, layernorm_modulate_backward
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    M, K = args.M, args.K
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

    # the gated residual round(x + round(y * gate)) (transformer.jl:272,293)
    # and its pullback (dy = round(dout * gate), dgate = sum dout * y)
    from reels_b200.lowvram import gated_residual, gated_residual_backward
    yres = torch.randn(M, K, device=dev).to(dt)
    gate = (0.1 * torch.randn(1, K, device=dev)).to(dt)
    res_out = torch.empty_like(x)

    def residual():
        gated_residual(x, yres, gate, out=res_out)

    def residual_bwd():
        gated_residual_backward(dout, yres, gate)

    best = _best_of_rounds(torch, dev, [("fused_fwd", fused), ("torch_fwd", torch_fwd),
                                        ("fused_bwd_with_param_grads", fused_bwd),
                                        ("gated_residual_fwd", residual),
                                        ("gated_residual_bwd_with_gate_grad", residual_bwd)], args.reps)
    hbm = float(load_peaks()[0]["hbm_gbs"])
    e = 2
    out = {"M": M, "K": K, "dtype": args.dtype}
    for name, us in best.items():
        out[name] = {"us": round(us, 1)}
    # bytes moved per pass, in units of M*K elements: LayerNorm forward reads
    # x and writes out (2); its backward reads x and dout, writes dx, and reads
    # x and dout again for the parameter sums (5); the gated residual reads x
    # and y and writes out (3); its pullback reads dout, writes dy, and reads
    # dout and y again for dgate (4)
    for name, arrays in (("fused_fwd", 2), ("fused_bwd_with_param_grads", 5), ("gated_residual_fwd", 3),
                         ("gated_residual_bwd_with_gate_grad", 4)):
        gb = arrays * M * K * e / (best[name] * 1e-6) / 1e9
        out[name].update(gbs=round(gb, 1), hbm_frac=round(gb / hbm, 3))
    print(json.dumps(out), flush=True)


def mode_adamw(args):
    """The optimizer step over the adapter tensors of Wan 2.1 14B at rank 32
    (40 blocks; per block 8 square 5120 linears and the 13824-wide FFN pair,
    each an A and a B tensor; 153.4 M parameters in 800 tensors), bf16
    parameters, fp32 gradients: the norm launch and the clipped AdamW launch.
    Bandwidth counts 4 bytes per element for the norm and 30 for the update
    (g, m, v, master read; m, v, master written; the 2-byte parameter
    written)."""
    import torch
    from reels_b200 import _native as nat
    from reels_b200 import build as native_build
    from reels_b200.optim import AdamWState
    native_build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r, d, f = 32, 5120, 13824
    shapes = []
    for _ in range(40):
        shapes += [(r * d, r * d)] * 8 + [(r * d, r * f), (r * f, r * d)]
    sizes = [n for pair in shapes for n in pair]
    params = [torch.zeros(n, dtype=torch.bfloat16, device=dev) for n in sizes]
    grads = [torch.randn(n, device=dev) * 1e-3 for n in sizes]
    total = sum(sizes)
    state = AdamWState(params)
    sumsq = torch.empty((), dtype=torch.float32, device=dev)
    ws = state._prepare(params, grads, None)
    L = nat.lib()
    st = torch.cuda.current_stream(dev).cuda_stream

    def norm():
        nat.check("norm", L.reels_grad_norm_sq(ws.data_ptr(), 1.0, sumsq.data_ptr(), st))

    def upd():
        nat.check("adamw", L.reels_adamw_update(ws.data_ptr(), 1e-4, 0.9, 0.999, 1e-8, 0.01, 0.1, 0.001, 1.0,
                                                sumsq.data_ptr(), 1.0, st))

    best = _best_of_rounds(torch, dev, [("norm", norm), ("adamw", upd)], args.reps)
    hbm = float(load_peaks()[0]["hbm_gbs"])
    out = {"params": total, "tensors": len(sizes)}
    for name, bpe in (("norm", 4), ("adamw", 30)):
        us = best[name]
        gbs = bpe * total / (us * 1e-6) / 1e9
        out[name] = {"us": round(us, 1), "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 3)}
    nat.check("device status", L.reels_lowvram_check_device_status(st))
    print(json.dumps(out), flush=True)


def mode_trace(args):
    """Per-role cycle counters of the weight-in-TMEM GEMM, from a debug build
    of the library (nvcc ... -DREELS_TS_TRACE, loaded through
    REELS_LOWVRAM_LIBRARY; the shipped library has no counters).  For each
    case, one launch of _weight_mul (fwd) or _weight_transpose_mul (dx) after
    three warm-up launches; per role (X producer, MMA, W producer, dequant,
    epilogue) the average cycles per CTA in [wait 0, wait 1, work, total]."""
    import ctypes
    import torch
    from reels_b200 import _native as nat
    L = nat.lib()
    if not hasattr(L, "reels_ts_trace_read"):
        raise SystemExit("the loaded library has no counters: build it with -DREELS_TS_TRACE and point "
                         "REELS_LOWVRAM_LIBRARY at it")
    L.reels_ts_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    nw = 19
    buf = (ctypes.c_ulonglong * (256 * nw * 4))()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    roles = {0: "xprod", 1: "mma", 2: "wprod"}
    roles.update({w: "deq" for w in range(3, 11)})
    roles.update({w: "epi" for w in range(11, 19)})
    cases = [(128, 5120, 13824, "f16", True), (128, 5120, 13824, "f16", False), (512, 5120, 13824, "f16", True),
             (32760, 1536, 1536, "bf16", True), (32760, 1536, 1536, "bf16", False), (8192, 1536, 8960, "bf16", True)]
    for (M, K, N, dtn, fwd) in cases:
        tdt, dt = (torch.float16, nat.F16) if dtn == "f16" else (torch.bfloat16, nat.BF16)
        x = torch.randn(M, K, device=dev).to(tdt)
        dy = torch.randn(M, N, device=dev).to(tdt)
        q = torch.randint(-127, 128, (K, N), device=dev, dtype=torch.int8)
        s = torch.rand(N, device=dev) * 1e-3 + 1e-4
        y = torch.empty(M, N, device=dev, dtype=tdt)
        dx = torch.empty(M, K, device=dev, dtype=tdt)
        wsn = max(L.reels_q8lora_workspace_bytes(M, K, N, 0, dt, p) for p in (0, 1))
        ws = torch.empty(max(wsn, 256), dtype=torch.uint8, device=dev)
        st = torch.cuda.current_stream(dev).cuda_stream

        def run():
            if fwd:
                nat.check("fwd", L.reels_q8_weight_mul(x.data_ptr(), q.data_ptr(), s.data_ptr(), 0, None, M, K, N,
                                                       dt, y.data_ptr(), ws.data_ptr(), wsn, st))
            else:
                nat.check("dx", L.reels_q8_weight_transpose_mul(dy.data_ptr(), q.data_ptr(), s.data_ptr(), 0, M, K,
                                                                N, dt, dx.data_ptr(), ws.data_ptr(), wsn, st))
        for _ in range(3):
            run()
        L.reels_ts_trace_read(None, 0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3
        L.reels_ts_trace_read(buf, len(buf))
        info = (ctypes.c_int64 * 7)()
        L.reels_q8_plan(M, N if fwd else K, K if fwd else N, 0, 0, info)
        ctas = [c for c in range(256) if buf[(c * nw + 1) * 4 + 3] > 0]
        agg = {}
        for c in ctas:
            for w in range(nw):
                a = agg.setdefault(roles[w], [0, 0, 0, 0, 0])
                for k in range(4):
                    a[k] += buf[(c * nw + w) * 4 + k]
                a[4] += 1
        out = {"shape": [M, K, N, dtn, "fwd" if fwd else "dx"], "us": round(us, 1), "plan": list(info),
               "ctas": len(ctas)}
        for role, a in agg.items():
            out[role] = [round(a[k] / a[4]) for k in range(4)]
        print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="block", choices=["block", "cfg1", "ffn8k", "wan14b", "wan14b-stack", "ltx"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-small-m", action="store_true", help="skip the small-token record of the default line")
    ap.add_argument("--bucket-mb", type=float, default=None,
                    help="all-reduce bucket size (default: per linear, 64 MB for the 40-block stack)")
    ap.add_argument("--mode", default="step", choices=["step", "sweep", "gemm", "norm", "adamw", "trace"])
    # measurement modes
    ap.add_argument("--N", type=int, default=13824)
    ap.add_argument("--K", type=int, default=5120)
    ap.add_argument("--M", type=int, default=32760)
    ap.add_argument("--tokens", default="128,512,2048,8192,32760")
    ap.add_argument("--ranks", default="8,64")
    ap.add_argument("--dtype", default=None, choices=["f16", "bf16"])
    ap.add_argument("--loss-scale", type=float, default=1024.0)
    ap.add_argument("--dropout", type=float, default=0.0)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--shape", default="8192,1536,8960", help="gemm mode: M,K,N")
    ap.add_argument("--layout", type=int, default=0)
    ap.add_argument("--gelu", action="store_true")
    ap.add_argument("--once", action="store_true")
    args = ap.parse_args()
    if args.dtype is None:
        args.dtype = "f16" if args.mode == "sweep" else "bf16"
    if args.warmup < 3:
        args.warmup = 3
    if args.mode != "step":
        {"sweep": mode_sweep, "gemm": mode_gemm, "norm": mode_norm, "adamw": mode_adamw,
         "trace": mode_trace}[args.mode](args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
