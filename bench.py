"""Benchmark: Int8-weight LoRA linear forward + backward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config block|cfg1]

Workload (the default "block"): every linear of one
Wan-2.1-1.3B DiT block at 32760 tokens per sample -- self-attention q/k/v/o
and cross-attention q/o (1536x1536 over 32760 tokens), cross-attention k/v
(1536x1536 over 512 context tokens), FFN up 1536->8960 and down 8960->1536 --
int8 per-row weights from N(0, 0.02), LoRA rank 32 / alpha 32 on every
linear, bf16 activations ~N(0,1).  One step = the forward of the ten linears,
then their backward in reverse order (dX, dA, dB), and at N > 1 the fp32
all-reduce of every LoRA gradient (per layer, overlapped with the backward).
Data-parallel weak scaling: each rank processes its own 32760-token sample.

Our arm prints one JSON line (rank 0).  ``--impl reference`` times the
reference's CPU code path (oracle/numpy_port.py: dequantise-materialise plus
OpenBLAS sgemm, the op order of src/layers/lora.jl:56-118) on the host cores
instead; the reference itself is Julia and cannot run in this image.
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
    if config == "cfg1":
        return dict(name="wan21-1.3b-ffn-up", layers=[("ffn_up", 1280, 1536, 8960)], tokens=1280, rank=16,
                    alpha=16.0)
    if config == "ffn8k":
        # One FFN up-projection at 8192 tokens: operands larger than L2 but a
        # few hundred MB in total, the case the ncu captures use.
        return dict(name="wan21-1.3b-ffn-up-8k", layers=[("ffn_up", 8192, 1536, 8960)], tokens=8192, rank=32,
                    alpha=32.0)
    if config == "wan14b":
        # BASELINE config 3, per GPU: one Wan 2.1 14B block (hidden 5120, FFN 13824)
        return dict(name="wan21-14b-block-linears", layers=block_layers(32760, 512, 5120, 13824), tokens=32760,
                    rank=32, alpha=32.0, context=512)
    if config == "ltx":
        # BASELINE config 4, per GPU: one LTX-2.3 block (hidden 4096, FFN 16384), 2 x 6144 tokens, context 2048
        return dict(name="ltx23-block-linears", layers=block_layers(12288, 2048, 4096, 16384), tokens=12288,
                    rank=64, alpha=64.0, context=2048)
    return dict(name="wan21-1.3b-block-linears", layers=block_layers(32760), tokens=32760, rank=32, alpha=32.0)


def step_flops(layers, r):
    # 4*M*N*K (forward + dX) + 6*M*r*(K+N) (LoRA forward and backward).
    return float(sum(4.0 * M * N * K + 6.0 * M * r * (K + N) for (_, M, K, N) in layers))


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
def cpu_sample(layers, r, alpha, tokens_sample, seconds, seed=0, context=CONTEXT):
    """Time the reference CPU path (numpy + OpenBLAS fp32) on the block with
    `tokens_sample` tokens per sample; returns (tokens/s, iters, threads)."""
    from oracle import numpy_port
    import oracle
    g = np.random.default_rng(seed)
    data = []
    for (_, M, K, N) in layers:
        m = M if M == context else min(M, tokens_sample)  # the context linears keep their length
        X = g.standard_normal((m, K), dtype=np.float32)
        dY = g.standard_normal((m, N), dtype=np.float32)
        W = (0.02 * g.standard_normal((K, N), dtype=np.float32))
        q, s = oracle.quantize(W, 0)
        A = (g.standard_normal((K, r), dtype=np.float32) / np.sqrt(K)).astype(np.float32)
        B = (0.01 * g.standard_normal((r, N), dtype=np.float32)).astype(np.float32)
        data.append((X, dY, q, s, A, B))
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info() if i.get("internal_api") == "openblas"]
                      or [1])
    except Exception:
        threads = os.cpu_count() or 1

    def one():
        for (X, dY, q, s, A, B) in data:
            numpy_port.lora_step(X, dY, q, s, 0, A, B, alpha)

    one()  # warm-up
    t0 = time.perf_counter()
    it = 0
    while True:
        one()
        it += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return tokens_sample * it / dt, it, threads, dt


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
    layers, r, alpha = wl["layers"], wl["rank"], wl["alpha"]
    bf = torch.bfloat16
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    class Lin:
        pass

    lins = []
    for i, (name, M, K, N) in enumerate(layers):
        o = Lin()
        o.name, o.M, o.K, o.N = name, M, K, N
        w = torch.empty((K, N), device=dev).normal_(0.0, 0.02, generator=gen).t()   # (out, in) column-major
        qm = quantize_frozen_matrix(w)
        del w
        o.q, o.s = qm.values, qm.scales
        o.A = (torch.randn((K, r), device=dev, generator=gen) / K ** 0.5).to(bf)     # [K][r] memory
        o.B = (0.01 * torch.randn((r, N), device=dev, generator=gen)).to(bf)         # [r][N] memory
        o.x = torch.randn((M, K), device=dev, generator=gen).to(bf)
        o.dy = torch.randn((M, N), device=dev, generator=gen).to(bf)
        o.y = torch.empty((M, N), device=dev, dtype=bf)
        o.dx = torch.empty((M, K), device=dev, dtype=bf)
        o.saved = torch.empty((max(L.reels_q8lora_saved_bytes(M, r, nat.BF16), 16),), dtype=torch.uint8,
                              device=dev)
        o.grad = torch.zeros((r * (K + N),), dtype=torch.float32, device=dev)     # [dA (K*r) | dB (r*N)]
        lins.append(o)
    wsn = max(max(L.reels_q8lora_workspace_bytes(o.M, o.K, o.N, r, nat.BF16, p) for p in (0, 1)) for o in lins)
    ws = torch.empty((wsn,), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    reducer = rd.OverlappedGradReducer(rt, dev)

    def fwd(o):
        nat.check("forward", L.reels_q8lora_forward(
            o.x.data_ptr(), o.q.data_ptr(), o.s.data_ptr(), 0, o.A.data_ptr(), o.B.data_ptr(), None, o.M, o.K,
            o.N, r, alpha, nat.BF16, o.y.data_ptr(), o.saved.data_ptr(), ws.data_ptr(), wsn, sp))

    def bwd(o):
        nat.check("backward", L.reels_q8lora_backward(
            o.x.data_ptr(), o.dy.data_ptr(), o.q.data_ptr(), o.s.data_ptr(), 0, o.A.data_ptr(), o.B.data_ptr(),
            o.saved.data_ptr(), o.M, o.K, o.N, r, alpha, 1.0, nat.BF16, o.dx.data_ptr(), o.grad.data_ptr(),
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
    flops = step_flops(layers, r)

    # ---------------- end to end through the C ABI with host buffers ----------------
    e2e_steps = max(1, min(args.steps, 10))
    hx = [o.x.cpu().pin_memory() for o in lins]
    hdy = [o.dy.cpu().pin_memory() for o in lins]
    hgrad = [torch.empty(o.grad.shape, dtype=torch.float32).pin_memory() for o in lins]
    h2d = sum(t.numel() * t.element_size() for t in hx + hdy)
    d2h = sum(t.numel() * t.element_size() for t in hgrad)

    # The step's inputs cross PCIe on a copy stream in the order the step
    # consumes them (x forward, dy backward), each layer waiting only for its
    # own: the copies overlap the compute, which alone is several times
    # shorter.  A step's copies start once the previous step has finished
    # reading the buffers.
    copy_stream = torch.cuda.Stream(dev)

    def e2e_step():
        ev_x, ev_dy = [], {}
        copy_stream.wait_stream(stream)
        with torch.cuda.stream(copy_stream):
            for o, a in zip(lins, hx):
                o.x.copy_(a, non_blocking=True)
                e = torch.cuda.Event()
                e.record(copy_stream)
                ev_x.append(e)
            for i in reversed(range(len(lins))):
                lins[i].dy.copy_(hdy[i], non_blocking=True)
                e = torch.cuda.Event()
                e.record(copy_stream)
                ev_dy[i] = e
        for o, e in zip(lins, ev_x):
            stream.wait_event(e)
            fwd(o)
        for i in reversed(range(len(lins))):
            stream.wait_event(ev_dy[i])
            bwd(lins[i])
            reducer.layer_done(lins[i].grad)
        reducer.finish()
        for o, h in zip(lins, hgrad):
            h.copy_(o.grad, non_blocking=True)

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
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    ratio, ratio_src = load_traffic_ratio()
    alg_bytes, alg_n = q8_algorithmic_bytes(layers, r)
    alg_per_launch = alg_bytes / alg_n
    traffic = ratio * alg_per_launch if ratio is not None else None

    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            sample = 512 if args.config == "block" else 256
            tps, it, threads, secs = cpu_sample(layers, r, alpha, sample, args.cpu_seconds,
                                                context=wl.get("context", CONTEXT))
            cpu = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{args.config} linears fwd+bwd at {sample} tokens/sample (context {wl.get('context', CONTEXT)}), "
                             f"numpy+OpenBLAS fp32, {it} iterations in {secs:.1f} s"}
        result = {
            "metric": "int8-W LoRA linear fwd+bwd tokens/s (TFLOP/s and % of roofline alongside)",
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
            "config": {"workload": wl["name"], "tokens_per_sample": tokens, "context_tokens": wl.get("context", CONTEXT),
                       "linears": [list(l) for l in layers], "rank": r, "alpha": alpha,
                       "weight_layout": "out-contiguous (reference)", "global_batch": world,
                       "parallelism": f"dp{world}",
                       "l2": l2_note(layers)},
            "tflops": flops * world * args.steps / (ms / 1e3) / 1e12,
            "roofline": {"bound": "tensor", "kernel": "q8ts_gemm_kernel (forward Y and dX)",
                         "achieved": q8_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": (q8_tflops / peak) if q8_tflops else None,
                         "peak_source": f"bf16_tflops_sustained of {peak_kind}",
                         "launches": q8_n, "algorithmic_flops_per_launch": (q8_flops / q8_n) if q8_n else None,
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": alg_per_launch,
                         "traffic_source": (f"ncu DRAM read+write of the same kernel's launches on a smaller case "
                                            f"({ratio_src}) as a fraction of their algorithmic bytes ({ratio:.3f}), "
                                            f"times this workload's algorithmic bytes per launch"
                                            if ratio is not None else None)},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps},
            "gpu_launches": launches,
            "clocks": clk,
        }
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
    layers, r, alpha = wl["layers"], wl["rank"], wl["alpha"]
    from oracle import numpy_port
    import oracle
    sample = 512 if args.config == "block" else 256
    g = np.random.default_rng(0)
    data = []
    ctx = wl.get("context", CONTEXT)
    for (_, M, K, N) in layers:
        m = M if M == ctx else min(M, sample)  # the context linears keep their length
        W = (0.02 * g.standard_normal((K, N), dtype=np.float32))
        q, s = oracle.quantize(W, 0)
        data.append((g.standard_normal((m, K), dtype=np.float32), g.standard_normal((m, N), dtype=np.float32), q,
                     s, (g.standard_normal((K, r), dtype=np.float32) / np.sqrt(K)).astype(np.float32),
                     (0.01 * g.standard_normal((r, N), dtype=np.float32)).astype(np.float32)))
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info() if i.get("internal_api") == "openblas"]
                      or [1])
    except Exception:
        threads = os.cpu_count() or 1

    def one():
        for (X, dY, q, s, A, B) in data:
            numpy_port.lora_step(X, dY, q, s, 0, A, B, alpha)

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    secs = time.perf_counter() - t0
    value = sample * args.steps / secs
    res = {
        "impl": "reference",
        "metric": "int8-W LoRA linear fwd+bwd tokens/s (TFLOP/s and % of roofline alongside)",
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
        "config": {"workload": wl["name"], "tokens_per_sample": wl["tokens"], "sample_tokens": sample,
                   "context_tokens": wl.get("context", CONTEXT), "rank": r, "alpha": alpha, "parallelism": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"each step: {wl['name']} fwd+bwd at {sample} tokens/sample through "
                                   "oracle/numpy_port.py (Julia is not installed, so the reference's CPU "
                                   "path is run as its numpy+OpenBLAS restatement)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="block", choices=["block", "cfg1", "ffn8k", "wan14b", "ltx"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
