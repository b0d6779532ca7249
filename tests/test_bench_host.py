"""CPU checks of bench.py's host logic: the clock sampler's timed-region
window (with a stand-in for nvidia-smi), the device-id mapping and the
algorithmic FLOP count the roofline divides."""
import datetime
import os
import stat
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _line(t, sm, reasons=("Not Active",) * 4):
    return ", ".join([t.strftime("%Y/%m/%d %H:%M:%S.%f")[:-3], "0", str(sm), "1965", "700.0", "0x0"] + list(reasons))


def test_summary_keeps_only_the_timed_region():
    s = bench.ClockSampler(0)
    base = datetime.datetime(2026, 1, 1, 12, 0, 0)
    s.t0, s.t1 = base + datetime.timedelta(seconds=1), base + datetime.timedelta(seconds=2)
    idle = [_line(base + datetime.timedelta(milliseconds=100 * i), 1965) for i in range(5)]
    load = [_line(base + datetime.timedelta(milliseconds=1000 + 100 * i), 1800 + i,
                  ("Not Active", "Not Active", "Not Active", "Active")) for i in range(1, 10)]
    after = [_line(base + datetime.timedelta(milliseconds=2500), 1965)]
    out = s.summarise("\n".join(idle + load + after))
    assert out["samples"] == 9 and out["sm_mhz"] == 1805 and out["window"] == "timed region"
    assert out["reasons"] == ["sw_power_cap"] and out["sm_max_mhz"] == 1965


def test_summary_falls_back_to_the_nearest_sample():
    s = bench.ClockSampler(0)
    base = datetime.datetime(2026, 1, 1, 12, 0, 0)
    s.t0, s.t1 = base + datetime.timedelta(milliseconds=130), base + datetime.timedelta(milliseconds=170)
    out = s.summarise("\n".join([_line(base, 1965), _line(base + datetime.timedelta(milliseconds=190), 1700),
                                 "garbage", ""]))
    assert out["samples"] == 1 and out["sm_mhz"] == 1700 and out["window"].startswith("nearest")
    assert s.summarise("") is None


def test_slowdown_reasons_are_reported():
    s = bench.ClockSampler(0)
    now = datetime.datetime(2026, 1, 1)
    s.t0, s.t1 = now, now + datetime.timedelta(seconds=1)
    out = s.summarise(_line(now + datetime.timedelta(milliseconds=500), 1200,
                            ("Active", "Not Active", "Active", "Not Active")))
    assert out["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]


def test_sampler_process_round_trip(tmp_path):
    """start/begin/end/stop against a stand-in that prints a timestamped
    sample every 20 ms until it is terminated."""
    fake = tmp_path / "fake-smi"
    fake.write_text(f"#!{sys.executable}\n"
                    "import datetime, sys, time\n"
                    "while True:\n"
                    "    t = datetime.datetime.now().strftime('%Y/%m/%d %H:%M:%S.%f')[:-3]\n"
                    "    print(t + ', 0, 1850, 1965, 800.0, 0x4, Not Active, Not Active, Not Active, Active', flush=True)\n"
                    "    time.sleep(0.02)\n")
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    s = bench.ClockSampler(0, command=str(fake))
    s.start()
    time.sleep(1.0)  # the stand-in is an interpreter: let it come up even on a loaded host
    s.begin()
    time.sleep(0.5)
    s.end()
    out = s.stop()
    assert out is not None and out["window"] == "timed region" and out["samples"] >= 3
    assert out["sm_mhz"] == 1850 and out["reasons"] == ["sw_power_cap"]


def test_missing_sampler_gives_no_clock_record():
    s = bench.ClockSampler(0, command="/nonexistent/nvidia-smi")
    s.start()
    s.begin()
    s.end()
    assert s.stop() is None


def test_smi_device_follows_visible_devices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "5,GPU-1234")
    assert bench.smi_device(0) == "5" and bench.smi_device(1) == "GPU-1234" and bench.smi_device(2) == "2"
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.smi_device(3) == "3"


def test_step_flops_match_the_algorithmic_count():
    # config 1: 4*M*N*K + 6*M*r*(K+N) = 70.5 G + 1.29 G
    f = bench.step_flops([("ffn_up", 1280, 1536, 8960)], 16)
    assert f == pytest.approx(71.75e9, rel=1e-3)
    layers = bench.block_layers(32760)
    assert len(layers) == 10 and sum(1 for l in layers if l[1] == 512) == 2


def _run_bench(args, env_extra=None):
    import json
    import subprocess
    env = dict(os.environ)
    env.update(env_extra or {})
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         env=env, timeout=600)
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    return res.returncode, [json.loads(l) for l in lines], res.stderr


def test_reference_arm_contract():
    """--impl reference times the CPU restatement and prints one JSON line
    with the reference fields the driver reads; it needs no GPU."""
    rc, lines, err = _run_bench(["--impl", "reference", "--config", "cfg1", "--steps", "1", "--warmup", "3"])
    assert rc == 0, err[-2000:]
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] >= 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "wan21-1.3b-ffn-up"


def test_reference_arm_other_ranks_print_nothing():
    rc, lines, err = _run_bench(["--impl", "reference", "--config", "cfg1", "--steps", "1", "--warmup", "3"],
                                {"RANK": "1", "WORLD_SIZE": "2"})
    assert rc == 0, err[-2000:]
    assert lines == []


def test_peak_follows_the_timed_region():
    peaks = {"bf16_tflops": 1678.0, "bf16_tflops_sustained": 1420.7}
    at_max = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0}
    p, why = bench.pick_peak(peaks, "measured", 0.15, at_max)
    assert p == 1678.0 and "burst" in why
    p, why = bench.pick_peak(peaks, "measured", 5.0, at_max)
    assert p == 1420.7 and "sustained" in why
    p, why = bench.pick_peak(peaks, "measured", 0.15, {"sm_mhz": 1400.0, "sm_max_mhz": 1965.0})
    assert p == 1420.7
    assert bench.pick_peak(peaks, "measured", 0.15, None)[0] == 1420.7


def test_cpu_step_extrapolates_the_sample_affinely(monkeypatch):
    """The CPU baseline times the token linears at two sample sizes and the
    context linears once; the full workload's time is the affine
    extrapolation (a per-call cost plus a per-token cost) plus the context."""
    wl = dict(name="t", layers=[("a", 1000, 16, 16), ("ctx", 7, 16, 16)], tokens=1000, rank=2, alpha=2.0,
              context=7, blocks=3)
    cs = bench.CpuStep(wl, small=100, large=200)
    assert len(cs.tok) == 1 and len(cs.ctx) == 1 and cs.tok[0][0].shape == (200, 16)
    cost = {100: 1.0 + 0.01 * 100, 200: 1.0 + 0.01 * 200}

    def fake_run(group, m=None):
        return cost[m] if m is not None else 0.5
    monkeypatch.setattr(cs, "_run", fake_run)
    est, took = cs.sample()
    assert est == pytest.approx(3 * ((1.0 + 0.01 * 1000) + 0.5))
    assert took == pytest.approx(2.0 + 3.0 + 0.5)
