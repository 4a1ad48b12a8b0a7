"""Host-side pieces of bench.py that decide whether a run is valid: the
defaults (at least 3 warm-up steps), the clock record taken during the timed
region (median SM clock, throttle reasons) and the CPU arm's thread count.
No GPU and no library compute."""
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def _summary(tmp_path, lines):
    s = bench.ClockSampler(0)
    s.path = tmp_path / "clocks.csv"
    s.path.write_text("\n".join(lines) + "\n")
    return s.summary()


def test_defaults_keep_three_warmup_steps(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert a.gpus == 1 and a.warmup >= 3 and a.steps >= 1 and a.impl == "native"
    assert a.batch == 8 and (a.height, a.width) == (480, 856)


def test_clock_summary_median_and_power_cap(tmp_path):
    # index, sm, max sm, power, active mask, hw_slowdown, hw_thermal, sw_thermal, sw_power_cap
    rows = [f"0, {mhz}, 1965, 990.1, 0x4, Not Active, Not Active, Not Active, Active"
            for mhz in (1500, 1560, 1590, 1620, 1440)]
    s = _summary(tmp_path, rows)
    assert s["sm_mhz"] == 1560 and s["sm_max_mhz"] == 1965 and s["samples"] == 5
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_reports_thermal_and_hw_slowdown(tmp_path):
    rows = ["0, 1200, 1965, 700.0, 0x48, Active, Not Active, Active, Not Active",
            "0, 1300, 1965, 710.0, 0x0, Not Active, Not Active, Not Active, Not Active",
            "garbage line"]
    s = _summary(tmp_path, rows)
    assert s["sm_mhz"] == 1250 and s["samples"] == 2
    assert s["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]


def test_clock_summary_without_samples(tmp_path):
    s = bench.ClockSampler(0)
    s.path = tmp_path / "missing.csv"
    assert s.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}


def test_cpu_arm_uses_every_allowed_cpu_despite_omp_one(monkeypatch):
    monkeypatch.setenv("OMP_NUM_THREADS", "1")  # what torch.distributed.run sets per rank
    n = bench.host_threads()
    expect = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    assert n == expect and n >= 1


def test_frame_pair_flops_constant():
    """3 x VAE (fwd + dX + dW on frame k) + 2 x encoder forward on frames 0
    and 16 + the U-Net's training pass = 10.16 TFLOP per frame-pair."""
    per_pair = 3 * bench.VAE_FWD_PER_FRAME + 2 * bench.ENC_FWD_PER_FRAME + \
        bench.MOTION_TRAIN_PER_SAMPLE
    assert abs(per_pair - 10.16e12) < 0.01e12
