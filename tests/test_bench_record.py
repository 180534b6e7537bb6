"""Host-side pieces of bench.py's record (no GPU): the clock summary that
decides whether a run counts (median SM clock under load, the throttle
reasons seen), the algorithmic work per config used by the roofline, and
the command-line contract the driver relies on."""
import importlib.util
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", REPO / "bench.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    return b


def test_clock_summary_median_and_reasons():
    b = _bench()
    c = b.ClockSampler(0)
    c.lines = [
        "0, 1300, 1965, 990.1, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1350, 1965, 995.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1400, 1965, 970.2, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
    ]
    s = c.summary()
    assert s["samples"] == 3 and s["sm_mhz"] == 1350 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    c.lines = ["0, 900, 1965, 400.0, 0x40, Active, Not Active, Not Active, Not Active"]
    assert c.summary()["reasons"] == ["hw_slowdown"]


def test_clock_summary_without_samples():
    b = _bench()
    c = b.ClockSampler(0)
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_flops_per_step_matches_the_stated_configs():
    b = _bench()
    # 2·T·d·E (router) + 6·T·k·d·F (experts): c5 is 46.2 TFLOP, c1 6.45 GFLOP
    assert abs(b.flops_per_step(b.CONFIGS["c5"]) / 46.2e12 - 1) < 0.01
    assert abs(b.flops_per_step(b.CONFIGS["c1"]) / 6.45e9 - 1) < 0.01


def test_command_line_contract():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--help"], capture_output=True,
                         text=True, timeout=120)
    assert out.returncode == 0
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--config", "--stage-times"):
        assert flag in out.stdout
