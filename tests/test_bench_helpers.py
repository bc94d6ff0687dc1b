"""bench.py's own logic on CPU: the clock summary that decides whether a
timed run is rejected (throttle reasons, clocks under load), and the
workload naming in the JSON line."""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _line(mhz, reasons=("Not Active",) * 4, max_mhz=1965):
    # index, clocks.sm, clocks.max.sm, power.draw, active, then the four
    # reasons: hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown,
    # sw_power_cap
    return ", ".join(["0", str(mhz), str(max_mhz), "700.0", "0x0"] +
                     list(reasons))


def test_clock_summary_uses_only_the_timed_region():
    c = bench.ClockSampler(0)
    c.lines = [(0.0, _line(900)),          # warm-up, before the region
               (1.0, _line(1965)), (1.1, _line(1950)), (1.2, _line(1965)),
               (9.0, _line(600))]          # after the region
    c.t_begin, c.t_end = 0.95, 1.25
    s = c.summary()
    assert s["samples"] == 3
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == []


def test_clock_summary_reports_active_reasons():
    c = bench.ClockSampler(0)
    c.lines = [(1.0, _line(1400, ("Not Active", "Not Active", "Not Active",
                                  "Active"))),
               (1.1, _line(1300, ("Active", "Not Active", "Not Active",
                                  "Not Active")))]
    c.t_begin, c.t_end = 0.9, 1.2
    s = c.summary()
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert s["sm_mhz"] == 1350.0


def test_clock_summary_ignores_malformed_lines():
    c = bench.ClockSampler(0)
    c.lines = [(1.0, "garbage"), (1.05, "0, [N/A], 1965, 1, 0x0, a, b, c, d"),
               (1.1, _line(1965))]
    c.t_begin, c.t_end = 0.9, 1.2
    s = c.summary()
    assert s["samples"] == 1 and s["sm_mhz"] == 1965.0


def test_workload_names():
    a = argparse.Namespace(blocks=4096, layers=32, gpus=1)
    cfg = bench.workload_config(a, 2 << 20)
    assert cfg["workload"] == "llama3-8b-kv-2MiB-x4096"
    assert "exceed the 126 MB L2" in cfg["l2"]
    b = argparse.Namespace(blocks=4096, layers=2, gpus=8)
    assert bench.workload_config(b, 128 << 10)["workload"] == \
        "llama3-8b-kv-128KiB-x4096"
