"""Host-side pieces of bench.py that need no GPU: the clock summary the
bench line carries, and the device time it derives from the library's
phase events."""
import importlib.util
import os

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def row(sm, mx, *active):
    """One nvidia-smi line: index, clocks.sm, clocks.max.sm, power, the active
    bitmask, then hw_slowdown, hw_thermal, sw_thermal, sw_power_cap."""
    flags = ["Active" if k in active else "Not Active" for k in range(4)]
    return ["0", str(sm), str(mx), "700.0", "0x0"] + flags


def test_clock_summary_uses_samples_inside_the_region(bench):
    c = bench.ClockSampler(0)
    c.rows = [row(1965, 1965)]  # taken at start-up, before the region
    c.first = 1
    c.rows += [row(1500, 1965, 3), row(1560, 1965, 3), row(1530, 1965, 3)]
    s = c.summary()
    assert s["sm_mhz"] == 1530.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["samples"] == 3
    assert "sampled_before_region" not in s


def test_clock_summary_of_a_region_shorter_than_the_period(bench):
    c = bench.ClockSampler(0)
    c.rows, c.first = [row(1965, 1965)], 1
    s = c.summary()
    assert s["sm_mhz"] == 1965.0 and s["samples"] == 1 and s["sampled_before_region"] is True


def test_clock_summary_reports_throttling_and_no_sampler(bench):
    c = bench.ClockSampler(0)
    c.rows = [row(1200, 1965, 0, 1)]
    s = c.summary()
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]
    assert bench.ClockSampler(0).summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}


def test_device_time_excludes_the_copies(bench):
    t = {"h2d": 0.5, "d2h": 0.25, "total": 10.0}
    assert bench.device_ms(t) == pytest.approx(9.25)
