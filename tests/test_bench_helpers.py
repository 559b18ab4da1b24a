"""bench.py's host helpers on CPU: the clock-sample summary (median SM clock under load and every throttle reason
seen, which decide whether a timed run is kept) and the roofline peak lookup."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def line(mhz, watts, hw="Not Active", thermal="Not Active", sw_thermal="Not Active", cap="Not Active"):
    # index, clocks.sm, clocks.max.sm, power.draw, reasons.active, hw_slowdown, hw_thermal, sw_thermal, power cap
    return f"0, {mhz}, 1965, {watts}, 0x0, {hw}, {thermal}, {sw_thermal}, {cap}"


def test_summary_takes_the_median_under_load_and_every_reason(bench):
    s = bench.ClockSampler(0)
    s.lines = [line(600, 120.0), line(1600, 900.0, cap="Active"), line(1700, 950.0), line(1650, 980.0),
               "garbage", line(1500, 990.0, sw_thermal="Active")]
    got = s.summary()
    assert got["sm_mhz"] == 1625.0                  # median of the four samples above 250 W
    assert got["sm_max_mhz"] == 1965.0
    assert got["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    assert got["samples"] == 4


def test_summary_without_samples_says_so(bench):
    s = bench.ClockSampler(0)
    s.lines = []
    assert s.summary()["reasons"] == ["unsampled"]


def test_summary_falls_back_to_idle_samples(bench):
    s = bench.ClockSampler(0)
    s.lines = [line(1965, 100.0, hw="Active")]
    got = s.summary()
    assert got["sm_mhz"] == 1965.0 and got["reasons"] == ["hw_slowdown"]


def test_peaks_come_from_the_measured_file_or_the_stated_fallback(bench):
    pk = bench.peaks()
    assert pk["source"] in ("measured", "fallback")
    assert pk["hbm_gbs"] > 1000.0
    if not (ROOT / "MEASURED_PEAKS.json").exists():
        assert pk == {"hbm_gbs": 6650.0, "source": "fallback"}
