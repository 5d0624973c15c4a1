"""bench.py's host-side measurement logic, no GPU: the clock sampler keeps only the samples
whose own nvidia-smi timestamp lies inside the timed window, and reports throttle reasons."""
import datetime
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _line(t, mhz, reasons=("Not Active",) * 4):
    ts = t.strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return ", ".join([ts, str(mhz), "1965", "700.00", "0x0000000000000000", *reasons])


def test_clock_summary_keeps_the_timed_window(bench):
    s = bench.ClockSampler(0)
    t0 = datetime.datetime(2026, 1, 1, 12, 0, 0)
    s.out = [_line(t0 + datetime.timedelta(milliseconds=20 * i), 1000 if i < 5 or i > 14 else 1965)
             for i in range(20)]
    s.t0 = t0 + datetime.timedelta(milliseconds=100)          # samples 5..14 inside
    s.t1 = t0 + datetime.timedelta(milliseconds=290)
    out = s.summary()
    assert out["samples"] == 10 and out["sm_mhz"] == 1965.0 and out["reasons"] == []
    assert abs(out["window_s"] - 0.19) < 1e-9


def test_clock_summary_reports_throttle_reasons(bench):
    s = bench.ClockSampler(0)
    t0 = datetime.datetime(2026, 1, 1, 12, 0, 0)
    s.out = [_line(t0 + datetime.timedelta(milliseconds=10), 1800,
                   ("Not Active", "Active", "Not Active", "Active")),
             "garbage line", ""]
    s.t0, s.t1 = t0, t0 + datetime.timedelta(seconds=1)
    out = s.summary()
    assert out["samples"] == 1 and out["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]


def test_configs_name_the_baseline_workloads(bench):
    assert {"cfg3", "cfg4", "cfg5"} <= set(bench.CONFIGS)
    c3 = bench.CONFIGS["cfg3"]
    assert (c3["num_docs"], c3["batch"], c3["nc"], c3["K"], c3["k_top"]) == (2_000_000, 256, 32, 4096, 10)
