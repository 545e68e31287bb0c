"""bench.py's clock record: samples are binned over the device-timed window.

The sampler polls NVML in a thread; here the samples are planted directly,
so the summary logic (window, median, slowdown reasons, samples whose
reasons could not be read) is checked without a GPU. So is the paired
check-overhead estimator, which compares the two variants within each
round of interleaved launches.
"""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_summary_covers_only_the_timed_window(bench):
    s = bench.ClockSampler(["abc"])
    s.source = "planted"
    power_cap = dict(bench.ClockSampler.REASONS)["sw_power_cap"]
    thermal = dict(bench.ClockSampler.REASONS)["hw_thermal_slowdown"]
    s.samples = [(0.5, 210.0, 1965.0, 90.0, 0),                # idle, before the window
                 (1.0, 1965.0, 1965.0, 700.0, 0),
                 (1.1, 1905.0, 1965.0, 999.0, power_cap),
                 (1.2, 1800.0, 1965.0, 998.0, power_cap),
                 (2.5, 1200.0, 1965.0, 500.0, thermal)]        # after the window
    out = s.summary(1.0, 1.2)
    assert out["samples"] == 3 and out["window"] == "timed"
    assert out["sm_mhz"] == 1905.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    assert out["power_w_max"] == 999.0


def test_summary_reports_an_empty_window_and_unreadable_reasons(bench):
    s = bench.ClockSampler(["abc"])
    s.samples = [(5.0, 1965.0, 1965.0, 300.0, -1)]
    empty = s.summary(1.0, 2.0)
    assert empty["samples"] == 0 and empty["sm_mhz"] is None and empty["samples_in_run"] == 1
    out = s.summary(4.0, 6.0)
    assert out["sm_mhz"] == 1965.0 and out["reasons"] == [] and out["reasons_unavailable_samples"] == 1


def test_uuids_get_the_nvml_prefix(bench):
    s = bench.ClockSampler(["58a0e2b8-0000", "GPU-1234"])
    assert s.uuids == ["GPU-58a0e2b8-0000", "GPU-1234"]


def test_paired_overhead_cancels_drift_between_rounds(bench):
    """Each round's checked / unchecked ratio is taken within the round, so a
    clock step between rounds (every launch of round 3 slower) does not move
    the estimate, while the ratio of medians would."""
    off = [100.0, 100.0, 100.0, 150.0, 150.0]
    chk = [107.0, 107.0, 107.0, 160.5, 160.5]
    assert bench.paired_overhead_pct(chk, off) == pytest.approx(7.0)
    assert bench.paired_overhead_pct([110.0, 90.0, 105.0], [100.0, 100.0, 100.0]) == pytest.approx(5.0)
