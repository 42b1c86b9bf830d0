"""Bandwidth arithmetic, percentiles and the clock-record rules used by the
benchmarks (no GPU needed)."""

import math

import pytest

from numa_allreduce_b200.utils.timing import (ClockSampler, _summarise, algbw_gbs, busbw_gbs, clocks_ok,
                                              percentile)


def test_bandwidth_conventions():
    # nccl-tests: algbw = S/t, busbw = algbw * 2(n-1)/n
    assert algbw_gbs(1 << 30, 1.0) == pytest.approx((1 << 30) / 1e9)
    assert busbw_gbs(1 << 30, 1.0, 8) == pytest.approx((1 << 30) / 1e9 * 14 / 8)
    assert busbw_gbs(1 << 30, 1.0, 1) == 0.0 and algbw_gbs(1, 0.0) == 0.0


def test_percentile():
    assert percentile([3.0, 1.0, 2.0], 0.5) == 2.0
    assert percentile([1.0, 2.0, 3.0, 4.0], 0.5) == pytest.approx(2.5)
    assert math.isnan(percentile([], 0.5))


def test_summary_and_rejection_rules():
    rows = [(1900.0, 1965.0, 700.0, set()), (1300.0, 1965.0, 998.0, {"sw_power_cap"}),
            (1950.0, 1965.0, 650.0, set())]
    s = _summarise(rows)
    assert s["sm_mhz"] == 1900.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    assert clocks_ok(s) is None  # too few samples to vouch for the run
    s = _summarise(rows * 4)
    assert clocks_ok(s) is True  # power capping is kept (and noted)
    for bad in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"):
        assert clocks_ok(dict(s, reasons=[bad])) is False
    # clocks stuck well below the maximum with no reason: a leftover lock
    assert clocks_ok(dict(s, sm_mhz=1100.0, reasons=[])) is False
    assert clocks_ok(dict(s, sm_mhz=1300.0, reasons=["sw_power_cap"])) is True
    assert _summarise([]) == {"available": False, "samples": 0}
    assert clocks_ok({"available": False}) is None
    assert clocks_ok(None) is None


def test_sampler_without_a_gpu_returns_a_record():
    rec = ClockSampler([], interval_ms=10).start(wait_s=2.0).stop(0.0, 1e12)
    assert isinstance(rec, dict)
    assert "available" in rec or "samples" in rec
