"""The clock summary that bench.py and the config runner attach to every
measurement (median SM clock, max clock, throttle reasons seen)."""

from confkv_b200.clocks import summarize

IDLE = "0, 1965, 1965, 180.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"
CAPPED = "0, 1320, 1965, 998.7, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
HOT = "0, 1500, 1965, 700.0, 0x0000000000000020, Not Active, Not Active, Active, Not Active"


def test_median_and_max_over_samples():
    out = summarize("\n".join([IDLE, IDLE, CAPPED]))
    assert out == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}


def test_every_active_reason_is_reported():
    out = summarize("\n".join([CAPPED, HOT, IDLE, HOT]))
    assert out["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    assert out["sm_mhz"] == 1500.0 and out["samples"] == 4


def test_cut_off_and_foreign_lines_are_skipped():
    out = summarize("\n".join([IDLE, "0, 19", "No devices were found", IDLE[:40], IDLE]))
    assert out["samples"] == 2 and out["reasons"] == []


def test_no_samples():
    assert summarize("") is None
    assert summarize("garbage\n") is None
