"""bench.py's clocks record, from nvidia-smi CSV lines as its sampler writes
them during the timed region (no GPU needed): the median SM clock, the
highest max clock and every throttle reason seen active, so that a run with a
slowdown reason is flagged and one under the power cap is kept and noted."""
import bench

# index, clocks.sm, clocks.max.sm, power.draw, reasons bitmask, hw_slowdown,
# hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap
ROW = "0, {sm}, 1965, 980.12, 0x0000000000000004, {hw}, Not Active, Not Active, {cap}"


def rows(*samples):
    return [ROW.format(sm=sm, hw=hw, cap=cap) for sm, hw, cap in samples]


def test_median_clock_and_power_cap_reason():
    got = bench.ClockSampler.summarize(rows((1900, "Not Active", "Not Active"), (1950, "Not Active", "Active"),
                                            (1965, "Not Active", "Not Active")))
    assert got == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}


def test_a_slowdown_seen_once_is_reported():
    got = bench.ClockSampler.summarize(rows((1965, "Not Active", "Not Active"), (1200, "Active", "Active")))
    assert got["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert got["sm_mhz"] == (1965 + 1200) / 2


def test_malformed_and_unavailable_fields_are_skipped():
    lines = rows((1800, "Not Active", "Not Active")) + ["", "garbage", "0, [N/A], [N/A], [N/A], [N/A], [N/A], "
                                                                      "[N/A], [N/A], [N/A]"]
    got = bench.ClockSampler.summarize(lines)
    assert got["sm_mhz"] == 1800.0 and got["sm_max_mhz"] == 1965.0 and got["reasons"] == []
    assert got["samples"] == 2  # the [N/A] row is a sample without a clock reading


def test_no_samples_gives_no_record():
    assert bench.ClockSampler.summarize([]) is None
    assert bench.ClockSampler.summarize(["too, short"]) is None
