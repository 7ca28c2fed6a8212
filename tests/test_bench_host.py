"""Host logic of bench.py's clock record (no GPU, no nvidia-smi): the samples
kept for the timed region and the throttle reasons read from them, which decide
whether a bench line is kept or measured again."""
import bench


def _line(sm, hw="Not Active", hwt="Not Active", swt="Not Active", pcap="Not Active"):
    return f"0, {sm}, 1965, 640.5, 0x0000000000000000, {hw}, {hwt}, {swt}, {pcap}\n"


def test_mark_keeps_only_the_timed_region():
    c = bench.ClockSampler(0)
    c.lines = [_line(1200, hwt="Active")] * 3  # before the region: dropped
    c.mark()
    c.lines += [_line(1965), _line(1965), _line(1950)]
    c.__exit__(None, None, None)  # no process was started
    s = c.summary()
    assert s["samples"] == 3
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == []


def test_reasons_are_read_from_the_active_columns():
    c = bench.ClockSampler(0)
    c.lines = [_line(1965), _line(1300, pcap="Active"), _line(1400, swt="Active"),
               "garbage line\n", _line(1965, hw="Active")]
    c.__exit__(None, None, None)
    s = c.summary()
    assert s["samples"] == 4
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap", "sw_thermal_slowdown"]


def test_no_samples_gives_no_summary():
    c = bench.ClockSampler(0)
    c.__exit__(None, None, None)
    assert c.summary() is None
