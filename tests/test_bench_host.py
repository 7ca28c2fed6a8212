"""Host logic of bench.py (no GPU, no nvidia-smi): the clock record -- the
samples kept for the timed region and the throttle reasons read from them,
which decide whether a bench line is kept or measured again -- and the
algorithmic bytes behind the roofline and the CPU baseline's GB/s."""
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


def test_algorithmic_bytes_and_cpu_rate_of_the_configs():
    """Per-step algorithmic bytes V*d + 4V + B*(4d + 4H + 4): C2's 545,620,996 B
    (one stream), C3's per 64 streams, and a CPU rate in GB/s from tokens/s."""
    from lal_b200 import synth
    c2 = synth.CONFIGS["c2_qwen"]
    assert bench.algorithmic_bytes(c2, 1) == 545_620_996
    c3 = synth.CONFIGS["c3_batch"]
    assert bench.algorithmic_bytes(c3, 64) == 152064 * 3584 + 4 * 152064 + 64 * (
        4 * 3584 + 4 * c3.hist + 4)
    # 1000 tokens/s of single-stream steps stream 1000 x 545.6 MB
    assert bench.cpu_gbs(c2, 1000.0) == round(545_620_996 * 1000 / 1e9, 3)
    # B tokens a step: the rate counts steps, not tokens
    assert bench.cpu_gbs(c3, 64 * 10.0) == round(bench.algorithmic_bytes(c3, 64) * 10 / 1e9, 3)
    # a rank's slice of the vocab at N shards
    assert bench.algorithmic_bytes(c2, 1, rows=19008) == 19008 * 3584 + 4 * 19008 + 4 * 3584 \
        + 4 * c2.hist + 4
