"""bench.py's clock window: samples inside the timed region, or the samples
bracketing a region shorter than the sampling period (no GPU needed)."""
import bench


def _sampler(samples):
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.samples, c.proc = samples, None
    return c


def _row(mhz, power_cap="Not Active", thermal="Not Active"):
    return ["0", str(mhz), "1965", "700", "0x0", "Not Active", "Not Active", thermal, power_cap]


def test_window_inside():
    c = _sampler([(0.0, _row(1965)), (0.1, _row(1900, "Active")), (0.2, _row(1880, "Active")),
                  (0.3, _row(1965))])
    w = c.window(0.05, 0.25)
    assert w["samples"] == 2 and w["sm_mhz"] == 1890 and w["reasons"] == ["sw_power_cap"]
    assert "bracketing" not in w


def test_window_short_region_bracketed():
    c = _sampler([(0.0, _row(1965)), (0.1, _row(1965, thermal="Active")), (0.2, _row(1950))])
    w = c.window(0.12, 0.15)  # 30 ms region between two samples
    assert w["bracketing"] and w["samples"] == 2
    assert w["sm_mhz"] == (1965 + 1950) / 2
    assert w["reasons"] == ["sw_thermal_slowdown"]


def test_window_unsampled():
    w = _sampler([]).window(0.0, 1.0)
    assert w["samples"] == 0 and w["reasons"] == ["unsampled"]


def test_bracketing_reasons_kept_apart():
    """One sample inside the region and a throttled sample just after it: the
    region's reasons come from the inside sample alone; the bracketing
    samples' reasons are listed separately."""
    c = _sampler([(0.0, _row(1965)), (0.1, _row(1965)), (0.2, _row(1700, thermal="Active"))])
    w = c.window(0.05, 0.15)
    assert w["bracketing"] and w["samples_inside"] == 1
    assert w["reasons"] == []
    assert w["reasons_bracketing"] == ["sw_thermal_slowdown"]
