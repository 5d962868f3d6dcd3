"""bench.py's host-side logic on CPU: the clock sampler's summary (the clocks field of the bench line, from
which a run with a slowdown reason is rejected) for both sample formats it collects."""
import bench


def _sampler(lines, nvml):
    c = bench.ClockSampler(0)
    c.lines = lines
    c.thread = object() if nvml else None
    return c


def test_clock_summary_nvml_lines():
    # index, SM MHz, max SM MHz, W, reason bits, then hw_slowdown, hw_thermal, sw_thermal, sw_power_cap
    lines = ["0,1965,1965,600.0,0x0,Not Active,Not Active,Not Active,Not Active",
             "0,1800,1965,990.5,0x4,Not Active,Not Active,Not Active,Active",
             "0,1700,1965,995.0,0x4,Not Active,Not Active,Not Active,Active"]
    s = _sampler(lines, nvml=True).summary()
    assert s["sm_mhz"] == 1800 and s["sm_max_mhz"] == 1965 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"] and s["power_w"] == 990.5
    assert s["sampler"].startswith("nvml")


def test_clock_summary_reports_slowdowns_and_skips_bad_lines():
    lines = ["0, 1500, 1965, 700.00, 0x0000000000000008, Active, Not Active, Not Active, Not Active",
             "0, [N/A], 1965, 700.00, 0x0, Not Active, Not Active, Not Active, Not Active",
             "garbage",
             "0, 1400, 1965, 700.00, 0x0000000000000060, Not Active, Active, Active, Not Active"]
    s = _sampler(lines, nvml=False).summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1450
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]
    assert s["sampler"].startswith("nvidia-smi")


def test_clock_summary_without_samples():
    s = _sampler([], nvml=False).summary()
    assert s["samples"] == 0 and s["sm_mhz"] is None and s["reasons"] == []
