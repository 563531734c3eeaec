"""CPU: the clock record of the bench line (bench.ClockSampler.summary) from
injected NVML samples: median SM clock, max clock, and every clock-event
reason seen during the timed region (idle excluded)."""
import bench


def sampler(samples, max_mhz=1965):
    s = bench.ClockSampler.__new__(bench.ClockSampler)   # no NVML here: inject the state
    s.ok, s.samples, s.max_mhz = True, samples, max_mhz
    return s


def test_median_and_reasons():
    # (time, SM MHz, reasons bitmask): idle 0x1 and power cap 0x4 seen, thermal 0x20 once
    samples = [(0.0, 1965, 0x1), (0.2, 1950, 0x4), (0.4, 1430, 0x4), (0.6, 1440, 0x4 | 0x20), (0.8, 1965, 0)]
    rec = sampler(samples).summary()
    assert rec["sm_mhz"] == 1950 and rec["sm_max_mhz"] == 1965 and rec["samples"] == 5
    assert rec["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]       # gpu_idle is not a throttle


def test_clean_run_and_no_nvml():
    rec = sampler([(0.0, 1965, 0), (0.2, 1965, 0)]).summary()
    assert rec["reasons"] == [] and rec["sm_mhz"] == 1965
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.ok, s.samples, s.err = False, [], "NVML Shared Library Not Found"
    rec = s.summary()
    assert rec["sm_mhz"] is None and rec["samples"] == 0 and "NVML" in rec["note"]


def test_every_rejecting_reason_has_a_name():
    names = set(bench.ClockSampler.REASONS.values())
    assert {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"} <= names
