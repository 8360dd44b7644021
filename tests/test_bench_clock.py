"""bench.py's clock record: only samples inside the timed region count, the
throttle-reason bits map to the names the timing rules use, and a region
shorter than one sample interval falls back to the samples around it."""
import importlib.util
import os
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_clock_summary_keeps_the_timed_region():
    b = _bench()
    c = b.ClockSampler(0)
    t = time.monotonic()
    # (monotonic time, SM MHz, max MHz, NVML clocks-event-reason bits)
    c.rows = [(t - 1.0, 900.0, 1965.0, 0x40),          # before the region: thermal slowdown, ignored
              (t + 0.001, 1965.0, 1965.0, 0x4),        # power cap inside the region
              (t + 0.002, 1950.0, 1965.0, 0x0),
              (t + 5.0, 800.0, 1965.0, 0x8)]           # after the region: ignored
    c.t0, c.t1 = t, t + 0.003
    s = c.summary()
    assert s["samples"] == 2 and s["window"] == "timed region"
    assert s["sm_mhz"] == 1957.5 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_short_region_and_reason_names():
    b = _bench()
    assert set(b.ClockSampler.REASONS.values()) == {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                                     "sw_power_cap"}
    c = b.ClockSampler(0)
    t = time.monotonic()
    c.rows = [(t - 0.004, 1965.0, 1965.0, 0x20)]
    c.t0, c.t1 = t, t + 0.0005                          # no sample inside: the neighbours within 10 ms
    s = c.summary()
    assert s["samples"] == 1 and s["window"] == "timed region +- 10 ms"
    assert s["reasons"] == ["sw_thermal_slowdown"]
    c.rows = []
    assert c.summary()["samples"] == 0
