"""bench.py's clock record, on CPU with a fake NVML.

The bench line must carry the SM clock seen during the timed region and the
clock-event reasons that were active (hw_slowdown, hw_thermal_slowdown,
sw_thermal_slowdown, sw_power_cap). The sampler decodes NVML's reason bit mask;
these tests feed it samples through a stand-in NVML module and check the
median, the maximum, the decoded reasons, the polling wait, and the empty
record when no sample was taken.
"""
import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class FakeNvml:
    NVML_CLOCK_SM = 1
    nvmlClocksEventReasonHwSlowdown = 0x8
    nvmlClocksEventReasonHwThermalSlowdown = 0x40
    nvmlClocksEventReasonSwThermalSlowdown = 0x20
    nvmlClocksEventReasonSwPowerCap = 0x4

    def __init__(self, clocks, reasons):
        self.clocks, self.reasons, self.i = list(clocks), list(reasons), 0

    def nvmlDeviceGetClockInfo(self, handle, kind):
        return self.clocks[min(self.i, len(self.clocks) - 1)]

    def nvmlDeviceGetCurrentClocksEventReasons(self, handle):
        r = self.reasons[min(self.i, len(self.reasons) - 1)]
        self.i += 1
        return r


def _sampler(bench, nvml):
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.gpu, c.proc, c.lines, c.samples, c.thread = 0, None, [], [], None
    c.nvml, c.handle, c.max_sm = nvml, object(), 1965.0
    return c


def test_reasons_are_decoded_and_the_clock_is_the_median():
    bench = _bench()
    c = _sampler(bench, FakeNvml([1965, 1800, 1965], [0x0, 0x4, 0x1]))  # 0x1 (GPU idle) is not reported
    for _ in range(3):
        c._sample()
    s = c.summary()
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"] and s["source"] == "nvml"
    c2 = _sampler(bench, FakeNvml([1200], [0x8 | 0x40 | 0x20]))
    c2._sample()
    assert c2.summary()["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_wait_samples_until_the_event_completes():
    bench = _bench()

    class Event:
        def __init__(self):
            self.polls = 0

        def query(self):
            self.polls += 1
            return self.polls > 5

    c = _sampler(bench, FakeNvml([1965], [0]))
    c.wait(Event())
    assert c.summary()["samples"] == 5


def test_no_sample_gives_an_empty_record():
    bench = _bench()
    c = _sampler(bench, None)
    s = c.summary()
    assert s["sm_mhz"] is None and s["samples"] == 0 and s["reasons"] == []
    c.wait(None)  # without NVML, waiting samples nothing and returns at once
