"""bench.py's clock record: nvidia-smi CSV samples of the timed region reduce to the median
SM clock, the max clock and the throttle reasons seen, for the benchmark's GPUs only."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


class FakeProc:
    def __init__(self, text):
        self.text = text

    def terminate(self):
        pass

    def communicate(self, timeout=None):
        return self.text, ""


def test_clock_sampler_summary():
    rows = [
        "0, 1900, 1965, 950.1, 0x0, Not Active, Not Active, Not Active, Active",
        "0, 1800, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active",
        "1, 1000, 1965, 100.0, 0x0, Active, Not Active, Not Active, Not Active",  # not ours
        "0, 1700, 1965, 999.9, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
        "0, [N/A], 1965, 1.0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    s = bench.ClockSampler([0])
    s.proc = FakeProc("\n".join(rows))
    rec = s.stop()
    assert rec["sm_mhz"] == 1800 and rec["sm_max_mhz"] == 1965
    assert rec["reasons"] == ["sw_power_cap"] and rec["samples"] == 3
    none = bench.ClockSampler([0])
    assert none.stop()["reasons"] == ["nvidia-smi unavailable"]
