"""bench.py's clock record: nvidia-smi CSV lines reduced to the samples inside the timed loops. CPU only."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _line(t: datetime.datetime, sm: int, reasons=()):
    flags = ["Active" if n in reasons else "Not Active" for n in bench.Clocks.NAMES]
    return ", ".join([t.strftime("%Y/%m/%d %H:%M:%S.%f")[:-3], str(sm), "1965", "812.34", "0x0000000000000000"] + flags)


def test_window_selects_the_timed_samples():
    base = datetime.datetime(2026, 12, 2, 10, 0, 0)
    lines = [_line(base + datetime.timedelta(milliseconds=50 * i), 1200 if i < 4 else 1965,
                   ("sw_power_cap",) if i == 6 else ()) for i in range(12)]
    t0 = (base + datetime.timedelta(milliseconds=200)).timestamp()
    t1 = (base + datetime.timedelta(milliseconds=400)).timestamp()
    got = bench.Clocks.summarize(lines, t0, t1)
    assert got["window"] == "timed loops"
    assert got["sm_mhz"] == 1965 and got["sm_max_mhz"] == 1965
    assert got["reasons"] == ["sw_power_cap"]
    assert 5 <= got["samples"] <= 7  # 200..400 ms plus 50 ms of slack each side


def test_fallbacks():
    base = datetime.datetime(2026, 12, 2, 10, 0, 0)
    lines = [_line(base + datetime.timedelta(milliseconds=50 * i), 1900 + i) for i in range(3)]
    far = (base + datetime.timedelta(hours=1)).timestamp()
    got = bench.Clocks.summarize(lines, far, far + 1)  # nothing inside: every sample
    assert got["window"] == "whole run" and got["samples"] == 3 and got["sm_mhz"] == 1901
    got = bench.Clocks.summarize(lines)
    assert got["samples"] == 3
    odd = ["garbage", "", "[N/A], [N/A], [N/A], 1, 2, 3, 4, 5, 6",
           "not a time, 1965, 1965, 700, 0x0, Not Active, Not Active, Active, Not Active"]
    got = bench.Clocks.summarize(odd, 0.0, 1.0)  # one usable row without a timestamp
    assert got["samples"] == 1 and got["reasons"] == ["sw_thermal_slowdown"] and got["window"] == "whole run"
    assert bench.Clocks.summarize([], 0.0, 1.0) is None
