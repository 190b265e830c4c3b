"""The bench's clock sampler summary (utils/clocks.py), on nvidia-smi CSV
lines written here: parsing, the median under load, throttle reasons, the
timed-window selection and the no-nvidia-smi path. Read-only by design: the
sampler only runs ``nvidia-smi --query-gpu``."""
import datetime

from sched_pass_b200.utils import clocks


def line(t, sm, smax=1965, reasons=("Not Active",) * 4, active="0x0"):
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return ", ".join([ts, "0", str(sm), str(smax), "700.5", active, *reasons])


def test_parse_line_fields_and_reasons():
    r = clocks.parse_line(line(1000.25, 1950, reasons=("Not Active", "Not Active", "Not Active", "Active")))
    ts, sm, smax, active = r
    assert abs(ts - 1000.25) < 1e-3 and sm == 1950 and smax == 1965
    assert active == {"hw_slowdown": False, "hw_thermal_slowdown": False, "sw_thermal_slowdown": False,
                      "sw_power_cap": True}
    assert clocks.parse_line("garbage") is None
    assert clocks.parse_line("a, b, [N/A], [N/A], x, y, z, w, v, u") is None  # clocks not numbers


def test_summary_median_under_load_and_reasons():
    rows = [clocks.parse_line(line(1000 + 0.02 * i, sm)) for i, sm in enumerate([345, 1965, 1950, 1965, 1965])]
    rows.append(clocks.parse_line(line(1000.2, 1310, reasons=("Active", "Not Active", "Not Active", "Active"))))
    s = clocks.summarize(rows)
    # idle samples (below half the peak) are left out of the median
    assert s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965 and s["samples"] == 6
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_window_keeps_inside_samples_and_one_neighbour_each_side():
    rows = [clocks.parse_line(line(1000 + 0.1 * i, 1000 + i)) for i in range(10)]
    s = clocks.summarize(rows, window=(1000.35, 1000.55))
    # inside: t = .4, .5; neighbours: .3 and .6
    assert s["samples"] == 4
    assert s["sm_mhz"] == (1004 + 1005) / 2
    # a window shorter than the period keeps its two neighbours
    s = clocks.summarize(rows, window=(1000.41, 1000.42))
    assert s["samples"] == 2


def test_empty_and_unavailable():
    assert clocks.summarize([])["samples"] == 0
    sampler = clocks.ClockSampler()
    sampler.proc = None  # as after start() on a host without nvidia-smi
    s = sampler.stop()
    assert s["samples"] == 0 and s["reasons"] == ["nvidia-smi unavailable"]
