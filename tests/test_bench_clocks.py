"""bench.py's clock sampler: samples are kept only inside the timed region's host-clock
window (plus one sampling period of slack), medians and throttle reasons come from those."""

import datetime


def _line(t: float, mhz: int, power_cap: bool = False, thermal: bool = False) -> str:
    stamp = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    flag = lambda on: "Active" if on else "Not Active"  # noqa: E731
    return (f"{stamp}, 0, {mhz}, 1965, 900.0, 0x0, Not Active, {flag(thermal)}, Not Active, {flag(power_cap)}")


def test_summary_keeps_only_the_timed_window():
    from bench import ClockSampler

    s = ClockSampler(None)
    t0 = 1_800_000_000.0
    s.t0, s.t1 = t0, t0 + 1.0
    s.lines = [_line(t0 - 3.0, 900, thermal=True),   # warm-up, long before: dropped
               _line(t0 - 0.05, 1900),               # within the slack before the start
               _line(t0 + 0.4, 1700, power_cap=True),
               _line(t0 + 0.8, 1800),
               _line(t0 + 2.0, 600, thermal=True)]   # after the region: dropped
    out = s.summary()
    assert out["samples"] == 3
    assert out["sm_mhz"] == 1800.0
    assert out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]


def test_summary_without_marks_uses_every_sample_and_disabled_sampler_is_empty():
    from bench import ClockSampler

    s = ClockSampler(None)
    s.lines = [_line(1_800_000_000.0, 1500), _line(1_800_000_000.2, 1600)]
    assert s.summary()["samples"] == 2
    with ClockSampler(None) as idle:  # the ranks that do not sample start nothing
        pass
    assert idle.proc is None and idle.summary()["samples"] == 0
