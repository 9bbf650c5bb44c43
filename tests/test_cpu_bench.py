"""bench.py's clock record: only nvidia-smi samples taken inside the timed window
count (idle samples before or after it would pull the median SM clock down and
hide or fake a throttled run), and throttle reasons seen inside it are reported."""
import datetime
import importlib.util
import os
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _line(t, mhz, power_cap):
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return "%s, 0, %d, 1965, 600.0, 0x0, Not Active, Not Active, Not Active, %s\n" % (
        ts, mhz, "Active" if power_cap else "Not Active")


def test_clock_summary_uses_the_timed_window_only(tmp_path):
    b = _bench()
    c = b.ClockSampler(0)
    c.path = str(tmp_path / "clocks.csv")
    c.proc = object()           # a sampler that ran
    c.t0 = time.time()
    c.t1 = c.t0 + 0.2
    with open(c.path, "w") as f:
        f.write(_line(c.t0 - 0.4, 120, False))     # idle, before the window
        f.write("garbage line\n")
        for i in range(5):
            f.write(_line(c.t0 + 0.03 + 0.04 * i, 1965 if i != 2 else 1800, i == 3))
        f.write(_line(c.t1 + 0.5, 120, False))     # idle, after the window
    s = c.summary()
    assert s["samples"] == 5
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_without_samples_is_none(tmp_path):
    b = _bench()
    c = b.ClockSampler(0)
    c.path = str(tmp_path / "clocks.csv")
    c.proc = object()
    c.t0 = time.time()
    c.t1 = c.t0 + 0.1
    with open(c.path, "w") as f:
        f.write(_line(c.t0 - 2.0, 120, False))
    assert c.summary() is None
