"""bench.py's clock record: only nvidia-smi samples taken inside the timed region count."""
import datetime
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _FakeSmi:
    def __init__(self, text):
        self.text = text

    def terminate(self):
        pass

    def communicate(self, timeout=None):
        return self.text, ""


def _row(ts, sm, power, cap="Not Active", thermal="Not Active"):
    return f"{ts}, 0, {sm}, 1965, {power}, 0x0, Not Active, Not Active, {thermal}, {cap}\n"


def test_samples_outside_the_timed_region_are_ignored():
    b = _bench()
    rows = (_row("2026/12/02 05:45:46.900", 345, 150.0)            # idle, before the region
            + _row("2026/12/02 05:45:47.100", 1965, 900.0)
            + _row("2026/12/02 05:45:47.150", 1800, 990.0, cap="Active")
            + _row("2026/12/02 05:45:48.100", 1000, 100.0, thermal="Active"))  # after the region
    cs = b.ClockSampler(0)
    cs.proc = _FakeSmi(rows)
    t0 = datetime.datetime.strptime("2026/12/02 05:45:47.000", "%Y/%m/%d %H:%M:%S.%f").timestamp()
    cs.window(t0, t0 + 0.5)
    rec = cs.stop()
    assert rec["samples"] == 2 and rec["samples_from"] == "timed region"
    assert rec["sm_mhz"] == (1965 + 1800) / 2 and rec["sm_max_mhz"] == 1965
    assert rec["reasons"] == ["sw_power_cap"]  # the thermal sample after the region is not counted
    assert rec["power_w_max"] == 990.0


def test_without_samples_in_the_window_the_whole_run_is_reported():
    b = _bench()
    cs = b.ClockSampler(0)
    cs.proc = _FakeSmi(_row("2026/12/02 05:45:46.900", 1965, 500.0))
    cs.window(0.0, 1.0)
    rec = cs.stop()
    assert rec["samples"] == 1 and rec["samples_from"] == "whole run"
