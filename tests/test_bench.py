"""CPU tests of bench.py's host logic: the clock sampler keeps only the
samples taken inside the timed region, and a region shorter than the
sampling interval falls back to the first sample after it began, saying so."""

from __future__ import annotations

import bench


class _FakeProc:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0

    def kill(self):
        pass


def _line(mhz: float, power_cap: bool = False) -> str:
    cap = "Active" if power_cap else "Not Active"
    return f"0, {mhz}, 1965, 480.5, 0x0, Not Active, Not Active, Not Active, {cap}"


def _sampler(samples):
    sampler = bench.ClockSampler(0)
    sampler.proc = _FakeProc()
    sampler.lines = list(samples)
    return sampler


def test_clock_samples_come_from_the_timed_region():
    sampler = _sampler([(1.0, _line(900)), (2.0, _line(1965)), (2.1, _line(1965, True)),
                        (2.2, _line(1950)), (9.0, _line(700))])
    clocks = sampler.stop(1.5, 2.5)
    assert clocks["samples"] == 3
    assert clocks["sm_mhz"] == 1965.0
    assert clocks["sm_max_mhz"] == 1965.0
    assert clocks["reasons"] == ["sw_power_cap"]
    assert clocks["window"] == "timed region"


def test_short_region_takes_the_next_sample_and_says_so():
    sampler = _sampler([(1.0, _line(900)), (3.0, _line(1965)), (3.1, _line(1800))])
    clocks = sampler.stop(2.0, 2.05)
    assert clocks["samples"] == 1
    assert clocks["sm_mhz"] == 1965.0
    assert clocks["window"].startswith("first sample after")


def test_unparseable_lines_are_ignored():
    sampler = _sampler([(2.0, "[N/A]"), (2.1, _line(1965))])
    assert sampler.stop(1.0, 3.0)["samples"] == 1
