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


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` runs the reference's CPU codec (or the C
    restatement where that library is absent) and prints one JSON line with
    the device arm's metric, unit, config and the e2e / cpu_baseline objects."""
    import json
    import subprocess
    import sys

    result = subprocess.run([sys.executable, str(bench.ROOT / "bench.py"), "--impl", "reference",
                             "--steps", "1", "--warmup", "1"],
                            capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stderr
    lines = [line for line in result.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["config"] == bench.arm_config("capsule", 1)
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": bench.UNIT,
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_nothing_on_other_ranks():
    """Under torchrun only rank 0 runs the CPU reference; other ranks exit 0."""
    import os
    import subprocess
    import sys

    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    result = subprocess.run([sys.executable, str(bench.ROOT / "bench.py"), "--impl", "reference",
                             "--gpus", "2", "--steps", "1", "--warmup", "1"],
                            capture_output=True, text=True, timeout=300, env=env)
    assert result.returncode == 0, result.stderr
    assert not [line for line in result.stdout.splitlines() if line.startswith("{")]
