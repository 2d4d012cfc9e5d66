"""CPU proofs of the kernels' division routines (no GPU needed).

The quantizer and the projection replace IEEE division by faster sequences
that must round exactly like IEEE division for the codes to stay bit-exact:
  * a / 127 as fma(a, zh, RN(a * zl)) -- checked for every float with
    |a| >= 2^-112 (the kernels send smaller |a| to IEEE division);
  * a / c from the two-term reciprocal RN(1/c), RN((1 - c RN(1/c)) RN(1/c))
    with one fma correction -- checked on hundreds of millions of operands
    over the kernels' fast-path ranges, including quotients next to rounding
    midpoints and at the bottom of the range.
tests/division_check.c holds the restatements; the device versions are
compared with IEEE division on the GPU by test_gpu_division.py.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

SOURCE = Path(__file__).resolve().parent / "division_check.c"
THREADS = max(1, min(16, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def checker(tmp_path_factory) -> Path:
    exe = tmp_path_factory.mktemp("division") / "division_check"
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
                    "-o", str(exe), str(SOURCE), "-lm", "-lpthread"], check=True)
    return exe


def _run(exe: Path, *args: str) -> str:
    result = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stdout + result.stderr
    return result.stdout.strip()


def test_div127_exhaustive(checker):
    line = _run(checker, "div127", str(THREADS))
    fields = dict(item.split("=") for item in line.split()[1:])
    assert int(fields["mismatches"]) == 0, line
    # every finite float with |a| >= 2^-112, both signs, plus 5 specials
    assert int(fields["checked"]) == 2 * (0x7F800000 - 0x07800000) + 5


def test_markstein_quotients(checker):
    line = _run(checker, "markstein", str(THREADS), str(4_000_000))
    fields = dict(item.split("=") for item in line.split()[1:])
    assert int(fields["mismatches"]) == 0, line
    assert int(fields["checked"]) > 10_000_000


def test_code_rule(checker):
    line = _run(checker, "codes", str(THREADS), str(2_000_000))
    fields = dict(item.split("=") for item in line.split()[1:])
    assert int(fields["mismatches"]) == 0, line
    assert int(fields["checked"]) > 10_000_000
    # the flag band is narrow: random values are flagged about 2^-13 of the time
    assert int(fields["random_flagged"]) < int(fields["random"]) // 1000
