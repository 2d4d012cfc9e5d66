"""CPU checks of the committed ncu summaries: each gives the full command that
made it, the command runs committed files only (bench.py with its own flags),
every ncu invocation keeps the GPU clocks unlocked, and the folder holds text
summaries only."""

from __future__ import annotations

import re
import shlex
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PROFILES = ROOT / "profiles"
SUMMARIES = sorted(PROFILES.glob("*.md"))


def _command(text: str) -> str:
    blocks = re.findall(r"```\n(.*?)```", text, flags=re.S)
    assert len(blocks) == 1, "one command block per summary"
    return blocks[0].replace("\\\n", " ")


def test_profiles_folder_holds_text_summaries_only():
    allowed = {".md", ".txt", ".json"}
    assert SUMMARIES
    assert all(p.suffix in allowed for p in PROFILES.iterdir())


@pytest.mark.parametrize("summary", SUMMARIES, ids=lambda p: p.name)
def test_summary_command_runs_committed_files(summary):
    command = _command(summary.read_text())
    for part in re.split(r"&&|>|;", command):
        words = shlex.split(part)
        if not words:
            continue
        if words[0] == "timeout":  # a bound around the command: timeout [-k N] SECONDS ...
            words = words[words.index("python"):] if "python" in words else []
        if words[0:1] == ["ncu"]:
            assert "--clock-control" in words and \
                words[words.index("--clock-control") + 1] == "none", part
            words = words[words.index("python"):] if "python" in words else []
        if words[:3] == ["python", "-m", "pytest"]:
            for path in (w for w in words[3:] if not w.startswith("-")):
                assert (ROOT / path).exists(), path
            continue
        if words[:3] == ["python", "-m", "torch.distributed.run"]:
            words = ["python"] + words[words.index("bench.py"):]
        if words[:1] == ["python"]:
            assert words[1] == "bench.py", part
            assert (ROOT / words[1]).is_file()
            for flag in (w for w in words[2:] if w.startswith("--")):
                assert f'"{flag}"' in (ROOT / "bench.py").read_text(), flag
