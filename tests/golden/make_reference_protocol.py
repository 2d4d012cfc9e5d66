"""Write tests/golden/reference_runtime_protocol.json: the launch sequence of
the reference plugin's own GdnStateCodecRuntime (src/gdn_state_codec/
runtime.py, with the three edits of INTEGRATION.md section 2) over one slot of
32 heads: the quant-only encode and 18 decode steps across a window refit,
every pointer named by the buffer the plugin allocated for it.

Run in a container that holds the reference source tree (GDN_REFERENCE_ROOT,
or a directory `reference` beside this repository):

    python tests/golden/make_reference_protocol.py

tests/test_reference_plugin.py re-records it from the reference and compares;
tests/test_gpu_reference_protocol.py replays it on the GPU without the
reference tree.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT / "tests"), str(ROOT / "gdn-state-codec_b200")]

import reference_plugin  # noqa: E402
from gdn_state_codec import _native  # noqa: E402

OUT = HERE / "reference_runtime_protocol.json"


def main() -> None:
    root = reference_plugin.reference_root()
    if root is None:
        raise SystemExit("reference source tree not found (set GDN_REFERENCE_ROOT)")
    config, runtime = reference_plugin.load_reference_plugin(root)
    protocol = reference_plugin.record_protocol(config, runtime, _native.library_dir())
    OUT.write_text(json.dumps(protocol, indent=1) + "\n")
    print(f"wrote {OUT}: {len(protocol['calls'])} launches, {len(protocol['buffers'])} buffers")


if __name__ == "__main__":
    main()
