"""Generates tests/golden/plan_traces.json.gz: the reference's frozen WebGPU dispatch lists
(``tests/golden/k28/dispatch-traces.json.gz`` of the reference checkout, recorded by
``tests/plan_trace.test.ts`` through a mock GPU) for the GLiNER2 (DeBERTa-v3 small/base) and
Julia (ModernBERT) plans, restricted to the plain forward modes (``normal``: all rows,
``normal100``: 100 rows per sequence). Each trace lists the input writes, the Julia type-row
copies, every pipeline with its override constants, every bind group and dispatch size, and the
output copy; buffers carry their sizes and the sha256 of their build-time contents (relidx,
cossin, zero). Run in the build container, where the reference exists:

    python tests/golden/make_plan_traces.py <path to the reference checkout>

The tests read the fixture only; they never open the reference.
"""
from __future__ import annotations

import gzip
import json
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "plan_traces.json.gz"


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_plan_traces.py <path to the reference checkout>")
    ref = Path(sys.argv[1])
    frozen = json.loads(gzip.decompress((ref / "tests/golden/k28/dispatch-traces.json.gz").read_bytes()))
    keep = {k: {"buffers": v["buffers"], "events": v["events"]}
            for k, v in frozen["traces"].items() if k.endswith("-normal") or k.endswith("-normal100")}
    blob = json.dumps({"sourceCommit": frozen["sourceCommit"], "traces": keep}, separators=(",", ":"))
    OUT.write_bytes(gzip.compress(blob.encode(), 9, mtime=0))
    print(f"{len(keep)} traces -> {OUT} ({OUT.stat().st_size} B)")


if __name__ == "__main__":
    main()
