"""Generate tests/golden/kbench_yhash.json from the reference's recorded kbench results.

The reference's kbench (engine/bench/kbench.c:181-260) runs its Q4K x A8 kernel on seeded
inputs (kb_fill_matrix seed 42, kb_fill_vec seed 7) and records yhash = FNV-1a of the fp32
outputs Y[n][rows] (kbench.c:212-214) in the RESULT lines saved under bench/results/*.json.
This script collects every Q4K yhash recorded there, keeps only values that every run agrees
on, and writes them as a fixture. It needs the reference checkout and runs only where one is
mounted; the fixture it writes is what the tests read.

    python tests/golden/make_kbench_yhash.py /path/to/reference
"""
from __future__ import annotations

import glob
import json
import os
import sys
from collections import defaultdict
from pathlib import Path


def collect(ref: Path) -> dict:
    seen: dict[tuple, set] = defaultdict(set)
    files: dict[tuple, set] = defaultdict(set)

    def walk(o, fname):
        if isinstance(o, dict):
            if o.get("dtype") == "q4k" and "yhash" in o and o.get("bench", "kbench") == "kbench":
                key = (o["shape"], int(o["rows"]), int(o["cols"]), int(o["n"]))
                seen[key].add(o["yhash"])
                files[key].add(fname)
            for v in o.values():
                walk(v, fname)
        elif isinstance(o, list):
            for v in o:
                walk(v, fname)

    for f in sorted(glob.glob(str(ref / "bench" / "results" / "*.json"))):
        try:
            data = json.loads(Path(f).read_text())
        except (OSError, ValueError):
            continue
        walk(data, Path(f).name)
    cases = []
    for key in sorted(seen):
        if len(seen[key]) != 1:      # disagreeing records pin nothing
            continue
        shape, rows, cols, n = key
        cases.append({"shape": shape, "rows": rows, "cols": cols, "n": n,
                      "yhash": next(iter(seen[key])), "sources": sorted(files[key])[:3]})
    return {"about": "Q4K x A8 yhash values recorded by the reference's kbench "
                     "(FNV-1a over fp32 Y[n][rows]); inputs kb_fill_matrix(seed 42), "
                     "kb_fill_vec(seed 7)", "matrix_seed": 42, "vec_seed": 7, "cases": cases}


def main() -> None:
    # the reference checkout: argument, $NB_REFERENCE, else `reference` beside this repository
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else
               os.environ.get("NB_REFERENCE", Path(__file__).resolve().parents[3] / "reference"))
    out = Path(__file__).with_name("kbench_yhash.json")
    out.write_text(json.dumps(collect(ref), indent=1) + "\n")
    print(f"wrote {out}")


if __name__ == "__main__":
    main()
