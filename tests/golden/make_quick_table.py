"""Generate tests/golden/quick_table_128.json from the reference's published quick run (test
infrastructure).

tools/validated/quick.csv is the reference evaluator's CSV (evaluation/evaluate.cpp --quick) from the
reference's own device: the table suite at n = 128 (seed 7, uniform(-1, 1); Scheme I with the table's fixed
slice counts, Scheme II with fixed_bits 54 and one reconstruction pass). This keeps its rows for the
formats built on B200 (BF16, FP16, TF32, FP8, INT8): what the plan reported and the output hash. Run
where the reference tree exists (OZTT_REFERENCE_DIR, or a directory named `reference` beside the
repository); the GPU machine reads the fixture.

    OZTT_REFERENCE_DIR=<reference tree> python tests/golden/make_quick_table.py
"""

from __future__ import annotations

import csv
import json
import os
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
SOURCE = Path(os.environ.get("OZTT_REFERENCE_DIR", REPO.parent / "reference")) / "tools" / "validated" / "quick.csv"
OUT = Path(__file__).resolve().parent / "quick_table_128.json"
FORMATS = ("BF16", "FP16", "TF32", "FP8", "INT8")
KEEP = ("scheme", "format", "slices", "integer_bits", "moduli", "passes", "partial_products", "output_hash",
        "effective_bits", "relative_fro")


def main() -> None:
    rows = []
    with SOURCE.open() as f:
        for i, row in enumerate(csv.DictReader(f), start=2):  # line 1 is the header
            if row["suite"] == "table" and row["n"] == "128" and row["format"] in FORMATS:
                rec = {key: row[key] for key in KEEP}
                rec["source_line"] = i
                rows.append(rec)
    OUT.write_text(json.dumps({"source": "tools/validated/quick.csv", "rows": rows}, indent=1) + "\n")
    print(f"wrote {OUT} ({len(rows)} rows)")


if __name__ == "__main__":
    main()
