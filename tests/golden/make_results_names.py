"""Extract the row names of the reference's published results table into
``reference_results_row_names.json`` (names only, in file order).

    python tests/golden/make_results_names.py <reference checkout>/results/rtx4070-laptop.json

The reference's checkout is not needed to run the tests: the extracted list is
committed beside this script.
"""

from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    src = sys.argv[1]
    with open(src, encoding="utf-8") as f:
        doc = json.load(f)
    out = {
        "source": "results/" + os.path.basename(src) + " of the reference (rows[].name)",
        "top_level_keys": list(doc),
        "row_keys": sorted({k for r in doc["rows"] for k in r}),
        "names": [r["name"] for r in doc["rows"]],
    }
    with open(os.path.join(HERE, "reference_results_row_names.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(f"{len(out['names'])} names")


if __name__ == "__main__":
    main()
