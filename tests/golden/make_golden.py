"""Regenerate the golden fixtures under tests/golden/ from the reference's own test data.

The reference holds one numeric golden vector for this path:
``tests/fixtures/motif_parity_cases.json`` -> ``component_checks`` ->
``polynorm_reference_2x3`` (consumed by its ``tests/test_swift_parity_fixtures.py:58``).
This script copies that entry verbatim into ``polynorm_reference_2x3.json``, and the same file's
``configs`` (two tiny model configs with the shape expectations its
``tests/test_swift_parity_fixtures.py:24-44`` checks) into ``model_configs.json``.

Usage: python tests/golden/make_golden.py /path/to/reference/checkout
(runs only where the reference checkout exists; the fixture is committed).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    src = Path(ref_root) / "tests" / "fixtures" / "motif_parity_cases.json"
    cases = json.loads(src.read_text())
    out = dict(configs=cases["configs"], source="reference tests/fixtures/motif_parity_cases.json configs")
    (HERE / "model_configs.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote model_configs.json")
    for entry in cases["component_checks"]:
        if entry["name"] == "polynorm_reference_2x3":
            out = dict(entry, source="reference tests/fixtures/motif_parity_cases.json component_checks")
            (HERE / "polynorm_reference_2x3.json").write_text(json.dumps(out, indent=1) + "\n")
            print("wrote polynorm_reference_2x3.json")
            return
    raise SystemExit("polynorm_reference_2x3 not found")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py /path/to/reference/checkout")
    main(sys.argv[1])
