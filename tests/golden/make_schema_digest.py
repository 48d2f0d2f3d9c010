"""Derive tests/golden/plan_schema_digest.json from the reference's plan schema.

    python tests/golden/make_schema_digest.py --reference <tt-flow source tree>

The digest keeps, for every object in tensixflow's schema/plan.schema.json, its
required keys, whether extra keys are allowed, and each property's JSON type
(and enum, if any): enough for tests/test_front.py to check the plan JSON that
this backend emits against the reference's contract without reading the
reference at test time.
"""

import argparse
import os
import json
from pathlib import Path


def digest(node):
    out = {"type": node.get("type")}
    if "enum" in node:
        out["enum"] = node["enum"]
    if node.get("type") == "object":
        out["required"] = node.get("required", [])
        out["additional"] = node.get("additionalProperties", True)
        out["properties"] = {k: digest(v) for k, v in node.get("properties", {}).items()}
    if node.get("type") == "array" and "items" in node:
        out["items"] = digest(node["items"])
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TENSIXFLOW_REFERENCE"),
                    help="root of a tt-flow source tree (default: $TENSIXFLOW_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("name the tt-flow source tree with --reference or TENSIXFLOW_REFERENCE")
    schema = json.loads((Path(a.reference) / "schema" / "plan.schema.json").read_text())
    out = Path(__file__).resolve().parent / "plan_schema_digest.json"
    out.write_text(json.dumps(digest(schema), indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
