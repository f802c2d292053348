"""Writes tests/golden/reference_cases.json: the case specifications of the reference's own
forecast tests (its tests/cases.json: batch, variates, context, horizon, seed, series shape,
missingness and covariate layout of each case), restricted to the cases it runs on its tiny
checkpoint. tests/test_reference_cases_gpu.py drives the GPU forecast and the oracle with the
inputs these specifications describe (timestral_b200.synthetic.reference_case_inputs).

Run from the repository root with the reference checkout at $TIMESTRAL_REFERENCE or beside
the repository:
    python tests/golden/make_reference_cases.py
"""
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
KEYS = ("name", "B", "V", "T", "H", "seed", "series", "missing", "past", "known", "cat_past", "cat_known")


def main():
    env = os.environ.get("TIMESTRAL_REFERENCE")
    cands = ([Path(env)] if env else []) + [ROOT.parent / "reference"]
    src = next((c / "tests" / "cases.json" for c in cands if (c / "tests" / "cases.json").is_file()), None)
    if src is None:
        sys.exit("reference checkout not found (set TIMESTRAL_REFERENCE)")
    cases = json.loads(src.read_text())["cases"]
    out = [{k: c[k] for k in KEYS if k in c} for c in cases if c.get("tiny")]
    (Path(__file__).resolve().parent / "reference_cases.json").write_text(json.dumps(out, indent=1) + "\n")
    print(f"{len(out)} cases")


if __name__ == "__main__":
    main()
