"""Write tests/golden/config_cases.json: the reference's coded rows for cut-down batches of every
benchmark configuration, with that configuration's exact tables (cases in tests/config_cases.py).

The reference CPU path is run from its compiled sources (``oracle/build_ref.py`` -> oracle/_ref):
``rans*_push`` / ``rans*_pop`` (and their alias / inverse-cdf forms) exactly as its callers bind
them, alias tables from its own ``rans_alias_build_table``, and the ragged case one stream at a
time (B = 1).  For each case the file keeps the digest of the inputs, the pushed stream's row
width, each row's length and the SHA-256 of its payload bytes, and the same after the full pop.

Run where the reference checkout exists ($TORCH_ANS_REFERENCE, or ``reference`` beside this
repository):
    python oracle/build_ref.py && python tests/golden/make_config_golden.py
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402
from tests import config_cases as CC  # noqa: E402


def main():
    build_ref.build()
    ref = build_ref.load()
    if ref is None:
        raise SystemExit("compiled reference not available (run oracle/build_ref.py)")
    out = {}
    for case in CC.CASES:
        out[case.name] = CC.reference_record(case, ref)
        print(case.name, out[case.name]["streams"], "streams", out[case.name]["symbols"], "symbols")
    with open(CC.FIXTURE, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", CC.FIXTURE, os.path.getsize(CC.FIXTURE), "bytes")


if __name__ == "__main__":
    main()
