"""Regenerate tests/golden/trunc_tapes.npz: composite tapes of truncation gates
written by the reference's own code (gates::composite_gen_trunc_gate with
mt19937_64(seed), then gates::composite_write_tapes), run by
oracle/_ref/tape_fixture (oracle/tape_fixture.cpp, built from the reference
headers and src/compiler/suf_to_pfss.cpp with the adapter in dealer-only mode;
needs the reference checkout, found by oracle.reference_root():
$SUF_REFERENCE or BASELINE.json's reference_path).

Cases: FaithfulTR, FaithfulARS and GapARS at f = 12 (seeds 1, 2) and f = 1
(seed 3: r_low = 1; seed 5: r_low = 0, no carry queries).  Per case i the
archive holds tape0_i / tape1_i (uint8) and a row of meta (kind, f, seed,
r_in, bit_order, pred-key count).
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
KINDS = {"tr": 0, "ars": 1, "gapars": 2}  # SUFB200_TRUNC_* numbering


def main() -> None:
    sys.path.insert(0, str(ROOT))
    from oracle.oracle import reference_root

    ref = reference_root()
    if ref is None:
        raise SystemExit("no reference checkout: set SUF_REFERENCE")
    subprocess.run(["make", "-C", str(ROOT / "oracle"), f"REF={ref}", "tape"], check=True)
    out = subprocess.run([str(ROOT / "oracle" / "_ref" / "tape_fixture")], check=True, capture_output=True,
                         text=True).stdout
    cases = json.loads(out)["cases"]
    arrays = {}
    meta = np.zeros((len(cases), 6), dtype=np.uint64)
    for i, c in enumerate(cases):
        arrays[f"tape0_{i}"] = np.frombuffer(bytes.fromhex(c["tape0"]), dtype=np.uint8)
        arrays[f"tape1_{i}"] = np.frombuffer(bytes.fromhex(c["tape1"]), dtype=np.uint8)
        meta[i] = [KINDS[c["kind"]], c["frac_bits"], c["seed"], int(c["r_in"]), c["bit_order"], c["pred_keys"]]
    np.savez(HERE / "trunc_tapes.npz", meta=meta, **arrays)
    print("wrote", HERE / "trunc_tapes.npz", file=sys.stderr)


if __name__ == "__main__":
    main()
