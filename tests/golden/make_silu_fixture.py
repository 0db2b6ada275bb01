"""Regenerate tests/golden/silu_gate_f12_seed3.json: the reference's own dealer
for the SiLU spline gate (configs[2]: f = 12, 16 segments, seed 3), run by
oracle/_ref/silu_fixture (oracle/silu_fixture.cpp, built from the reference
headers and src/compiler/suf_to_pfss.cpp with the adapter in dealer-only
mode; needs the reference checkout, found by oracle.reference_root():
$SUF_REFERENCE or BASELINE.json's reference_path).

The fixture holds the compiled coefficient program's shape (interval-LUT
mode, degree 0, r = 4 coefficient words c0..c3), r_in, the output masks and
both parties' shares of them, both parties' interval-LUT keys (reference
IntervalKeyHeader blobs), the gate's SUF table (alpha cutpoints, per-piece
coefficient words) and suf::eval_suf_ref on 256 sample inputs (Gaussian
sigma = 4 at f = 12 plus the spline's breakpoints and the ring's extremes).
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def main() -> None:
    sys.path.insert(0, str(ROOT))
    from oracle.oracle import reference_root

    ref = reference_root()
    if ref is None:
        raise SystemExit("no reference checkout: set SUF_REFERENCE")
    subprocess.run(["make", "-C", str(ROOT / "oracle"), f"REF={ref}", "silu"], check=True)
    out = subprocess.run([str(ROOT / "oracle" / "_ref" / "silu_fixture"), "12", "3", "256"], check=True,
                         capture_output=True, text=True).stdout
    data = json.loads(out)
    (HERE / "silu_gate_f12_seed3.json").write_text(json.dumps(data, indent=0) + "\n")
    print("wrote", HERE / "silu_gate_f12_seed3.json", file=sys.stderr)


if __name__ == "__main__":
    main()
