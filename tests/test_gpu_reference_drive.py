"""The reference's own composite-FSS truncation pipeline (composite_gen_trunc_gate
+ composite_eval_batch_with_postproc + its postproc hooks, compiled from the
reference sources into oracle/_ref/ref_composite_drive) with
proto::SufB200Backend plugged in as its PFSS backend: keygen through our
gen_dcf, evaluation through our eval_dcf_many_u64 (host x^) and
eval_dcf_many_u64_device_broadcast (device x^), reconstruction checked against
plaintext and the reference's ClearBackend."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
EXE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "ref_composite_drive"


@pytest.mark.skipif(not EXE.exists(), reason="oracle/_ref/ref_composite_drive not built (needs the reference checkout)")
def test_reference_composite_pipeline_on_b200_backend(torch_cuda):
    r = subprocess.run([str(EXE)], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().endswith("OK")
